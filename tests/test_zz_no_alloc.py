"""h2c_q4_matvec_noalloc: the Q4_0 matvec for callers that cannot call cudaMalloc.

Such callers (a host that owns all device memory through its own pool, or a latency-critical thread like a voice
pipeline's audio callback, where cudaMalloc can block and synchronize the device) get the same result as
h2c_q4_matvec without passing scratch memory: the library keeps a fixed 256 KiB device array for it. This file
is collected last so that a failure here cannot hide the rest of the suite, and it must pass both alone in a
fresh process and after the other tests.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from e2e_browser_voice_agent_b200 import _lib
from e2e_browser_voice_agent_b200 import gguf as G

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def packed_matrix(L, N, K, seed):
    rng = np.random.default_rng(seed)
    blocks = G.q4_0_quantize(rng.standard_normal(N * K, dtype=np.float32) * np.float32(0.02))
    packed = np.zeros(L.h2c_q4_matrix_bytes(N, K), np.uint8)
    assert L.h2c_q4_pack(blocks.ctypes.data, N, K, packed.ctypes.data) == 0
    return torch.from_numpy(packed).cuda()


@pytest.mark.parametrize("N,K,M", [(896, 896, 1), (4864, 896, 3), (896, 4864, 2), (151936, 896, 1)])
def test_noalloc_matches_scratch_entry_point_twice(N, K, M):
    """Two calls in a row (different inputs and ops) agree bit for bit with h2c_q4_matvec on the same inputs."""
    assert torch.cuda.is_available()
    L = _lib.load()
    w = packed_matrix(L, N, K, seed=N + K)
    scratch = torch.zeros(L.h2c_q4_matvec_scratch_bytes(M, K), dtype=torch.uint8, device="cuda")
    rng = np.random.default_rng(M)
    bias = torch.from_numpy(rng.standard_normal(N, dtype=np.float32)).cuda()
    for call, op in enumerate((1, 2)):
        x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()
        y0 = torch.from_numpy(rng.standard_normal((M, N), dtype=np.float32)).cuda()
        y_ref, y_new = y0.clone(), y0.clone()
        b = bias.data_ptr() if op == 1 else None
        assert L.h2c_q4_matvec(w.data_ptr(), N, K, x.data_ptr(), M, y_ref.data_ptr(), op, b, scratch.data_ptr(), None) == 0
        rc = L.h2c_q4_matvec_noalloc(w.data_ptr(), N, K, x.data_ptr(), M, y_new.data_ptr(), op, b, None)
        assert rc == 0, L.h2c_last_error(None)
        torch.cuda.synchronize()
        assert np.array_equal(bits(y_new.cpu().numpy()), bits(y_ref.cpu().numpy())), f"call {call}"


def test_noalloc_rejects_inputs_beyond_its_buffer():
    L = _lib.load()
    M, K = 64, 4864
    assert L.h2c_q4_matvec_scratch_bytes(M, K) > 256 * 1024
    w = torch.zeros(L.h2c_q4_matrix_bytes(32, K), dtype=torch.uint8, device="cuda")
    x = torch.zeros((M, K), dtype=torch.float32, device="cuda")
    y = torch.zeros((M, 32), dtype=torch.float32, device="cuda")
    rc = L.h2c_q4_matvec_noalloc(w.data_ptr(), 32, K, x.data_ptr(), M, y.data_ptr(), 0, None, None)
    assert rc == _lib.ERR_INVALID
    assert b"static buffer" in L.h2c_last_error(None)


def test_noalloc_on_a_second_device():
    """The library sets its kernels' shared-memory limits and looks the scratch address up per device: a call on
    device 1 after calls on device 0 (no engine ever created on device 1) gives h2c_q4_matvec's result there."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two visible GPUs")
    L = _lib.load()
    N, K, M = 4864, 896, 3
    rng = np.random.default_rng(9)
    with torch.cuda.device(1):
        w = packed_matrix(L, N, K, seed=5).to("cuda:1")
        x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).to("cuda:1")
        scratch = torch.zeros(L.h2c_q4_matvec_scratch_bytes(M, K), dtype=torch.uint8, device="cuda:1")
        y_ref = torch.zeros((M, N), dtype=torch.float32, device="cuda:1")
        y_new = torch.zeros((M, N), dtype=torch.float32, device="cuda:1")
        assert L.h2c_q4_matvec_noalloc(w.data_ptr(), N, K, x.data_ptr(), M, y_new.data_ptr(), 0, None, None) == 0, \
            L.h2c_last_error(None)
        assert L.h2c_q4_matvec(w.data_ptr(), N, K, x.data_ptr(), M, y_ref.data_ptr(), 0, None, scratch.data_ptr(),
                               None) == 0
        torch.cuda.synchronize()
        assert np.array_equal(bits(y_new.cpu().numpy()), bits(y_ref.cpu().numpy()))


def test_noalloc_reports_a_misaligned_input():
    L = _lib.load()
    N, K, M = 32, 96, 1
    w = torch.zeros(L.h2c_q4_matrix_bytes(N, K), dtype=torch.uint8, device="cuda")
    x = torch.zeros(K + 4, dtype=torch.float32, device="cuda")
    y = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    rc = L.h2c_q4_matvec_noalloc(w.data_ptr(), N, K, x.data_ptr() + 4, M, y.data_ptr(), 0, None, None)
    assert rc == _lib.ERR_INVALID
    msg = L.h2c_last_error(None)
    assert msg.startswith(b"h2c_q4_matvec_noalloc:") and b"16-byte aligned" in msg
