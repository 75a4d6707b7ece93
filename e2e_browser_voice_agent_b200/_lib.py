"""ctypes binding of the CUDA library libh2cuda.so (include/h2cuda.h).

The library is built in-tree by build.py (nvcc, sm_100a). There is no fallback: if the shared library is
missing or cannot be loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libh2cuda.so")

OK = 0
ERR_INVALID, ERR_CONTEXT_FULL, ERR_BAD_TYPE, ERR_CUDA, ERR_NOT_READY, ERR_NO_MEMORY, ERR_TIMEOUT, ERR_UNSUPPORTED = \
    range(-1, -9, -1)
TP_ID_BYTES = 128
GGML_F32, GGML_Q4_0, GGML_Q8_0 = 0, 2, 8
KIND_QKV, KIND_O, KIND_GATE_UP, KIND_DOWN, KIND_ATTN_NORM, KIND_FFN_NORM, KIND_QKV_BIAS, KIND_EMBED, KIND_OUTPUT, \
    KIND_OUTPUT_NORM = range(10)
NPROF = 11
DECODE_AUTO, DECODE_GRAPH, DECODE_PERSISTENT = 0, 1, 2
MATMUL_AUTO, MATMUL_MMA_SYNC, MATMUL_TCGEN05 = 0, 1, 2
PROFILE_NAMES = ["embed", "norm+quantize", "matvec qkv", "rope+kv", "attention", "quantize", "matvec o",
                 "matvec gate+up", "swiglu+quantize", "matvec down", "matvec output"]  # cpu-worker.js:32

# the exported symbols of include/h2cuda.h
EXPORTS = ["h2c_create", "h2c_set_tensor", "h2c_forward", "h2c_forward_batch", "h2c_generate_batch", "h2c_batch_kernels", "h2c_generate", "h2c_decode_kernels", "h2c_set_decode_mode",
           "h2c_decode_path", "h2c_trace_decode", "h2c_decode_ctas", "h2c_set_decode_fault", "h2c_read_logits",
           "h2c_profile", "h2c_destroy", "h2c_selftest_math",
           "h2c_last_error", "h2c_device_bytes", "h2c_q4_matrix_bytes", "h2c_q4_pack", "h2c_q4_matvec_scratch_bytes",
           "h2c_q4_matvec", "h2c_q4_matvec_noalloc", "h2c_set_matmul_kernel", "h2c_matmul_kernel",
           "h2c_tp_unique_id", "h2c_create_tp", "h2c_tp_rank", "h2c_tp_world"]


class Config(C.Structure):
    _fields_ = [("dim", C.c_int32), ("layers", C.c_int32), ("ffn", C.c_int32), ("heads", C.c_int32),
                ("kv_heads", C.c_int32), ("vocab", C.c_int32), ("ctx", C.c_int32), ("max_chunk", C.c_int32),
                ("max_seqs", C.c_int32), ("eps", C.c_float), ("rope_theta", C.c_double)]


class H2CError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


_lib = None


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load libh2cuda.so once; raise if it is absent (the engine has no CPU path)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} is not built; run __graft_entry__.build() (nvcc, sm_100a)")
    L = C.CDLL(path)
    p, i32, u32, u64, i64 = C.c_void_p, C.c_int32, C.c_uint32, C.c_uint64, C.c_int64
    L.h2c_create.argtypes = [C.c_int, C.POINTER(Config), C.POINTER(p)]
    L.h2c_set_tensor.argtypes = [p, C.c_int, C.c_int, C.c_int, p, u64]
    L.h2c_forward.argtypes = [p, C.c_int, p, i32, i32, C.c_double, u32, C.POINTER(i32)]
    L.h2c_forward_batch.argtypes = [p, i32, p, p, p, C.c_double, u32, p]
    L.h2c_generate_batch.argtypes = [p, i32, p, p, p, i32, p, C.POINTER(C.c_float)]
    L.h2c_batch_kernels.argtypes = [p, i32]
    L.h2c_generate.argtypes = [p, C.c_int, i32, i32, i32, p, C.POINTER(C.c_float)]
    L.h2c_decode_kernels.argtypes = [p]
    L.h2c_set_decode_mode.argtypes = [p, C.c_int]
    L.h2c_decode_path.argtypes = [p]
    L.h2c_trace_decode.argtypes = [p, C.c_int, i32, i32, i32, p, i64]
    L.h2c_decode_ctas.argtypes = [p]
    L.h2c_set_decode_fault.argtypes = [p, C.c_int, i64]
    L.h2c_selftest_math.argtypes = [C.c_int, p]
    L.h2c_read_logits.argtypes = [p, C.c_int, p, i64]
    L.h2c_profile.argtypes = [p, C.c_int, p, i32, i32, C.POINTER(C.c_double)]
    L.h2c_destroy.argtypes = [p]
    L.h2c_last_error.argtypes = [p]
    L.h2c_last_error.restype = C.c_char_p
    L.h2c_device_bytes.argtypes = [p]
    L.h2c_device_bytes.restype = i64
    L.h2c_q4_matrix_bytes.argtypes = [i32, i32]
    L.h2c_q4_matrix_bytes.restype = u64
    L.h2c_q4_pack.argtypes = [p, i32, i32, p]
    L.h2c_q4_matvec_scratch_bytes.argtypes = [i32, i32]
    L.h2c_q4_matvec_scratch_bytes.restype = u64
    L.h2c_q4_matvec.argtypes = [p, i32, i32, p, i32, p, i32, p, p, p]
    L.h2c_q4_matvec_noalloc.argtypes = [p, i32, i32, p, i32, p, i32, p, p]
    L.h2c_set_matmul_kernel.argtypes = [C.c_int]
    L.h2c_matmul_kernel.argtypes = []
    L.h2c_tp_unique_id.argtypes = [p]
    L.h2c_create_tp.argtypes = [C.c_int, C.POINTER(Config), i32, i32, p, i32, C.POINTER(p)]
    L.h2c_tp_rank.argtypes = [p]
    L.h2c_tp_rank.restype = i32
    L.h2c_tp_world.argtypes = [p]
    L.h2c_tp_world.restype = i32
    for name in ("h2c_create", "h2c_set_tensor", "h2c_forward", "h2c_forward_batch", "h2c_generate_batch", "h2c_batch_kernels", "h2c_generate", "h2c_decode_kernels", "h2c_set_decode_mode",
                 "h2c_decode_path", "h2c_trace_decode", "h2c_decode_ctas", "h2c_set_decode_fault", "h2c_read_logits",
                 "h2c_profile", "h2c_selftest_math",
                 "h2c_destroy", "h2c_q4_pack", "h2c_q4_matvec", "h2c_q4_matvec_noalloc", "h2c_set_matmul_kernel",
                 "h2c_matmul_kernel", "h2c_tp_unique_id", "h2c_create_tp"):
        getattr(L, name).restype = C.c_int
    _lib = L
    return L


def check(rc: int, handle=None) -> None:
    if rc != OK:
        msg = load().h2c_last_error(handle)
        raise H2CError(rc, (msg or b"").decode(errors="replace") or f"h2cuda error {rc}")


def tp_unique_id() -> bytes:
    """A new tensor-parallel group id (rank 0 creates it; every rank passes it to CudaBackend(tp=...))."""
    L = load()
    buf = (C.c_uint8 * TP_ID_BYTES)()
    check(L.h2c_tp_unique_id(C.cast(buf, C.c_void_p)), None)
    return bytes(buf)
