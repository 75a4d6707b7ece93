"""Benchmark: batch-1 greedy decode of the seeded Qwen2.5-0.5B-architecture Q4_0 model (tied Q4_0 lm_head), the
configuration the reference's headline metric is quoted on: 24 layers, hidden 896, 14 q / 2 kv heads, FFN 4864,
vocab 151936, 32 uniform-random prompt ids, then greedy decode of 64 tokens.

A step is one decode token. The timed region runs K steps as rounds of the 64-token decode (positions 32..95,
restarting from the prompt's cache after each round), so every step reads all 278 MB of weights plus its KV cache.
The weights (278 MB) exceed the 126 MB L2, so no L2 flush is needed between steps.

  value  tokens/s over all ranks, device-timed with CUDA events around K device-chained decode steps (the next
         token never leaves the GPU; inputs resident in HBM).
  e2e    the same K steps through the reference-facing per-token call (h2c_forward, as LLM.generateIds drives
         be.forward): each step passes its token id and position from the host and reads the next id back.

The same line carries the other configurations of the hot path as nested records, measured in the same process on
every rank (so a multi-GPU run records each at every N):
  multi_session  32 concurrent sessions per GPU (128-token prompts, then batched greedy decode steps: every weight
                 byte read once per step for all 32 tokens), device-timed; e2e through the per-step batched call;
  prefill        prompt passes of 32 (the C1 prompt), 128, 512 and 4096 tokens through h2c_forward;
  microbench     the Q4_0 matvec shapes (one token), with weight copies rotated so that bytes come from HBM, and
                 the two small shapes also L2-resident;
  long_context   a 4096-token prompt, then device-chained greedy decode at positions 4096..
  c5_7b          the 7B architecture: 512-token prompt, then 256 device-chained greedy decode steps; on N GPUs
                 tensor-parallel groups (tp.plan: TP 2 on 2 GPUs, TP 4 on 4, two TP-4 groups on 8) with NCCL
                 all-gathers inside the decode step's CUDA graph
Multi-GPU (torchrun, one rank per GPU): independent sessions per rank, weights replicated, no collective on the
data path ("weak" scaling); timing barriers and the max-over-ranks reduction use NCCL.

--workload c4 prints the multi-session record alone as the line; --workload prefill the prompt passes and the
long-context decode alone.
--impl reference: the reference's own CPU kernels (kernels.c, compiled natively through oracle/shim into
oracle/_ref, driven like cpu-worker.js) on this host's cores, same workload and config, rank 0 only (one CPU
process whatever N is; the other ranks exit without work).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s @bs1 Qwen2-0.5B Q4_0"
UNIT = "tok/s"
PROMPT = 32
ROUND = 64
# algorithmic bytes of one decode step at the 0.5B configuration (tied Q4_0 lm_head): layer weights, norms and
# biases, lm_head, plus 24,576 B of fp32 KV read per cached position and 24,576 B written per step
LAYER_WEIGHT_BYTES = 201_277_440
NORM_BIAS_BYTES = 286_208
LM_HEAD_BYTES = 76_575_744
WEIGHT_BYTES = LAYER_WEIGHT_BYTES + NORM_BIAS_BYTES + LM_HEAD_BYTES
KV_BYTES_PER_POS = 24 * 2 * 64 * 4 * 2
EMBED_ROW_BYTES = 504
# multiply-accumulates per token of the 0.5B layers (Q4_0: 18 bytes per 32 weights)
LAYER_MACS = LAYER_WEIGHT_BYTES // 18 * 32

# DRAM bytes (read + write) of one decode step of k_decode_persistent, from the ncu capture of a 4-step launch at
# positions 32..35: 1,123,380,992 B / 4
NCU_TRAFFIC_PER_STEP = 280_845_248
# DRAM bytes (read + write) of one batched 32-session step, ncu launch list of two steps of the timed region
# (bench.py --workload c4 --steps 2): 933,209,344 B / 2
NCU_TRAFFIC_C4_STEP = 466604672

C1_CONFIG = {"workload": "qwen2-0.5b Q4_0 tied lm_head, batch 1, 32-token prompt then greedy decode rounds of 64 "
                         "(positions 32..95)",
             "l2": "no flush: 278 MB of weights per step > 126 MB L2"}

C4_SESSIONS = 32
C4_PROMPT = 128
C4_DECODE = 128
C4_METRIC = "decode tok/s multi-session (32 concurrent per GPU) Qwen2-0.5B Q4_0"
C3_PROMPT = 4096
C3_DECODE = 64
C2_SHAPES = [(896, 896), (128, 896), (4864, 896), (896, 4864), (151936, 896)]
# the 7B configuration: 512-token prompt, 256 greedy decode tokens; bytes per decode token (Q4_0 layers, norms and
# biases, untied Q4_0 lm_head) and KV bytes per cached position (28 layers x 4 kv heads x 128 dims x f32 x K,V)
C5_PROMPT = 512
C5_DECODE = 256
C5_WEIGHT_BYTES = 3_670_474_752 + 1_333_248 + 306_561_024
C5_KV_BYTES_PER_POS = 28 * 4 * 128 * 4 * 2
C5_LAYER_PARAMS = 6_525_288_448  # 28 layers x 233,046,016 weights


def step_bytes(pos: int) -> int:
    """Bytes one decode step at position pos must move (T = pos + 1 cached positions read, one written)."""
    return WEIGHT_BYTES + KV_BYTES_PER_POS * (pos + 1) + KV_BYTES_PER_POS + EMBED_ROW_BYTES


def c1_positions(steps: int):
    """Positions of K timed C1 steps (rounds of the 64-token decode starting at the prompt's end)."""
    return [PROMPT + (k % ROUND) for k in range(steps)]


def peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, source) from MEASURED_PEAKS.json, else the documented fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class Clocks:
    """SM clocks and throttle reasons sampled through NVML by a thread while the timed region runs (every 2 ms, so
    short regions get samples too)."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap"}

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self.stop_ev = threading.Event()
        self.th = None
        self.ok = False

    def _run(self, h, N):
        while True:
            try:
                self.samples.append((N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM),
                                     N.nvmlDeviceGetCurrentClocksEventReasons(h)))
            except Exception:
                pass
            if self.stop_ev.wait(0.002):
                break

    def start(self):
        try:
            import pynvml as N
            N.nvmlInit()
            dev = os.environ.get("CUDA_VISIBLE_DEVICES")
            idx = int(dev.split(",")[self.gpu]) if dev and dev.split(",")[0].isdigit() else self.gpu
            h = N.nvmlDeviceGetHandleByIndex(idx)
            self.max = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            self.th = threading.Thread(target=self._run, args=(h, N), daemon=True)
            self.th.start()
            self.ok = True
        except Exception:
            self.ok = False

    def stop(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        self.stop_ev.set()
        self.th.join(timeout=2)
        sm = [s for s, _ in self.samples]
        reasons = sorted({name for _, r in self.samples for bit, name in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max, "reasons": reasons,
                "samples": len(sm), "source": "NVML, every 2 ms during the timed region"}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    return world, rank, local


def host_cores():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def c1_config(world: int):
    return dict(C1_CONFIG, global_batch=world, seq_len=PROMPT + ROUND, parallelism=f"sessions x{world}")


def reference_arm(args, world, rank):
    """The reference's CPU path (oracle/_ref) on this host: rank 0 only, one CPU process whatever N is."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from e2e_browser_voice_agent_b200 import synth

    kind = "ref_mt" if O.available("ref_mt") else "oracle"
    cores = host_cores()
    decode_threads = max(1, math.ceil(cores / 2))  # cpu.js:23 default for generation
    path = synth.ensure("qwen2-0.5b")
    eng = O.open_model(kind, path, ctx=PROMPT + ROUND + 1, mt=16, threads=cores, decode_threads=decode_threads)
    prompt = synth.prompt_ids(151936, PROMPT, seed=1)
    first = eng.forward(prompt, 0)["next"]
    steps = args.steps if args.steps is not None else 64
    warm = args.warmup

    def run(n):
        nxt, k = first, 0
        t = 0.0
        while k < n:
            pos = PROMPT + (k % ROUND)
            if k % ROUND == 0:
                nxt = first
            t0 = time.perf_counter()
            nxt = eng.forward([nxt], pos)["next"]
            t += time.perf_counter() - t0
            k += 1
        return t

    run(warm)
    t = run(steps)
    v = steps / t
    line = {"metric": METRIC, "value": round(v, 3), "unit": UNIT, "impl": "reference", "n_gpus": world,
            "steps": steps, "warmup": warm, "ms_per_step": round(t / steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot / f32 accumulate (Q4_0 weights)",
            "data": "synthetic: seeded GGUF, N(0,0.02) weights quantised to Q4_0, uniform-random prompt ids",
            "config": c1_config(world),
            "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": decode_threads,
                             "kind": "reference" if kind == "ref_mt" else "port",
                             "sample": f"{steps} decode steps (positions 32..95), {cores} host cores visible, "
                                       f"{decode_threads} decode threads (cpu.js:23 default); one CPU process on "
                                       f"rank 0's host for any number of GPUs"},
            "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline_sample():
    """Reference CPU path timed on this host (rank 0 only): 64 decode steps of the same workload."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from e2e_browser_voice_agent_b200 import synth
    kind = "ref_mt" if O.available("ref_mt") else "oracle"
    cores = host_cores()
    dt = max(1, math.ceil(cores / 2))
    eng = O.open_model(kind, synth.ensure("qwen2-0.5b"), ctx=PROMPT + ROUND + 1, mt=16, threads=cores,
                       decode_threads=dt)
    nxt = eng.forward(synth.prompt_ids(151936, PROMPT, seed=1), 0)["next"]
    t0 = time.perf_counter()
    for i in range(ROUND):
        nxt = eng.forward([nxt], PROMPT + i)["next"]
    t = time.perf_counter() - t0
    return {"value": round(ROUND / t, 3), "unit": UNIT, "cores": dt,
            "kind": "reference" if kind == "ref_mt" else "port",
            "sample": f"{ROUND} greedy decode steps after the 32-token prompt (the full per-token workload), "
                      f"{dt} decode threads of {cores} host cores (cpu.js:23 default)"}


class nvtx_range:
    """An NVTX range around a timed region (for profiler launch filters such as ncu --nvtx-include "c4_timed/")."""

    def __init__(self, name):
        self.name = name

    def __enter__(self):
        import torch
        torch.cuda.nvtx.range_push(self.name)

    def __exit__(self, *a):
        import torch
        torch.cuda.nvtx.range_pop()


class Ctx:
    """Per-process benchmark context: rank, world, barrier and max-over-ranks."""

    def __init__(self, world, rank, local):
        self.world, self.rank, self.local = world, rank, local

    def barrier(self):
        import torch
        from e2e_browser_voice_agent_b200 import sessions
        sessions.barrier()
        torch.cuda.synchronize()

    def max(self, x: float) -> float:
        from e2e_browser_voice_agent_b200 import sessions
        return sessions.max_over_ranks(x, device="cuda")


def measure_c4(cx: Ctx, steps: int, warm: int):
    """Multi-session serving: 32 sessions per GPU in batched decode steps. Returns the record."""
    from e2e_browser_voice_agent_b200 import backend, sessions, synth
    S = C4_SESSIONS
    steps = min(steps, C4_DECODE)
    be = backend.open_model(synth.ensure("qwen2-0.5b"), ctx=C4_PROMPT + C4_DECODE + 1, prefill_chunk=S, max_seqs=S,
                            device=cx.local)
    sids = sessions.shard(S * cx.world, cx.world, cx.rank)  # rank r serves sessions r, r + world, ...
    prompts = [synth.prompt_ids(151936, C4_PROMPT, seed=sessions.session_seed(sid)) for sid in sids]
    # prefill of the 32 prompts (one h2c_forward each, 4 chunks of 32 tokens), wall clock
    cx.barrier()
    t0 = time.perf_counter()
    first = [be.forward(p, 0, seq=i) for i, p in enumerate(prompts)]
    prefill_s = cx.max(time.perf_counter() - t0)
    seqs = list(range(S))
    pos = [C4_PROMPT] * S
    be.generate_batch(seqs, first, pos, warm)
    clocks = Clocks(cx.local)
    cx.barrier()
    clocks.start()
    with nvtx_range("c4_timed"):
        _, ms = be.generate_batch(seqs, first, pos, steps)
    cx.barrier()
    ck = clocks.stop()
    ms = cx.max(ms)
    value = cx.world * S * steps / (ms / 1e3)

    def host_steps(n):
        cur, p = list(first), list(pos)
        for _ in range(n):
            cur = be.forward_batch(seqs, cur, p)
            p = [x + 1 for x in p]

    host_steps(warm)
    cx.barrier()
    t0 = time.perf_counter()
    host_steps(steps)
    cx.barrier()
    e2e_s = cx.max(time.perf_counter() - t0)
    e2e = cx.world * S * steps / e2e_s
    # bytes: weights once per step + every session's KV (positions C4_PROMPT .. C4_PROMPT + steps - 1)
    tot = sum(WEIGHT_BYTES + S * (KV_BYTES_PER_POS * (p + 2) + EMBED_ROW_BYTES)
              for p in range(C4_PROMPT, C4_PROMPT + steps))
    bytes_step = tot / steps
    hbm, _, src = peaks()
    achieved = bytes_step / (ms / steps / 1e3) / 1e9
    kernels = be.batch_kernels(S)
    be.destroy()
    return {
        "metric": C4_METRIC, "value": round(value, 2), "unit": UNIT, "steps": steps, "warmup": warm,
        "ms_per_step": round(ms / steps, 5), "higher_is_better": True, "scaling": "weak",
        "config": {"workload": f"c4: {S} concurrent sessions per GPU, {C4_PROMPT}-token prompts, batched greedy "
                               f"decode steps (positions {C4_PROMPT}..{C4_PROMPT + steps - 1})",
                   "global_batch": S * cx.world, "seq_len": C4_PROMPT + steps, "parallelism": f"sessions x{cx.world}",
                   "l2": "no flush: 278 MB of weights per step > 126 MB L2"},
        "roofline": {"bound": "hbm", "kernel": f"batched decode step ({kernels} kernels in one CUDA graph)",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "peak_source": src, "bytes_per_step": round(bytes_step), "traffic": NCU_TRAFFIC_C4_STEP,
                     "traffic_note": "DRAM read+write bytes per batched step, ncu launch list of the step's kernels"},
        "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": 4 * 4 + 3 * 4 * 256,
                "d2h_bytes_per_step": 4 * S},
        "prompt_prefill_ms": round(prefill_s * 1e3, 2),
        "gpu_launches": kernels * steps, "clocks": ck,
    }


def measure_prefill_and_c3(cx: Ctx, decode_steps: int):
    """Prompt passes of 128, 512 and 4096 tokens (one engine with 256-token chunks), then the long-context decode
    after the 4096-token prompt. Returns (prefill records, long-context record)."""
    import torch
    from e2e_browser_voice_agent_b200 import backend, synth
    _, bf16, src = peaks()
    int8_peak = 2 * bf16  # the dense int8 tensor rate is twice the bf16 rate
    be = backend.open_model(synth.ensure("qwen2-0.5b"), ctx=C3_PROMPT + C3_DECODE + 2, prefill_chunk=256,
                            device=cx.local)
    pre = {}
    for n in (128, 512, 4096):
        prompt = synth.prompt_ids(151936, n, seed=7 + n)
        reps = 3 if n < 4096 else 1
        be.forward(prompt[:64], 0)  # warm-up
        ts = []
        for _ in range(reps):
            cx.barrier()
            t0 = time.perf_counter()
            with nvtx_range(f"prefill_{n}"):
                first = be.forward(prompt, 0)
            torch.cuda.synchronize()
            ts.append(time.perf_counter() - t0)
        t = cx.max(min(ts))
        ops = 2 * LAYER_MACS * n
        pre[str(n)] = {"tokens": n, "ms": round(t * 1e3, 3), "tok_per_s": round(n / t, 1),
                       "roofline": {"bound": "tensor", "achieved": round(ops / t / 1e12, 2), "peak": int8_peak,
                                    "unit": "int8 TOP/s", "frac": round(ops / t / 1e12 / int8_peak, 5),
                                    "peak_source": f"2 x {src} bf16 (dense int8 rate)",
                                    "ops": ops, "ops_note": "2 x layer weights x tokens (attention excluded)"}}
    # long context: device-chained greedy decode after the 4096-token prompt (first = that prompt's next token)
    be.generate(first, C3_PROMPT, 4)
    clocks = Clocks(cx.local)
    cx.barrier()
    clocks.start()
    with nvtx_range("c3_timed"):
        _, ms = be.generate(first, C3_PROMPT, decode_steps)
    cx.barrier()
    ck = clocks.stop()
    ms = cx.max(ms)
    hbm, _, src = peaks()
    tot = sum(step_bytes(p) for p in range(C3_PROMPT, C3_PROMPT + decode_steps))
    achieved = tot / (ms / 1e3) / 1e9
    lc = {"metric": "decode tok/s long context (4096-token prompt) Qwen2-0.5B Q4_0",
          "value": round(cx.world * decode_steps / (ms / 1e3), 2), "unit": UNIT, "steps": decode_steps,
          "ms_per_step": round(ms / decode_steps, 5), "positions": [C3_PROMPT, C3_PROMPT + decode_steps - 1],
          "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                       "frac": round(achieved / hbm, 4), "peak_source": src,
                       "bytes_per_step": round(tot / decode_steps)},
          "kernel": be.decode_path, "clocks": ck}
    be.destroy()
    return pre, lc


def measure_c2(cx: Ctx):
    """The Q4_0 matvec shapes (one token): us per call and GB/s with weight copies rotated (>= 256 MB in rotation,
    so the bytes come from HBM), and the two small shapes also L2-resident (the same copy back to back)."""
    import numpy as np
    import torch
    from e2e_browser_voice_agent_b200 import _lib
    from e2e_browser_voice_agent_b200 import gguf as G
    L = _lib.load()
    hbm, _, src = peaks()
    dev = torch.device("cuda", cx.local)
    stream = torch.cuda.current_stream(dev)
    out = {}
    rng = np.random.default_rng(0)
    for N, K in C2_SHAPES:
        blocks = G.q4_0_quantize(rng.standard_normal(N * K, dtype=np.float32) * np.float32(0.02))
        packed = np.zeros(L.h2c_q4_matrix_bytes(N, K), np.uint8)
        assert L.h2c_q4_pack(blocks.ctypes.data, N, K, packed.ctypes.data) == 0
        w0 = torch.from_numpy(packed).to(dev)
        copies = max(1, math.ceil(256e6 / packed.nbytes))
        ws = [w0] + [w0.clone() for _ in range(copies - 1)]
        x = torch.from_numpy(rng.standard_normal(K, dtype=np.float32)).to(dev)
        y = torch.zeros(N, dtype=torch.float32, device=dev)
        scratch = torch.zeros(L.h2c_q4_matvec_scratch_bytes(1, K), dtype=torch.uint8, device=dev)
        algo = N * K // 32 * 18 + 4 * K + 4 * N

        def run(seq):
            for w in seq:
                rc = L.h2c_q4_matvec(w.data_ptr(), N, K, x.data_ptr(), 1, y.data_ptr(), 0, None, scratch.data_ptr(),
                                     stream.cuda_stream)
                if rc:
                    _lib.check(rc)

        rec = {"bytes": algo}
        for mode, seq in (("hbm", ws * max(1, 200 // len(ws))), ("l2", [w0] * 200)):
            if mode == "l2" and N * K > 4864 * 896:
                continue
            run(seq[:20])
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(stream)
            run(seq)
            e1.record(stream)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / len(seq)
            gbs = algo / (us * 1e-6) / 1e9
            rec[mode] = {"us_per_call": round(us, 3), "gbs": round(gbs, 1), "frac": round(gbs / hbm, 4),
                         "calls": len(seq)}
        out[f"{N}x{K}"] = rec
        del ws
    return {"note": "h2c_q4_matvec, one token: quantize_row kernel + matvec kernel per call (2 launches), CUDA events "
                    "on the launching stream; 'hbm' rotates weight copies (>= 256 MB), 'l2' repeats one copy",
            "peak": hbm, "peak_source": src, "shapes": out}


def measure_c5(cx: Ctx):
    """The 7B configuration: seeded weights generated on the device (synth.device_tensors), a 512-token prompt (two
    256-token passes on the tcgen05 matmul), then 256 device-chained greedy decode steps (per-op CUDA graph path; the
    7B rows are too long for the persistent kernel's tiles). On N GPUs: tensor-parallel groups of G = tp.plan(N)
    ranks (NCCL all-gathers inside the step's CUDA graph), N / G groups decoding independent sequences."""
    import torch
    from e2e_browser_voice_agent_b200 import _lib, backend, synth, tp
    t0 = time.perf_counter()
    cfg, src = synth.device_tensors("qwen2-7b", seed=0, device=cx.local)
    G, reps = tp.plan(cfg, cx.world)
    tpa = None
    if G > 1:
        tpa = (G, cx.rank % G, tp.exchange_ids(cx.world, cx.rank, G, _lib.tp_unique_id))
    be = backend.CudaBackend(src, None, cfg, ctx=C5_PROMPT + C5_DECODE + 2, prefill_chunk=256, device=cx.local,
                             tp=tpa, tp_timeout_ms=120000)
    load_s = time.perf_counter() - t0
    prompt = synth.prompt_ids(cfg["vocab"], C5_PROMPT, seed=5 + cx.rank // G)
    be.forward(prompt[:64], 0)  # warm-up
    ts = []
    for _ in range(2):
        cx.barrier()
        t1 = time.perf_counter()
        with nvtx_range("c5_prefill"):
            first = be.forward(prompt, 0)
        torch.cuda.synchronize()
        ts.append(time.perf_counter() - t1)
    pre = cx.max(min(ts))
    be.generate(first, C5_PROMPT, 3)
    clocks = Clocks(cx.local)
    cx.barrier()
    clocks.start()
    with nvtx_range("c5_timed"):
        _, ms = be.generate(first, C5_PROMPT, C5_DECODE)
    cx.barrier()
    ck = clocks.stop()
    ms = cx.max(ms)
    hbm, bf16, src_kind = peaks()
    # bytes one rank reads per step: its 1/G of the weights and of the KV cache
    tot = sum(C5_WEIGHT_BYTES + C5_KV_BYTES_PER_POS * (p + 2) for p in range(C5_PROMPT, C5_PROMPT + C5_DECODE)) / G
    achieved = tot / (ms / 1e3) / 1e9
    ops = 2 * C5_LAYER_PARAMS * C5_PROMPT / G  # one rank's share of the prompt pass's multiply-adds
    path, mem = be.decode_path, be.memory_bytes
    be.destroy()
    par = "none (TP 1)" if G == 1 and reps == 1 else f"tensor parallel {G} (NCCL all-gathers) x {reps} replica(s)"
    return {"metric": "decode tok/s @bs1 Qwen2-7B-architecture Q4_0 (1 GPU)" if cx.world == 1 else
            f"decode tok/s @bs1 Qwen2-7B-architecture Q4_0 ({cx.world} GPUs: TP {G} x {reps})",
            "value": round(reps * C5_DECODE / (ms / 1e3), 2), "unit": UNIT, "steps": C5_DECODE, "n_gpus": cx.world,
            "tp": G, "replicas": reps,
            "ms_per_step": round(ms / C5_DECODE, 5), "positions": [C5_PROMPT, C5_PROMPT + C5_DECODE - 1],
            "config": {"workload": "c5: 28 layers, hidden 3584, 28/4 heads of 128, FFN 18944, vocab 152064, untied "
                                   "Q4_0 lm_head; 512-token prompt then 256 greedy steps", "parallelism": par,
                       "weights": "seeded N(0,0.02) generated on the device, Q4_0", "device_bytes": mem,
                       "load_s": round(load_s, 1)},
            "roofline": {"bound": "hbm", "kernel": f"decode step ({path}), per rank", "achieved": round(achieved, 1),
                         "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4), "peak_source": src_kind,
                         "bytes_per_step": round(tot / C5_DECODE)},
            "prefill": {"tokens": C5_PROMPT, "ms": round(pre * 1e3, 2), "tok_per_s": round(C5_PROMPT / pre, 1),
                        "roofline": {"bound": "tensor", "achieved": round(ops / pre / 1e12, 2), "peak": 2 * bf16,
                                     "unit": "int8 TOP/s", "frac": round(ops / pre / 1e12 / (2 * bf16), 5),
                                     "peak_source": f"2 x {src_kind} bf16 (dense int8 rate)", "ops": ops}},
            "clocks": ck}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="C1 only, without the nested records")
    ap.add_argument("--workload", default="c1", choices=["c1", "c4", "prefill", "c5"])
    args = ap.parse_args()
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        return reference_arm(args, world, rank)

    import torch
    import torch.distributed as dist
    from e2e_browser_voice_agent_b200 import backend, sessions, synth

    torch.cuda.set_device(local)
    if world > 1:
        sessions.init("nccl")
    cx = Ctx(world, rank, local)
    warm = max(3, args.warmup)
    if args.workload == "c5":  # the 7B record alone
        rec = measure_c5(cx)
        if rank == 0:
            print(json.dumps(rec), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.workload == "prefill":  # the prompt passes and the long-context decode alone (one JSON object)
        pre, lc = measure_prefill_and_c3(cx, C3_DECODE)
        if rank == 0:
            print(json.dumps({"prefill": pre, "long_context": lc}), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.workload == "c4":
        rec = measure_c4(cx, args.steps if args.steps is not None else C4_DECODE, warm)
        if rank == 0:
            rec.update({"n_gpus": world, "vs_baseline": None, "dtype": "int8 dot / f32 accumulate (Q4_0 weights)",
                        "data": "synthetic: seeded GGUF, N(0,0.02) weights quantised to Q4_0, uniform-random prompt ids"})
            print(json.dumps(rec), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    steps = args.steps if args.steps is not None else 3200
    path = synth.ensure("qwen2-0.5b")
    be = backend.open_model(path, ctx=PROMPT + ROUND + 1, prefill_chunk=16, device=local)
    # one session per rank (weak scaling): rank r serves session r of a world-sized set
    (sid,) = sessions.shard(world, world, rank)
    prompt = synth.prompt_ids(151936, PROMPT, seed=sessions.session_seed(sid))
    first = be.forward(prompt, 0)

    def device_rounds(n):
        """n decode steps as rounds of the 64-token decode; returns (device ms, generate calls)."""
        ms, k, calls = 0.0, 0, 0
        while k < n:
            s = min(ROUND, n - k)
            _, t = be.generate(first, PROMPT, s)
            ms += t
            k += s
            calls += 1
        return ms, calls

    # ---- value: device-chained decode, device time
    device_rounds(warm)
    clocks = Clocks(local)
    cx.barrier()
    clocks.start()
    with nvtx_range("c1_timed"):
        ms, calls = device_rounds(steps)
    cx.barrier()
    ck = clocks.stop()
    ms = cx.max(ms)
    value = world * steps / (ms / 1e3)

    # ---- e2e: the per-token reference-facing call, host buffers, host<->device transfers in the timed region
    def host_rounds(n):
        k, nxt = 0, first
        while k < n:
            pos = PROMPT + (k % ROUND)
            if k % ROUND == 0:
                nxt = first
            nxt = be.forward([nxt], pos)
            k += 1

    e2e_steps = min(steps, 640)
    host_rounds(warm)
    cx.barrier()
    t0 = time.perf_counter()
    host_rounds(e2e_steps)
    cx.barrier()
    e2e_s = cx.max(time.perf_counter() - t0)
    e2e = world * e2e_steps / e2e_s

    # ---- roofline of the decode step, from the device-timed region and the positions it actually ran
    bytes_step = sum(step_bytes(p) for p in c1_positions(steps)) / steps
    hbm, _, src = peaks()
    achieved = bytes_step / (ms / steps / 1e3) / 1e9
    kernels = be.decode_kernels()
    persistent = be.decode_path == "persistent"
    if persistent:  # one cooperative launch runs a whole generate call (up to 64 device-chained steps)
        kdesc = "k_decode_persistent (one cooperative launch per 64-step round, 1 CTA per SM)"
        launches = calls
        h2d = 3 * 4  # sequence, position and token id, carried in the launch's parameter block
        d2h = 5 * 4  # the record CTA 0 writes into mapped host memory: launch number, next id, 3 status words
    else:
        kdesc = f"decode step ({kernels} kernels in one CUDA graph)"
        launches = kernels * steps
        h2d = 4 * 5  # pass parameters (position, length, sequence, pad, token id)
        d2h = 4
    be.destroy()

    extra = {}
    if not args.no_extra:
        t_extra = time.perf_counter()
        extra["multi_session"] = measure_c4(cx, steps, warm)
        extra["prefill"], extra["long_context"] = measure_prefill_and_c3(cx, C3_DECODE)
        extra["microbench"] = measure_c2(cx)
        extra["c5_7b"] = measure_c5(cx)
        extra["extra_wall_s"] = round(time.perf_counter() - t_extra, 1)

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline_sample()
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"value": None, "unit": UNIT, "cores": 0, "kind": "reference", "sample": f"failed: {ex}"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": steps,
            "warmup": warm, "ms_per_step": round(ms / steps, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 dot / f32 accumulate (Q4_0 weights)",
            "data": "synthetic: seeded GGUF, N(0,0.02) weights quantised to Q4_0, uniform-random prompt ids",
            "config": c1_config(world),
            "roofline": {"bound": "hbm", "kernel": kdesc,
                         "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "peak_source": src,
                         "bytes_per_step": round(bytes_step),
                         "traffic": NCU_TRAFFIC_PER_STEP if persistent else None,
                         "traffic_note": "DRAM read+write bytes per decode step, ncu capture of k_decode_persistent"},
            "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "clocks": ck,
            "cpu_baseline": cpu,
            **extra,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
