"""Benchmark: batch-1 greedy decode of the seeded Qwen2.5-0.5B-architecture Q4_0 model (tied Q4_0 lm_head), the
configuration the reference's headline metric is quoted on: 24 layers, hidden 896, 14 q / 2 kv heads, FFN 4864,
vocab 151936, 32 uniform-random prompt ids, then greedy decode of 64 tokens.

A step is one decode token. The timed region runs K steps as rounds of the 64-token decode (positions 32..95,
restarting from the prompt's cache after each round), so every step reads all 278 MB of weights plus its KV cache.
The weights (278 MB) exceed the 126 MB L2, so no L2 flush is needed between steps.

  value  tokens/s over all ranks, device-timed with CUDA events around K device-chained decode steps (the next
         token never leaves the GPU; inputs resident in HBM).
  e2e    the same K steps through the reference-facing per-token call (h2c_forward, as LLM.generateIds drives
         be.forward): each step copies its token id and position host -> device and reads the next id back.

Multi-GPU (torchrun, one rank per GPU): independent sessions, one per rank, weights replicated, no collective on
the data path ("weak" scaling); timing barriers and the max-over-ranks reduction use NCCL.

--workload c4: multi-session serving, 32 concurrent sessions per GPU (128-token prompts, then greedy decode) in
batched steps (h2c_forward_batch / h2c_generate_batch: every weight byte read once per step for all 32 tokens).
A step is one batched decode step (32 tokens); value = tokens/s over all ranks, device-timed around K device-chained
batched steps; e2e = the same steps through the host-driven per-step call (ids and positions copied in, 32 next
ids read back).

--impl reference: the reference's own CPU kernels (kernels.c, compiled natively through oracle/shim into
oracle/_ref, driven like cpu-worker.js) on this host's cores, same workload, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
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
WEIGHT_BYTES = 201_277_440 + 286_208 + 76_575_744
KV_BYTES_PER_POS = 24 * 2 * 64 * 4 * 2


# DRAM bytes (read + write) of one decode step of k_decode_persistent, from the ncu capture of a 4-step launch at
# positions 32..35 (profiles/k_decode_persistent_qwen2-0.5b_full.md): 1,123,380,992 B / 4
NCU_TRAFFIC_PER_STEP = 280_845_248


def step_bytes(pos: int) -> int:
    """Bytes one decode step at position pos must move (T = pos + 1 cached positions read, one written)."""
    return WEIGHT_BYTES + KV_BYTES_PER_POS * (pos + 1) + KV_BYTES_PER_POS + 504


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.out = None

    def start(self):
        try:
            self.out = tempfile.TemporaryFile(mode="w+")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.gpu)], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.seek(0)
        sm, mx, reasons, n = [], None, set(), 0
        for line in self.out.read().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            n += 1
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": n}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    return world, rank, local


def reference_arm(args, world, rank):
    """The reference's CPU path (oracle/_ref) on this host: rank 0 only."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from e2e_browser_voice_agent_b200 import synth

    kind = "ref_mt" if O.available("ref_mt") else "oracle"
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
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
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot / f32", "data": "synthetic (seeded GGUF)",
            "config": {"workload": "qwen2-0.5b Q4_0 tied, batch 1, 32 prompt + greedy decode rounds of 64",
                       "prompt": PROMPT, "decode_round": ROUND},
            "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": decode_threads,
                             "kind": "reference" if kind == "ref_mt" else "port",
                             "sample": f"{steps} decode steps (positions 32..95), {cores} host cores visible, "
                                       f"{decode_threads} decode threads (cpu.js:23 default)"},
            "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline_sample():
    """Reference CPU path timed on this host (rank 0 only): 64 decode steps of the same workload."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from e2e_browser_voice_agent_b200 import synth
    kind = "ref_mt" if O.available("ref_mt") else "oracle"
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
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


C4_SESSIONS = 32
C4_PROMPT = 128
C4_DECODE = 128
C4_METRIC = "decode tok/s multi-session (32 concurrent per GPU) Qwen2-0.5B Q4_0"


def bench_c4(args, world, rank, local):
    import torch
    import torch.distributed as dist
    from e2e_browser_voice_agent_b200 import backend, sessions, synth

    torch.cuda.set_device(local)
    if world > 1:
        sessions.init("nccl")
    steps = min(args.steps if args.steps is not None else C4_DECODE, C4_DECODE)
    warm = max(3, args.warmup)
    S = C4_SESSIONS
    path = synth.ensure("qwen2-0.5b")
    be = backend.open_model(path, ctx=C4_PROMPT + C4_DECODE + 1, prefill_chunk=S, max_seqs=S, device=local)
    # rank r serves sessions r, r + world, ... of a 32 x world set (weak scaling), 32 at a time
    sids = sessions.shard(S * world, world, rank)
    first = []
    for i, sid in enumerate(sids):
        first.append(be.forward(synth.prompt_ids(151936, C4_PROMPT, seed=sessions.session_seed(sid)), 0, seq=i))
    seqs = list(range(S))
    pos = [C4_PROMPT] * S

    def barrier():
        sessions.barrier()
        torch.cuda.synchronize()

    be.generate_batch(seqs, first, pos, warm)
    clocks = Clocks(local)
    barrier()
    clocks.start()
    _, ms = be.generate_batch(seqs, first, pos, steps)
    barrier()
    ck = clocks.stop()
    ms = sessions.max_over_ranks(ms, device="cuda")
    value = world * S * steps / (ms / 1e3)

    def host_steps(n):
        cur, p = list(first), list(pos)
        for _ in range(n):
            cur = be.forward_batch(seqs, cur, p)
            p = [x + 1 for x in p]

    host_steps(warm)
    barrier()
    t0 = time.perf_counter()
    host_steps(steps)
    barrier()
    e2e_s = sessions.max_over_ranks(time.perf_counter() - t0, device="cuda")
    e2e = world * S * steps / e2e_s

    mean_pos = C4_PROMPT + (steps - 1) / 2
    bytes_step = WEIGHT_BYTES + S * (KV_BYTES_PER_POS * (int(round(mean_pos)) + 2) + 504)
    peak, peak_kind = measured_peaks()
    achieved = bytes_step / (ms / steps / 1e3) / 1e9
    kernels = be.batch_kernels(S)
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline_sample()
            cpu["sample"] += "; sessions run one after another on the CPU, so its multi-session rate is the same"
        except Exception as ex:
            cpu = {"value": None, "unit": UNIT, "cores": 0, "kind": "reference", "sample": f"failed: {ex}"}
    be.destroy()
    if rank == 0:
        line = {
            "metric": C4_METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": steps,
            "warmup": warm, "ms_per_step": round(ms / steps, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 dot / f32 accumulate (Q4_0 weights)",
            "data": "synthetic: seeded GGUF, N(0,0.02) weights quantised to Q4_0, uniform-random prompt ids",
            "config": {"workload": f"c4: {S} concurrent sessions per GPU, {C4_PROMPT}-token prompts, batched greedy "
                                   f"decode steps (positions {C4_PROMPT}..{C4_PROMPT + steps - 1})",
                       "global_batch": S * world, "seq_len": C4_PROMPT + steps, "parallelism": f"sessions x{world}",
                       "l2": "no flush: 278 MB of weights per step > 126 MB L2"},
            "roofline": {"bound": "hbm", "kernel": f"batched decode step ({kernels} kernels in one CUDA graph; "
                                                   "k_matmul_tc: int8 tensor-core block dots, 32 tokens per weight load)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind, "bytes_per_step": bytes_step,
                         "traffic": None},
            "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": 4 * 4 + 3 * 4 * 256,
                    "d2h_bytes_per_step": 4 * S},
            "gpu_launches": kernels * steps,
            "clocks": ck,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="c1", choices=["c1", "c4"])
    args = ap.parse_args()
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        return reference_arm(args, world, rank)
    if args.workload == "c4":
        return bench_c4(args, world, rank, local)

    import torch
    import torch.distributed as dist
    from e2e_browser_voice_agent_b200 import backend, sessions, synth

    torch.cuda.set_device(local)
    if world > 1:
        sessions.init("nccl")
    steps = args.steps if args.steps is not None else 3200
    warm = max(3, args.warmup)

    def barrier():
        sessions.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        return sessions.max_over_ranks(x, device="cuda")

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
    barrier()
    clocks.start()
    ms, calls = device_rounds(steps)
    barrier()
    ck = clocks.stop()
    ms = max_over_ranks(ms)
    value = world * steps / (ms / 1e3)

    # ---- e2e: the per-token reference-facing call, host buffers, host<->device copies in the timed region
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
    barrier()
    t0 = time.perf_counter()
    host_rounds(e2e_steps)
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e = world * e2e_steps / e2e_s

    # ---- roofline of the decode step (the unit the kernels of one step form), from the device-timed region
    mean_pos = PROMPT + (ROUND - 1) / 2
    bytes_step = step_bytes(int(round(mean_pos)))
    peak, peak_kind = measured_peaks()
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

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline_sample()
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"value": None, "unit": UNIT, "cores": 0, "kind": "reference", "sample": f"failed: {ex}"}
    be.destroy()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": steps,
            "warmup": warm, "ms_per_step": round(ms / steps, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 dot / f32 accumulate (Q4_0 weights)",
            "data": "synthetic: seeded GGUF, N(0,0.02) weights quantised to Q4_0, uniform-random prompt ids",
            "config": {"workload": "qwen2-0.5b Q4_0 tied lm_head, batch 1, 32-token prompt then greedy decode "
                                   "rounds of 64 (positions 32..95)",
                       "global_batch": world, "seq_len": PROMPT + ROUND, "parallelism": f"sessions x{world}",
                       "l2": "no flush: 278 MB of weights per step > 126 MB L2"},
            "roofline": {"bound": "hbm", "kernel": kdesc,
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "bytes_per_step": bytes_step,
                         "traffic": NCU_TRAFFIC_PER_STEP if persistent else None,
                         "traffic_note": "DRAM read+write bytes per decode step, ncu capture of k_decode_persistent"},
            "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "clocks": ck,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
