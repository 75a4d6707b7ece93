"""Regenerate the golden fixtures of this directory from the reference's own CPU kernels.

The fixtures pin the oracle restatement (oracle/h2_oracle.c) without needing the reference at test time: each
one holds, for a seeded model built by e2e_browser_voice_agent_b200.synth, the SHA-256 of the GGUF file, the
prompt, the teacher-forced token stream and the logits of every step, as computed by oracle/_ref/libh2ref_st.so
(h2-own-inference-engine/engine/kernels.c compiled unmodified through oracle/shim, driven by oracle/oracle.py,
which restates cpu-worker.js). Run from the repository root after `make -C oracle`:

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle")]

import oracle as O  # noqa: E402
from e2e_browser_voice_agent_b200 import synth  # noqa: E402

CASES = [
    # name, model config, prompt length, chunk (mt), decode steps, prompt seed, forced-token seed
    ("tiny_mt4", "tiny", 9, 4, 6, 11, 12),
    ("small_mt16", "small", 20, 16, 5, 21, 22),
    ("gqa7_mt3", "gqa7", 7, 3, 4, 31, 32),
    ("smallq8_mt16", "small-q8", 12, 16, 4, 41, 42),
]


def make(name, model, n_prompt, mt, steps, s_prompt, s_forced):
    path = synth.ensure(model)
    eng = O.open_model("ref_st", path, ctx=64, mt=mt)
    V = eng.cfg["vocab"]
    prompt = synth.prompt_ids(V, n_prompt, seed=s_prompt)
    forced = synth.prompt_ids(V, steps, seed=s_forced)
    logits, nexts = [], []
    r = eng.forward(prompt, 0, want_logits=True)
    logits.append(r["logits"])
    nexts.append(r["next"])
    pos = n_prompt
    for t in forced:
        r = eng.forward([int(t)], pos, want_logits=True)
        logits.append(r["logits"])
        nexts.append(r["next"])
        pos += 1
    np.savez_compressed(os.path.join(HERE, name + ".npz"), model=model, sha256=synth.file_sha256(path),
                        prompt=prompt, forced=forced, mt=mt, logits=np.stack(logits), next=np.array(nexts, np.int32),
                        generator="oracle/_ref/libh2ref_st.so (reference kernels.c)")


if __name__ == "__main__":
    for c in CASES:
        make(*c)
        print("wrote", c[0])
