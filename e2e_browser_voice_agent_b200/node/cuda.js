// The "cuda" backend of the H2 engine for Node.js: the same object createCPU returns
// (h2-own-inference-engine/engine/cpu.js:52-68), with its work in libh2cuda on a B200 through the N-API addon
// h2cuda.node (h2cuda_node.cc). LLM.load selects it with one more branch (llm.js:23-29):
//
//   } else if (backend === "cuda") {
//     const { createCUDA } = await import("./cuda.js");
//     be = await createCUDA(gguf, bytes, cfg, { ctx, ...opts });
//   }
//
// UNVERIFIED: this build image has no Node.js, so this file runs nowhere here. Its Python counterpart,
// e2e_browser_voice_agent_b200/backend.py, drives the same C ABI and is what the tests exercise.
import { createRequire } from "node:module";

const require = createRequire(import.meta.url);
const h2c = require("./build/Release/h2cuda.node");

// tensor kinds of the reference's set_tensor (kernels.c:422-430)
const KIND = { qkv: 0, o: 1, gu: 2, down: 3, attn_norm: 4, ffn_norm: 5, bqkv: 6, embd: 7, out: 8, out_norm: 9 };
const GGML = { F32: 0, Q4_0: 2, Q8_0: 8 };

export const tpUniqueId = () => h2c.tpUniqueId();

export async function createCUDA(gguf, bytes, cfg, opts = {}) {
  const ctx = opts.ctx || 2048;
  const maxSeqs = opts.maxSeqs || 1;
  const ccfg = {
    dim: cfg.dim, layers: cfg.layers, ffn: cfg.ffn, heads: cfg.heads, kv_heads: cfg.kvHeads, vocab: cfg.vocab,
    ctx, max_chunk: opts.prefillChunk || 16, max_seqs: maxSeqs, eps: cfg.eps, rope_theta: cfg.ropeTheta,
  };
  // opts.tp = {world, rank, id} (id: the Buffer h2c.tpUniqueId() made on rank 0): one rank of a tensor-parallel
  // group, one process per GPU; every rank loads the same file and makes the same calls
  const eng = opts.tp ? h2c.createTp(opts.device ?? 0, ccfg, opts.tp.world, opts.tp.rank, opts.tp.id, opts.tp.timeoutMs ?? 0)
                      : h2c.create(opts.device ?? 0, ccfg);
  const T = gguf.tensors;  // parseGGUF offsets (gguf.js:15-70)
  const need = (name, type) => {
    const t = T[name];
    if (!t) throw new Error(`${name}: missing`);
    if (t.type !== type) throw new Error(`${name}: expected ${type === GGML.Q4_0 ? "Q4_0" : "F32"}`);  // cpu-worker.js:105, 112
    return t;
  };
  const part = (t) => ({ type: t.type, offset: t.offset, nbytes: t.nbytes });
  const put = (kind, layer, t) => h2c.setTensor(eng, kind, layer, t.type, bytes, t.offset, t.nbytes);
  const cat = (kind, layer, ...ts) => h2c.setTensorConcat(eng, kind, layer, bytes, ts.map(part));
  for (let l = 0; l < cfg.layers; l++) {
    const p = `blk.${l}.`;
    const q4 = (n) => need(p + n, GGML.Q4_0), f32 = (n) => need(p + n, GGML.F32);
    cat(KIND.qkv, l, q4("attn_q.weight"), q4("attn_k.weight"), q4("attn_v.weight"));
    put(KIND.o, l, q4("attn_output.weight"));
    cat(KIND.gu, l, q4("ffn_gate.weight"), q4("ffn_up.weight"));
    put(KIND.down, l, q4("ffn_down.weight"));
    put(KIND.attn_norm, l, f32("attn_norm.weight"));
    put(KIND.ffn_norm, l, f32("ffn_norm.weight"));
    cat(KIND.bqkv, l, f32("attn_q.bias"), f32("attn_k.bias"), f32("attn_v.bias"));
    opts.onProgress?.(l + 1, cfg.layers);
  }
  put(KIND.embd, 0, need("token_embd.weight", GGML.Q4_0));
  if (T["output.weight"]) put(KIND.out, 0, T["output.weight"]);  // Q8_0 (or Q4_0); absent: tied to token_embd
  put(KIND.out_norm, 0, need("output_norm.weight", GGML.F32));

  const memoryBytes = h2c.deviceBytes(eng);
  let lastLogits = null;
  return {
    name: "cuda", ctx, threads: 1, build: "libh2cuda.so (sm_100a)", memoryBytes,
    info: `B200 sm_100a, ${maxSeqs} sequence(s) x ${ctx} positions, ${(memoryBytes / 2 ** 20).toFixed(0)} MiB on device`,
    // writes ids at pos and returns the next token; rejects with Error("context full") when pos + ids.length >= ctx
    async forward(ids, pos, { temperature = 0, seed = 1, wantLogits = false, seq = 0 } = {}) {
      const next = await h2c.forward(eng, seq, Int32Array.from(ids), pos, temperature, seed >>> 0);
      lastLogits = wantLogits || opts.keepLogits ? h2c.readLogits(eng, seq, cfg.vocab) : null;
      return next;
    },
    async readLogits() { return lastLogits; },
    rawForward: async (ids, pos) => {
      const t0 = performance.now();
      const next = await h2c.forward(eng, 0, Int32Array.from(ids), pos, 0, 1);
      return { next, ms: performance.now() - t0, logits: h2c.readLogits(eng, 0, cfg.vocab) };
    },
    profile: async (ids, pos) => h2c.profile(eng, 0, Int32Array.from(ids), pos),
    // multi-session serving (no reference counterpart): one decode step of every listed session, token ids[k] of
    // session seqs[k] at position pos[k]; the same tokens as one forward() per session
    forwardBatch: async (seqs, ids, pos, { temperature = 0, seed = 1 } = {}) =>
      Array.from(await h2c.forwardBatch(eng, Int32Array.from(seqs), Int32Array.from(ids), Int32Array.from(pos),
                                        temperature, seed >>> 0)),
    destroy: () => h2c.destroy(eng),
  };
}
