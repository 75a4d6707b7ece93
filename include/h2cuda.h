/* h2cuda: the B200 (sm_100a) backend of the H2 engine's Qwen2 Q4_0 token loop, as a plain C ABI.
 *
 * This is the drop-in boundary. It replaces the reference's WebAssembly kernel exports
 * (h2-own-inference-engine/engine/kernels.c:418-496: set_config / set_tensor / set_buffers / run /
 * profile_* / run_read_test), which its CPU backend host binds (cpu-worker.js:85-137, 169-182), and it
 * implements the backend object contract of cpu.js:52-68 / webgpu.js:616-620 one layer up:
 *   forward(ids, pos, {temperature, seed, wantLogits}) -> next token id   => h2c_forward
 *   readLogits()                                                          => h2c_read_logits
 *   profile(ids, pos)                                                     => h2c_profile
 *   destroy()                                                             => h2c_destroy
 *
 * Ownership differs from the reference on purpose: there, JavaScript owns all memory (set_buffers); here the
 * library owns the device weights, the KV cache, the scratch buffers and the CUDA graph of a decode step, and
 * callers pass only host pointers. No torch types cross this boundary.
 *
 * Every call returns a status (H2C_OK = 0, negative on error) and never aborts; h2c_last_error() gives the
 * message of the last failing call on that engine. Calls on one engine must be serialised by the caller (the
 * reference keeps a single outstanding request per backend, cpu.js:33-50).
 */
#ifndef H2CUDA_H
#define H2CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define H2C_OK 0
#define H2C_ERR_INVALID (-1)      /* bad argument or call order */
#define H2C_ERR_CONTEXT_FULL (-2) /* pos + n >= ctx: "context full", cpu-worker.js:173, webgpu.js:552 */
#define H2C_ERR_BAD_TYPE (-3)     /* unsupported tensor type: cpu-worker.js:105, 112, 126 */
#define H2C_ERR_CUDA (-4)         /* a CUDA runtime call failed */
#define H2C_ERR_NOT_READY (-5)    /* forward before every tensor was set */
#define H2C_ERR_NO_MEMORY (-6)    /* device or pinned allocation failed */
#define H2C_ERR_TIMEOUT (-7)      /* a bounded device-side wait expired (persistent decode kernel, tcgen05 matmul) or a
                                     tensor-parallel peer did not answer within the engine's deadline */
#define H2C_ERR_UNSUPPORTED (-8)  /* tensor parallelism without an NCCL library (libnccl.so.2) in the process */

/* GGML tensor types accepted by h2c_set_tensor (gguf.js:6) */
#define H2C_GGML_F32 0
#define H2C_GGML_Q4_0 2
#define H2C_GGML_Q8_0 8

/* tensor kinds: the numbering of the reference's set_tensor (kernels.c:422-430) */
#define H2C_KIND_QKV 0         /* [Wq; Wk; Wv] rows concatenated, Q4_0 (cpu-worker.js:60, 108-115) */
#define H2C_KIND_O 1           /* attn_output, Q4_0 */
#define H2C_KIND_GATE_UP 2     /* [Wgate; Wup] rows concatenated, Q4_0 */
#define H2C_KIND_DOWN 3        /* ffn_down, Q4_0 */
#define H2C_KIND_ATTN_NORM 4   /* F32 [dim] */
#define H2C_KIND_FFN_NORM 5    /* F32 [dim] */
#define H2C_KIND_QKV_BIAS 6    /* F32 [dim + 2*kv_heads*head_dim]: [bq; bk; bv] */
#define H2C_KIND_EMBED 7       /* token_embd, Q4_0 [vocab][dim] */
#define H2C_KIND_OUTPUT 8      /* output.weight, Q8_0 (the reference's only type) or Q4_0; unset = tied to EMBED */
#define H2C_KIND_OUTPUT_NORM 9 /* F32 [dim] */

/* Model and runtime configuration: set_config(dim, layers, ffn, heads, kvh, vocab, ctx, mt, eps)
 * (kernels.c:418-421) plus the RoPE base the reference host uses for its table (cpu-worker.js:131-135). */
typedef struct h2c_config {
  int32_t dim, layers, ffn, heads, kv_heads, vocab;
  int32_t ctx;        /* positions per sequence (KV cache length); forward needs pos + n < ctx */
  int32_t max_chunk;  /* tokens per prefill pass (the reference's mt / prefillChunk: cpu.js:46) */
  int32_t max_seqs;   /* independent sequences (sessions), each with its own KV cache; >= 1 */
  float eps;          /* RMSNorm epsilon */
  double rope_theta;  /* RoPE frequency base (gguf.js:82) */
} h2c_config;

typedef struct h2c_engine h2c_engine;

/* Per-operation device time of one forward pass, in the reference's profile order (cpu-worker.js:32). */
#define H2C_NPROF 11
/* 0 embed, 1 norm+quantize, 2 matvec qkv, 3 rope+kv, 4 attention, 5 quantize, 6 matvec o, 7 matvec gate+up,
 * 8 swiglu+quantize, 9 matvec down, 10 matvec output */

/* Create an engine on CUDA device `device`: allocates the KV cache and scratch (replaces set_config +
 * set_buffers, kernels.c:418-437 and the layout of cpu-worker.js:52-88). With max_chunk >= 32 the scratch includes
 * the score buffer of prompt passes: heads x max_chunk x ctx floats, at most 256 MB (the environment variable
 * H2C_PROMPT_SCORES_MB, read here, sets another cap; longer passes then run in query blocks, same results). */
int h2c_create(int device, const h2c_config* cfg, h2c_engine** out);

/* Tensor parallelism over G GPUs of one node, one process (or thread) per GPU: the 7B configuration split so that
 * each rank reads 1/G of the weights per token (no reference counterpart: the reference runs one CPU process).
 * Every matrix is split by output rows, so each output value is computed whole, in the reference's order, by one
 * rank, and the results stay bit-identical to one GPU's: rank r owns query heads [r*H/G, (r+1)*H/G) with their
 * kv heads (and that part of the KV cache), rows [r*D/G, (r+1)*D/G) of O and of down, rows [r*F/G, (r+1)*F/G) of
 * gate and of up, and rows [r*Vp, r*Vp + Vp) of the lm_head (Vp = vocab / G rounded up to 32 rows). NCCL
 * all-gathers of the attention output, of the residual after O and after down, of the quantized FFN activation and
 * of the logits give every rank the full vectors in between; every rank computes the same token. Requires
 * kv_heads, dim / 32 and ffn / 32 divisible by G (Qwen2-7B: G = 1, 2 or 4; 4 kv heads cannot be split 8 ways).
 *
 * h2c_tp_unique_id: rank 0 creates the group's id (H2C_TP_ID_BYTES bytes) and the host hands it to every rank.
 * h2c_create_tp: every rank calls it at about the same time with the same cfg and id; the engine then takes the
 * FULL tensors in h2c_set_tensor and keeps this rank's rows. Every rank must then make the same calls with the same
 * arguments (h2c_forward, h2c_generate, h2c_profile). timeout_ms (<= 0: 120 s) bounds the group's set-up and each
 * call's wait: a peer that never joins or stops answering ends in H2C_ERR_TIMEOUT with the communicator aborted
 * (the engine then only accepts h2c_destroy). Not available with tensor parallelism: h2c_forward_batch,
 * h2c_generate_batch, the persistent decode kernel (steps run on the CUDA graph path), h2c_trace_decode. NCCL is
 * loaded at run time (libnccl.so.2 of the process, else the system's): H2C_ERR_UNSUPPORTED without one. G = 1
 * behaves as h2c_create. */
#define H2C_TP_ID_BYTES 128
int h2c_tp_unique_id(uint8_t* id);
int h2c_create_tp(int device, const h2c_config* cfg, int32_t world, int32_t rank, const uint8_t* id,
                  int32_t timeout_ms, h2c_engine** out);
/* This engine's rank and group size (0 and 1 without tensor parallelism). */
int32_t h2c_tp_rank(const h2c_engine* e);
int32_t h2c_tp_world(const h2c_engine* e);

/* Upload one tensor from host memory holding raw GGUF bytes of `ggml_type` (blocks for Q4_0 / Q8_0, floats for
 * F32). Replaces set_tensor (kernels.c:423-431) and the repack of cpu-worker.js:97-128: the library splits
 * GGUF blocks into its own device layout. `layer` is ignored for kinds 7..9. */
int h2c_set_tensor(h2c_engine* e, int kind, int layer, int ggml_type, const void* data, uint64_t nbytes);

/* Run ids[0..n) of sequence `seq` at positions pos..pos+n-1 (prefill when n > 1, one decode step when n == 1)
 * and return the next token in *next: greedy argmax (ties to the lowest id) when temperature <= 0, else a
 * sample of softmax(logits / temperature) with mulberry32 seeded by (seed + pos) (cpu-worker.js:154-180), drawn on
 * the device (the logits never leave it). temperature is a double, as the reference's JavaScript number is.
 * Prompts run in chunks of max_chunk tokens; logits exist for the last token only (kernels.c:404-414).
 * Replaces run() (kernels.c:454-465) plus the host loop of cpu-worker.js:169-182. */
int h2c_forward(h2c_engine* e, int seq, const int32_t* ids, int32_t n, int32_t pos, double temperature,
                uint32_t seed, int32_t* next);

/* One decode step of n sessions at once (the multi-session serving form, forwardBatch of the CUDA backend; no
 * reference counterpart: the reference serves one session per backend, cpu.js:33-50). Token ids[m] of sequence
 * seqs[m] (distinct) is processed at position pos[m]; next[m] receives its next token, chosen as by h2c_forward
 * (greedy, or sampled with seed + pos[m]). Each weight byte is read once for the whole batch; every token's
 * arithmetic is the single-token arithmetic, so the results equal n separate h2c_forward calls bit for bit.
 * 1 <= n <= min(max_chunk, 256). h2c_read_logits(seqs[m]) returns token m's logits afterwards. */
int h2c_forward_batch(h2c_engine* e, int32_t n, const int32_t* seqs, const int32_t* ids, const int32_t* pos,
                      double temperature, uint32_t seed, int32_t* next);

/* Greedy decode of `steps` tokens of each of n sessions entirely on the device: batched steps as h2c_forward_batch,
 * each step's tokens fed to the next without a host round trip. out_tokens (nullable) receives [n][steps] ids;
 * device_ms (nullable) the CUDA-event time of the steps. Needs pos[m] + steps < ctx. */
int h2c_generate_batch(h2c_engine* e, int32_t n, const int32_t* seqs, const int32_t* ids, const int32_t* pos,
                       int32_t steps, int32_t* out_tokens, float* device_ms);

/* Greedy decode of `steps` tokens of sequence `seq` entirely on the device: first_id is processed at `pos`, each
 * step's argmax becomes the next step's input without a host round trip (the WebGPU backend keeps its sampled
 * token on the GPU the same way, webgpu.js:391, 553-574). out_tokens (nullable) receives the `steps` generated
 * ids; device_ms (nullable) the CUDA-event time of the steps on the engine's stream. Needs pos + steps < ctx.
 * Equivalent to steps calls of h2c_forward(e, seq, &id, 1, pos + i, 0, 0, &id). */
int h2c_generate(h2c_engine* e, int seq, int32_t first_id, int32_t pos, int32_t steps, int32_t* out_tokens,
                 float* device_ms);

/* Decode-step implementations. AUTO (default) uses the persistent kernel when the model fits it (one cooperative
 * launch runs every layer of one or more tokens; weights stream into shared memory ahead of use) and otherwise
 * the CUDA graph of per-operation kernels. Both give bit-identical results. */
#define H2C_DECODE_AUTO 0
#define H2C_DECODE_GRAPH 1
#define H2C_DECODE_PERSISTENT 2
/* Select the decode path; H2C_DECODE_PERSISTENT fails with H2C_ERR_INVALID if the model does not fit it. */
int h2c_set_decode_mode(h2c_engine* e, int mode);
/* The path single-token steps will take: H2C_DECODE_GRAPH or H2C_DECODE_PERSISTENT (< 0 on error). */
int h2c_decode_path(h2c_engine* e);

/* The kernel of passes of several tokens (prompt chunks, batched decode steps), process-wide (no reference
 * counterpart: the reference has one CPU matmul). TCGEN05 takes the Blackwell tensor-core form (tcgen05.mma into
 * TMEM) for Q4_0 matrices, MMA_SYNC the warp-level int8 mma.sync form; AUTO (default) the tcgen05 form for passes of
 * 64 or more tokens and the mma.sync form for fewer (the faster of the two at each size on B200). All are
 * bit-identical to the reference. Takes effect for passes enqueued afterwards (a batch step's CUDA graph keeps the
 * kernel it was captured with). */
#define H2C_MATMUL_AUTO 0
#define H2C_MATMUL_MMA_SYNC 1
#define H2C_MATMUL_TCGEN05 2
int h2c_set_matmul_kernel(int kind);
/* The current setting (H2C_MATMUL_AUTO, _MMA_SYNC or _TCGEN05). */
int h2c_matmul_kernel(void);

/* Profiling aid for the persistent decode kernel: runs h2c_generate's device-side greedy decode once with
 * %globaltimer stamps (nanoseconds) taken at the stage boundaries of every CTA. out receives
 * h2c_decode_ctas(e) * steps * (layers + 1) * 16 entries: [cta][step][layer or lm_head][point], 0 where a point
 * does not apply. The per-operation profile of the reference (profile_start/get, kernels.c:481-483) for this
 * path. Allocates a temporary device buffer. */
int h2c_trace_decode(h2c_engine* e, int seq, int32_t first_id, int32_t pos, int32_t steps, uint64_t* out, int64_t n);

/* Grid size (CTAs) of the persistent decode kernel, 0 when the model takes the graph path; < 0 on error. */
int h2c_decode_ctas(h2c_engine* e);

/* Test aid for the persistent kernel's failure detection (no reference counterpart): every bounded wait of the
 * kernel gives up after timeout_ns (default 2 s), and with stall_cta >= 0 that CTA never publishes its QKV rows,
 * so the CTAs that need them wait until the limit, record the error and every CTA returns; the next
 * h2c_forward / h2c_generate then fails with H2C_ERR_TIMEOUT and the engine stays usable (the affected positions
 * of the KV cache must be recomputed). stall_cta = -1 restores normal operation. No fault, trap or hang. */
int h2c_set_decode_fault(h2c_engine* e, int stall_cta, int64_t timeout_ns);

/* Self-test of the decode kernels' correctly rounded arithmetic (no reference counterpart): compares the fast
 * division by 127 and by 896, reciprocal and square root used on the quantization and RMSNorm paths with CUDA's
 * IEEE-rounded __fdiv_rn / __fsqrt_rn over all 2^32 float bit patterns on `device` and writes the four mismatch
 * counts (all 0 when the fast forms are exact on this GPU) to mismatches[0..3]. */
int h2c_selftest_math(int device, uint64_t* mismatches);

/* Number of kernels one batched decode step of n sessions launches (the kernel nodes of its CUDA graph, which the
 * first h2c_forward_batch / h2c_generate_batch of that size builds); 0 before that; < 0 on error. */
int h2c_batch_kernels(h2c_engine* e, int32_t n);

/* Number of kernels one decode step launches (the kernel nodes of the decode-step CUDA graph); < 0 on error. */
int h2c_decode_kernels(h2c_engine* e);

/* Copy the logits of the last forward of `seq` (vocab floats) to host memory (cpu.js:60-62, webgpu.js:605-611). */
int h2c_read_logits(h2c_engine* e, int seq, float* out, int64_t n);

/* One forward pass like h2c_forward with greedy sampling, timing each operation with CUDA events (no graph):
 * ms[H2C_NPROF] receives milliseconds per operation class (profile_start/get/stop, kernels.c:481-483). */
int h2c_profile(h2c_engine* e, int seq, const int32_t* ids, int32_t n, int32_t pos, double* ms);

/* Free everything the engine owns (cpu.js:67 destroy). Safe on NULL. */
int h2c_destroy(h2c_engine* e);

/* Message of the last error on this engine; with e NULL, of the last failed call on this thread that has no engine
 * (h2c_create, h2c_q4_matvec, h2c_q4_matvec_noalloc). */
const char* h2c_last_error(const h2c_engine* e);

/* Bytes of device memory the engine holds (cpu.js:53 memoryBytes / webgpu.js uploadedBytes). */
int64_t h2c_device_bytes(const h2c_engine* e);

/* ---- Q4_0 matvec, the reference's matmul_q4 (kernels.c:200-273) with its quantize_row (kernels.c:90-114)
 * as a stand-alone device operation: the Q4_0 matvec microbench. Pointers are DEVICE pointers. ---- */

/* Bytes of the device layout of an N x K Q4_0 matrix (values, then fp16 scales). */
uint64_t h2c_q4_matrix_bytes(int32_t n_rows, int32_t k);
/* Convert raw GGUF Q4_0 blocks (host) to the device layout (host buffer of h2c_q4_matrix_bytes). */
int h2c_q4_pack(const void* gguf_blocks, int32_t n_rows, int32_t k, void* packed_host);
/* Scratch bytes h2c_q4_matvec needs for m tokens of length k (the int8 activations and their scales). */
uint64_t h2c_q4_matvec_scratch_bytes(int32_t m, int32_t k);
/* y[m][n] (op)= W[n] . quantize(x[m]) for m < M on `stream` (a cudaStream_t, 0 = default).
 * op: 0 store, 1 add bias[n], 2 accumulate into y (the reference's put(): kernels.c:190-194).
 * w: packed matrix (h2c_q4_pack layout) on the device; x: float32 [M][K]; y: float32 [M][N]; bias: float32 [N]
 * or NULL; scratch: h2c_q4_matvec_scratch_bytes(M, K) bytes of device memory, 16-byte aligned. */
int h2c_q4_matvec(const void* w, int32_t n_rows, int32_t k, const float* x, int32_t m, float* y, int32_t op,
                  const float* bias, void* scratch, void* stream);

/* h2c_q4_matvec without any allocation, for callers that cannot call cudaMalloc (a host that owns all device
 * memory through its own pool, or a latency-critical thread such as a voice pipeline's audio callback, where
 * cudaMalloc can block and synchronize the device). This entry point has no counterpart in the reference.
 * Same arguments and result as h2c_q4_matvec, minus `scratch`: the scratch lives in a fixed 256 KiB
 * __device__ array inside this library (held on every GPU that loads it until the process exits), so m and k are
 * limited to h2c_q4_matvec_scratch_bytes(m, k) <= 262144 (for example m = 32 tokens of k = 4864); larger inputs
 * are rejected with H2C_ERR_INVALID and a message in h2c_last_error(NULL). The first call on a device looks the
 * array's device address up (make it before any stream capture). All calls share the array: calls that overlap
 * on the GPU race and must be serialised by the caller. */
int h2c_q4_matvec_noalloc(const void* w, int32_t n_rows, int32_t k, const float* x, int32_t m, float* y,
                          int32_t op, const float* bias, void* stream);

#ifdef __cplusplus
}
#endif
#endif
