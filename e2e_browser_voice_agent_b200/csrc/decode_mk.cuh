// Persistent decode kernel: every layer of one or more greedy decode steps in a single cooperative launch.
//
// One CTA per SM (grid <= SM count, co-resident by cooperative launch). Each CTA owns a fixed share of every
// matrix, and the engine lays those shares out in HBM in the order the CTA consumes them ("stream layout"). A
// producer warp streams that contiguous region tile by tile into a ring of shared-memory slots with 1D TMA bulk
// copies (cp.async.bulk, completion on an mbarrier), independently of the data dependencies, so the weights of
// the next stages (and of the next token) are on chip before their inputs arrive. Sixteen compute warps run the
// stages.
//
// Batch-1 decode is bound by dependency latency, not bandwidth, so the partition minimises global round trips.
// Data crossing CTAs travels as 64-bit "tagged words" (32-bit payload, 32-bit epoch): a reader spins until the word
// carries the epoch it needs, so the read is itself the synchronisation (one L2 round trip; no counters). Per layer
// (E = layer epoch):
//   all CTAs:          x (tag 2E-1; the embedding at layer 0) -> RMSNorm + int8 quantization -> their QKV rows in
//                      pairs (i, i + HD/2) of a head -> bias, RoPE -> q (tag E); k, v appended to the KV cache and
//                      published (tag E).
//   head CTAs h < H:   q of head h, k and v of its KV head -> attention over the cache (earlier positions
//                      prefetched into shared memory at the start of the layer) -> att[h] (tag E).
//   other CTAs:        att (tag E) -> quantization -> their O rows, x[n] += o[n] -> x rows (tag 2E).
//   all CTAs:          x (tag 2E) -> RMSNorm + quantization -> gate/up rows of whole 32-value act blocks ->
//                      silu(g) * u -> quantized act block (tag E).
//   other CTAs:        act (tag E) -> their down rows, x[n] += down[n] -> x rows (tag 2E+1).
// After the last layer every CTA takes x, the final RMSNorm, its lm_head rows and a local argmax, publishes the
// (value, index) pair and merges all pairs, so every CTA knows the next token without another round trip.
// Tagged words carry their own payload, so relaxed stores and loads suffice, except for the k/v words: their
// writers also store KV-cache rows that other CTAs read at later steps, so those words are released and acquired.
//
// Arithmetic is the reference's, bit for bit (kernels.cuh): lane-ordered float sums as short chains, exact
// integer block dots. Every wait is bounded (a %globaltimer timeout plus an abort word any CTA can set): on
// expiry the kernel records an error code, stops issuing copies, waits (bounded) for the copies in flight and
// returns. It never traps.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "kernels.cuh"

namespace h2 {

constexpr int MK_SLOT = 32768;                   // bytes per ring slot (one tile)
constexpr int MK_NSLOT = 3;                      // ring depth
constexpr int MK_MAX_TILES = 256;                // per-CTA tile table kept in shared memory
constexpr int MK_WARPS = 16;                     // compute warps
constexpr int MK_NT = MK_WARPS * 32;             // compute threads
constexpr int MK_THREADS = MK_NT + 32;           // + one producer warp
constexpr int MK_TILE_ROWS = 64;                 // rows per tile (lm_head, q/k/v)
constexpr int MK_TRACE_PTS = 16;
constexpr int MK_ACT_WORDS = 16;                 // tagged words per act block: 8 int8 quads, d, 4 lane sums
#ifndef MK_POLL_NS
#define MK_POLL_NS 0                             // back-off between polls of a tagged word
#endif

enum { MK_OK = 0, MK_TIMEOUT_WAIT = 1, MK_TIMEOUT_SLOT = 2, MK_ABORTED = 3 };

struct MkTile {          // one entry of a CTA's stream table
  uint64_t off;          // byte offset from the stream base
  uint32_t bytes;        // multiple of 16
  uint16_t rows, nb;     // rows in the tile, 32-value blocks per row
};

struct MkParams {
  int D, F, H, KVH, HD, QKV, L, V, ctx, ncta;
  float eps;
  const uint8_t* stream;          // all tiles
  const MkTile* tiles;            // [ncta][tile_stride]
  const int* tile_count;          // [ncta] tiles per token of each CTA
  int tile_stride;
  int prod_items;                 // float4 entries of the product buffer (max rows * blocks of any tile)
  int kv_stage;                   // cached positions a head CTA stages in shared memory (0: read from L2)
  const float* attn_norm;         // [L][D]
  const float* ffn_norm;          // [L][D]
  const float* bqkv;              // [L][QKV]
  const float* out_norm;          // [D]
  const float* rope;              // [ctx][HD]
  const uint8_t* embd_qs;         // grouped Q4_0 layout
  const __half* embd_d;
  float* kc;
  float* vc;
  float* logits;                  // [V]
  unsigned long long* xw;         // [D] tagged x
  unsigned long long* qw;         // [D] tagged q (after bias and RoPE)
  unsigned long long* kvw;        // [2 KVH HD] tagged k then v of the current position
  unsigned long long* attw;       // [D] tagged att
  unsigned long long* actw;       // [F/32][MK_ACT_WORDS] tagged act blocks
  unsigned long long* lmw;        // [ncta][2] tagged lm_head partials (value, index)
  unsigned long long* kvdone;     // [ncta] epoch of the last layer whose KV-cache rows this CTA has released
  int* err;                       // [4]: code, cta, stage, abort flag
  int32_t* prm;                   // pass parameters (P_POS0, P_M, P_SEQ, P_IDS)
  int32_t* toklog;                // [seqs][ctx + 1]
  int32_t* next;
  int steps;
  unsigned long long timeout_ns;
  unsigned long long* trace;      // optional: [2][steps * (L + 1)][MK_TRACE_PTS] %globaltimer stamps of CTA 0
                                  // and of the last CTA (profiling)
};

// dynamic shared memory of k_decode_persistent without the K/V staging area (must match the carve-up below)
__host__ __device__ inline size_t mk_smem_base(int D, int F, int HD, int ctx, int prod_items) {
  const int nbf = F / 32;
  const int outn = 3 * HD > 64 ? 3 * HD : 64;
  return (size_t)MK_NSLOT * MK_SLOT + (size_t)prod_items * 16 + (size_t)((F + 127) & ~127) +
         (size_t)((nbf + 3) & ~3) * 4 + (size_t)nbf * 16 + (size_t)D * 4 + 64 * 4 + (size_t)outn * 4 + 32 * 4 + 64 +
         (size_t)MK_MAX_TILES * 16 + (size_t)D * 4 * 3 + (size_t)64 * 4 + (size_t)HD * 4 +
         (size_t)((ctx + 3) & ~3) * 4;
}

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned long long ld_acquire64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed64(unsigned long long* p, uint32_t payload, uint32_t tag) {
  const unsigned long long v = ((unsigned long long)tag << 32) | payload;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void st_release64(unsigned long long* p, uint32_t payload, uint32_t tag) {
  const unsigned long long v = ((unsigned long long)tag << 32) | payload;
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int ld_volatile_i(const int* p) { return *(const volatile int*)p; }
__device__ __forceinline__ void compute_bar() { asm volatile("bar.sync 1, %0;" ::"n"(MK_NT) : "memory"); }

// bounded wait on an mbarrier phase; false on timeout or abort
__device__ __forceinline__ bool mbar_wait(uint64_t* b, unsigned parity, const MkParams& p) {
  if (mbar_try_wait(b, parity)) return true;
  const unsigned long long t0 = gtimer();
  for (unsigned it = 0;; it++) {
    if (mbar_try_wait(b, parity)) return true;
    if ((it & 63) == 63) {
      if (ld_volatile_i(p.err + 3)) return false;
      if (gtimer() - t0 > p.timeout_ns) return false;
    }
  }
}

__device__ __forceinline__ void mk_fail(const MkParams& p, int code, int stage) {
  if (atomicCAS(p.err, 0, code) == 0) {
    p.err[1] = blockIdx.x;
    p.err[2] = stage;
  }
  atomicExch(p.err + 3, 1);
  __threadfence();
}

// Spin (bounded) until tagged word w carries an epoch >= tag; returns its payload. On timeout or abort sets
// *abort_s (a shared flag that is only ever raised). ACQ: acquire load (for words published with release).
template <bool ACQ = false>
__device__ __forceinline__ uint32_t wait_word(const unsigned long long* w, uint32_t tag, const MkParams& p, int stage,
                                              int* abort_s) {
  unsigned long long v = ACQ ? ld_acquire64(w) : ld_relaxed64(w);
  if ((uint32_t)(v >> 32) >= tag) return (uint32_t)v;
  const unsigned long long t0 = gtimer();
  for (unsigned it = 0;; it++) {
    __nanosleep(MK_POLL_NS);
    v = ACQ ? ld_acquire64(w) : ld_relaxed64(w);
    if ((uint32_t)(v >> 32) >= tag) return (uint32_t)v;
    if ((it & 31) == 31) {
      if (*(volatile int*)abort_s || ld_volatile_i(p.err + 3)) break;
      if (gtimer() - t0 > p.timeout_ns) {
        mk_fail(p, MK_TIMEOUT_WAIT, stage);
        break;
      }
    }
  }
  *(volatile int*)abort_s = 1;
  return 0;
}

// ---------------------------------------------------------------- shared building blocks

// s = ((s + p[0]) + p[stride]) + ... over n terms in order. The shared-memory loads of the next 16 terms issue
// before the adds of the current 16, so a step costs one add latency, not a load latency.
__device__ __forceinline__ float chain_sum(float s, const float* p, int stride, int n) {
  float a[16], nx[16];
  const int n16 = n & ~15;
  if (n16) {
#pragma unroll
    for (int u = 0; u < 16; u++) a[u] = p[u * stride];
    for (int k = 16; k < n16; k += 16) {
#pragma unroll
      for (int u = 0; u < 16; u++) nx[u] = p[(k + u) * stride];
#pragma unroll
      for (int u = 0; u < 16; u++) s = __fadd_rn(s, a[u]);
#pragma unroll
      for (int u = 0; u < 16; u++) a[u] = nx[u];
    }
#pragma unroll
    for (int u = 0; u < 16; u++) s = __fadd_rn(s, a[u]);
  }
  const int rem = n - n16;
#pragma unroll
  for (int u = 0; u < 16; u++) a[u] = u < rem ? p[(n16 + u) * stride] : 0.f;
#pragma unroll
  for (int u = 0; u < 16; u++)
    if (u < rem) s = __fadd_rn(s, a[u]);
  return s;
}

// the thread -> (block, first row, row step) map of mk_tile_dot for rows of nb blocks, computed once per stage
struct TileMap {
  int b, r0, rstep;
};
__device__ __forceinline__ TileMap tile_map(int nb) {
  TileMap m;
  m.rstep = MK_NT / nb;
  m.b = threadIdx.x % nb;
  m.r0 = threadIdx.x / nb;
  return m;
}

// quantization of nblk 32-value blocks: value i of block b is f(b * 32 + lane); two blocks per warp at a time
template <typename Fn>
__device__ __forceinline__ void mk_quant_blocks(int nblk, Fn f, int8_t* xq, float* xd, int4* xs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int b = warp; b < nblk; b += 2 * MK_WARPS) {
    const int b2 = b + MK_WARPS;
    const float v0 = f(b * 32 + lane);
    const float v1 = b2 < nblk ? f(b2 * 32 + lane) : 0.f;
    quant_block_redux(v0, lane, xq + b * 32, xd + b, xs + b);
    if (b2 < nblk) quant_block_redux(v1, lane, xq + b2 * 32, xd + b2, xs + b2);
  }
  compute_bar();
}

// RMSNorm of xf[0..D) (shared) into int8 blocks xq/xd/xs (shared), the reference's lane order (kernels.c:80-114):
// the squares are formed by all threads into sq (shared, D floats), then thread l < 4 adds sq[4k + l] over k in
// order and ((l0 + l1) + l2) + l3 combines the four chains.
__device__ void mk_norm_quant(const float* xf, const float* w, int D, float eps, int8_t* xq, float* xd, int4* xs,
                              float* red, float* sq) {
  const int tid = threadIdx.x;
  for (int i = tid; i < D; i += MK_NT) sq[i] = __fmul_rn(xf[i], xf[i]);
  compute_bar();
  if (tid < 4) red[tid] = chain_sum(0.f, sq + tid, 4, D / 4);
  compute_bar();
  const float ss = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[1]), red[2]), red[3]);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), eps)));
  mk_quant_blocks(D / 32, [&](int i) { return __fmul_rn(__fmul_rn(xf[i], r), w[i]); }, xq, xd, xs);
}

// plain quantization of xf[0..K) (shared) into shared int8 blocks
__device__ void mk_quant(const float* xf, int K, int8_t* xq, float* xd, int4* xs) {
  mk_quant_blocks(K / 32, [&](int i) { return xf[i]; }, xq, xd, xs);
}

// One tile (R rows, nb blocks; row-major: values [R][nb][16 B], then fp16 scales [R][nb]) against the shared
// int8 input: out[r] = ((l0 + l1) + l2) + l3 of the reference's lane chains (kernels.c:121-139, 209-229).
// Phase 1: a thread owns one 32-value block b (its activations stay in registers) and walks rows r, r + NT/nb, ...
// computing the four exact lane dots and the products f32(p_l) * (dw * dx) into prod (rows padded to 4 nb + 4
// floats so the phase-2 reads are conflict-free). Phase 2: thread (r, l) adds its lane's products in block order.
// Requires nb <= MK_NT.
__device__ __forceinline__ int mk_prod_stride(int nb) { return 4 * nb + 4; }

__device__ void mk_tile_dot(const uint8_t* tile, int R, int nb, const TileMap& m, const int8_t* xq, const float* xd,
                            const int4* xs, float4* prod, float* out) {
  const int tid = threadIdx.x;
  const __half* wd = reinterpret_cast<const __half*>(tile + (((size_t)nb * R * 16 + 15) & ~(size_t)15));
  const int PS = mk_prod_stride(nb);
  float* pf = reinterpret_cast<float*>(prod);
  if (m.r0 < m.rstep) {
    const int b = m.b;
    const int4 x0 = *reinterpret_cast<const int4*>(xq + b * 32);
    const int4 x1 = *reinterpret_cast<const int4*>(xq + b * 32 + 16);
    const int4 s = xs[b];
    const float dx = xd[b];
    for (int r = m.r0; r < R; r += m.rstep) {
      const int it = r * nb + b;
      const uint4 w = *reinterpret_cast<const uint4*>(tile + (size_t)it * 16);
      const float sc = __fmul_rn(__half2float(wd[it]), dx);
      *reinterpret_cast<float4*>(pf + r * PS + 4 * b) =
          make_float4(__fmul_rn(q4_lane(w.x, x0.x, x1.x, s.x), sc), __fmul_rn(q4_lane(w.y, x0.y, x1.y, s.y), sc),
                      __fmul_rn(q4_lane(w.z, x0.z, x1.z, s.z), sc), __fmul_rn(q4_lane(w.w, x0.w, x1.w, s.w), sc));
    }
  }
  compute_bar();
  const int chains = R * 4;
  if (tid < ((chains + 31) & ~31)) {
    float acc = 0.f;
    if (tid < chains) acc = chain_sum(0.f, pf + (tid >> 2) * PS + (tid & 3), 4, nb);
    const float v = hsum4_quad(acc);
    if (tid < chains && (tid & 3) == 0) out[tid >> 2] = v;
  }
  compute_bar();
}

// ---------------------------------------------------------------- the kernel
__global__ void __launch_bounds__(MK_THREADS, 1) k_decode_persistent(const MkParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int D = p.D, F = p.F, H = p.H, KVH = p.KVH, HD = p.HD, L = p.L;
  const int nbd = D / 32, nbf = F / 32;
  uint8_t* ring = smem;                                                     // MK_NSLOT * MK_SLOT
  float4* prod = reinterpret_cast<float4*>(ring + MK_NSLOT * MK_SLOT);      // p.prod_items
  int8_t* xq = reinterpret_cast<int8_t*>(prod + p.prod_items);             // F int8
  float* xd = reinterpret_cast<float*>(xq + ((F + 127) & ~127));          // F/32
  int4* xs = reinterpret_cast<int4*>(xd + ((nbf + 3) & ~3));              // F/32
  float* xf = reinterpret_cast<float*>(xs + nbf);                          // D
  float* xown = xf + D;                                                    // 64 (this CTA's x rows)
  float* outv = xown + 64;                                                 // max(3 HD, 64) (tile results)
  float* red = outv + (3 * HD > 64 ? 3 * HD : 64);                         // 32
  int8_t* actq = reinterpret_cast<int8_t*>(red + 32);                     // 32 B int8, 4 B d, 16 B sums
  float* actd = reinterpret_cast<float*>(actq + 32);
  int4* acts = reinterpret_cast<int4*>(actq + 48);
  MkTile* tsm = reinterpret_cast<MkTile*>(actq + 64);                     // MK_MAX_TILES (this CTA's table)
  float* nw1 = reinterpret_cast<float*>(tsm + MK_MAX_TILES);              // D: attn_norm of the layer
  float* nw2 = nw1 + D;                                                    // D: ffn_norm of the layer
  float* onw = nw2 + D;                                                    // D: output norm
  float* bsm = onw + D;                                                    // 64: bias of this CTA's QKV rows
  float* rsm = bsm + 64;                                                   // HD: RoPE row of the position
  float* sc = rsm + HD;                                                    // ctx (scores)
  const int HDP = HD + 4;                                                  // padded K rows: conflict-free dots
  float* kst = sc + ((p.ctx + 3) & ~3);                                    // kv_stage * HDP
  float* vst = kst + (size_t)p.kv_stage * HDP;                             // kv_stage * HD
  __shared__ __align__(8) uint64_t full[MK_NSLOT], empty[MK_NSLOT];
  __shared__ int abort_s;
  __shared__ int tok_s;

  const int tid = threadIdx.x, cta = blockIdx.x, ncta = p.ncta;
  const MkTile* my_tiles = p.tiles + (size_t)cta * p.tile_stride;

  if (tid == 0) {
    for (int s = 0; s < MK_NSLOT; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_s = 0;
  }
  __syncthreads();

  const int my_count = p.tile_count[cta];
  const int total_tiles = my_count * p.steps;
  // this CTA's tile table and the output norm go to shared memory once (no global load per tile)
  for (int i = tid; i < my_count; i += MK_THREADS) tsm[i] = my_tiles[i];
  for (int i = tid; i < D; i += MK_THREADS) onw[i] = p.out_norm[i];
  __syncthreads();

  // ------------------------------------------------------------ producer warp: stream the CTA's tiles
  if (tid >= MK_NT) {
    if (tid == MK_NT) {
      int issued = 0;
      for (int i = 0; i < total_tiles; i++) {
        const int s = i % MK_NSLOT;
        if (i >= MK_NSLOT) {
          if (!mbar_wait(&empty[s], ((i / MK_NSLOT) - 1) & 1, p)) {
            if (!ld_volatile_i(p.err + 3)) mk_fail(p, MK_TIMEOUT_SLOT, -1);
            break;
          }
        }
        if (ld_volatile_i(p.err + 3)) break;
        const MkTile t = tsm[i % my_count];
        if (t.bytes == 0 || t.bytes > MK_SLOT || (t.bytes & 15) || (t.off & 15)) {
          mk_fail(p, MK_ABORTED, -2);
          break;
        }
        mbar_expect_tx(&full[s], t.bytes);
        bulk_g2s(ring + (size_t)s * MK_SLOT, p.stream + t.off, t.bytes, &full[s]);
        issued = i + 1;
      }
      // drain: every issued copy must land before the CTA exits (bounded; the source is valid memory)
      for (int i = (issued > MK_NSLOT ? issued - MK_NSLOT : 0); i < issued; i++) {
        const unsigned long long t0 = gtimer();
        while (!mbar_try_wait(&full[i % MK_NSLOT], (i / MK_NSLOT) & 1))
          if (gtimer() - t0 > p.timeout_ns) break;
      }
    }
    return;
  }

  // ------------------------------------------------------------ compute warps
  int tile_i = 0;
  // wait for the next tile; the table entry must describe the rows and blocks this stage expects
  auto next_tile = [&](int stage, int rows, int nb) -> const uint8_t* {
    const int s = tile_i % MK_NSLOT;
    if (tid == 0) {
      const MkTile t = tsm[tile_i % my_count];
      if (t.rows != rows || t.nb != nb) {
        mk_fail(p, MK_ABORTED, stage);
        abort_s = 1;
      } else if (!mbar_wait(&full[s], (tile_i / MK_NSLOT) & 1, p)) {
        if (!ld_volatile_i(p.err + 3)) mk_fail(p, MK_TIMEOUT_SLOT, stage);
        abort_s = 1;
      }
    }
    compute_bar();
    return abort_s ? nullptr : ring + (size_t)s * MK_SLOT;
  };
  auto release_tile = [&]() {
    compute_bar();
    if (tid == 0) mbar_arrive(&empty[tile_i % MK_NSLOT]);
    tile_i++;
  };
  // read D tagged floats (x or att) into xf
  auto read_vec = [&](const unsigned long long* src, uint32_t tag, int stage) -> bool {
    for (int i = tid; i < D; i += MK_NT) xf[i] = __uint_as_float(wait_word(src + i, tag, p, stage, &abort_s));
    compute_bar();
    return !abort_s;
  };

  const TileMap map_d = tile_map(nbd), map_f = tile_map(nbf);
  float* sqs = reinterpret_cast<float*>(prod);  // norm squares (prod is free between tiles)
  const bool head = cta < H;
  const int nh = ncta - H;                  // CTAs that own O / down rows
  const int j = cta - H;
  const int o_lo = head ? 0 : (int)((long long)j * D / nh), o_hi = head ? 0 : (int)((long long)(j + 1) * D / nh);
  const int v_lo = (int)((long long)cta * p.V / ncta), v_hi = (int)((long long)(cta + 1) * p.V / ncta);
  const int npair = p.QKV / 2, half = HD / 2;
  const int pr_lo = (int)((long long)cta * npair / ncta), pr_hi = (int)((long long)(cta + 1) * npair / ncta);
  const int G = H / KVH, kh = head ? cta / G : 0;
  const int kv_pair_lo = H * half, kv_pair_hi = (H + 2 * KVH) * half;  // QKV row pairs of the k and v heads
  const bool my_kv = pr_lo < kv_pair_hi && pr_hi > kv_pair_lo;
  const int seq = p.prm[P_SEQ];
  int pos = p.prm[P_POS0];
  int tok = p.prm[P_IDS];
  uint32_t E = 0;  // layer epoch (1-based within the launch)
  unsigned long long* trace = nullptr;
  if (p.trace && (cta == 0 || cta == ncta - 1))
    trace = p.trace + (cta == 0 ? 0 : (size_t)p.steps * (L + 1) * MK_TRACE_PTS);
#define MK_TRACE(row, k) \
  do { if (trace && tid == 0) trace[(size_t)(row) * MK_TRACE_PTS + (k)] = gtimer(); } while (0)

  for (int step = 0; step < p.steps; step++, pos++) {
    // token start: the RoPE row of this position; the embedding row (kernels.c:313-322), from which the O/down
    // owners start their x rows
    if (tid < HD / 4) cp_async16(rsm + 4 * tid, p.rope + (size_t)pos * HD + 4 * tid);
    {
      const int g = tok >> 5, r = tok & 31;
      for (int i = tid; i < D / 2; i += MK_NT) {
        const int blk = i >> 4, jj = i & 15;
        const size_t e = ((size_t)g * nbd + blk) * 32 + r;
        const uint8_t b = p.embd_qs[e * 16 + invperm16(jj)];
        const float s = __half2float(p.embd_d[e]);
        xf[32 * blk + jj] = __fmul_rn((float)((b & 15) - 8), s);
        xf[32 * blk + 16 + jj] = __fmul_rn((float)((b >> 4) - 8), s);
      }
      compute_bar();
      for (int n = o_lo + tid; n < o_hi; n += MK_NT) xown[n - o_lo] = xf[n];
    }

    for (int l = 0; l < L; l++) {
      E++;
      const int trow = step * (L + 1) + l;
      MK_TRACE(trow, 0);
      if (trace && tid == 0) trace[(size_t)trow * MK_TRACE_PTS + 15] = (unsigned long long)clock64();
      const size_t cbase = (((size_t)seq * L + l) * KVH + kh) * (size_t)p.ctx * HD;
      const bool staged = head && pos <= p.kv_stage;
      {
        // this layer's norm weights and QKV bias arrive while the layer's inputs are in flight
        for (int i = tid; i < D / 4; i += MK_NT) {
          cp_async16(nw1 + 4 * i, p.attn_norm + (size_t)l * D + 4 * i);
          cp_async16(nw2 + 4 * i, p.ffn_norm + (size_t)l * D + 4 * i);
        }
        if (tid < 2 * (pr_hi - pr_lo)) {
          const int pidx = pr_lo + (tid >> 1), row = (pidx / half) * HD + pidx % half + (tid & 1) * half;
          cp_async4(bsm + tid, p.bqkv + (size_t)l * p.QKV + row);
        }
        if (head && E > (uint32_t)L) {
          // acquire the KV-cache rows that the k/v owners released at this layer of earlier steps of this launch
          // (rows of earlier launches are ordered by the launch boundary)
          if (tid < ncta) {
            const int c_lo = (int)((long long)tid * npair / ncta), c_hi = (int)((long long)(tid + 1) * npair / ncta);
            if (c_lo < kv_pair_hi && c_hi > kv_pair_lo) wait_word<true>(p.kvdone + tid, E - L, p, 10 * l + 9, &abort_s);
          }
          compute_bar();
          if (abort_s) goto out;
        }
        if (staged) {  // a head CTA's earlier cache positions are final: stage them now
          const float* kb = p.kc + cbase;
          const float* vb = p.vc + cbase;
          for (int i = tid; i < pos * (HD / 4); i += MK_NT) {
            const int t = i / (HD / 4), c4 = i - t * (HD / 4);
            cp_async16(kst + (size_t)t * HDP + 4 * c4, kb + (size_t)t * HD + 4 * c4);
            cp_async16(vst + 4 * i, vb + 4 * i);
          }
        }
        cp_async_commit();
      }

      // ---- A (all CTAs): norm, QKV pairs, bias, RoPE, KV append (kernels.c:328-352)
      if (l > 0 && !read_vec(p.xw, 2 * (E - 1) + 1, 10 * l + 0)) goto out;
      cp_async_wait_all();
      compute_bar();
      MK_TRACE(trow, 1);
      mk_norm_quant(xf, nw1, D, p.eps, xq, xd, xs, red, sqs);
      MK_TRACE(trow, 2);
      {
        const int R = 2 * (pr_hi - pr_lo);
        const uint8_t* t = next_tile(1, R, nbd);
        if (!t) goto out;
        mk_tile_dot(t, R, nbd, map_d, xq, xd, xs, prod, outv);
        release_tile();
        for (int jp = tid; jp < pr_hi - pr_lo; jp += MK_NT) {
          const int pidx = pr_lo + jp, hh = pidx / half, i = pidx % half;
          const float a = __fadd_rn(outv[2 * jp], bsm[2 * jp]);
          const float b = __fadd_rn(outv[2 * jp + 1], bsm[2 * jp + 1]);
          if (hh < H + KVH) {  // q or k head: rotate (kernels.c:341-344)
            const float c = rsm[2 * i], s = rsm[2 * i + 1];
            const float r0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
            const float r1 = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
            if (hh < H) {
              st_relaxed64(p.qw + hh * HD + i, __float_as_uint(r0), E);
              st_relaxed64(p.qw + hh * HD + i + half, __float_as_uint(r1), E);
            } else {
              const int kk = hh - H;
              const size_t base = ((((size_t)seq * L + l) * KVH + kk) * p.ctx + pos) * HD;
              p.kc[base + i] = r0;
              p.kc[base + i + half] = r1;
              st_relaxed64(p.kvw + kk * HD + i, __float_as_uint(r0), E);
              st_relaxed64(p.kvw + kk * HD + i + half, __float_as_uint(r1), E);
            }
          } else {  // v head: appended as is
            const int kk = hh - H - KVH;
            const size_t base = ((((size_t)seq * L + l) * KVH + kk) * p.ctx + pos) * HD;
            p.vc[base + i] = a;
            p.vc[base + i + half] = b;
            st_relaxed64(p.kvw + (KVH + kk) * HD + i, __float_as_uint(a), E);
            st_relaxed64(p.kvw + (KVH + kk) * HD + i + half, __float_as_uint(b), E);
          }
        }
        compute_bar();  // outv is reused below
        // Release of this layer's KV-cache rows (read by the head CTAs from the next step on): one gpu-scope fence
        // after the barrier that orders the CTA's cache stores, then the CTA's kvdone word. Off the critical path:
        // the warp that fences next waits for other CTAs' results anyway.
        if (my_kv && tid == 0) {
          __threadfence();
          st_relaxed64(p.kvdone + cta, E, E);
        }
      }
      MK_TRACE(trow, 3);

      if (head) {
        // ---- B: attention of head h over the cache (kernels.c:355-377)
        const int T = pos + 1;
        float* q_s = outv;
        float* knew = outv + HD;
        float* vnew = outv + 2 * HD;
        for (int i = tid; i < 3 * HD; i += MK_NT) {
          float v;
          if (i < HD) v = __uint_as_float(wait_word(p.qw + cta * HD + i, E, p, 10 * l + 1, &abort_s));
          else if (i < 2 * HD) v = __uint_as_float(wait_word<true>(p.kvw + kh * HD + (i - HD), E, p, 10 * l + 1, &abort_s));
          else v = __uint_as_float(wait_word<true>(p.kvw + (KVH + kh) * HD + (i - 2 * HD), E, p, 10 * l + 1, &abort_s));
          outv[i] = v;
        }
        compute_bar();
        if (abort_s) goto out;
        MK_TRACE(trow, 4);
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
        float mx = -1e30f;
        for (int t = tid; t < T; t += MK_NT) {
          float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
          if (t == pos || staged) {
            const float4* kr = reinterpret_cast<const float4*>(t == pos ? knew : kst + (size_t)t * HDP);
#pragma unroll 8
            for (int i = 0; i < HD / 4; i++) {
              const float4 k4 = kr[i];
              s0 = __fadd_rn(s0, __fmul_rn(q_s[4 * i], k4.x));
              s1 = __fadd_rn(s1, __fmul_rn(q_s[4 * i + 1], k4.y));
              s2 = __fadd_rn(s2, __fmul_rn(q_s[4 * i + 2], k4.z));
              s3 = __fadd_rn(s3, __fmul_rn(q_s[4 * i + 3], k4.w));
            }
          } else {
            const float4* kg = reinterpret_cast<const float4*>(p.kc + cbase + (size_t)t * HD);
#pragma unroll 8
            for (int i = 0; i < HD / 4; i++) {
              const float4 k4 = __ldcg(kg + i);
              s0 = __fadd_rn(s0, __fmul_rn(q_s[4 * i], k4.x));
              s1 = __fadd_rn(s1, __fmul_rn(q_s[4 * i + 1], k4.y));
              s2 = __fadd_rn(s2, __fmul_rn(q_s[4 * i + 2], k4.z));
              s3 = __fadd_rn(s3, __fmul_rn(q_s[4 * i + 3], k4.w));
            }
          }
          const float v = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3), scale);
          sc[t] = v;
          mx = fmaxf(mx, v);
        }
        mx = warp_max(mx);
        if ((tid & 31) == 0) red[tid >> 5] = mx;
        compute_bar();
        mx = warp_max(red[tid & (MK_WARPS - 1)]);
        for (int t = tid; t < T; t += MK_NT) sc[t] = fast_exp_ref(__fsub_rn(sc[t], mx));
        compute_bar();
        MK_TRACE(trow, 5);
        if (tid == 0) red[16] = chain_sum(0.f, sc, 1, T);  // softmax sum in position order (kernels.c:368)
        compute_bar();
        const float sum = red[16];
        for (int t = tid; t < T; t += MK_NT) sc[t] = __fdiv_rn(sc[t], sum);
        compute_bar();
        MK_TRACE(trow, 6);
        if (tid < HD) {  // o = sum_t p_t v_t in position order (kernels.c:372-375)
          float o = 0.f;
          if (staged) {  // products issue 16 positions ahead of the dependent adds
            const float* vp = vst + tid;
            int t = 0;
            for (; t + 16 <= pos; t += 16) {
              float v[16];
#pragma unroll
              for (int u = 0; u < 16; u++) v[u] = __fmul_rn(sc[t + u], vp[(size_t)(t + u) * HD]);
#pragma unroll
              for (int u = 0; u < 16; u++) o = __fadd_rn(o, v[u]);
            }
            for (; t < pos; t++) o = __fadd_rn(o, __fmul_rn(sc[t], vp[(size_t)t * HD]));
          } else {
            const float* vp = p.vc + cbase + tid;
#pragma unroll 8
            for (int t = 0; t < pos; t++) o = __fadd_rn(o, __fmul_rn(sc[t], __ldcg(vp + (size_t)t * HD)));
          }
          o = __fadd_rn(o, __fmul_rn(sc[pos], vnew[tid]));
          st_relaxed64(p.attw + (size_t)cta * HD + tid, __float_as_uint(o), E);
        }
        MK_TRACE(trow, 7);
      } else {
        // ---- C: O rows with the residual (kernels.c:379-382)
        if (!read_vec(p.attw, E, 10 * l + 2)) goto out;
        MK_TRACE(trow, 8);
        mk_quant(xf, D, xq, xd, xs);
        const uint8_t* t = next_tile(3, o_hi - o_lo, nbd);
        if (!t) goto out;
        mk_tile_dot(t, o_hi - o_lo, nbd, map_d, xq, xd, xs, prod, outv);
        release_tile();
        for (int n = o_lo + tid; n < o_hi; n += MK_NT) {
          const float v = __fadd_rn(xown[n - o_lo], outv[n - o_lo]);
          xown[n - o_lo] = v;
          st_relaxed64(p.xw + n, __float_as_uint(v), 2 * E);
        }
        MK_TRACE(trow, 9);
      }

      // ---- D (all CTAs): norm + gate/up rows of whole act blocks, silu * up, quantize (kernels.c:385-397)
      if (!read_vec(p.xw, 2 * E, 10 * l + 3)) goto out;
      MK_TRACE(trow, 10);
      mk_norm_quant(xf, nw2, D, p.eps, xq, xd, xs, red, sqs);
      for (int ab = cta; ab < nbf; ab += ncta) {
        const uint8_t* t = next_tile(4, 64, nbd);
        if (!t) goto out;
        mk_tile_dot(t, 64, nbd, map_d, xq, xd, xs, prod, outv);
        release_tile();
        if (tid < 32) {
          const float gt = outv[tid], up = outv[32 + tid];
          const float v = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, fast_exp_ref(-gt))), up);
          quant_block_redux(v, tid, actq, actd, acts);
          __syncwarp();
          unsigned long long* dst = p.actw + (size_t)ab * MK_ACT_WORDS;
          if (tid < 8) st_relaxed64(dst + tid, reinterpret_cast<const uint32_t*>(actq)[tid], E);
          else if (tid == 8) st_relaxed64(dst + 8, __float_as_uint(*actd), E);
          else if (tid < 13) st_relaxed64(dst + tid, reinterpret_cast<const uint32_t*>(acts)[tid - 9], E);
          __syncwarp();
        }
      }
      MK_TRACE(trow, 11);

      // ---- E (other CTAs): down rows over the quantized act, residual (kernels.c:399-400)
      if (!head) {
        for (int i = tid; i < nbf * 13; i += MK_NT) {
          const int ab = i / 13, w = i - ab * 13;
          const uint32_t v = wait_word(p.actw + (size_t)ab * MK_ACT_WORDS + w, E, p, 10 * l + 4, &abort_s);
          if (w < 8) reinterpret_cast<uint32_t*>(xq)[ab * 8 + w] = v;
          else if (w == 8) xd[ab] = __uint_as_float(v);
          else reinterpret_cast<uint32_t*>(xs)[ab * 4 + (w - 9)] = v;
        }
        compute_bar();
        if (abort_s) goto out;
        MK_TRACE(trow, 12);
        const uint8_t* t = next_tile(5, o_hi - o_lo, nbf);
        if (!t) goto out;
        mk_tile_dot(t, o_hi - o_lo, nbf, map_f, xq, xd, xs, prod, outv);
        release_tile();
        for (int n = o_lo + tid; n < o_hi; n += MK_NT) {
          const float v = __fadd_rn(xown[n - o_lo], outv[n - o_lo]);
          xown[n - o_lo] = v;
          st_relaxed64(p.xw + n, __float_as_uint(v), 2 * E + 1);
        }
        MK_TRACE(trow, 13);
      }
    }

    // ---- output norm, lm_head rows, argmax (kernels.c:404-414, cpu-worker.js:154-158)
    const int lrow = step * (L + 1) + L;
    MK_TRACE(lrow, 0);
    if (!read_vec(p.xw, 2 * E + 1, 9999)) goto out;
    MK_TRACE(lrow, 1);
    mk_norm_quant(xf, onw, D, p.eps, xq, xd, xs, red, sqs);
    MK_TRACE(lrow, 2);
    {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int r0 = v_lo; r0 < v_hi; r0 += MK_TILE_ROWS) {
        const int R = v_hi - r0 < MK_TILE_ROWS ? v_hi - r0 : MK_TILE_ROWS;
        const uint8_t* t = next_tile(8, R, nbd);
        if (!t) goto out;
        mk_tile_dot(t, R, nbd, map_d, xq, xd, xs, prod, outv);
        release_tile();
        for (int r = tid; r < R; r += MK_NT) p.logits[r0 + r] = outv[r];
        if (tid < 32) {  // rows in increasing order, ties to the lowest index (cpu-worker.js:156-157)
          float v = -INFINITY;
          int idx = 0x7fffffff;
          for (int r = tid; r < R; r += 32) amax_merge(v, idx, outv[r], r0 + r);
#pragma unroll
          for (int o = 16; o; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
            amax_merge(v, idx, v2, i2);
          }
          amax_merge(bv, bi, v, idx);
        }
      }
      MK_TRACE(lrow, 3);
      if (tid == 0) {
        st_relaxed64(p.lmw + 2 * cta, __float_as_uint(bv), step + 1);
        st_relaxed64(p.lmw + 2 * cta + 1, (uint32_t)bi, step + 1);
      }
    }
    if (tid < 32) {
      float v = -INFINITY;
      int idx = 0x7fffffff;
      for (int i = tid; i < ncta; i += 32) {
        const float v2 = __uint_as_float(wait_word(p.lmw + 2 * i, step + 1, p, 9998, &abort_s));
        const int i2 = (int)wait_word(p.lmw + 2 * i + 1, step + 1, p, 9998, &abort_s);
        amax_merge(v, idx, v2, i2);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
        amax_merge(v, idx, v2, i2);
      }
      if (tid == 0) tok_s = idx == 0x7fffffff ? 0 : idx;
    }
    compute_bar();
    if (abort_s) goto out;
    MK_TRACE(lrow, 4);
    tok = tok_s;
    if (cta == 0 && tid == 0) {  // like k_argmax2: log the token and advance the pass parameters
      *p.next = tok;
      if (pos + 1 <= p.ctx) p.toklog[(size_t)seq * (p.ctx + 1) + pos + 1] = tok;
      p.prm[P_POS0] = pos + 1;
      p.prm[P_M] = 1;
      p.prm[P_IDS] = tok;
    }
  }
out:
  cp_async_wait_all();  // no shared-memory copy may still be in flight when the CTA exits
  return;
#undef MK_TRACE
}

}  // namespace h2
