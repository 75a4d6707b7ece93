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
constexpr int MK_NSLOT = 4;                      // ring depth (two tiles in use, two in flight)
constexpr int MK_MAX_TILES = 256;                // per-CTA tile table kept in shared memory
constexpr int MK_WARPS = 16;                     // compute warps
constexpr int MK_NT = MK_WARPS * 32;             // compute threads
constexpr int MK_THREADS = MK_NT;                // 16 warps: the 128-register limit of a 512-thread block
constexpr int MK_TILE_ROWS = 64;                 // rows per tile (lm_head, q/k/v)
constexpr int MK_TRACE_PTS = 16;
constexpr int MK_ACT_WORDS = 8;                  // words per act block: its 32 int8 values and scale (36 bytes) as six
                                                 // 48-bit payloads under a 16-bit epoch tag (words 6, 7 unused)
#ifndef MK_SQ_SINK
#define MK_SQ_SINK true                          // the x reads also store x^2 for the RMSNorm
#endif
#ifndef MK_PACE
#define MK_PACE true                             // defer ring refills inside the layers to the next RMSNorm
#endif

#ifndef MK_POLL_NS
#define MK_POLL_NS 0                             // back-off between polls of a tagged word
#endif
#ifndef MK_SETTLE_O
#define MK_SETTLE_O 1000                         // cycles the O owners pause after publishing x before polling it
#endif
#ifndef MK_SETTLE_LM
#define MK_SETTLE_LM 1000                        // cycles every CTA pauses after the lm_head partial publish
#endif
#ifndef MK_SETTLE_QKV
#define MK_SETTLE_QKV 0                          // cycles the head CTAs pause after the QKV publish
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
  unsigned long long* actw;       // [F/32][MK_ACT_WORDS] act blocks, 48-bit payload | 16-bit epoch
  unsigned long long* lmw;        // [ncta][2] tagged lm_head partials (value, index)
  unsigned long long* kvdone;     // [ncta] epoch of the last layer whose KV-cache rows this CTA has released
  unsigned long long* rawact;     // [nsplit][32] tagged act values of the split blocks
  unsigned long long* lcmax;      // [H][ncta rounded up to 4] long-context attention: members' partial score maxes
  unsigned long long* lce;        // [H][ctx rounded up to 4] long-context attention: exp(s_t - max) per position
  unsigned long long* lcsum;      // [H] long-context attention: the softmax sum
  int stall_cta;                  // test aid: this CTA never publishes its QKV rows (-1: none), so waits expire
  int nsplit;                     // act blocks beyond one per CTA, computed in 4 pieces of 16 gate/up rows by the
                                  // last 4 nsplit CTAs and quantized by the consumers (0: whole blocks only)
  int* err;                       // [4]: code, cta, stage, abort flag
  int32_t* prm;                   // pass parameters (P_POS0, P_M, P_SEQ, P_IDS)
  int arg_seq, arg_pos, arg_tok;  // the first step's sequence, position and token when args_given (else from prm)
  int args_given;
  int32_t* toklog;                // [seqs][ctx + 1]
  int32_t* next;
  int32_t* done;                  // optional record in mapped host memory, written by CTA 0 when it finishes:
                                  // {launch_seq, next token, error code, error CTA, error stage}
  int32_t launch_seq;
  int steps;
  uint32_t epoch0;                // layer epoch before this launch: tags keep growing across launches, so words of
                                  // earlier launches never read as fresh and need no clearing
  uint32_t lm0;                   // decode steps before this launch (tags of the lm_head partials)
  unsigned long long timeout_ns;
  unsigned long long* trace;      // optional: [ncta][steps * (L + 1)][MK_TRACE_PTS] %globaltimer stamps
                                  // (profiling)
};

// dynamic shared memory of k_decode_persistent without the K/V staging area (must match the carve-up below)
__host__ __device__ inline size_t mk_smem_base(int D, int F, int HD, int ctx, int prod_items) {
  const int nbf = F / 32;
  const int outn = 3 * HD > 128 ? 3 * HD : 128;
  const int nbp = ((D / 32) + 3) & ~3;
  return (size_t)MK_NSLOT * MK_SLOT + (size_t)prod_items * 16 + (size_t)((F + 127) & ~127) +
         (size_t)((nbf + 3) & ~3) * 4 + (size_t)nbf * 16 + (size_t)D * 4 + 64 * 4 + (size_t)outn * 4 + 32 * 4 + 128 +
         (size_t)MK_MAX_TILES * 16 + (size_t)D * 4 * 3 + (size_t)64 * 4 + (size_t)HD * 4 + (size_t)nbp * 13 * 4 +
         (size_t)((ctx + 3) & ~3) * 4;
}

// ---------------------------------------------------------------- chain tiles
// QKV, O, gate/up and lm_head tiles use the "chain" layout: for R rows of nb blocks (nbp = nb rounded up to 4),
// values [R][4 lanes][nbp] as 32-bit words (word (r, l, b) = the 4 bytes wasm lane l of block b consumes), then fp16
// scales [R][nbp]; padding blocks are zero. Thread (r, l) reads its lane's words of 4 blocks with one 16-byte load
// and keeps the lane's running sum in a register. The int8 input is in the matching per-lane layout (MkX).
__host__ __device__ constexpr int mk_nbp(int nb) { return (nb + 3) & ~3; }

struct MkX {       // int8 input of a chain tile, per lane: x0[l][b] = word l of block b's low half, x1 = high half,
  int* x0;         // xs[l][b] = MK_MAGIC - 8 x (sum of lane l's values), dx[b] = scale; [4][nbp] ints, dx [nbp];
  int* x1;         // padding blocks hold zeros, which make every padding product -0 (exact no-op in the sums)
  int* xs;
  float* dx;
};

// thread (r, l) of a chain tile: acc_l = (((0 + f32(p_0) * (dw_0 * dx_0)) + ...) over the blocks in order
// (dot_q4_q8, kernels.c:121-139)
__device__ __forceinline__ float mk_lane_chain(const uint8_t* tile, int R, int nbp, int r, int l, const MkX& x) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(tile) + (size_t)(r * 4 + l) * nbp;
  const __half* d = reinterpret_cast<const __half*>(tile + (size_t)R * nbp * 16) + (size_t)r * nbp;
  const int *x0 = x.x0 + l * nbp, *x1 = x.x1 + l * nbp, *xs = x.xs + l * nbp;
  float acc = 0.f;
  for (int b = 0; b < nbp; b += 4) {
    const uint4 ww = *reinterpret_cast<const uint4*>(w + b);
    const uint2 dd = *reinterpret_cast<const uint2*>(d + b);
    const int4 a0 = *reinterpret_cast<const int4*>(x0 + b), a1 = *reinterpret_cast<const int4*>(x1 + b);
    const int4 as = *reinterpret_cast<const int4*>(xs + b);
    const float4 dx = *reinterpret_cast<const float4*>(x.dx + b);
    const __half2 d01 = *reinterpret_cast<const __half2*>(&dd.x), d23 = *reinterpret_cast<const __half2*>(&dd.y);
    const float p0 = q4_lane(ww.x, a0.x, a1.x, as.x), p1 = q4_lane(ww.y, a0.y, a1.y, as.y);
    const float p2 = q4_lane(ww.z, a0.z, a1.z, as.z), p3 = q4_lane(ww.w, a0.w, a1.w, as.w);
    acc = __fadd_rn(acc, __fmul_rn(p0, __fmul_rn(__low2float(d01), dx.x)));
    acc = __fadd_rn(acc, __fmul_rn(p1, __fmul_rn(__high2float(d01), dx.y)));
    acc = __fadd_rn(acc, __fmul_rn(p2, __fmul_rn(__low2float(d23), dx.z)));
    acc = __fadd_rn(acc, __fmul_rn(p3, __fmul_rn(__high2float(d23), dx.w)));
  }
  return acc;
}

// ---------------------------------------------------------------- PTX helpers
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
// four consecutive tagged words (32-byte aligned) in one request; each 64-bit element is read atomically
__device__ __forceinline__ void ld_relaxed64x4(const unsigned long long* p, unsigned long long* v) {
  asm volatile("ld.relaxed.gpu.global.v4.u64 {%0, %1, %2, %3}, [%4];"
               : "=l"(v[0]), "=l"(v[1]), "=l"(v[2]), "=l"(v[3])
               : "l"(p)
               : "memory");
}
__device__ __forceinline__ void st_relaxed64(unsigned long long* p, uint32_t payload, uint32_t tag) {
  const unsigned long long v = ((unsigned long long)tag << 32) | payload;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_release64(unsigned long long* p, uint32_t payload, uint32_t tag) {
  const unsigned long long v = ((unsigned long long)tag << 32) | payload;
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// A local pause (no memory traffic) of the given number of SM cycles.
__device__ __forceinline__ void mk_settle(long long cycles) {
  const long long c0 = clock64();
  while (clock64() - c0 < cycles) {
  }
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

// Out of line: a failure path that is taken at most once, called from many sites, and kept out of the
// instruction stream of the per-layer code (the kernel's code exceeds the instruction cache; inlined cold paths
// measured 5% slower per decode step).
__device__ __noinline__ void mk_fail(const MkParams& p, int code, int stage) {
  if (atomicCAS(p.err, 0, code) == 0) {
    p.err[1] = blockIdx.x;
    p.err[2] = stage;
  }
  __threadfence();  // the code, CTA and stage words before the abort flag
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

// Read `count` tagged words (word k at src(k)) that must carry epoch >= tag. Words are read in aligned quads
// (src(4m) .. src(4m) + 3 contiguous and 32-byte aligned; words of the last quad beyond count are read but
// ignored, so the allocation must extend to the quad's end): thread t takes quads t, t + MK_NT. A quad is one
// 32-byte request, and strong loads are not merged across threads, so the request count per poll round, which
// sets its latency, is a quarter of the word count. Stale quads are re-read together until every word carries
// the tag (bounded like wait_word). sink(k, payload) stores each payload. On timeout or abort sets *abort_s and
// returns early.
template <typename Src, typename Sink>
__device__ __forceinline__ void read_words(int count, Src src, uint32_t tag, Sink sink, const MkParams& p, int stage,
                                           int* abort_s) {
  const int nquad = (count + 3) >> 2;
  for (int m0 = threadIdx.x; m0 < nquad; m0 += 2 * MK_NT) {
    unsigned long long v[8];
    unsigned pending = 0;  // bit 4 j + e: word e of quad j still to deliver
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int m = m0 + j * MK_NT;
      v[4 * j] = v[4 * j + 1] = v[4 * j + 2] = v[4 * j + 3] = 0;
      if (m < nquad) {
        ld_relaxed64x4(src(4 * m), v + 4 * j);
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (4 * m + e < count) pending |= 1u << (4 * j + e);
      }
    }
    unsigned long long t0 = 0;
    for (unsigned it = 0;; it++) {
#pragma unroll
      for (int j = 0; j < 2; j++)
#pragma unroll
        for (int e = 0; e < 4; e++)
          if (((pending >> (4 * j + e)) & 1u) && (uint32_t)(v[4 * j + e] >> 32) >= tag) {
            sink(4 * (m0 + j * MK_NT) + e, (uint32_t)v[4 * j + e]);
            pending &= ~(1u << (4 * j + e));
          }
      if (!pending) break;
      if (it == 0) {
        t0 = gtimer();
      } else if ((it & 31) == 31) {
        if (*(volatile int*)abort_s || ld_volatile_i(p.err + 3)) {
          *(volatile int*)abort_s = 1;
          return;
        }
        if (gtimer() - t0 > p.timeout_ns) {
          mk_fail(p, MK_TIMEOUT_WAIT, stage);
          *(volatile int*)abort_s = 1;
          return;
        }
      }
#pragma unroll
      for (int j = 0; j < 2; j++)
        if ((pending >> (4 * j)) & 15u) ld_relaxed64x4(src(4 * (m0 + j * MK_NT)), v + 4 * j);
    }
  }
}

// ---------------------------------------------------------------- shared building blocks

// s = ((s + p[0]) + p[stride]) + ... over n terms in order. Two 16-register buffers alternate: the shared-memory
// loads of the next 16 terms issue before the adds of the current 16, so a step costs one add latency, not a load
// latency (and no register moves between the buffers).
__device__ __forceinline__ float chain_sum(float s, const float* p, int stride, int n) {
  float a[16], b[16];
  const int n32 = n & ~31;
  if (n32) {
#pragma unroll
    for (int u = 0; u < 16; u++) a[u] = p[u * stride];
    for (int k = 0; k < n32; k += 32) {
#pragma unroll
      for (int u = 0; u < 16; u++) b[u] = p[(k + 16 + u) * stride];
#pragma unroll
      for (int u = 0; u < 16; u++) s = __fadd_rn(s, a[u]);
      if (k + 32 < n32) {
#pragma unroll
        for (int u = 0; u < 16; u++) a[u] = p[(k + 32 + u) * stride];
      }
#pragma unroll
      for (int u = 0; u < 16; u++) s = __fadd_rn(s, b[u]);
    }
  }
  const int rem = n - n32;  // 0..31 trailing terms
#pragma unroll
  for (int u = 0; u < 16; u++) a[u] = u < rem ? p[(n32 + u) * stride] : 0.f;
#pragma unroll
  for (int u = 0; u < 16; u++) b[u] = u + 16 < rem ? p[(n32 + 16 + u) * stride] : 0.f;
#pragma unroll
  for (int u = 0; u < 16; u++)
    if (u < rem) s = __fadd_rn(s, a[u]);
#pragma unroll
  for (int u = 0; u < 16; u++)
    if (u + 16 < rem) s = __fadd_rn(s, b[u]);
  return s;
}

// Quantize two 32-value blocks b0 and b1 (one value of each per lane) into a chain input, the arithmetic of
// quant_block_redux (kernels.c:90-114) for each, written interleaved so that the reductions and divisions of the
// two blocks overlap; the int8 values are stored per lane, then lanes 0-3 (b0) and 4-7 (b1) form their lane sums
// and lane 0 stores the scales.
__device__ __forceinline__ void mk_quant_chain2(float v0, float v1, int lane, int b0, int b1, int nbp, const MkX& x) {
  const unsigned m0 = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v0)));
  const unsigned m1 = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v1)));
  float d0, d1, i0, i1;
  block_scales2(__uint_as_float(m0), __uint_as_float(m1), d0, d1, i0, i1);
  const int q0 = max(-128, min(127, __float2int_rn(__fmul_rn(v0, i0))));
  const int q1 = max(-128, min(127, __float2int_rn(__fmul_rn(v1, i1))));
  const int pos = (lane & 16) | invperm16(lane & 15);
  int8_t* dst = reinterpret_cast<int8_t*>(pos < 16 ? x.x0 : x.x1) + ((((pos & 15) >> 2) * nbp) * 4 + (pos & 3));
  dst[b0 * 4] = (int8_t)q0;
  dst[b1 * 4] = (int8_t)q1;
  __syncwarp();
  if (lane < 8) {  // lane l of block b0 (lanes 0-3) / b1 (lanes 4-7): its words of the two halves, dp4a against ones
    const int i = (lane & 3) * nbp + (lane < 4 ? b0 : b1);
    x.xs[i] = MK_MAGIC - 8 * __dp4a(x.x0[i], 0x01010101, __dp4a(x.x1[i], 0x01010101, 0));
  }
  if (lane == 0) {
    x.dx[b0] = d0;
    x.dx[b1] = d1;
  }
}

// quantization of nblk 32-value blocks: value i of block b is f(b * 32 + lane); two blocks per warp at a time
template <typename Fn>
__device__ __forceinline__ void mk_quant_blocks(int nblk, Fn f, const MkX& x) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nbp = mk_nbp(nblk);
  for (int b = warp; b < nblk; b += 2 * MK_WARPS) {
    // a warp without a second block quantizes its block twice into the same place (the same values and stores):
    // one code path instead of a one-block variant beside the two-block one
    const int b2 = b + MK_WARPS < nblk ? b + MK_WARPS : b;
    mk_quant_chain2(f(b * 32 + lane), f(b2 * 32 + lane), lane, b, b2, nbp, x);
  }
  compute_bar();
}

// The squares of the RMSNorm are kept lane-major: the square of element k is at sq[(k % 4) * mk_sq_stride(D) + k / 4],
// so lane chain l's terms are contiguous (16-byte loads) and the four lane rows start in different banks.
__host__ __device__ constexpr int mk_sq_stride(int D) { return D / 4 + 4; }
__device__ __forceinline__ int mk_sq_index(int k, int D) { return (k & 3) * mk_sq_stride(D) + (k >> 2); }

// s = ((s + p[0]) + p[1]) + ... over n terms in order, p 16-byte aligned and n a multiple of 4: four float4 loads
// of the next 16 terms issue before the adds of the current 16 (alternating buffers).
__device__ __forceinline__ float chain_sum4(float s, const float* p, int n) {
  const float4* q = reinterpret_cast<const float4*>(p);
  const int n4 = n >> 2;
  float4 a[4], b[4];
#pragma unroll
  for (int u = 0; u < 4; u++) a[u] = u < n4 ? q[u] : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < n4; k += 8) {
#pragma unroll
    for (int u = 0; u < 4; u++)
      if (k + 4 + u < n4) b[u] = q[k + 4 + u];
#pragma unroll
    for (int u = 0; u < 4; u++)
      if (k + u < n4) {
        s = __fadd_rn(s, a[u].x);
        s = __fadd_rn(s, a[u].y);
        s = __fadd_rn(s, a[u].z);
        s = __fadd_rn(s, a[u].w);
      }
#pragma unroll
    for (int u = 0; u < 4; u++)
      if (k + 8 + u < n4) a[u] = q[k + 8 + u];
#pragma unroll
    for (int u = 0; u < 4; u++)
      if (k + 4 + u < n4) {
        s = __fadd_rn(s, b[u].x);
        s = __fadd_rn(s, b[u].y);
        s = __fadd_rn(s, b[u].z);
        s = __fadd_rn(s, b[u].w);
      }
  }
  return s;
}

// RMSNorm of xf[0..D) (shared) into int8 blocks xq/xd/xs (shared), the reference's lane order (kernels.c:80-114):
// the squares are formed by all threads into sq (shared, lane-major as above), then thread 32 + l (warp 1, so that
// thread 0 can issue weight copies meanwhile) adds the squares of elements 4k + l over k in order and
// ((l0 + l1) + l2) + l3 combines the four chains.
__device__ __forceinline__ void mk_norm_quant(const float* xf, const float* w, int D, float eps, const MkX& x, float* red,
                                              float* sq, bool have_sq = false) {
  const int tid = threadIdx.x;
  if (!have_sq) {  // (the x reads can deliver the squares with x)
    for (int i = tid; i < D; i += MK_NT) sq[mk_sq_index(i, D)] = __fmul_rn(xf[i], xf[i]);
    compute_bar();
  }
  if (tid >= 32 && tid < 36) red[tid - 32] = chain_sum4(0.f, sq + (tid - 32) * mk_sq_stride(D), D / 4);
  compute_bar();
  const float ss = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[1]), red[2]), red[3]);
  const float r = norm_scale(ss, D, eps);
  mk_quant_blocks(D / 32, [&](int i) { return __fmul_rn(__fmul_rn(xf[i], r), w[i]); }, x);
}

// plain quantization of xf[0..K) (shared) into shared int8 blocks
__device__ __forceinline__ void mk_quant(const float* xf, int K, const MkX& x) {
  mk_quant_blocks(K / 32, [&](int i) { return xf[i]; }, x);
}

// Down tiles are row-major (values [R][nb][16 B], then fp16 scales [R][nb]); their products go to a shared buffer,
// lane-major: row r's lane-l products of blocks 0 .. nb-1 are contiguous at (4 r + l) * mk_prod_lane_stride(nb)
// (16-byte aligned; the padding spreads the 4 R chain threads' 16-byte reads over the banks).
__host__ __device__ constexpr int mk_prod_lane_stride(int nb) { return ((nb + 3) & ~3) + 4; }
// row stride (floats) of the products of a few-row chain tile: at least nbp, 16-byte aligned, 4 banks apart
__host__ __device__ constexpr int mk_small_stride(int nbp) { return (nbp + 27) / 32 * 32 + 4; }
// act blocks beyond one per CTA (nbf blocks over ncta CTAs, nh of which own O / down rows): up to 8 are split into
// 16-row gate/up pieces on the last 4 nsplit CTAs (returns nsplit), else (0) every CTA takes whole blocks
__host__ __device__ constexpr int mk_nsplit(int nbf, int ncta, int nh) {
  return (nbf > ncta && nbf - ncta <= 8 && 4 * (nbf - ncta) <= nh) ? nbf - ncta : 0;
}
// a few-row chain tile of R rows and nb blocks fits the two-phase form: 4 R chain threads, products in prod
__host__ __device__ constexpr bool mk_small_tile_fits(int R, int nb, int prod_items) {
  return 4 * R <= MK_NT && 4 * R * mk_small_stride(mk_nbp(nb)) <= 4 * prod_items;
}

// ---------------------------------------------------------------- the kernel
// Shape parameters TD (hidden), TF (ffn), TH (q heads), TKVH (kv heads), THD (head dim) fix the model shape at
// compile time when non-zero, so buffer offsets and loop bounds are constants (fewer live registers in this
// single large kernel); 0 takes the shape from MkParams. TNCTA likewise fixes the grid size (and with it the
// split of the act blocks) when non-zero. TR compiles in the optional timestamp trace (p.trace), TLC the
// long-context attention (positions beyond kv_stage; a TLC = false instance serves launches whose positions all stay
// within kv_stage): the instances without them carry none of their code (the kernel's code exceeds the instruction
// cache).
template <int TD, int TF, int TH, int TKVH, int THD, int TNCTA, bool TR, bool TLC>
__global__ void __launch_bounds__(MK_THREADS, 1) k_decode_persistent(const MkParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int D = TD ? TD : p.D, F = TF ? TF : p.F, H = TH ? TH : p.H, KVH = TKVH ? TKVH : p.KVH,
            HD = THD ? THD : p.HD, L = p.L;
  const int nbd = D / 32, nbf = F / 32;
  const int QKV = D + 2 * KVH * HD;
  // fixed-size regions first (constant offsets for a fixed shape), then the context-dependent ones
  uint8_t* ring = smem;                                                     // MK_NSLOT * MK_SLOT
  int8_t* xq = reinterpret_cast<int8_t*>(ring + MK_NSLOT * MK_SLOT);       // F int8
  float* xd = reinterpret_cast<float*>(xq + ((F + 127) & ~127));          // F/32
  int4* xs = reinterpret_cast<int4*>(xd + ((nbf + 3) & ~3));              // F/32
  float* xf = reinterpret_cast<float*>(xs + nbf);                          // D
  float* xown = xf + D;                                                    // 64 (this CTA's x rows)
  float* outv = xown + 64;                                                 // max(3 HD, 128) (tile results)
  float* red = outv + (3 * HD > 128 ? 3 * HD : 128);                       // 32
  uint8_t* actb = reinterpret_cast<uint8_t*>(red + 32);                   // 2 x (32 B int8, 4 B d, 16 B sums, pad)
  MkTile* tsm = reinterpret_cast<MkTile*>(actb + 128);                    // MK_MAX_TILES (this CTA's table)
  float* nw1 = reinterpret_cast<float*>(tsm + MK_MAX_TILES);              // D: attn_norm of the layer
  float* nw2 = nw1 + D;                                                    // D: ffn_norm of the layer
  float* onw = nw2 + D;                                                    // D: output norm
  float* bsm = onw + D;                                                    // 64: bias of this CTA's QKV rows
  float* rsm = bsm + 64;                                                   // HD: RoPE row of the position
  const int nbpd = mk_nbp(nbd);
  int* xcw = reinterpret_cast<int*>(rsm + HD);                             // chain input: 13 nbpd words
  const MkX xc{xcw, xcw + 4 * nbpd, xcw + 8 * nbpd, reinterpret_cast<float*>(xcw + 12 * nbpd)};
  float4* prod = reinterpret_cast<float4*>(xcw + 13 * nbpd);              // p.prod_items
  float* sc = reinterpret_cast<float*>(prod + p.prod_items);              // ctx (scores)
  const int HDP = HD + 4;                                                  // padded K rows: conflict-free dots
  float* kst = sc + ((p.ctx + 3) & ~3);                                    // kv_stage * HDP
  float* vst = kst + (size_t)p.kv_stage * HDP;                             // kv_stage * HD
  __shared__ __align__(8) uint64_t full[MK_NSLOT];
  __shared__ int abort_s;
  __shared__ int tok_s;
  __shared__ int ndone_s;       // act blocks whose down products are in prod
  __shared__ __align__(16) uint8_t splitq_s[8][64];  // quantized split act blocks: 32 B int8, d, lane sums

  const int tid = threadIdx.x, cta = blockIdx.x, ncta = TNCTA ? TNCTA : p.ncta;
  const int nsplit = TNCTA ? mk_nsplit(nbf, TNCTA, TNCTA - H) : p.nsplit;
  const MkTile* my_tiles = p.tiles + (size_t)cta * p.tile_stride;

  if (tid == 0) {
    for (int s = 0; s < MK_NSLOT; s++) mbar_init(&full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_s = 0;
  }
  __syncthreads();

  const int my_count = p.tile_count[cta];
  const int total_tiles = my_count * p.steps;
  // this CTA's tile table and the output norm go to shared memory once (no global load per tile)
  for (int i = tid; i < my_count; i += MK_THREADS) tsm[i] = my_tiles[i];
  for (int i = tid; i < D; i += MK_THREADS) onw[i] = p.out_norm[i];
  for (int i = tid; i < 13 * nbpd; i += MK_THREADS) xcw[i] = 0;
  __syncthreads();

  // ------------------------------------------------------------ the weight ring
  // Thread 0 streams the CTA's tiles into the ring with bulk copies: tile k goes to slot k % MK_NSLOT once tile
  // k - MK_NSLOT has been released (after a CTA barrier, so no thread still reads the slot). Weight streaming
  // competes with the cross-CTA exchanges for L2 and memory bandwidth, and slots free up at stage ends, right when
  // results are exchanged; so inside the layers the refills wait for the start of the next RMSNorm, which reads no
  // global memory, or for a stage that finds its tile not yet issued. The lm_head refills as soon as a slot frees.
  int tile_i = 0;    // tiles consumed (every thread)
  int tpos = 0;      // tile_i % my_count: table entry of the next tile to consume
  int issued = 0;    // tiles issued (thread 0)
  int ipos = 0;      // issued % my_count (thread 0)
  bool pace = false; // thread 0: defer refills to the next RMSNorm
  auto refill = [&]() {  // thread 0: issue every tile whose slot is free
    const int lim = min(total_tiles, tile_i + MK_NSLOT);
    if (issued < lim) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    while (issued < lim) {
      const int s = issued % MK_NSLOT;
      const MkTile t = tsm[ipos];
      if (t.bytes == 0 || t.bytes > MK_SLOT || (t.bytes & 15) || (t.off & 15)) {
        mk_fail(p, MK_ABORTED, -2);
        abort_s = 1;
        return;
      }
      mbar_expect_tx(&full[s], t.bytes);
      bulk_g2s(ring + (size_t)s * MK_SLOT, p.stream + t.off, t.bytes, &full[s]);
      issued++;
      if (++ipos == my_count) ipos = 0;
    }
  };
  if (tid == 0) refill();

  unsigned long long* trace = nullptr;
  if (TR && p.trace) trace = p.trace + (size_t)cta * p.steps * (L + 1) * MK_TRACE_PTS;
  // thread 0: the next n (1 or 2) tiles have landed and their table entries describe the rows and blocks the stage
  // expects. A stage's thread 0 may do this ahead (during the RMSNorm before it, whose chains run on warp 1), so
  // that the stage itself only passes the barrier.
  int verified = 0;  // thread 0: tiles [0, verified) have landed and were checked (in consumption order)
  auto wait_tiles = [&](int stage, int ahead, int n, int rows0, int rows1, int nb) {  // tiles tile_i + ahead + h
    for (int h = 0; h < n && !abort_s; h++) {
      const int ti = tile_i + ahead + h;
      if (ti < verified) continue;
      int tp = tpos + ahead + h;
      while (tp >= my_count) tp -= my_count;
      const MkTile t = tsm[tp];
      if (ti >= issued) refill();  // not issued yet: refill now
      if (t.rows != (h ? rows1 : rows0) || t.nb != nb) {
        mk_fail(p, MK_ABORTED, stage);
        abort_s = 1;
      } else if (!mbar_wait(&full[ti % MK_NSLOT], (ti / MK_NSLOT) & 1, p)) {
        if (!ld_volatile_i(p.err + 3)) mk_fail(p, MK_TIMEOUT_SLOT, stage);
        abort_s = 1;
      }
      if (!abort_s) verified = ti + 1;
    }
  };
  // wait for the next n (1 or 2) tiles; each table entry must describe the rows and blocks this stage expects
  auto next_tiles = [&](int stage, int n, int rows0, int rows1, int nb) -> bool {
    if (tid == 0) wait_tiles(stage, 0, n, rows0, rows1, nb);
    compute_bar();
    return !abort_s;
  };
  auto release_tiles = [&](int n) {
    compute_bar();
    tile_i += n;
    tpos += n;
    while (tpos >= my_count) tpos -= my_count;
    if (tid == 0 && !pace) refill();
  };
  // n chain tiles at once (tile h on warps 8h .. 8h + 7, thread (r, l) = (t / 4, t % 4)); row r of tile h lands in
  // outv[64 h + r]
  auto chain_tiles = [&](int stage, int n, int rows0, int rows1, int nb) -> bool {
    if (!next_tiles(stage, n, rows0, rows1, nb)) return false;
    const int h = tid >> 8, t = tid & 255, R = h ? rows1 : rows0;
    if (h < n && (t & ~31) < 4 * R) {  // whole warps: hsum4_quad shuffles over all 32 lanes
      const uint8_t* tl = ring + (size_t)((tile_i + h) % MK_NSLOT) * MK_SLOT;
      const int r = t >> 2;
      const float a = r < R ? mk_lane_chain(tl, R, mk_nbp(nb), r, t & 3, xc) : 0.f;
      const float v = hsum4_quad(a);
      if (r < R && (t & 3) == 0) outv[64 * h + r] = v;
    }
    release_tiles(n);
    return true;
  };
  // One chain tile of few rows (QKV, O: 4 R lane chains would leave 15 of 16 warps idle): all warps form the
  // R x 4 x nb lane products into shared memory (prod, one padded row per (r, l)), then thread (r, l) adds its
  // lane's products in block order; the same arithmetic and order as mk_lane_chain. Row r lands in outv[r].
  auto small_tile = [&](int stage, int R, int nb) -> bool {
    const int nbp = mk_nbp(nb), PSS = mk_small_stride(nbp);
    // (the fixed-shape instance has no fallback: the host checks mk_small_tile_fits for its shape)
    if (TD == 0 && !mk_small_tile_fits(R, nb, p.prod_items)) return chain_tiles(stage, 1, R, 0, nb);
    if (!next_tiles(stage, 1, R, 0, nb)) return false;
    const uint8_t* tl = ring + (size_t)(tile_i % MK_NSLOT) * MK_SLOT;
    const uint32_t* w = reinterpret_cast<const uint32_t*>(tl);
    const __half* dws = reinterpret_cast<const __half*>(tl + (size_t)R * nbp * 16);
    float* pp = reinterpret_cast<float*>(prod);
    for (int i = tid; i < 4 * R * nb; i += MK_NT) {
      const int rl = i / nb, b = i - rl * nb, l = rl & 3;
      const float q = q4_lane(w[(size_t)rl * nbp + b], xc.x0[l * nbp + b], xc.x1[l * nbp + b], xc.xs[l * nbp + b]);
      pp[rl * PSS + b] = __fmul_rn(q, __fmul_rn(__half2float(dws[(rl >> 2) * nbp + b]), xc.dx[b]));
    }
    compute_bar();
    if ((tid & ~31) < 4 * R) {  // whole warps: hsum4_quad shuffles over all 32 lanes
      const int r = tid >> 2;
      float a = 0.f;
      if (r < R) a = (nb & 3) == 0 ? chain_sum4(0.f, pp + tid * PSS, nb) : chain_sum(0.f, pp + tid * PSS, 1, nb);
      const float v = hsum4_quad(a);
      if (r < R && (tid & 3) == 0) outv[r] = v;
    }
    release_tiles(1);
    return true;
  };
  // read D tagged floats (x or att) into xf
  float* sqs = reinterpret_cast<float*>(prod);  // norm squares (prod is free between tiles)
  // read D tagged floats into xf; with_sq also stores their squares into sqs for the RMSNorm that follows
  auto read_vec = [&](const unsigned long long* src, uint32_t tag, int stage, bool with_sq = false) -> bool {
    if (with_sq)
      read_words(
          D, [&](int k) { return src + k; }, tag,
          [&](int k, uint32_t v) {
            const float f = __uint_as_float(v);
            xf[k] = f;
            sqs[mk_sq_index(k, D)] = __fmul_rn(f, f);
          },
          p, stage, &abort_s);
    else
      read_words(D, [&](int k) { return src + k; }, tag, [&](int k, uint32_t v) { xf[k] = __uint_as_float(v); }, p,
                 stage, &abort_s);
    compute_bar();
    return !abort_s;
  };

  const bool head = cta < H;
  const int nh = ncta - H;                  // CTAs that own O / down rows
  const int j = cta - H;
  const int o_lo = head ? 0 : (int)((long long)j * D / nh), o_hi = head ? 0 : (int)((long long)(j + 1) * D / nh);
  const int v_lo = (int)((long long)cta * p.V / ncta), v_hi = (int)((long long)(cta + 1) * p.V / ncta);
  const int npair = QKV / 2, half = HD / 2;
  const int pr_lo = (int)((long long)cta * npair / ncta), pr_hi = (int)((long long)(cta + 1) * npair / ncta);
  const int G = H / KVH, kh = head ? cta / G : 0;
  const int kv_pair_lo = H * half, kv_pair_hi = (H + 2 * KVH) * half;  // QKV row pairs of the k and v heads
  const bool my_kv = pr_lo < kv_pair_hi && pr_hi > kv_pair_lo;
  const int seq = p.args_given ? p.arg_seq : p.prm[P_SEQ];
  int pos = p.args_given ? p.arg_pos : p.prm[P_POS0];
  int tok = p.args_given ? p.arg_tok : p.prm[P_IDS];
  uint32_t E = p.epoch0;  // layer epoch (grows by one per layer, across launches)

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

      const size_t cbase = (((size_t)seq * L + l) * KVH + kh) * (size_t)p.ctx * HD;
      const bool staged = head && pos <= p.kv_stage;
      // long context: more positions than a head CTA stages; every CTA then works on attention (below)
      const bool lc = TLC && pos > p.kv_stage;
      {
        // this layer's norm weights and QKV bias arrive while the layer's inputs are in flight
        for (int i = tid; i < D / 4; i += MK_NT) {
          cp_async16(nw1 + 4 * i, p.attn_norm + (size_t)l * D + 4 * i);
          cp_async16(nw2 + 4 * i, p.ffn_norm + (size_t)l * D + 4 * i);
        }
        if (tid < 2 * (pr_hi - pr_lo)) {
          const int pidx = pr_lo + (tid >> 1), row = (pidx / half) * HD + pidx % half + (tid & 1) * half;
          cp_async4(bsm + tid, p.bqkv + (size_t)l * QKV + row);
        }
        if ((head || lc) && E > p.epoch0 + (uint32_t)L) {
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
      if (l > 0 && !read_vec(p.xw, 2 * (E - 1) + 1, 10 * l + 0, MK_SQ_SINK)) goto out;
      cp_async_wait_all();
      compute_bar();
      MK_TRACE(trow, 1);
      if (tid == 0) {
        pace = MK_PACE;
        refill();
        wait_tiles(1, 0, 1, 2 * (pr_hi - pr_lo), 0, nbd);  // the QKV tile, while warp 1 runs the norm's chains
      }
      mk_norm_quant(xf, nw1, D, p.eps, xc, red, sqs, MK_SQ_SINK && l > 0);
      MK_TRACE(trow, 2);
      {
        const int R = 2 * (pr_hi - pr_lo);
        if (!small_tile(1, R, nbd)) goto out;
        const int npub = cta == p.stall_cta ? 0 : pr_hi - pr_lo;
        for (int jp = tid; jp < npub; jp += MK_NT) {
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
      if (MK_SETTLE_QKV > 0 && head) mk_settle(MK_SETTLE_QKV);
      if (!head && !lc && tid == 0) wait_tiles(3, 0, 1, o_hi - o_lo, 0, nbd);  // the O tile, while attention runs

      if (lc) {
        // ---- B' (long context, all CTAs): the CTAs of head hg's group (the head CTA and every non-head CTA j with
        // (j - H) % H == hg) split the positions for the scores and the head dims for the ordered p.v sums; the
        // head CTA adds the softmax sum in position order (kernels.c:355-377, same arithmetic and order as B).
        const int T = pos + 1;
        const int hg = head ? cta : (cta - H) % H, khg = hg / G;
        const int gcount = hg < nh ? (nh - 1 - hg) / H + 1 : 0;  // non-head members
        const int GS = 1 + gcount, gi = head ? 0 : 1 + (cta - H) / H;
        const int t0 = (int)((long long)gi * T / GS), t1 = (int)((long long)(gi + 1) * T / GS);
        const int d0 = gi * HD / GS, d1 = (gi + 1) * HD / GS, nd = d1 - d0;
        const size_t gbase = (((size_t)seq * L + l) * KVH + khg) * (size_t)p.ctx * HD;
        // per-head rows of the exchange arrays start on 4-word boundaries (read_words reads aligned quads)
        unsigned long long* lcm = p.lcmax + (size_t)hg * ((ncta + 3) & ~3);
        unsigned long long* lce = p.lce + (size_t)hg * ((p.ctx + 3) & ~3);
        float* q_s = outv;
        float* knew = outv + HD;
        float* vnew = outv + 2 * HD;
        read_words(
            3 * HD,
            [&](int k) {
              return k < HD ? p.qw + hg * HD + k
                            : (k < 2 * HD ? p.kvw + khg * HD + (k - HD) : p.kvw + (KVH + khg) * HD + (k - 2 * HD));
            },
            E, [&](int k, uint32_t v) { outv[k] = __uint_as_float(v); }, p, 10 * l + 1, &abort_s);
        compute_bar();
        if (abort_s) goto out;
        if (head) MK_TRACE(trow, 4);
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
        float mx = -1e30f;
        for (int t = t0 + tid; t < t1; t += MK_NT) {  // this member's positions
          float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
          const float4* kr = reinterpret_cast<const float4*>(t == pos ? knew : p.kc + gbase + (size_t)t * HD);
#pragma unroll 16
          for (int i = 0; i < HD / 4; i++) {
            const float4 k4 = t == pos ? kr[i] : __ldcg(kr + i);
            s0 = __fadd_rn(s0, __fmul_rn(q_s[4 * i], k4.x));
            s1 = __fadd_rn(s1, __fmul_rn(q_s[4 * i + 1], k4.y));
            s2 = __fadd_rn(s2, __fmul_rn(q_s[4 * i + 2], k4.z));
            s3 = __fadd_rn(s3, __fmul_rn(q_s[4 * i + 3], k4.w));
          }
          const float v = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3), scale);
          sc[t] = v;
          mx = fmaxf(mx, v);
        }
        mx = warp_max(mx);
        if ((tid & 31) == 0) red[tid >> 5] = mx;
        compute_bar();
        mx = warp_max(red[tid & (MK_WARPS - 1)]);
        if (tid == 0) st_relaxed64(lcm + gi, __float_as_uint(mx), E);
        // the group's max (exact in any order), then exp of this member's positions, published
        read_words(GS, [&](int k) { return lcm + k; }, E,
                   [&](int k, uint32_t v) { xf[k] = __uint_as_float(v); }, p, 10 * l + 6, &abort_s);  // (xf is free)
        compute_bar();
        if (abort_s) goto out;
        mx = -1e30f;
        for (int k = 0; k < GS; k++) mx = fmaxf(mx, xf[k]);
        for (int t = t0 + tid; t < t1; t += MK_NT) {
          const float e = fast_exp_ref(__fsub_rn(sc[t], mx));
          st_relaxed64(lce + t, __float_as_uint(e), E);
        }
        // every member collects all T exponentials; the head CTA adds them in position order (kernels.c:368)
        read_words(T, [&](int k) { return lce + k; }, E,
                   [&](int k, uint32_t v) { sc[k] = __uint_as_float(v); }, p, 10 * l + 7, &abort_s);
        compute_bar();
        if (abort_s) goto out;
        if (head) {
          MK_TRACE(trow, 5);
          if (tid == 0) st_relaxed64(p.lcsum + hg, __float_as_uint(chain_sum(0.f, sc, 1, T)), E);
        }
        if (tid == 0) red[16] = __uint_as_float(wait_word(p.lcsum + hg, E, p, 10 * l + 8, &abort_s));
        compute_bar();
        if (abort_s) goto out;
        const float sum = red[16];
        for (int t = tid; t < T; t += MK_NT) sc[t] = __fdiv_rn(sc[t], sum);
        compute_bar();
        if (head) MK_TRACE(trow, 6);
        // o_d = sum_t p_t v_td in position order for this member's dims. Warps 1-15 form the products p_t v_td of the
        // next chunk of positions straight from the cache into the staging area (double-buffered) while warp 0's
        // threads d < nd add the current chunk's products in order: a step of the ordered sum is one add.
        if (nd > 0) {
          const int C = (int)((size_t)p.kv_stage * (2 * HD + 4) / (2 * nd));  // positions per chunk
          float* pb = kst;                                                     // [2][nd][C] products
          const float* vg = p.vc + gbase + d0;
          auto make_chunk = [&](int c, int buf) {  // threads 32 ..: eight loads in flight per thread
            const int ta = c * C, n = (min(pos, ta + C) - ta) * nd;
            constexpr int U = 8, NL = MK_NT - 32;
            for (int i0 = tid - 32; i0 < n; i0 += U * NL) {
              float v[U];
#pragma unroll
              for (int u = 0; u < U; u++) {
                const int i = i0 + u * NL, t = i / nd, dd = i - t * nd;
                v[u] = i < n ? __ldcg(vg + (size_t)(ta + t) * HD + dd) : 0.f;
              }
#pragma unroll
              for (int u = 0; u < U; u++) {
                const int i = i0 + u * NL, t = i / nd, dd = i - t * nd;
                if (i < n) pb[((size_t)buf * nd + dd) * C + t] = __fmul_rn(sc[ta + t], v[u]);
              }
            }
          };
          const int nch = (pos + C - 1) / C;  // chunks of cached positions 0 .. pos - 1
          float o = 0.f;
          if (tid >= 32 && nch > 0) make_chunk(0, 0);
          for (int c = 0; c < nch; c++) {
            compute_bar();  // chunk c's products are in place; the other buffer is free
            if (tid >= 32) {
              if (c + 1 < nch) make_chunk(c + 1, (c + 1) & 1);
            } else if (tid < nd) {
              o = chain_sum(o, pb + ((size_t)(c & 1) * nd + tid) * C, 1, min(pos, c * C + C) - c * C);
            }
          }
          compute_bar();  // the product buffers are free again
          if (tid < nd) {
            o = __fadd_rn(o, __fmul_rn(sc[pos], vnew[d0 + tid]));
            st_relaxed64(p.attw + (size_t)hg * HD + d0 + tid, __float_as_uint(o), E);
          }
        }
        if (head) MK_TRACE(trow, 7);
      } else if (head) {
        // ---- B: attention of head h over the cache (kernels.c:355-377)
        const int T = pos + 1;
        float* q_s = outv;
        float* knew = outv + HD;
        float* vnew = outv + 2 * HD;
        read_words(
            3 * HD,
            [&](int k) {
              return k < HD ? p.qw + cta * HD + k
                            : (k < 2 * HD ? p.kvw + kh * HD + (k - HD) : p.kvw + (KVH + kh) * HD + (k - 2 * HD));
            },
            E, [&](int k, uint32_t v) { outv[k] = __uint_as_float(v); }, p, 10 * l + 1, &abort_s);
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
        MK_TRACE(trow, 12);
        mx = warp_max(mx);
        if ((tid & 31) == 0) red[tid >> 5] = mx;
        compute_bar();
        mx = warp_max(red[tid & (MK_WARPS - 1)]);
        MK_TRACE(trow, 13);
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
      }
      if (!head) {
        // ---- C: O rows with the residual (kernels.c:379-382)
        if (!read_vec(p.attw, E, 10 * l + 2)) goto out;
        MK_TRACE(trow, 8);
        mk_quant(xf, D, xc);
        if (!small_tile(3, o_hi - o_lo, nbd)) goto out;
        for (int n = o_lo + tid; n < o_hi; n += MK_NT) {
          const float v = __fadd_rn(xown[n - o_lo], outv[n - o_lo]);
          xown[n - o_lo] = v;
          st_relaxed64(p.xw + n, __float_as_uint(v), 2 * E);
        }
        MK_TRACE(trow, 9);
        // The O owners pause before polling x (the next stage's read), which includes the rows they just stored:
        // polled at once, the last owners' rows became visible about 1.2 us later than after a 1000-cycle pause
        // (measured 17-26 us per decode step). The down -> x exchange needs none: the next layer's start (the
        // weight copies it issues) already separates the publish from the first poll.
        if (MK_SETTLE_O > 0) mk_settle(MK_SETTLE_O);
      }

      // ---- D (all CTAs): norm + gate/up rows of whole act blocks, silu * up, quantize (kernels.c:385-397)
      if (!read_vec(p.xw, 2 * E, 10 * l + 3, MK_SQ_SINK)) goto out;
      MK_TRACE(trow, 10);
      if (tid == 0) {
        refill();
        // the gate/up tiles of the first (or only) pair of act blocks, ahead as above (waiting for the down tile
        // here as well measured 36 us per step slower)
        if (nsplit == 0) {
          if (cta < nbf) wait_tiles(4, 0, cta + ncta < nbf ? 2 : 1, 64, 64, nbd);
        } else {
          wait_tiles(4, 0, cta >= ncta - 4 * nsplit ? 2 : 1, 64, 16, nbd);
        }
      }
      mk_norm_quant(xf, nw2, D, p.eps, xc, red, sqs, MK_SQ_SINK);
      MK_TRACE(trow, 14);
      auto publish_act = [&](int h, int ab) {  // warp 8h: silu(gate) * up of tile h, quantized and published
        const int lane = tid & 31;
        const float gt = outv[64 * h + lane], up = outv[64 * h + 32 + lane];
        const float v = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, fast_exp_ref(-gt))), up);
        int8_t* aq = reinterpret_cast<int8_t*>(actb + 64 * h);
        float* ad = reinterpret_cast<float*>(actb + 64 * h + 32);
        quant_block_nosum(v, lane, aq, ad);  // (the consumers form the lane sums themselves)
        __syncwarp();
        if (lane < 6) {  // bytes 6 lane .. 6 lane + 5 of the int8 block and its scale, under the epoch's low 16 bits
          const uint8_t* bb = actb + 64 * h;
          const int off = 6 * lane, a = off & ~7, sh = (off & 7) * 8;
          const unsigned long long lo = *reinterpret_cast<const unsigned long long*>(bb + a);
          const unsigned long long hi = *reinterpret_cast<const unsigned long long*>(bb + a + 8);
          const unsigned long long v48 = (sh ? (lo >> sh) | (hi << (64 - sh)) : lo) & 0xFFFFFFFFFFFFull;
          const unsigned long long wv = ((unsigned long long)(E & 0xFFFFu) << 48) | v48;
          asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p.actw + (size_t)ab * MK_ACT_WORDS + lane), "l"(wv)
                       : "memory");
        }
        __syncwarp();
      };
      if (nsplit == 0) {
        for (int ab0 = cta; ab0 < nbf; ab0 += 2 * ncta) {  // act blocks ab0 and ab0 + ncta: two tiles at once
          const int n = ab0 + ncta < nbf ? 2 : 1;
          if (!chain_tiles(4, n, 64, 64, nbd)) goto out;
          const int h = tid >> 8;
          if (h < n && (tid & 255) < 32) publish_act(h, ab0 + h * ncta);
        }
      } else {
        // act block cta on warps 0-7; the last 4 nsplit CTAs also take piece q (8 gate + 8 up rows of block
        // ncta + q / 4) on warps 8-9 and publish its 8 act values unquantized
        const int q = cta - (ncta - 4 * nsplit);
        if (!chain_tiles(4, q >= 0 ? 2 : 1, 64, 16, nbd)) goto out;
        if (tid < 32) publish_act(0, cta);
        if (q >= 0 && tid >= 256 && tid < 256 + 8) {
          const int j = tid - 256;
          const float gt = outv[64 + j], up = outv[64 + 8 + j];
          const float v = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, fast_exp_ref(-gt))), up);
          st_relaxed64(p.rawact + (size_t)(q >> 2) * 32 + 8 * (q & 3) + j, __float_as_uint(v), E);
        }
      }
      MK_TRACE(trow, 11);

      // ---- E (other CTAs): down rows over the quantized act, residual (kernels.c:399-400). Pipelined over the act
      // blocks: thread b (warps 0-5) polls act block b and, as soon as it lands, forms its products for every down
      // row of the CTA; warps 8.. quantize the split blocks the same way; warps 6-7 then add each (row, lane)
      // chain in block order once all blocks are in.
      if (!head) {
        const int R = o_hi - o_lo, LS = mk_prod_lane_stride(nbf);
        const int nq = nbf - nsplit;  // blocks published quantized
        if (tid == 0) ndone_s = 0;
        if (!next_tiles(5, 1, R, 0, nbf)) goto out;
        MK_TRACE(trow, 7);
        const uint8_t* tl = ring + (size_t)(tile_i % MK_NSLOT) * MK_SLOT;
        const __half* wdn = reinterpret_cast<const __half*>(tl + (((size_t)nbf * R * 16 + 15) & ~(size_t)15));
        float* pf = reinterpret_cast<float*>(prod);
        auto products = [&](int b, int r, const int4& x0, const int4& x1, const int4& xs4, float dx) {
          const int it = r * nbf + b;
          const uint4 w = *reinterpret_cast<const uint4*>(tl + (size_t)it * 16);
          const float sc = __fmul_rn(__half2float(wdn[it]), dx);
          float* o = pf + (size_t)(4 * r) * LS + b;
          o[0] = __fmul_rn(q4_lane(w.x, x0.x, x1.x, xs4.x), sc);
          o[LS] = __fmul_rn(q4_lane(w.y, x0.y, x1.y, xs4.y), sc);
          o[2 * LS] = __fmul_rn(q4_lane(w.z, x0.z, x1.z, xs4.z), sc);
          o[3 * LS] = __fmul_rn(q4_lane(w.w, x0.w, x1.w, xs4.w), sc);
        };
        if (tid < 192) {
          // warp w takes blocks 32 w + 192 k ...: its lanes poll the blocks' words together (each load instruction
          // reads 256 contiguous bytes: lane j of round t holds word (32 t + j) % 16 of block (32 t + j) / 16), park
          // the payloads in xq / xd / xs, then lane j forms the products of its block
          const int warp = tid >> 5, lane = tid & 31;
          // lane j reads words 4 j .. 4 j + 3: half j % 2 of block j / 2 (the six payload words of a block are words
          // 0-3 and 4-5); every act word is rewritten each layer, so its 16-bit tag differs from the previous one
          const uint16_t tg = (uint16_t)E;
          for (int b0 = 16 * warp; b0 < nq; b0 += 6 * 16) {
            const int nbw = min(16, nq - b0);
            const unsigned long long* src = p.actw + (size_t)b0 * MK_ACT_WORDS;
            unsigned long long v[4] = {0, 0, 0, 0};
            unsigned pending = 0;
            if ((lane >> 1) < nbw) {
              ld_relaxed64x4(src + 4 * lane, v);
              pending = (lane & 1) ? 0x3u : 0xFu;
            }
            const unsigned long long t0 = gtimer();
            for (unsigned it = 0;; it++) {
#pragma unroll
              for (int e = 0; e < 4; e++)
                if (((pending >> e) & 1u) && (uint16_t)(v[e] >> 48) == tg) pending &= ~(1u << e);
              if (__all_sync(0xffffffffu, pending == 0)) break;
              if ((it & 31) == 31) {
                int bad = 0;
                if (*(volatile int*)&abort_s || ld_volatile_i(p.err + 3)) bad = 1;
                else if (gtimer() - t0 > p.timeout_ns) bad = 2;
                if (__any_sync(0xffffffffu, bad != 0)) {
                  if (bad == 2) mk_fail(p, MK_TIMEOUT_WAIT, 10 * l + 4);
                  abort_s = 1;
                  break;
                }
              }
              if (pending) ld_relaxed64x4(src + 4 * lane, v);
            }
            if (*(volatile int*)&abort_s) break;
            if (trace && lane == 0 && (warp == 0 || b0 + 16 >= nq))
              trace[(size_t)trow * MK_TRACE_PTS + (warp == 0 ? 4 : 5)] = gtimer();
            // lane b (< 16) gathers block b's six payloads from lanes 2 b and 2 b + 1 and unpacks the 36 bytes
            const unsigned long long M48 = 0xFFFFFFFFFFFFull;
            const int s0 = 2 * (lane & 15);
            const unsigned long long c0 = __shfl_sync(0xffffffffu, v[0], s0) & M48;
            const unsigned long long c1 = __shfl_sync(0xffffffffu, v[1], s0) & M48;
            const unsigned long long c2 = __shfl_sync(0xffffffffu, v[2], s0) & M48;
            const unsigned long long c3 = __shfl_sync(0xffffffffu, v[3], s0) & M48;
            const unsigned long long c4 = __shfl_sync(0xffffffffu, v[0], s0 + 1) & M48;
            const unsigned long long c5 = __shfl_sync(0xffffffffu, v[1], s0 + 1) & M48;
            if (lane < nbw) {
              const int b = b0 + lane;
              const unsigned long long w0 = c0 | (c1 << 48), w1 = (c1 >> 16) | (c2 << 32), w2 = (c2 >> 32) | (c3 << 16),
                                       w3 = c4 | (c5 << 48);
              const int4 x0 = make_int4((int)w0, (int)(w0 >> 32), (int)w1, (int)(w1 >> 32));
              const int4 x1 = make_int4((int)w2, (int)(w2 >> 32), (int)w3, (int)(w3 >> 32));
              const float dx = __uint_as_float((uint32_t)(c5 >> 16));
              // lane l's accumulator start: MK_MAGIC - 8 x (sum of its eight int8 values, word l of each half)
              const int4 xs4 = make_int4(MK_MAGIC - 8 * __dp4a(x0.x, 0x01010101, __dp4a(x1.x, 0x01010101, 0)),
                                         MK_MAGIC - 8 * __dp4a(x0.y, 0x01010101, __dp4a(x1.y, 0x01010101, 0)),
                                         MK_MAGIC - 8 * __dp4a(x0.z, 0x01010101, __dp4a(x1.z, 0x01010101, 0)),
                                         MK_MAGIC - 8 * __dp4a(x0.w, 0x01010101, __dp4a(x1.w, 0x01010101, 0)));
              for (int r = 0; r < R; r++) products(b, r, x0, x1, xs4, dx);
              __threadfence_block();
              atomicAdd(&ndone_s, 1);
            }
            __syncwarp();
          }
        } else if (tid >= 256 && (tid >> 5) - 8 < nsplit) {
          const int k = (tid >> 5) - 8, lane = tid & 31, b = nq + k;
          const float v = __uint_as_float(wait_word(p.rawact + (size_t)k * 32 + lane, E, p, 10 * l + 5, &abort_s));
          if (trace && k == 0 && lane == 0) trace[(size_t)trow * MK_TRACE_PTS + 6] = gtimer();
          int8_t* sq8 = reinterpret_cast<int8_t*>(splitq_s[k]);
          quant_block_redux(v, lane, sq8, reinterpret_cast<float*>(splitq_s[k] + 32), reinterpret_cast<int4*>(splitq_s[k] + 48));
          __syncwarp();
          if (lane < R)
            products(b, lane, *reinterpret_cast<const int4*>(sq8), *reinterpret_cast<const int4*>(sq8 + 16),
                     *reinterpret_cast<const int4*>(splitq_s[k] + 48), *reinterpret_cast<const float*>(splitq_s[k] + 32));
          __syncwarp();
          if (lane == 0) {
            __threadfence_block();
            atomicAdd(&ndone_s, 1);
          }
        } else if (tid >= 192 && tid < 192 + ((4 * R + 31) & ~31)) {
          const int c = tid - 192;
          const unsigned long long t0 = gtimer();
          for (unsigned it = 0; *(volatile int*)&ndone_s < nbf; it++) {
            if ((it & 63) == 63) {
              if (*(volatile int*)&abort_s || ld_volatile_i(p.err + 3)) break;
              if (gtimer() - t0 > p.timeout_ns) {
                mk_fail(p, MK_TIMEOUT_WAIT, 10 * l + 6);
                abort_s = 1;
                break;
              }
            }
          }
          __threadfence_block();
          if (trace && c == 0) trace[(size_t)trow * MK_TRACE_PTS + 12] = gtimer();
          float acc = 0.f;
          if (c < 4 * R && !*(volatile int*)&abort_s)
            acc = (nbf & 3) == 0 ? chain_sum4(0.f, pf + (size_t)c * LS, nbf) : chain_sum(0.f, pf + (size_t)c * LS, 1, nbf);
          const float hv = hsum4_quad(acc);
          if (c < 4 * R && (c & 3) == 0) outv[c >> 2] = hv;
        }
        compute_bar();
        if (abort_s) goto out;
        release_tiles(1);
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
    if (!read_vec(p.xw, 2 * E + 1, 9999, MK_SQ_SINK)) goto out;
    MK_TRACE(lrow, 1);
    if (tid == 0) {  // the lm_head streams freely
      pace = false;
      refill();
    }
    mk_norm_quant(xf, onw, D, p.eps, xc, red, sqs, MK_SQ_SINK);
    MK_TRACE(lrow, 2);
    {
      // two tiles at once; the quad leader of each row stores its logit, and every warp keeps the running argmax
      // of its rows (ties to the lowest index, cpu-worker.js:156-157; the merge is order-independent)
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int r0 = v_lo; r0 < v_hi; r0 += 2 * MK_TILE_ROWS) {
        const int R0 = min(MK_TILE_ROWS, v_hi - r0);
        const int R1 = min(MK_TILE_ROWS, max(0, v_hi - r0 - MK_TILE_ROWS));
        const int n = R1 > 0 ? 2 : 1;
        if (!next_tiles(8, n, R0, R1, nbd)) goto out;
        const int h = tid >> 8, t = tid & 255, R = h ? R1 : R0;
        if (h < n && (t & ~31) < 4 * R) {  // whole warps (shuffles over all 32 lanes)
          const uint8_t* tl = ring + (size_t)((tile_i + h) % MK_NSLOT) * MK_SLOT;
          const int r = t >> 2;
          const float a = r < R ? mk_lane_chain(tl, R, nbpd, r, t & 3, xc) : 0.f;
          const float v = hsum4_quad(a);
          float vv = -INFINITY;
          int vi = 0x7fffffff;
          if (r < R && (t & 3) == 0) {
            p.logits[r0 + 64 * h + r] = v;
            vv = v;
            vi = r0 + 64 * h + r;
          }
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {  // the warp's 8 quad leaders
            const float v2 = __shfl_xor_sync(0xffffffffu, vv, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, vi, o);
            amax_merge(vv, vi, v2, i2);
          }
          amax_merge(bv, bi, vv, vi);
        }
        release_tiles(n);
      }
      MK_TRACE(lrow, 3);
      if ((tid & 31) == 0) {  // each warp's best
        red[tid >> 5] = bv;
        reinterpret_cast<int*>(red)[16 + (tid >> 5)] = bi;
      }
      compute_bar();
      if (tid == 0) {
        for (int w = 1; w < MK_WARPS; w++) amax_merge(bv, bi, red[w], reinterpret_cast<const int*>(red)[16 + w]);
        st_relaxed64(p.lmw + 2 * cta, __float_as_uint(bv), p.lm0 + step + 1);
        st_relaxed64(p.lmw + 2 * cta + 1, (uint32_t)bi, p.lm0 + step + 1);
      }
    }
    // (a pause before polling the words just published, as after the O publish: 1.3 us per step)
    if (MK_SETTLE_LM > 0) mk_settle(MK_SETTLE_LM);
    {  // every CTA's (value, index) pair, all words read at once
      uint32_t* lmv = reinterpret_cast<uint32_t*>(prod);
      read_words(2 * ncta, [&](int k) { return p.lmw + k; }, p.lm0 + step + 1, [&](int k, uint32_t v) { lmv[k] = v; }, p,
                 9998, &abort_s);
      compute_bar();
    }
    if (tid < 32) {
      const uint32_t* lmv = reinterpret_cast<const uint32_t*>(prod);
      float v = -INFINITY;
      int idx = 0x7fffffff;
      for (int i = tid; i < ncta; i += 32) amax_merge(v, idx, __uint_as_float(lmv[2 * i]), (int)lmv[2 * i + 1]);
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
  if (tid == 0)  // every issued bulk copy must land before the CTA exits (bounded; the sources are valid memory)
    for (int k = tile_i; k < issued; k++) {
      const unsigned long long t0 = gtimer();
      while (!mbar_try_wait(&full[k % MK_NSLOT], (k / MK_NSLOT) & 1))
        if (gtimer() - t0 > p.timeout_ns) break;
    }
  cp_async_wait_all();  // no shared-memory copy may still be in flight when the CTA exits
  if (p.done && cta == 0 && tid == 0) {
    // CTA 0 finishes after every CTA has published its last lm_head partial, so the launch's outcome is known:
    // the host polls this record instead of copying and synchronising
    volatile int32_t* d = p.done;
    d[1] = tok;
    d[2] = ld_volatile_i(p.err);
    d[3] = ld_volatile_i(p.err + 1);
    d[4] = ld_volatile_i(p.err + 2);
    __threadfence_system();
    d[0] = p.launch_seq;
  }
  return;
#undef MK_TRACE
}

}  // namespace h2
