// Device kernels of the H2 Qwen2 token loop for sm_100a, bit-exact with the reference CPU path.
//
// Why bit-exact: the reference quantizes every matrix input to int8 per 32 values (kernels.c:90-114). That
// re-quantization turns a 1-ulp difference anywhere upstream into a flipped int8 somewhere downstream, and 24
// layers amplify it: reordering only the RMSNorm sum moves the 0.5B model's logits by ~1.4% of their range, far
// outside the 2e-3 parity tolerance. So every floating-point result here is produced by the reference's own
// operation order and roundings (IEEE round-to-nearest intrinsics; no fused multiply-add):
//   - four "lanes" per vector, as the reference's 128-bit SIMD computes them: element i goes to lane i mod 4 in
//     RMSNorm and attention dots (kernels.c:80-86, 362-366); lane l of a Q4_0/Q8_0 block dot sums elements
//     {2l, 2l+1, 8+2l, 9+2l} of each half (the i32x4.dot_i16x8 lanes of kernels.c:121-139, 157-170);
//   - each lane accumulates in block (or position) order; lanes are added ((l0 + l1) + l2) + l3;
//   - softmax sums and the probability-weighted V sums run in position order (kernels.c:367-375).
// The parallel part of every op (integer block dots, products, exponentials) runs wide; only those ordered
// float sums run as short per-output chains.
//
// Data layout in HBM:
//   Q4_0 matrix [N][K]: rows in groups of 32; group g holds values [K/32][32 rows][16 B] then (separately) scales
//     [K/32][32 rows] fp16, so one warp-wide 16-byte load of block b reads 32 rows contiguously. Within each
//     16-byte block the bytes are permuted so that 32-bit word l holds the bytes of lane l (PERM below): word l =
//     GGUF bytes {2l, 2l+1, 8+2l, 9+2l}; its low nibbles are elements {2l, 2l+1, 8+2l, 9+2l} and its high nibbles
//     elements 16 + those. N is padded to a multiple of 32 with zero blocks.
//   Q8_0 matrix: the same grouping with 32-byte blocks, each 16-byte half permuted the same way.
//   int8 activations xq [M][K]: per block of 32 the two halves (elements 0..15, 16..31) permuted like the
//     weights, scale xd [M][K/32] f32, and per lane the accumulator start of its Q4_0 block dot xs [M][K/32] int4
//     (-8 x the sum of its int8 values, for the nibble offset, plus the float-conversion constant MK_MAGIC).
//   activations: x [M][D] f32 residual stream; qkv [M][D + 2*KVH*HD]; att [M][D]; gu [M][2F].
//   KV cache [seq][layer][kv_head][ctx][HD] f32 (the reference's dtype and order, kernels.c:347-348).
#pragma once
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace h2 {

// device-resident parameters of one pass, written by the host with one copy before each pass:
// [P_POS0] first position, [P_M] tokens, [P_SEQ] sequence, [P_MODE] 0 = the tokens are positions pos0 .. pos0+M-1 of
// one sequence (a prompt chunk or one decode step), 1 = one decode token of each of M sequences (a batched decode
// step: token m is at position prm[P_IDS + P_CAP + m] of sequence prm[P_IDS + 2 P_CAP + m]); then the ids.
enum { P_POS0 = 0, P_M = 1, P_SEQ = 2, P_MODE = 3, P_IDS = 4, P_CAP = 256, P_WORDS = P_IDS + 3 * P_CAP };
__device__ __forceinline__ int tok_pos(const int32_t* prm, int m) {
  return prm[P_MODE] ? prm[P_IDS + P_CAP + m] : prm[P_POS0] + m;
}
__device__ __forceinline__ int tok_seq(const int32_t* prm, int m) {
  return prm[P_MODE] ? prm[P_IDS + 2 * P_CAP + m] : prm[P_SEQ];
}

// byte p of a permuted 16-byte block holds GGUF byte PERM[p]
__host__ __device__ constexpr int perm16(int p) { return ((p & 3) >> 1) * 8 + (p >> 2) * 2 + (p & 1); }
// position of GGUF byte j (0..15) in the permuted block
__host__ __device__ constexpr int invperm16(int j) { return (((j & 7) >> 1) << 2) | ((j >> 3) << 1) | (j & 1); }

__device__ __forceinline__ float fast_exp_ref(float x) {  // kernels.c:69-78
  if (x < -87.0f) return 0.0f;
  if (x > 88.0f) x = 88.0f;
  float n = floorf(__fadd_rn(__fmul_rn(x, 1.44269504f), 0.5f));
  float r = __fsub_rn(__fsub_rn(x, __fmul_rn(n, 0.693145752f)), __fmul_rn(n, 1.42860677e-6f));
  float p = __fadd_rn(0.00833333377f, __fmul_rn(r, 0.00138888892f));
  p = __fadd_rn(0.0416666679f, __fmul_rn(r, p));
  p = __fadd_rn(0.166666672f, __fmul_rn(r, p));
  p = __fadd_rn(0.5f, __fmul_rn(r, p));
  p = __fadd_rn(1.0f, __fmul_rn(r, p));
  p = __fadd_rn(1.0f, __fmul_rn(r, p));
  return __int_as_float(__float_as_int(p) + ((int)n << 23));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ((l0 + l1) + l2) + l3 across 4 consecutive threads; valid in the thread with (tid & 3) == 0.
__device__ __forceinline__ float hsum4_quad(float a) {
  const float a1 = __shfl_down_sync(0xffffffffu, a, 1), a2 = __shfl_down_sync(0xffffffffu, a, 2),
              a3 = __shfl_down_sync(0xffffffffu, a, 3);
  return __fadd_rn(__fadd_rn(__fadd_rn(a, a1), a2), a3);
}

// Correctly rounded division by 127, division by 896 (the 0.5B hidden size), reciprocal and square root for the
// latency-critical chains of the decode kernel (RMSNorm scale, int8 block scales). Each uses a short published
// method inside an input range where a comparison with the IEEE-rounded intrinsics over every float of the range
// found no difference on B200 (h2c_selftest_math repeats that comparison over all 2^32 inputs, fallbacks included),
// and the intrinsic itself outside the range; so every result equals the intrinsic's, about 8-25 cycles instead of
// 60-70 on the dependent path.
//  - x / y with the divisor known in advance (N. Brisebarre, J.-M. Muller, S. K. Raina, "Accelerating correctly
//    rounded floating-point division when the divisor is known in advance", IEEE Trans. Computers 53(8), 2004):
//    zh = RN(1/y), zl = RN(1/y - zh), q = RN(x zh + RN(x zl)); exact here for x >= 2^-100.
//  - 1/b and sqrt(a) (P. W. Markstein, "Computation of elementary functions on the IBM RISC System/6000
//    processor", IBM J. Res. Dev. 34(1), 1990): the hardware approximation refined by one Newton step whose residual
//    (1 - b y, resp. a - s^2) is exact through a fused multiply-add; exact here for normal b < 2^126, resp.
//    a >= 2^-102.
constexpr float H2_R127_HI = (float)(1.0 / 127.0);
constexpr float H2_R127_LO = (float)((1.0 - 127.0 * (double)H2_R127_HI) / 127.0);
constexpr float H2_R896_HI = (float)(1.0 / 896.0);
constexpr float H2_R896_LO = (float)((1.0 - 896.0 * (double)H2_R896_HI) / 896.0);
// The fast forms themselves (branch-free) and their input ranges. Callers that need several results test all the
// ranges once and fall back to the intrinsics together, so the common path has one branch instead of one per
// operation (each branch around a possible call to the intrinsics' slow path costs a warp re-convergence).
__device__ __forceinline__ bool div_fast_ok(float x) { return __float_as_uint(x) - 0x0D800000u < 0x72000000u; }
__device__ __forceinline__ float div127_fast(float x) { return __fmaf_rn(x, H2_R127_HI, __fmul_rn(x, H2_R127_LO)); }
__device__ __forceinline__ float div896_fast(float x) { return __fmaf_rn(x, H2_R896_HI, __fmul_rn(x, H2_R896_LO)); }
__device__ __forceinline__ bool rcp_fast_ok(float b) { return __float_as_uint(b) - 0x00800000u <= 0x7E000000u; }
__device__ __forceinline__ float rcp_fast(float b) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
  return __fmaf_rn(__fmaf_rn(-b, y, 1.0f), y, y);
}
__device__ __forceinline__ bool sqrt_fast_ok(float a) { return __float_as_uint(a) - 0x0C800000u < 0x73000000u; }
__device__ __forceinline__ float sqrt_fast(float a) {
  float r;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  const float s = __fmul_rn(a, r);
  return __fmaf_rn(__fmaf_rn(-s, s, a), __fmul_rn(0.5f, r), s);
}
__device__ __forceinline__ float div127_rn(float x) { return div_fast_ok(x) ? div127_fast(x) : __fdiv_rn(x, 127.0f); }
__device__ __forceinline__ float div896_rn(float x) { return div_fast_ok(x) ? div896_fast(x) : __fdiv_rn(x, 896.0f); }
__device__ __forceinline__ float rcp_rn(float b) { return rcp_fast_ok(b) ? rcp_fast(b) : __fdiv_rn(1.0f, b); }
__device__ __forceinline__ float sqrt_rn(float a) { return sqrt_fast_ok(a) ? sqrt_fast(a) : __fsqrt_rn(a); }
// The exact forms of the block scales and of the RMSNorm scale (plain correctly rounded divisions and square root),
// for arguments outside the fast forms' ranges. Out of line: rarely taken, and inlined at every quantizer they
// measured 1.5% slower per decode step in the persistent kernel, whose code exceeds the instruction cache.
__device__ __noinline__ float2 block_scales_exact(float amax) {
  const float d = __fdiv_rn(amax, 127.0f);
  return make_float2(d, d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f);
}
__device__ __noinline__ float norm_scale_exact(float ss, int D, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), eps)));
}

// the int8 block scale and its reciprocal: d = amax / 127, id = d ? 1 / d : 0 (kernels.c:96-97), for one block and
// for two blocks at once
__device__ __forceinline__ void block_scales(float amax, float& d, float& id) {
  d = div127_fast(amax);
  id = rcp_fast(d);
  if (!(div_fast_ok(amax) && rcp_fast_ok(d))) {
    const float2 e = block_scales_exact(amax);
    d = e.x;
    id = e.y;
  }
}
__device__ __forceinline__ void block_scales2(float a0, float a1, float& d0, float& d1, float& i0, float& i1) {
  d0 = div127_fast(a0);
  d1 = div127_fast(a1);
  i0 = rcp_fast(d0);
  i1 = rcp_fast(d1);
  if (!(div_fast_ok(a0) && div_fast_ok(a1) && rcp_fast_ok(d0) && rcp_fast_ok(d1))) {
    const float2 e0 = block_scales_exact(a0), e1 = block_scales_exact(a1);
    d0 = e0.x;
    i0 = e0.y;
    d1 = e1.x;
    i1 = e1.y;
  }
}
// the RMSNorm scale 1 / sqrt(ss / D + eps) (kernels.c:84), every step correctly rounded
__device__ __forceinline__ float norm_scale(float ss, int D, float eps) {
  if (D == 896) {
    const float m = __fadd_rn(div896_fast(ss), eps);
    const float q = sqrt_fast(m);
    const float r = rcp_fast(q);
    if (div_fast_ok(ss) && sqrt_fast_ok(m) && rcp_fast_ok(q)) return r;
  }
  return norm_scale_exact(ss, D, eps);
}

// Integers |p| < 2^22 converted to float without the (quarter-rate) int->float instruction: the bit pattern
// MK_MAGIC + p is the float 12582912 + p exactly, and subtracting 12582912 is exact. Block dots carry MK_MAGIC in
// their accumulator, so f32(p) = __int_as_float(acc) - 12582912.0f.
constexpr int MK_MAGIC = 0x4B400000;
__device__ __forceinline__ float magic_to_float(int acc) { return __fsub_rn(__int_as_float(acc), 12582912.0f); }

// Quantize the 32 values held one per lane (kernels.c:90-114): amax over the block (a max is exact in any order),
// d = amax / 127, q = nearest-even(x * (1 / d)) saturated to int8. Stores the permuted int8 block, the scale and,
// per lane l of the reference's dot (the owner of elements {2l, 2l+1, 8+2l, 9+2l} of each half),
// MK_MAGIC - 8 x (sum of the lane's int8 values): the accumulator start of the lane's Q4_0 block dot (the -8 nibble
// offset and the float-conversion constant folded in). The warp reductions run in hardware (redux.sync): amax is
// the integer max of the |x| bit patterns (order-preserving for non-negative floats); the four lane sums are two
// packed add-reductions of the biased values q + 128 (eight of them per lane sum fit 16 bits), lanes 0 and 1 in one
// word, 2 and 3 in the other.
// dT (optional): a second copy of the scale (the transposed scale array the tensor-core matmul reads); s may be null
// when no consumer needs the lane sums.
__device__ __forceinline__ void quant_block_redux(float v, int lane, int8_t* q, float* d, int4* s, float* dT = nullptr) {
  const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))));
  float dd, id;
  block_scales(amax, dd, id);
  const int qi = max(-128, min(127, __float2int_rn(__fmul_rn(v, id))));
  q[(lane & 16) | invperm16(lane & 15)] = (int8_t)qi;
  const int dl = (lane & 7) >> 1;  // the dot lane that owns this element
  const unsigned bq = (unsigned)(qi + 128) << ((dl & 1) * 16);
  const unsigned s01 = __reduce_add_sync(0xffffffffu, dl < 2 ? bq : 0u);
  const unsigned s23 = __reduce_add_sync(0xffffffffu, dl < 2 ? 0u : bq);
  if (lane == 0) {
    *d = dd;
    if (dT) *dT = dd;
    if (s)
      *s = make_int4(MK_MAGIC - 8 * ((int)(s01 & 0xffffu) - 1024), MK_MAGIC - 8 * ((int)(s01 >> 16) - 1024),
                     MK_MAGIC - 8 * ((int)(s23 & 0xffffu) - 1024), MK_MAGIC - 8 * ((int)(s23 >> 16) - 1024));
  }
}

// quant_block_redux without the lane sums (for blocks whose consumers form them from the int8 values)
__device__ __forceinline__ void quant_block_nosum(float v, int lane, int8_t* q, float* d) {
  const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))));
  float dd, id;
  block_scales(amax, dd, id);
  q[(lane & 16) | invperm16(lane & 15)] = (int8_t)max(-128, min(127, __float2int_rn(__fmul_rn(v, id))));
  if (lane == 0) *d = dd;
}

// x[m] = dequant(embedding row ids[m]) (kernels.c:313-322), from the grouped / permuted Q4_0 layout
static __global__ void k_embed(const int32_t* __restrict__ prm, const uint8_t* __restrict__ qs, const __half* __restrict__ dsc,
                        int D, float* __restrict__ x) {
  const int m = blockIdx.x;
  const int t = prm[P_IDS + m];
  const int nb = D / 32, g = t >> 5, r = t & 31;
  float* xr = x + (size_t)m * D;
  for (int i = threadIdx.x; i < D / 2; i += blockDim.x) {
    const int blk = i >> 4, j = i & 15;
    const size_t e = ((size_t)g * nb + blk) * 32 + r;
    const uint8_t b = qs[e * 16 + invperm16(j)];
    const float s = __half2float(dsc[e]);
    xr[32 * blk + j] = __fmul_rn((float)((b & 15) - 8), s);
    xr[32 * blk + 16 + j] = __fmul_rn((float)((b >> 4) - 8), s);
  }
}

// RMSNorm then int8 quantization of rows row0 + blockIdx.x (kernels.c:80-86, 90-114), one CTA of NQ_THREADS per row.
// All threads load x and w with 16-byte loads into shared memory and store the squares lane-major (element 4k + l at
// sqT[l][k], lane rows padded by 4 floats against bank conflicts); threads 0..3 then run the reference's four lane
// chains of the sum of squares (lane l: x[l]^2 + x[l+4]^2 + ... in index order) from 16-byte shared loads, the
// scale is formed from ((l0 + l1) + l2) + l3, and every warp quantizes 32-value blocks of (x * scale) * w.
// D a multiple of 32; dynamic smem nq_smem_bytes(D).
constexpr int NQ_THREADS = 1024;
__host__ __device__ constexpr size_t nq_smem_bytes(int D) { return ((size_t)2 * D + 4 * ((size_t)D / 4 + 4)) * 4; }
static __global__ void __launch_bounds__(NQ_THREADS) k_norm_quant(const float* __restrict__ x, int row0,
                                                                  const float* __restrict__ w, int D, float eps,
                                                                  int8_t* __restrict__ xq, float* __restrict__ xd,
                                                                  int4* __restrict__ xs,
                                                                  float* __restrict__ xdT = nullptr, int ldT = 0) {
  extern __shared__ __align__(16) float nsm[];
  float* xsm = nsm;
  float* wsm = nsm + D;
  float* sqT = nsm + 2 * D;
  const int L4 = D / 4 + 4;
  __shared__ float rs;
  const int slot = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)(row0 + slot) * D);
  const float4* wr = reinterpret_cast<const float4*>(w);
  for (int k = threadIdx.x; k < D / 4; k += blockDim.x) {
    const float4 a = xr[k], b = __ldg(wr + k);
    reinterpret_cast<float4*>(xsm)[k] = a;
    reinterpret_cast<float4*>(wsm)[k] = b;
    sqT[k] = __fmul_rn(a.x, a.x);
    sqT[L4 + k] = __fmul_rn(a.y, a.y);
    sqT[2 * L4 + k] = __fmul_rn(a.z, a.z);
    sqT[3 * L4 + k] = __fmul_rn(a.w, a.w);
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    float s = 0.f;
    if (threadIdx.x < 4) {
      const float4* p = reinterpret_cast<const float4*>(sqT + threadIdx.x * L4);
#pragma unroll 8
      for (int j = 0; j < D / 16; j++) {
        const float4 a = p[j];
        s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, a.x), a.y), a.z), a.w);
      }
    }
    const float s1 = __shfl_sync(0xffffffffu, s, 1), s2 = __shfl_sync(0xffffffffu, s, 2),
                s3 = __shfl_sync(0xffffffffu, s, 3);
    if (threadIdx.x == 0) rs = norm_scale(__fadd_rn(__fadd_rn(__fadd_rn(s, s1), s2), s3), D, eps);
  }
  __syncthreads();
  const float r = rs;
  const int nb = D / 32, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int b = warp; b < nb; b += nw) {
    const int i = b * 32 + lane;
    const float v = __fmul_rn(__fmul_rn(xsm[i], r), wsm[i]);
    quant_block_redux(v, lane, xq + (size_t)slot * D + b * 32, xd + (size_t)slot * nb + b, xs + (size_t)slot * nb + b,
                      xdT ? xdT + (size_t)b * ldT + slot : nullptr);
  }
}

// int8 quantization of M rows of length K (the attention output before the O projection, kernels.c:379):
// one warp per 32-value block. xs may be null (no lane sums); xdT (optional): the scales transposed ([block][ldT]).
static __global__ void k_quant(const float* __restrict__ x, int K, int M, int8_t* __restrict__ xq, float* __restrict__ xd,
                        int4* __restrict__ xs, float* __restrict__ xdT = nullptr, int ldT = 0) {
  const int nb = K / 32;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (gw >= M * nb) return;
  const int m = gw / nb, b = gw % nb;
  const float v = x[(size_t)m * K + b * 32 + lane];
  quant_block_redux(v, lane, xq + (size_t)m * K + b * 32, xd + (size_t)m * nb + b, xs ? xs + (size_t)m * nb + b : nullptr,
                    xdT ? xdT + (size_t)b * ldT + m : nullptr);
}

// act = silu(gate) * up, then int8 quantization (kernels.c:393-397); one warp per 32-value block of act.
// gu: [M][2F] (gate, then up); outputs with a row pitch of ldo values (ldo >= F: a tensor-parallel rank writes its
// F columns into rows of the full width).
static __global__ void k_swiglu_quant(const float* __restrict__ gu, int F, int M, int8_t* __restrict__ xq,
                               float* __restrict__ xd, int4* __restrict__ xs, float* __restrict__ xdT = nullptr,
                               int ldT = 0, int ldo = 0) {
  const int nb = F / 32;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (gw >= M * nb) return;
  if (ldo == 0) ldo = F;
  const int m = gw / nb, b = gw % nb, nbo = ldo / 32;
  const float* g = gu + (size_t)m * 2 * F;
  const float gt = g[b * 32 + lane], up = g[F + b * 32 + lane];
  const float v = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, fast_exp_ref(-gt))), up);
  quant_block_redux(v, lane, xq + (size_t)m * ldo + b * 32, xd + (size_t)m * nbo + b, xs + (size_t)m * nbo + b,
                    xdT ? xdT + (size_t)b * ldT + m : nullptr);
}

enum { OP_STORE = 0, OP_BIAS = 1, OP_ADD = 2 };
enum { WQ4 = 0, WQ8 = 1 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint4 ldg_stream(const void* p) {  // weights are read once per pass: no L1 allocation
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Lane l of a Q4_0 block dot as a float: sum over its 8 elements of (q - 8) * x = dp4a(low nibbles, x0 word l)
// + dp4a(high nibbles, x1 word l) - 8 * (sum of those 8 x); xsn (from the quantizer) starts the accumulator with
// that last term plus MK_MAGIC. Nibbles 0..15 equal their signed-byte values, so signed dp4a applies.
__device__ __forceinline__ float q4_lane(uint32_t w, int x0, int x1, int xsn) {
  return magic_to_float(__dp4a((int)(w & 0x0f0f0f0fu), x0, __dp4a((int)((w >> 4) & 0x0f0f0f0fu), x1, xsn)));
}

// y[m][n] (op)= sum over blocks of the reference's lane arithmetic (matmul_q4 / dot_q8_q8, kernels.c:121-273).
// One CTA (256 threads) takes ROWS rows (within one 32-row group) for up to MB tokens:
//   phase 1 (wide): every (block, row) item loads its 16 (Q4) or 32 (Q8) weight bytes once, computes the four
//     exact integer lane dots per token and the products f32(p_l) * (dw * dx) into shared memory;
//   phase 2 (ordered): thread (token, row, lane) adds its lane's products in block order; four threads then form
//     ((l0 + l1) + l2) + l3 and apply the epilogue (put(), kernels.c:190-194).
// dynamic smem: MB * (K/32) * ROWS * 16 bytes
template <int WT, int ROWS, int MB, int OP>
__global__ void __launch_bounds__(256) k_matvec(const uint8_t* __restrict__ qs, const __half* __restrict__ dsc, int N,
                                                int K, const int8_t* __restrict__ xq, const float* __restrict__ xd,
                                                const int4* __restrict__ xs, int M, float* __restrict__ y, int ldy,
                                                const float* __restrict__ bias) {
  extern __shared__ float4 prod[];  // [m][b][r]
  constexpr int BB = WT == WQ4 ? 16 : 32;
  const int nb = K / 32;
  const int n0 = blockIdx.x * ROWS;
  const int g = n0 >> 5, r0 = n0 & 31;
  const uint8_t* wg = qs + (size_t)g * nb * 32 * BB;
  const __half* dg = dsc + (size_t)g * nb * 32;
#pragma unroll 8  // (8 items' weight loads in flight per thread: one token's matvec is bound by memory parallelism)
  for (int it = threadIdx.x; it < nb * ROWS; it += blockDim.x) {
    const int b = it / ROWS, r = it % ROWS;
    const size_t e = (size_t)b * 32 + r0 + r;
    const float dw = __half2float(dg[e]);
    uint4 w0 = ldg_stream(wg + e * BB), w1;
    if (WT == WQ8) w1 = ldg_stream(wg + e * BB + 16);
#pragma unroll
    for (int m = 0; m < MB; m++) {
      if (m < M) {
        const int4* xp = reinterpret_cast<const int4*>(xq + (size_t)m * K + b * 32);
        const int4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
        const float sc = __fmul_rn(dw, __ldg(xd + (size_t)m * nb + b));
        float p0, p1, p2, p3;
        if (WT == WQ4) {
          const int4 s = __ldg(xs + (size_t)m * nb + b);
          p0 = q4_lane(w0.x, x0.x, x1.x, s.x);
          p1 = q4_lane(w0.y, x0.y, x1.y, s.y);
          p2 = q4_lane(w0.z, x0.z, x1.z, s.z);
          p3 = q4_lane(w0.w, x0.w, x1.w, s.w);
        } else {
          p0 = magic_to_float(__dp4a((int)w0.x, x0.x, __dp4a((int)w1.x, x1.x, MK_MAGIC)));
          p1 = magic_to_float(__dp4a((int)w0.y, x0.y, __dp4a((int)w1.y, x1.y, MK_MAGIC)));
          p2 = magic_to_float(__dp4a((int)w0.z, x0.z, __dp4a((int)w1.z, x1.z, MK_MAGIC)));
          p3 = magic_to_float(__dp4a((int)w0.w, x0.w, __dp4a((int)w1.w, x1.w, MK_MAGIC)));
        }
        prod[((size_t)m * nb + b) * ROWS + r] = make_float4(__fmul_rn(p0, sc), __fmul_rn(p1, sc),
                                                            __fmul_rn(p2, sc), __fmul_rn(p3, sc));
      }
    }
  }
  __syncthreads();
  // (MB * ROWS * 4 is a multiple of 32 or below 256, so whole warps take part in hsum4_quad)
  for (int t = threadIdx.x; t < ((MB * ROWS * 4 + 255) & ~255); t += blockDim.x) {
    const int l = t & 3, r = (t >> 2) % ROWS, m = (t >> 2) / ROWS;
    float acc = 0.f;
    if (m < M && m < MB) {
      const float* pp = reinterpret_cast<const float*>(prod) + ((size_t)m * nb * ROWS + r) * 4 + l;
#pragma unroll 8
      for (int b = 0; b < nb; b++) acc = __fadd_rn(acc, pp[(size_t)b * ROWS * 4]);
    }
    const float v = hsum4_quad(acc);
    const int n = n0 + r;
    if (l == 0 && m < M && m < MB && n < N) {
      float* o = y + (size_t)m * ldy + n;
      if (OP == OP_ADD) *o = __fadd_rn(*o, v);
      else if (OP == OP_BIAS) *o = __fadd_rn(v, bias[n]);
      else *o = v;
    }
  }
}

// One token's matvec y[n] (op)= W[n] . x (matmul_q4 / dot_q8_q8 with M = 1, kernels.c:121-273), the decode step's
// hot loop. CTA = R rows of one 32-row group (256 threads), streaming its rows' blocks in chunks of CB = 256 / R
// blocks (thread (j, r) of a chunk takes block j, row r):
//   - the weight bytes and fp16 scales of chunk c, and the token's int8 values, scales and lane sums of its blocks,
//     land in stage c % MV_P of a cp.async ring, MV_P - 1 chunks ahead;
//   - after the chunk's barrier every thread forms its item's four exact lane products f32(p_l) * (dw * dx) into
//     the product buffer of the chunk (two, alternating), while threads 0..4R-1 (row r = t / 4, lane l = t % 4)
//     add the previous chunk's products to their running lane sum in block order;
//   - at the end ((l0 + l1) + l2) + l3 and the epilogue (put(), kernels.c:190-194).
// Every product and every sum is the reference's; only the order of independent work differs.
// dynamic smem: mv_smem_bytes<WT, R>().
constexpr int MV_P = 6;
template <int WT, int R>
__host__ __device__ constexpr size_t mv_stage_bytes() {
  // weights, fp16 scales, then the token's values (32 B), lane sums (16 B) and scale (4 B) per block
  return (size_t)256 * (WT == WQ4 ? 16 : 32) + 512 + (size_t)(256 / R) * 52;
}
template <int WT, int R>
__host__ __device__ constexpr size_t mv_smem_bytes() { return (size_t)MV_P * mv_stage_bytes<WT, R>() + 2 * 256 * 16; }
template <int WT, int R, int OP>
__global__ void __launch_bounds__(256) k_mv(const uint8_t* __restrict__ qs, const __half* __restrict__ dsc, int N,
                                            int K, const int8_t* __restrict__ xq, const float* __restrict__ xd,
                                            const int4* __restrict__ xs, float* __restrict__ y,
                                            const float* __restrict__ bias) {
  constexpr int BB = WT == WQ4 ? 16 : 32;
  constexpr int CB = 256 / R;
  constexpr int WS = 256 * BB;            // weight bytes per stage
  constexpr int ST = (int)mv_stage_bytes<WT, R>();
  extern __shared__ __align__(16) uint8_t mvs[];
  float4* prod = reinterpret_cast<float4*>(mvs + MV_P * ST);  // [2][CB][R]
  const int nb = K / 32, nch = (nb + CB - 1) / CB;
  const int tid = threadIdx.x, n0 = blockIdx.x * R, g = n0 >> 5, r0 = n0 & 31;
  const uint8_t* wg = qs + (size_t)g * nb * 32 * BB;
  const __half* dg = dsc + (size_t)g * nb * 32;
  const int j = tid / R, r = tid % R;
  // stage s: [WS] weights [j][r], [512] scales [j][r], [CB * 32] token values, [CB * 16] lane sums, [CB * 4] scales
  auto stage_w = [&](int c) {  // chunk c's weights and their scales into stage c % MV_P
    uint8_t* st = mvs + (c % MV_P) * ST;
    const int b = c * CB + j;
    if (b < nb) {
      const size_t e = (size_t)b * 32 + r0 + r;
      uint8_t* dst = st + (j * R + r) * BB;
      cp_async16(dst, wg + e * BB);
      if (BB == 32) cp_async16(dst + 16, wg + e * BB + 16);
      if ((r & 1) == 0) cp_async4(st + WS + (j * R + r) * 2, dg + e);
    }
  };
  auto stage_x = [&](int c) {  // the token's values of chunk c's blocks into stage c % MV_P
    {
      uint8_t* st = mvs + (c % MV_P) * ST;
      const int b0 = c * CB;
      if (tid < 2 * CB) {  // the token's values of the chunk's blocks, 16 bytes per thread
        if (b0 + tid / 2 < nb) cp_async16(st + WS + 512 + tid * 16, xq + (size_t)b0 * 32 + tid * 16);
      } else if (tid < 3 * CB) {
        if (WT == WQ4 && b0 + tid - 2 * CB < nb)
          cp_async16(st + WS + 512 + CB * 32 + (tid - 2 * CB) * 16, xs + b0 + tid - 2 * CB);
      } else if (tid < 4 * CB) {
        if (b0 + tid - 3 * CB < nb) cp_async4(st + WS + 512 + CB * 48 + (tid - 3 * CB) * 4, xd + b0 + tid - 3 * CB);
      }
    }
  };
  auto stage = [&](int c) {  // chunk c into stage c % MV_P (an empty group past the last chunk)
    if (c < nch) {
      stage_w(c);
      stage_x(c);
    }
    cp_async_commit();
  };
  // the first chunks' weights first, then the token's values of those chunks (one more group)
#pragma unroll
  for (int c = 0; c < MV_P - 1; c++) {
    if (c < nch) stage_w(c);
    cp_async_commit();
  }
#pragma unroll
  for (int c = 0; c < MV_P - 1; c++)
    if (c < nch) stage_x(c);
  cp_async_commit();
  const int cr = tid >> 2, cl = tid & 3;
  float acc = 0.f;
  for (int c = 0; c <= nch; c++) {
    if (c == 0) cp_async_wait_all();                // the first chunk and the token's first values
    else if (c < nch) cp_async_wait_group<MV_P - 2>();  // chunk c has landed
    __syncthreads();
    stage(c + MV_P - 1);  // into the stage chunk c - 1 used (every thread is past it)
    if (c >= 1 && tid < R * 4) {  // the previous chunk's products, in block order
      const int cb = min(CB, nb - (c - 1) * CB);
      const float* pp = reinterpret_cast<const float*>(prod + ((c - 1) & 1) * 256) + cr * 4 + cl;
#pragma unroll 8
      for (int jj = 0; jj < cb; jj++) acc = __fadd_rn(acc, pp[jj * R * 4]);
    }
    const int b = c * CB + j;
    if (c < nch && b < nb) {
      const uint8_t* st = mvs + (c % MV_P) * ST;
      const uint4 w0 = *reinterpret_cast<const uint4*>(st + (j * R + r) * BB);
      const float dw = __half2float(*reinterpret_cast<const __half*>(st + WS + (j * R + r) * 2));
      const int4* xp = reinterpret_cast<const int4*>(st + WS + 512 + j * 32);
      const int4 x0 = xp[0], x1 = xp[1];
      const float sc = __fmul_rn(dw, *reinterpret_cast<const float*>(st + WS + 512 + CB * 48 + j * 4));
      float p0, p1, p2, p3;
      if (WT == WQ4) {
        const int4 sm = *reinterpret_cast<const int4*>(st + WS + 512 + CB * 32 + j * 16);
        p0 = q4_lane(w0.x, x0.x, x1.x, sm.x);
        p1 = q4_lane(w0.y, x0.y, x1.y, sm.y);
        p2 = q4_lane(w0.z, x0.z, x1.z, sm.z);
        p3 = q4_lane(w0.w, x0.w, x1.w, sm.w);
      } else {
        const uint4 w1 = *reinterpret_cast<const uint4*>(st + (j * R + r) * BB + 16);
        p0 = magic_to_float(__dp4a((int)w0.x, x0.x, __dp4a((int)w1.x, x1.x, MK_MAGIC)));
        p1 = magic_to_float(__dp4a((int)w0.y, x0.y, __dp4a((int)w1.y, x1.y, MK_MAGIC)));
        p2 = magic_to_float(__dp4a((int)w0.z, x0.z, __dp4a((int)w1.z, x1.z, MK_MAGIC)));
        p3 = magic_to_float(__dp4a((int)w0.w, x0.w, __dp4a((int)w1.w, x1.w, MK_MAGIC)));
      }
      prod[(c & 1) * 256 + j * R + r] = make_float4(__fmul_rn(p0, sc), __fmul_rn(p1, sc), __fmul_rn(p2, sc),
                                                    __fmul_rn(p3, sc));
    }
  }
  cp_async_wait_all();
  const float v = hsum4_quad(acc);  // (every warp takes part; threads past 4R hold 0)
  const int n = n0 + cr;
  if (tid < R * 4 && cl == 0 && n < N) {
    if (OP == OP_ADD) y[n] = __fadd_rn(y[n], v);
    else if (OP == OP_BIAS) y[n] = __fadd_rn(v, bias[n]);
    else y[n] = v;
  }
}

// y[m][n] (op)= the reference's lane arithmetic for several tokens at once (matmul_q4 M > 1 / dot_q8_q8,
// kernels.c:121-273), each weight byte read once per token group. CTA (token group, row range): the group's TG
// tokens' int8 activations, lane sums and scales stay in shared memory for the whole CTA; the range's weights stream
// through a double-buffered cp.async ring in chunks of MC_BC blocks x RT * H rows (a sub-range). Thread
// (m, h, l) keeps the running lane-l sums of token m for rows h, h + H, ... of the sub-range (H = 256 / (4 TG)) in
// registers and adds each block's product in block order: acc = (((0 + p_0 (dw_0 dx_0)) + p_1 (dw_1 dx_1)) + ...);
// at the sub-range's last block ((l0 + l1) + l2) + l3 and the epilogue (put(), kernels.c:190-194).
constexpr int MC_BC = 16;  // blocks per weight chunk
__host__ __device__ constexpr int mm_wb(int wt) { return wt == 0 ? 16 : 32; }
__host__ __device__ constexpr int mm_xq_stride(int nb) { return nb * 32 + 16; }  // bytes per token (padded)
__host__ __device__ constexpr int mm_xs_stride(int nb) { return nb * 16 + 16; }
__host__ __device__ constexpr int mm_xd_stride(int nb) { return nb + 1; }       // floats
__host__ __device__ constexpr int mm_act_bytes(int tg, int nb) {
  return tg * (mm_xq_stride(nb) + mm_xs_stride(nb)) + ((tg * mm_xd_stride(nb) * 4 + 15) & ~15);
}
__host__ __device__ constexpr int mm_chunk_bytes(int wt, int sr) {
  return sr * MC_BC * mm_wb(wt) + ((sr * MC_BC * 2 + 15) & ~15);
}
template <int WT, int TG, int RT, int OP>
__global__ void __launch_bounds__(256) k_matmul(const uint8_t* __restrict__ qs, const __half* __restrict__ dsc, int N,
                                                int K, const int8_t* __restrict__ xq, const float* __restrict__ xd,
                                                const int4* __restrict__ xs, int M, int rows_per_cta, float* __restrict__ y,
                                                int ldy, const float* __restrict__ bias) {
  constexpr int WB = mm_wb(WT), H = 256 / (TG * 4), SR = H * RT, CH = mm_chunk_bytes(WT, SR);
  constexpr int WSZ = SR * MC_BC * WB;
  extern __shared__ __align__(16) uint8_t msm[];
  const int nb = K / 32, ntg = (M + TG - 1) / TG;
  const int tg = blockIdx.x % ntg, m0 = tg * TG, mt = min(TG, M - m0);
  const int row_lo = (blockIdx.x / ntg) * rows_per_cta, row_hi = min(N, row_lo + rows_per_cta);
  const int tid = threadIdx.x, l = tid & 3, hp = (tid >> 2) % H, m = tid / (4 * H);
  uint8_t* axq = msm;
  uint8_t* axs = axq + TG * mm_xq_stride(nb);
  float* axd = reinterpret_cast<float*>(axs + TG * mm_xs_stride(nb));
  uint8_t* ring = msm + mm_act_bytes(TG, nb);
  // the token group's activations, once
  for (int i = tid; i < mt * nb * 2; i += 256) {
    const int hf = i & 1, b = (i >> 1) % nb, mm = (i >> 1) / nb;
    cp_async16(axq + mm * mm_xq_stride(nb) + b * 32 + hf * 16, xq + (size_t)(m0 + mm) * K + (size_t)b * 32 + hf * 16);
  }
  for (int i = tid; i < mt * nb; i += 256) {
    const int b = i % nb, mm = i / nb;
    if (WT == WQ4) cp_async16(axs + mm * mm_xs_stride(nb) + b * 16, xs + (size_t)(m0 + mm) * nb + b);
    cp_async4(axd + mm * mm_xd_stride(nb) + b, xd + (size_t)(m0 + mm) * nb + b);
  }
  const int nkc = (nb + MC_BC - 1) / MC_BC;
  const int nsub = (row_hi - row_lo + SR - 1) / SR;
  const int nchunk = nsub * nkc;
  auto stage = [&](int c) {  // chunk c: sub-range c / nkc, blocks (c % nkc) * MC_BC ..
    uint8_t* ws = ring + (c & 1) * CH;
    __half* ds = reinterpret_cast<__half*>(ws + WSZ);
    const int rb = row_lo + (c / nkc) * SR, b0 = (c % nkc) * MC_BC, bc = min(MC_BC, nb - b0);
    for (int i = tid; i < bc * SR * (WB / 16); i += 256) {
      const int piece = i % (WB / 16), r = (i / (WB / 16)) % SR, b = i / (WB / 16) / SR;
      const int n = rb + r;  // rows past N read the zero padding of their 32-row group, or are skipped
      if (n < ((N + 31) & ~31)) {
        const size_t e = ((size_t)(n >> 5) * nb + b0 + b) * 32 + (n & 31);
        cp_async16(ws + (b * SR + r) * WB + piece * 16, qs + e * WB + piece * 16);
      }
    }
    for (int i = tid; i < bc * (SR / 2); i += 256) {  // scales of two adjacent rows (same 32-row group) per copy
      const int rp = i % (SR / 2), b = i / (SR / 2), n = rb + 2 * rp;
      if (n < ((N + 31) & ~31))
        cp_async4(ds + b * SR + 2 * rp, dsc + ((size_t)(n >> 5) * nb + b0 + b) * 32 + (n & 31));
    }
    cp_async_commit();
  };
  float acc[RT];
#pragma unroll
  for (int j = 0; j < RT; j++) acc[j] = 0.f;
  if (nchunk > 0) stage(0);  // (committed together with the activations)
  for (int c = 0; c < nchunk; c++) {
    if (c + 1 < nchunk) {
      stage(c + 1);
      cp_async_wait_group<1>();
    } else {
      cp_async_wait_group<0>();
    }
    __syncthreads();
    const int kc = c % nkc, b0 = kc * MC_BC, bc = min(MC_BC, nb - b0);
    if (m < mt) {
      const uint8_t* ws = ring + (c & 1) * CH;
      const __half* ds = reinterpret_cast<const __half*>(ws + WSZ);
      const uint8_t* xqm = axq + m * mm_xq_stride(nb) + b0 * 32;
      const uint8_t* xsm = axs + m * mm_xs_stride(nb) + b0 * 16;
      const float* xdm = axd + m * mm_xd_stride(nb) + b0;
      for (int b = 0; b < bc; b++) {
        const int x0 = *reinterpret_cast<const int*>(xqm + b * 32 + 4 * l);
        const int x1 = *reinterpret_cast<const int*>(xqm + b * 32 + 16 + 4 * l);
        const int xsl = WT == WQ4 ? *reinterpret_cast<const int*>(xsm + b * 16 + 4 * l) : 0;
        const float dx = xdm[b];
#pragma unroll
        for (int j = 0; j < RT; j++) {
          const int r = hp + H * j;
          const uint8_t* wr = ws + (b * SR + r) * WB + 4 * l;
          float p;
          if (WT == WQ4) {
            p = q4_lane(*reinterpret_cast<const uint32_t*>(wr), x0, x1, xsl);
          } else {
            const int w0 = *reinterpret_cast<const int*>(wr), w1 = *reinterpret_cast<const int*>(wr + 16);
            p = magic_to_float(__dp4a(w0, x0, __dp4a(w1, x1, MK_MAGIC)));
          }
          acc[j] = __fadd_rn(acc[j], __fmul_rn(p, __fmul_rn(__half2float(ds[b * SR + r]), dx)));
        }
      }
    }
    if (kc == nkc - 1) {  // the sub-range's rows are complete
      const int rb = row_lo + (c / nkc) * SR;
#pragma unroll
      for (int j = 0; j < RT; j++) {
        const float v = hsum4_quad(acc[j]);
        acc[j] = 0.f;
        const int n = rb + hp + H * j;
        if (l == 0 && m < mt && n < row_hi) {
          float* o = y + (size_t)(m0 + m) * ldy + n;
          if (OP == OP_ADD) *o = __fadd_rn(*o, v);
          else if (OP == OP_BIAS) *o = __fadd_rn(v, bias[n]);
          else *o = v;
        }
      }
    }
    __syncthreads();  // the buffer is refilled by the next iteration's stage()
  }
  cp_async_wait_all();
}

// The same arithmetic with the exact integer block dots on the tensor cores (mma.sync m16n8k32, u8 x s8 for Q4_0
// nibbles, s8 x s8 for Q8_0). In the permuted block layout lane l of the reference's dot owns bytes 4l .. 4l+3 of
// each 16-byte half, which are the k = 4t .. 4t+3 and 16+4t .. 16+4t+3 slices of the MMA's A fragment of thread
// t = l; so an A tile whose row 4 r + l keeps only lane l's weights of weight row r gives, in one MMA, the four lane
// dots of 4 weight rows x 8 tokens for one block. The accumulator input is the lane's MK_MAGIC - 8 x (sum of its
// int8 activations) (Q4) or MK_MAGIC (Q8), so each result is the float bit pattern of 12582912 + dot, exactly the
// value q4_lane / dot_q8 form with dp4a. The float epilogue per block, in block order, is the reference's:
// acc_l += f32(dot_l) * (dw * dx), the conversion and the two products for two tokens at a time with the packed
// f32x2 forms (each half rounded as the scalar op). CTA: 8 warps x 4 weight rows = one 32-row group per sub-range; warp w holds the lane sums of rows 4w + (g / 4)
// and 4w + 2 + (g / 4) (lane g % 4) for tokens 8 j + 2 t, 8 j + 2 t + 1 (g = laneid / 4, t = laneid % 4). The token
// group's activations stay in shared memory (int8 blocks per token; lane sums as [block][lane][token]; scales as
// [block][token], so each thread's token pair is one 8-byte load); the weights stream through an MT_ST-stage
// cp.async ring of MC_BC-block chunks.
constexpr int MT_ST = 4;
__host__ __device__ constexpr int mt_xs_lane(int tg) { return tg + 8; }  // ints per lane row (padded)
__host__ __device__ constexpr int mt_act_bytes(int tg, int nb) {
  return tg * mm_xq_stride(nb) + nb * 4 * mt_xs_lane(tg) * 4 + nb * tg * 4;
}
__host__ __device__ constexpr int mt_smem_bytes(int wt, int tg, int nb) {
  return mt_act_bytes(tg, nb) + MT_ST * mm_chunk_bytes(wt, 32);
}
__device__ __forceinline__ unsigned long long f2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float f2_lo(unsigned long long v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(unsigned long long v) { return __uint_as_float((uint32_t)(v >> 32)); }

// One token's matvec on the tensor cores (mma.sync m16n8k32), y[n] (op)= W[n] . x, the decode step's hot loop
// (matmul_q4 / dot_q8_q8 with M = 1, kernels.c:121-273). Each warp owns 8 RG weight rows and walks their blocks in
// order; per block and per group of 8 rows one MMA:
//   - B = the 8 rows' block (k = the permuted byte order: 4t .. 4t+3 and 16+4t .. 16+4t+3 are lane t's bytes of the
//     two halves; u8 low and high nibbles for Q4_0, s8 for Q8_0), one 32-bit shared load per thread;
//   - A = the token's int8 block masked per reference lane: row m keeps only lane m's bytes (rows 4..15 zero), so
//     D[m][n] = lane m's exact integer dot of row n; the accumulator input is MK_MAGIC - 8 x (lane sum) for Q4_0 (the
//     -8 nibble offset folded in) or MK_MAGIC for Q8_0, so D holds the bit pattern of 12582912 + dot. A, the
//     accumulator input and the token's block scale are loaded once per block for the RG groups;
//   - thread t (t < 16) holds lane t / 4 of rows 2 (t % 4) and 2 (t % 4) + 1 of each group and keeps their running
//     sums in registers: acc += f32(dot) * (dw * dx) in block order; at the end ((l0 + l1) + l2) + l3 across four
//     threads and the epilogue (put(), kernels.c:190-194).
// The rows' weight bytes and scales stream through a per-warp cp.async ring of NSTG chunks of CK blocks; the token's
// values are staged in shared memory once per CTA. CTA: W warps; dynamic smem mt_smem_bytes<WT, W, RG, NSTG, CK>(K).
template <int WT>
__host__ __device__ constexpr int mt_bb() { return WT == WQ4 ? 16 : 32; }
template <int WT, int RG, int NSTG, int CK>
__host__ __device__ constexpr size_t mt_warp_bytes() { return (size_t)NSTG * CK * 8 * RG * (mt_bb<WT>() + 2); }
template <int WT, int W, int RG, int NSTG, int CK>
__host__ __device__ constexpr size_t mt_smem_bytes(int K) {
  return (size_t)W * mt_warp_bytes<WT, RG, NSTG, CK>() + (size_t)K + (((size_t)K / 32 * 4 + 15) & ~(size_t)15) +
         (WT == WQ4 ? (size_t)K / 32 * 16 : 0);
}
template <int WT, int W, int RG, int NSTG, int CK, int OP>
__global__ void __launch_bounds__(W * 32) k_mvt(const uint8_t* __restrict__ qs, const __half* __restrict__ dsc, int N,
                                                int K, const int8_t* __restrict__ xq, const float* __restrict__ xd,
                                                const int4* __restrict__ xs, float* __restrict__ y,
                                                const float* __restrict__ bias) {
  constexpr int BB = mt_bb<WT>();
  constexpr int RB = 8 * RG * BB;     // weight bytes of the warp's rows per block
  constexpr int SW = CK * RB;         // weight bytes per stage
  constexpr int SS = CK * 16 * RG;    // scale bytes per stage (8 RG fp16 per block)
  static_assert(SW % 512 == 0 && SS % 16 == 0, "stage sizes");
  extern __shared__ __align__(16) uint8_t mts[];
  const int nb = K / 32, nch = (nb + CK - 1) / CK;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = mts + warp * mt_warp_bytes<WT, RG, NSTG, CK>();  // [NSTG][SW], then [NSTG][SS] scales
  uint8_t* sring = ring + NSTG * SW;
  int8_t* xqs = reinterpret_cast<int8_t*>(mts + W * mt_warp_bytes<WT, RG, NSTG, CK>());
  float* xds = reinterpret_cast<float*>(xqs + K);
  int* xss = reinterpret_cast<int*>(xds + ((nb + 3) & ~3));
  const int n0 = (blockIdx.x * W + warp) * 8 * RG;
  const bool live = n0 < ((N + 31) & ~31);
  const int g32 = n0 >> 5, r0 = n0 & 31;
  const uint8_t* wg = qs + ((size_t)g32 * nb * 32 + r0) * BB;  // block b of the warp's rows: wg + b * 32 * BB
  const __half* dg = dsc + (size_t)g32 * nb * 32 + r0;          // their scales: dg + b * 32
  auto stage = [&](int c) {  // chunk c into stage c % NSTG (an empty group past the last chunk)
    if (live && c < nch) {
      const int b0 = c * CK;
      uint8_t* dst = ring + (c % NSTG) * SW;
#pragma unroll
      for (int i = 0; i < SW / 16 / 32; i++) {
        const int pc = lane + 32 * i, bl = pc / (RB / 16);
        if (b0 + bl < nb) cp_async16(dst + pc * 16, wg + (size_t)(b0 + bl) * 32 * BB + (pc % (RB / 16)) * 16);
      }
#pragma unroll
      for (int i = 0; i < (SS / 16 + 31) / 32; i++) {
        const int pc = lane + 32 * i, bl = pc / RG;
        if (pc < SS / 16 && b0 + bl < nb)
          cp_async16(sring + (c % NSTG) * SS + pc * 16, dg + (size_t)(b0 + bl) * 32 + (pc % RG) * 8);
      }
    }
    cp_async_commit();
  };
  // the first chunks' weights first, then the token's values (one more group)
#pragma unroll
  for (int c = 0; c < NSTG - 1; c++) stage(c);
  for (int i = threadIdx.x; i < K / 16; i += W * 32) cp_async16(xqs + 16 * i, xq + 16 * i);
  for (int i = threadIdx.x; i < nb; i += W * 32) {
    cp_async4(xds + i, xd + i);
    if (WT == WQ4) cp_async16(xss + 4 * i, xs + i);
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();  // the token's values, staged by all threads, are visible to every warp
  if (!live) return;
  // masks instead of branches: A keeps lane m's bytes only in row m (lanes 0, 5, 10, 15), C only in rows 0..3
  const int tq = lane & 3, lm = (lane >> 2) & 3;
  const int amask = (lane < 16 && (lane >> 2) == tq) ? -1 : 0;
  const int cmask = lane < 16 ? -1 : 0;
  const unsigned long long magic2 = f2(-12582912.0f, -12582912.0f);
  float acc[RG][2];  // (meaningful in lanes 0..15)
#pragma unroll
  for (int g = 0; g < RG; g++) acc[g][0] = acc[g][1] = 0.f;
  auto block = [&](const uint8_t* ws, const uint8_t* ss, int bl, int b) {
    const int* xb = reinterpret_cast<const int*>(xqs + b * 32);
    const int a0 = xb[tq] & amask, a2 = xb[4 + tq] & amask;
    const int c0 = (WT == WQ4 ? xss[4 * b + lm] : MK_MAGIC) & cmask;
    const float dx = xds[b];
    const unsigned long long dx2 = f2(dx, dx);
#pragma unroll
    for (int g = 0; g < RG; g++) {
      uint32_t b0r, b1r;
      if (WT == WQ4) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(ws + bl * RB + g * 128 + 4 * lane);
        b0r = w & 0x0f0f0f0fu;
        b1r = (w >> 4) & 0x0f0f0f0fu;
      } else {
        const uint8_t* wr = ws + bl * RB + g * 256 + (lane >> 2) * 32 + tq * 4;
        b0r = *reinterpret_cast<const uint32_t*>(wr);
        b1r = *reinterpret_cast<const uint32_t*>(wr + 16);
      }
      int d0, d1, d2, d3;
      if (WT == WQ4)
        asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%10, %11, %12, %13};"
            : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
            : "r"(a0), "r"(0), "r"(a2), "r"(0), "r"(b0r), "r"(b1r), "r"(c0), "r"(c0), "r"(0), "r"(0));
      else
        asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%10, %11, %12, %13};"
            : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
            : "r"(a0), "r"(0), "r"(a2), "r"(0), "r"(b0r), "r"(b1r), "r"(c0), "r"(c0), "r"(0), "r"(0));
      const float2 dw = __half22float2(*reinterpret_cast<const __half2*>(ss + (bl * RG + g) * 16 + 4 * tq));
      const unsigned long long p = f2_add(f2(__int_as_float(d0), __int_as_float(d1)), magic2);
      const unsigned long long q = f2_mul(p, f2_mul(f2(dw.x, dw.y), dx2));
      // (scalar adds for the running sums: a packed multiply feeding a packed add could become one fused op)
      acc[g][0] = __fadd_rn(acc[g][0], f2_lo(q));
      acc[g][1] = __fadd_rn(acc[g][1], f2_hi(q));
    }
  };
  for (int c = 0; c < nch; c++) {
    if (c > 0) cp_async_wait_group<NSTG - 2>();  // chunk c has landed
    __syncwarp();
    stage(c + NSTG - 1);  // into the stage of chunk c - 1 (every lane is past it)
    const int s = c % NSTG, b0 = c * CK;
    const uint8_t* ws = ring + s * SW;
    const uint8_t* ss = sring + s * SS;
    if (b0 + CK <= nb) {
#pragma unroll
      for (int bl = 0; bl < CK; bl++) block(ws, ss, bl, b0 + bl);
    } else {
      for (int bl = 0; bl < nb - b0; bl++) block(ws, ss, bl, b0 + bl);
    }
  }
  cp_async_wait_all();
  // lanes m = 0..3 of rows 2j, 2j+1 of a group sit at threads j, 4 + j, 8 + j, 12 + j
#pragma unroll
  for (int g = 0; g < RG; g++) {
#pragma unroll
    for (int k = 0; k < 2; k++) {
      const float a = acc[g][k];
      const float u1 = __shfl_down_sync(0xffffffffu, a, 4), u2 = __shfl_down_sync(0xffffffffu, a, 8),
                  u3 = __shfl_down_sync(0xffffffffu, a, 12);
      const int n = n0 + g * 8 + 2 * lane + k;
      if (lane < 4 && n < N) {
        const float v = __fadd_rn(__fadd_rn(__fadd_rn(a, u1), u2), u3);
        if (OP == OP_ADD) y[n] = __fadd_rn(y[n], v);
        else if (OP == OP_BIAS) y[n] = __fadd_rn(v, bias[n]);
        else y[n] = v;
      }
    }
  }
}


template <int WT, int TG, int OP>
__global__ void __launch_bounds__(256) k_matmul_tc(const uint8_t* __restrict__ qs, const __half* __restrict__ dsc,
                                                   int N, int K, const int8_t* __restrict__ xq,
                                                   const float* __restrict__ xd, const int4* __restrict__ xs, int M,
                                                   int rows_per_cta, float* __restrict__ y, int ldy,
                                                   const float* __restrict__ bias) {
  constexpr int WB = mm_wb(WT), SR = 32, CH = mm_chunk_bytes(WT, SR), NT = TG / 8, XL = mt_xs_lane(TG);
  constexpr int WSZ = SR * MC_BC * WB;
  extern __shared__ __align__(16) uint8_t msm[];
  const int nb = K / 32, ntg = (M + TG - 1) / TG, xqs = mm_xq_stride(nb);
  const int tg = blockIdx.x % ntg, m0 = tg * TG, mt = min(TG, M - m0);
  const int row_lo = (blockIdx.x / ntg) * rows_per_cta, row_hi = min(N, row_lo + rows_per_cta);
  const int tid = threadIdx.x, warp = tid >> 5, lid = tid & 31, g = lid >> 2, t = lid & 3, ln = g & 3;
  const int ra = 4 * warp + (g >> 2), rbw = ra + 2;  // the thread's two weight rows (sub-range local)
  uint8_t* axq = msm;                                                  // [TG][xqs]
  int* axs = reinterpret_cast<int*>(axq + TG * xqs);                   // [nb][4][XL]
  float* axd = reinterpret_cast<float*>(axs + nb * 4 * XL);            // [nb][TG]
  uint8_t* ring = msm + mt_act_bytes(TG, nb);
  // the token group's activations, once (tokens past M read as zeros)
  for (int i = tid; i < TG * nb * 2; i += 256) {
    const int hf = i & 1, b = (i >> 1) % nb, mm = (i >> 1) / nb;
    uint8_t* dst = axq + mm * xqs + b * 32 + hf * 16;
    if (mm < mt) cp_async16(dst, xq + (size_t)(m0 + mm) * K + (size_t)b * 32 + hf * 16);
    else *reinterpret_cast<int4*>(dst) = make_int4(0, 0, 0, 0);
  }
  for (int i = tid; i < TG * nb; i += 256) {
    const int mm = i % TG, b = i / TG;
    int4 s4 = make_int4(0, 0, 0, 0);
    float d = 0.f;
    if (mm < mt) {
      if (WT == WQ4) s4 = xs[(size_t)(m0 + mm) * nb + b];
      d = xd[(size_t)(m0 + mm) * nb + b];
    }
    int* sp = axs + (b * 4) * XL + mm;
    sp[0] = s4.x;
    sp[XL] = s4.y;
    sp[2 * XL] = s4.z;
    sp[3 * XL] = s4.w;
    axd[b * TG + mm] = d;
  }
  const int nkc = (nb + MC_BC - 1) / MC_BC;
  const int nsub = (row_hi - row_lo + SR - 1) / SR;
  const int nchunk = nsub * nkc;
  auto stage = [&](int c) {
    if (c < nchunk) {
      uint8_t* ws = ring + (c % MT_ST) * CH;
      __half* ds = reinterpret_cast<__half*>(ws + WSZ);
      const int rb = row_lo + (c / nkc) * SR, b0 = (c % nkc) * MC_BC, bc = min(MC_BC, nb - b0);
      for (int i = tid; i < bc * SR * (WB / 16); i += 256) {
        const int piece = i % (WB / 16), r = (i / (WB / 16)) % SR, b = i / (WB / 16) / SR;
        const int n = rb + r;
        if (n < ((N + 31) & ~31)) {
          const size_t e = ((size_t)(n >> 5) * nb + b0 + b) * 32 + (n & 31);
          cp_async16(ws + (b * SR + r) * WB + piece * 16, qs + e * WB + piece * 16);
        }
      }
      for (int i = tid; i < bc * (SR / 2); i += 256) {
        const int rp = i % (SR / 2), b = i / (SR / 2), n = rb + 2 * rp;
        if (n < ((N + 31) & ~31))
          cp_async4(ds + b * SR + 2 * rp, dsc + ((size_t)(n >> 5) * nb + b0 + b) * 32 + (n & 31));
      }
    }
    cp_async_commit();  // (an empty group past the last chunk keeps the group count uniform)
  };
  unsigned long long acc[NT][2];  // (row ra: tokens ta, tb), (row rbw: tokens ta, tb)
#pragma unroll
  for (int j = 0; j < NT; j++) acc[j][0] = acc[j][1] = 0ull;
  const unsigned long long magic2 = f2(-12582912.0f, -12582912.0f);
#pragma unroll
  for (int s = 0; s < MT_ST - 1; s++) stage(s);
  for (int c = 0; c < nchunk; c++) {
    stage(c + MT_ST - 1);
    cp_async_wait_group<MT_ST - 1>();
    __syncthreads();
    const int kc = c % nkc, b0 = kc * MC_BC, bc = min(MC_BC, nb - b0);
    const uint8_t* ws = ring + (c % MT_ST) * CH;
    const __half* ds = reinterpret_cast<const __half*>(ws + WSZ);
    const uint8_t* wa = ws + ra * WB + 4 * t;
    const uint8_t* wbp = ws + rbw * WB + 4 * t;
    const uint8_t* xb = axq + g * xqs + b0 * 32 + 4 * t;
    const int* cs = axs + (b0 * 4 + ln) * XL + 2 * t;
    const float* dxp = axd + b0 * TG + 2 * t;
    const bool own = t == ln;
#pragma unroll
    for (int b = 0; b < MC_BC; b++) {
      if (b < bc) {
        uint32_t a0, a1, a2, a3;
        if (WT == WQ4) {
          const uint32_t u0 = own ? *reinterpret_cast<const uint32_t*>(wa + b * SR * WB) : 0u;
          const uint32_t u1 = own ? *reinterpret_cast<const uint32_t*>(wbp + b * SR * WB) : 0u;
          a0 = u0 & 0x0f0f0f0fu;
          a2 = (u0 >> 4) & 0x0f0f0f0fu;
          a1 = u1 & 0x0f0f0f0fu;
          a3 = (u1 >> 4) & 0x0f0f0f0fu;
        } else {
          a0 = own ? *reinterpret_cast<const uint32_t*>(wa + b * SR * WB) : 0u;
          a2 = own ? *reinterpret_cast<const uint32_t*>(wa + b * SR * WB + 16) : 0u;
          a1 = own ? *reinterpret_cast<const uint32_t*>(wbp + b * SR * WB) : 0u;
          a3 = own ? *reinterpret_cast<const uint32_t*>(wbp + b * SR * WB + 16) : 0u;
        }
        const float dw0 = __half2float(ds[b * SR + ra]), dw1 = __half2float(ds[b * SR + rbw]);
        const unsigned long long w0 = f2(dw0, dw0), w1 = f2(dw1, dw1);
#pragma unroll
        for (int j = 0; j < NT; j++) {
          const uint8_t* xj = xb + 8 * j * xqs + b * 32;
          const uint32_t b0r = *reinterpret_cast<const uint32_t*>(xj), b1r = *reinterpret_cast<const uint32_t*>(xj + 16);
          int c0, c1;
          if (WT == WQ4) {
            const int2 cc = *reinterpret_cast<const int2*>(cs + b * 4 * XL + 8 * j);
            c0 = cc.x;
            c1 = cc.y;
          } else {
            c0 = c1 = MK_MAGIC;
          }
          int d0, d1, d2, d3;
          if (WT == WQ4)
            asm volatile(
                "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                "{%10, %11, %12, %13};"
                : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
                : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0r), "r"(b1r), "r"(c0), "r"(c1), "r"(c0), "r"(c1));
          else
            asm volatile(
                "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                "{%10, %11, %12, %13};"
                : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
                : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0r), "r"(b1r), "r"(c0), "r"(c1), "r"(c0), "r"(c1));
          const unsigned long long dx = *reinterpret_cast<const unsigned long long*>(dxp + b * TG + 8 * j);
          const unsigned long long p01 = f2_add(f2(__int_as_float(d0), __int_as_float(d1)), magic2);
          const unsigned long long p23 = f2_add(f2(__int_as_float(d2), __int_as_float(d3)), magic2);
          const unsigned long long q01 = f2_mul(p01, f2_mul(w0, dx)), q23 = f2_mul(p23, f2_mul(w1, dx));
          // the running sums are added as scalars: a packed multiply feeding a packed add may be fused into one
          // packed fused multiply-add by the compiler (one rounding instead of two), which the reference never does
          acc[j][0] = f2(__fadd_rn(f2_lo(acc[j][0]), f2_lo(q01)), __fadd_rn(f2_hi(acc[j][0]), f2_hi(q01)));
          acc[j][1] = f2(__fadd_rn(f2_lo(acc[j][1]), f2_lo(q23)), __fadd_rn(f2_hi(acc[j][1]), f2_hi(q23)));
        }
      }
    }
    if (kc == nkc - 1) {  // the sub-range's rows are complete: ((l0 + l1) + l2) + l3 across g, g + 1, g + 2, g + 3
      const int rb = row_lo + (c / nkc) * SR;
#pragma unroll
      for (int j = 0; j < NT; j++) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float v0 = (q & 1) ? f2_hi(acc[j][q >> 1]) : f2_lo(acc[j][q >> 1]);
          const float v1 = __shfl_down_sync(0xffffffffu, v0, 4), v2 = __shfl_down_sync(0xffffffffu, v0, 8),
                      v3 = __shfl_down_sync(0xffffffffu, v0, 12);
          const float v = __fadd_rn(__fadd_rn(__fadd_rn(v0, v1), v2), v3);
          const int mm = 8 * j + 2 * t + (q & 1), n = rb + ((q & 2) ? rbw : ra);
          if (ln == 0 && mm < mt && n < row_hi) {
            float* o = y + (size_t)(m0 + mm) * ldy + n;
            if (OP == OP_ADD) *o = __fadd_rn(*o, v);
            else if (OP == OP_BIAS) *o = __fadd_rn(v, bias[n]);
            else *o = v;
          }
        }
        acc[j][0] = acc[j][1] = 0ull;
      }
    }
    __syncthreads();
  }
  cp_async_wait_all();
}

// RoPE on the Q and K heads of each token (pairs (i, i + HD/2), table cos/sin), then K and V appended to the
// cache of (seq, layer) (kernels.c:337-352). grid (x, tokens): the (head, pair) tasks of a token spread over
// gridDim.x CTAs, one task per thread when the grid covers them.
static __global__ void k_rope_kv(const int32_t* __restrict__ prm, float* __restrict__ qkv, int QKV, const float* __restrict__ rope,
                          float* __restrict__ kc, float* __restrict__ vc, int H, int KVH, int HD, int ctx, int layers,
                          int layer) {
  const int m = blockIdx.y;
  const int pos = tok_pos(prm, m), seq = tok_seq(prm, m);
  const int D = H * HD, half = HD / 2;
  float* row = qkv + (size_t)m * QKV;
  const float* cs = rope + (size_t)pos * HD;
  for (int task = blockIdx.x * blockDim.x + threadIdx.x; task < (H + KVH) * half; task += gridDim.x * blockDim.x) {
    const int h = task / half, i = task % half;
    float* v = row + (size_t)h * HD;
    const float c = cs[2 * i], s = cs[2 * i + 1], x0 = v[i], x1 = v[i + half];
    const float r0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    const float r1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
    v[i] = r0;
    v[i + half] = r1;
    if (h >= H) {
      const int kh = h - H;
      const size_t base = ((((size_t)seq * layers + layer) * KVH + kh) * ctx + pos) * HD;
      const float* vs = row + D + KVH * HD + (size_t)kh * HD;
      kc[base + i] = r0;
      kc[base + i + half] = r1;
      vc[base + i] = vs[i];
      vc[base + i + half] = vs[i + half];
    }
  }
}

// Attention for one (head, token), kernels.c:355-377: scores q.k_t in four lanes of HD/4 products each,
// * 1/sqrt(HD); max; e_t = fast_exp(s_t - max); sum in position order; p_t = e_t / sum; o = sum_t p_t v_t in
// position order. Scores and exponentials run one position per thread (16 of a K row's 16-byte loads in flight per
// thread); the two ordered sums run as chains. The V rows of the p.v chains stream through shared memory in chunks of
// AT_VC positions, AT_NST chunks in flight (cp.async; the first ones are requested before the scores), so a chain
// step reads shared memory instead of waiting on a global load.
// grid (H, M), 128 threads, dynamic smem at_smem_bytes<HD>(T_max).
constexpr int AT_VC = 16;
constexpr int AT_NST = 4;
template <int HD>
__host__ __device__ constexpr size_t at_smem_bytes(int ctx) {
  return ((size_t)((ctx + 3) & ~3) + (size_t)AT_NST * AT_VC * HD) * 4;
}
template <int HD>
__global__ void __launch_bounds__(128) k_attention(const int32_t* __restrict__ prm, const float* __restrict__ qkv, int QKV,
                                                   const float* __restrict__ kc, const float* __restrict__ vc, int H,
                                                   int KVH, int ctx, int layers, int layer, float* __restrict__ att,
                                                   int D) {
  extern __shared__ __align__(16) float sc[];
  float* vst = sc + ((ctx + 3) & ~3);  // [AT_NST][AT_VC][HD]
  __shared__ float q_s[HD];
  __shared__ float red[4];
  __shared__ float sum_s;
  const int h = blockIdx.x, m = blockIdx.y, tid = threadIdx.x;
  const int T = tok_pos(prm, m) + 1, seq = tok_seq(prm, m);
  const int kh = h / (H / KVH);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  for (int i = tid; i < HD; i += blockDim.x) q_s[i] = qkv[(size_t)m * QKV + (size_t)h * HD + i];
  const size_t cbase = (((size_t)seq * layers + layer) * KVH + kh) * (size_t)ctx * HD;
  const float* kb = kc + cbase;
  const float* vb = vc + cbase;
  const int nvc = (T + AT_VC - 1) / AT_VC;
  auto stage_v = [&](int c) {  // V rows of chunk c into buffer c % AT_NST (an empty group past the last chunk)
    if (c < nvc) {
      const int t0 = c * AT_VC, tc = min(AT_VC, T - t0);
      float* dst = vst + (c % AT_NST) * AT_VC * HD;
      for (int i = tid; i < tc * (HD / 4); i += blockDim.x) cp_async16(dst + 4 * i, vb + (size_t)t0 * HD + 4 * i);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int c = 0; c < AT_NST - 1; c++) stage_v(c);
  __syncthreads();
  float mx = -1e30f;
  for (int t = tid; t < T; t += blockDim.x) {
    const float4* kr = reinterpret_cast<const float4*>(kb + (size_t)t * HD);
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll 16
    for (int i = 0; i < HD / 4; i++) {
      const float4 k4 = __ldg(kr + i);
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
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  for (int t = tid; t < T; t += blockDim.x) sc[t] = fast_exp_ref(__fsub_rn(sc[t], mx));
  __syncthreads();
  if (tid == 0) {
    float s = 0.f;
#pragma unroll 8
    for (int t = 0; t < T; t++) s = __fadd_rn(s, sc[t]);
    sum_s = s;
  }
  __syncthreads();
  const float sum = sum_s;
  for (int t = tid; t < T; t += blockDim.x) sc[t] = __fdiv_rn(sc[t], sum);
  // o[d] = sum_t p_t v_t[d] in position order (kernels.c:372-375), chain d per thread, V from shared memory
  constexpr int ND = (HD + 127) / 128;
  float o[ND];
#pragma unroll
  for (int k = 0; k < ND; k++) o[k] = 0.f;
  for (int cc = 0; cc < nvc; cc++) {
    const int t0 = cc * AT_VC, tc = min(AT_VC, T - t0);
    cp_async_wait_group<AT_NST - 2>();  // chunk cc has landed (the later ones may still be in flight)
    __syncthreads();                    // (also orders the p writes above before their first use)
    const float* vbuf = vst + (cc % AT_NST) * AT_VC * HD;
#pragma unroll
    for (int k = 0; k < ND; k++) {
      const int d = tid + 128 * k;
      if (d < HD) {
        float acc = o[k];
#pragma unroll 4
        for (int t = 0; t < tc; t++) acc = __fadd_rn(acc, __fmul_rn(sc[t0 + t], vbuf[t * HD + d]));
        o[k] = acc;
      }
    }
    __syncthreads();  // buffer cc % AT_NST is free again
    stage_v(cc + AT_NST - 1);
  }
  cp_async_wait_all();
#pragma unroll
  for (int k = 0; k < ND; k++) {
    const int d = tid + 128 * k;
    if (d < HD) att[(size_t)m * D + (size_t)h * HD + d] = o[k];
  }
}

// Single-token attention, kernels.c:355-377: V rows stream through a shared-memory ring of AP_NST chunks of AP_VC
// positions (cp.async).
constexpr int AP_VC = 128;  // positions per V stage
constexpr int AP_NST = 4;   // V stages in flight

// The attention of the decode step for one token: a cluster of AC_CL CTAs per head. CTA r of head h computes the
// scores of positions [r T / AC_CL, (r + 1) T / AC_CL) and stores each into every CTA of the cluster (distributed
// shared memory), so after the cluster barrier every CTA holds all T scores; each then takes the max, the
// exponentials, the ordered sum and p = e / sum itself, and runs the ordered p.v chains of its HD / AC_CL dims with V
// columns from the cp.async ring requested at the start. The two ordered sums stay single chains (bit-exact); the
// scores need no round trip through global memory.
// QNT: instead of writing the attention output, quantize it (the input of the O matrix, kernels.c:379): the CTAs of
// each 32-value block send their values to the block's first CTA (distributed shared memory), which quantizes it
// with one warp (quant_block_redux: the int8 values, the scale and the lane sums of block (h HD + r HD/8) / 32).
// grid (H x AC_CL), 128 threads, dynamic smem ac_smem_bytes<HD>(ctx).
constexpr int AC_CL = 8;
template <int HD>
__host__ __device__ constexpr size_t ac_smem_bytes(int ctx) {
  return ((size_t)((ctx + 3) & ~3) + (size_t)AP_NST * AP_VC * (HD / AC_CL)) * 4;
}
template <int HD, bool QNT>
__global__ void __cluster_dims__(AC_CL, 1, 1) __launch_bounds__(128)
    k_att_cl(const int32_t* __restrict__ prm, const float* __restrict__ qkv, const float* __restrict__ kc,
             const float* __restrict__ vc, int H, int KVH, int ctx, int layers, int layer, float* __restrict__ att,
             int8_t* __restrict__ xq, float* __restrict__ xd, int4* __restrict__ xs) {
  namespace cg = cooperative_groups;
  constexpr int DS = HD / AC_CL;
  cg::cluster_group cl = cg::this_cluster();
  extern __shared__ __align__(16) float sc[];
  float* vst = sc + ((ctx + 3) & ~3);  // [AP_NST][AP_VC][DS]
  __shared__ float q_s[HD];
  __shared__ float red[4];
  __shared__ float sum_s;
  const int h = blockIdx.x / AC_CL, rk = (int)cl.block_rank(), tid = threadIdx.x;
  const int T = tok_pos(prm, 0) + 1, seq = tok_seq(prm, 0);
  const int kh = h / (H / KVH);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  const size_t cbase = (((size_t)seq * layers + layer) * KVH + kh) * (size_t)ctx * HD;
  const float* kb = kc + cbase;
  const float* vb = vc + cbase + rk * DS;
  const int nvc = (T + AP_VC - 1) / AP_VC;
  auto stage_v = [&](int c) {  // V columns of this CTA's dims for chunk c into stage c % AP_NST
    if (c < nvc) {
      const int t0 = c * AP_VC, tc = min(AP_VC, T - t0);
      float* dst = vst + (c % AP_NST) * AP_VC * DS;
      for (int i = tid; i < tc * (DS / 4); i += blockDim.x) {
        const int t = i / (DS / 4), q = i % (DS / 4);
        cp_async16(dst + t * DS + 4 * q, vb + (size_t)(t0 + t) * HD + 4 * q);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int c = 0; c < AP_NST - 1; c++) stage_v(c);
  for (int i = tid; i < HD; i += blockDim.x) q_s[i] = qkv[(size_t)h * HD + i];
  cl.sync();  // every CTA of the cluster is running (its shared memory can be written) and q_s is in place
  const int t0 = (int)((long long)rk * T / AC_CL), t1 = (int)((long long)(rk + 1) * T / AC_CL);
  for (int t = t0 + tid; t < t1; t += blockDim.x) {
    const float4* kr = reinterpret_cast<const float4*>(kb + (size_t)t * HD);
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll 16
    for (int i = 0; i < HD / 4; i++) {
      const float4 k4 = __ldg(kr + i);
      s0 = __fadd_rn(s0, __fmul_rn(q_s[4 * i], k4.x));
      s1 = __fadd_rn(s1, __fmul_rn(q_s[4 * i + 1], k4.y));
      s2 = __fadd_rn(s2, __fmul_rn(q_s[4 * i + 2], k4.z));
      s3 = __fadd_rn(s3, __fmul_rn(q_s[4 * i + 3], k4.w));
    }
    const float v = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3), scale);
#pragma unroll
    for (int r = 0; r < AC_CL; r++) cl.map_shared_rank(sc, r)[t] = v;
  }
  cl.sync();  // all T scores in every CTA (no shared memory of another CTA is touched after this)
  float mx = -1e30f;
  for (int t = tid; t < T; t += blockDim.x) mx = fmaxf(mx, sc[t]);
  mx = warp_max(mx);
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  for (int t = tid; t < T; t += blockDim.x) sc[t] = fast_exp_ref(__fsub_rn(sc[t], mx));
  __syncthreads();
  if (tid == 0) {  // sum in position order
    float s = 0.f;
    const float4* p4 = reinterpret_cast<const float4*>(sc);
#pragma unroll 8
    for (int j = 0; j < T / 4; j++) {
      const float4 a = p4[j];
      s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, a.x), a.y), a.z), a.w);
    }
    for (int t = T & ~3; t < T; t++) s = __fadd_rn(s, sc[t]);
    sum_s = s;
  }
  __syncthreads();
  const float sum = sum_s;
  for (int t = tid; t < T; t += blockDim.x) sc[t] = __fdiv_rn(sc[t], sum);
  float acc = 0.f;
  for (int cc = 0; cc < nvc; cc++) {
    const int c0 = cc * AP_VC, tc = min(AP_VC, T - c0);
    cp_async_wait_group<AP_NST - 2>();  // chunk cc has landed
    __syncthreads();                    // (also orders the p writes before their first use)
    if (tid < DS) {
      const float* vbuf = vst + (cc % AP_NST) * AP_VC * DS + tid;
      const float* pp = sc + c0;
#pragma unroll 8
      for (int t = 0; t < tc; t++) acc = __fadd_rn(acc, __fmul_rn(pp[t], vbuf[t * DS]));
    }
    __syncthreads();  // stage cc % AP_NST is free again
    stage_v(cc + AP_NST - 1);
  }
  cp_async_wait_all();
  if (!QNT) {
    if (tid < DS) att[(size_t)h * HD + rk * DS + tid] = acc;
    return;
  }
  __shared__ float ob[32];
  constexpr int PER = 32 / DS;  // CTAs per 32-value block
  const int lead = rk - rk % PER;
  if (tid < DS) cl.map_shared_rank(ob, lead)[(rk % PER) * DS + tid] = acc;
  cl.sync();
  if (rk % PER == 0 && tid < 32) {
    const int b = (h * HD + rk * DS) / 32;
    quant_block_redux(ob[tid], tid, xq + (size_t)b * 32, xd + b, xs + b, nullptr);
  }
}

// The same attention for the G = H / KVH query heads that share kv head kh, one CTA per (kv head, token): each K row
// is loaded once for the G heads (scores one position per thread), the G softmax sums run as G chains in position
// order, and the G * HD ordered p.v chains advance together over chunks of AV_VC V rows, double-buffered in shared
// memory with cp.async (the first two chunks are requested before the scores, so they arrive meanwhile).
// grid (KVH, M), 256 threads; dynamic smem: attg_smem_bytes(G, ctx).
constexpr int AV_VC = 32;
template <int HD>
__host__ __device__ constexpr size_t attg_smem_bytes(int G, int ctx) {
  return ((size_t)G * HD + (size_t)G * ((ctx + 3) & ~3) + (size_t)2 * AV_VC * HD + 8 * 16 + 16) * 4;
}
template <int HD>
__global__ void __launch_bounds__(256) k_attention_gqa(const int32_t* __restrict__ prm, const float* __restrict__ qkv,
                                                       int QKV, const float* __restrict__ kc,
                                                       const float* __restrict__ vc, int H, int KVH, int ctx,
                                                       int layers, int layer, float* __restrict__ att, int D) {
  extern __shared__ __align__(16) float asm_[];
  const int kh = blockIdx.x, m = blockIdx.y, tid = threadIdx.x, G = H / KVH;
  const int ctxp = (ctx + 3) & ~3;
  float* q_s = asm_;                     // [G][HD]
  float* sc = q_s + G * HD;              // [G][ctxp]
  float* vst = sc + (size_t)G * ctxp;    // [2][AV_VC][HD]
  float* red = vst + 2 * AV_VC * HD;     // [8 warps][<= 16 heads]
  float* sum_s = red + 8 * 16;           // [G]
  const int T = tok_pos(prm, m) + 1, seq = tok_seq(prm, m);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  for (int i = tid; i < G * HD; i += 256) q_s[i] = qkv[(size_t)m * QKV + (size_t)kh * G * HD + i];
  __syncthreads();
  const size_t cbase = (((size_t)seq * layers + layer) * KVH + kh) * (size_t)ctx * HD;
  const float* kb = kc + cbase;
  const float* vb = vc + cbase;
  const int nvc = (T + AV_VC - 1) / AV_VC;
  auto stage_v = [&](int c) {  // V rows of chunk c into buffer c & 1 (an empty group past the last chunk)
    if (c < nvc) {
      const int t0 = c * AV_VC, tc = min(AV_VC, T - t0);
      float* dst = vst + (c & 1) * AV_VC * HD;
      for (int i = tid; i < tc * (HD / 4); i += 256) cp_async16(dst + 4 * i, vb + (size_t)t0 * HD + 4 * i);
    }
    cp_async_commit();
  };
  stage_v(0);
  stage_v(1);
  float mx[16];
#pragma unroll
  for (int g = 0; g < 16; g++) mx[g] = -1e30f;
  for (int t = tid; t < T; t += 256) {
    float4 kr[HD / 4];
    const float4* kp = reinterpret_cast<const float4*>(kb + (size_t)t * HD);
#pragma unroll
    for (int i = 0; i < HD / 4; i++) kr[i] = __ldg(kp + i);
#pragma unroll
    for (int g = 0; g < 16; g++) {
      if (g < G) {
        const float* qg = q_s + g * HD;
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int i = 0; i < HD / 4; i++) {
          s0 = __fadd_rn(s0, __fmul_rn(qg[4 * i], kr[i].x));
          s1 = __fadd_rn(s1, __fmul_rn(qg[4 * i + 1], kr[i].y));
          s2 = __fadd_rn(s2, __fmul_rn(qg[4 * i + 2], kr[i].z));
          s3 = __fadd_rn(s3, __fmul_rn(qg[4 * i + 3], kr[i].w));
        }
        const float v = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(s0, s1), s2), s3), scale);
        sc[g * ctxp + t] = v;
        mx[g] = fmaxf(mx[g], v);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < 16; g++) {
    if (g < G) {
      const float w = warp_max(mx[g]);
      if ((tid & 31) == 0) red[(tid >> 5) * 16 + g] = w;
    }
  }
  __syncthreads();
  for (int i = tid; i < G * T; i += 256) {
    const int g = i / T, t = i - g * T;
    float w = red[g];
    for (int k = 1; k < 8; k++) w = fmaxf(w, red[k * 16 + g]);
    sc[g * ctxp + t] = fast_exp_ref(__fsub_rn(sc[g * ctxp + t], w));
  }
  __syncthreads();
  if (tid < G) {  // softmax sums in position order (kernels.c:368)
    const float* e = sc + tid * ctxp;
    float s = 0.f;
#pragma unroll 8
    for (int t = 0; t < T; t++) s = __fadd_rn(s, e[t]);
    sum_s[tid] = s;
  }
  __syncthreads();
  for (int i = tid; i < G * T; i += 256) {
    const int g = i / T, t = i - g * T;
    sc[g * ctxp + t] = __fdiv_rn(sc[g * ctxp + t], sum_s[g]);
  }
  // o[g][d] = sum_t p[g][t] v[t][d] in position order (kernels.c:372-375); chains c = tid, tid + 256, ...
  constexpr int NC = 4;  // chains per thread (G * HD <= 1024)
  float o[NC];
#pragma unroll
  for (int k = 0; k < NC; k++) o[k] = 0.f;
  for (int cc = 0; cc < nvc; cc++) {
    const int t0 = cc * AV_VC, tc = min(AV_VC, T - t0);
    cp_async_wait_group<1>();  // chunk cc has landed (chunk cc + 1 may still be in flight)
    __syncthreads();           // (also orders the p writes above before their first use)
    const float* vbuf = vst + (cc & 1) * AV_VC * HD;
#pragma unroll
    for (int k = 0; k < NC; k++) {
      const int c = tid + 256 * k;
      if (c < G * HD) {
        const int g = c / HD, d = c - g * HD;
        const float* p = sc + g * ctxp + t0;
        float acc = o[k];
        for (int t = 0; t < tc; t++) acc = __fadd_rn(acc, __fmul_rn(p[t], vbuf[t * HD + d]));
        o[k] = acc;
      }
    }
    __syncthreads();  // buffer cc & 1 is free again
    stage_v(cc + 2);
  }
  cp_async_wait_all();
#pragma unroll
  for (int k = 0; k < NC; k++) {
    const int c = tid + 256 * k;
    if (c < G * HD) att[(size_t)m * D + (size_t)kh * G * HD + c] = o[k];
  }
}

// Greedy argmax, stage 1: per-CTA (value, index) with ties to the lowest index (cpu-worker.js:156-157 scans
// with a strict >).
__device__ __forceinline__ void amax_merge(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}
static __global__ void k_argmax1(const float* __restrict__ logits, int V, float* __restrict__ pv, int* __restrict__ pi) {
  __shared__ float sv[32];
  __shared__ int si[32];
  logits += (size_t)blockIdx.y * V;  // row blockIdx.y (one row per token of a batched step)
  pv += (size_t)blockIdx.y * gridDim.x;
  pi += (size_t)blockIdx.y * gridDim.x;
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) amax_merge(v, idx, logits[i], i);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    amax_merge(v, idx, v2, i2);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { sv[warp] = v; si[warp] = idx; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) amax_merge(v, idx, sv[w], si[w]);
    pv[blockIdx.x] = v;
    pi[blockIdx.x] = idx;
  }
}

// stage 2: one warp merges the partials and stores the token. Like the WebGPU backend (webgpu.js:391), the token
// stays on the device: it is logged at tokens[seq][pos0 + M] and the pass parameters are advanced to
// (pos0 + M, one token, that id), so the next decode step can start without the host.
static __global__ void k_argmax2(const float* __restrict__ pv, const int* __restrict__ pi, int np, int32_t* __restrict__ prm,
                          int32_t* __restrict__ toklog, int ctx, int32_t* __restrict__ out) {
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < np; i += 32) amax_merge(v, idx, pv[i], pi[i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    amax_merge(v, idx, v2, i2);
  }
  if (threadIdx.x == 0) {
    const int tok = idx == 0x7fffffff ? 0 : idx;
    const int next_pos = prm[P_POS0] + prm[P_M];
    *out = tok;
    if (next_pos <= ctx) toklog[(size_t)prm[P_SEQ] * (ctx + 1) + next_pos] = tok;
    prm[P_POS0] = next_pos;
    prm[P_M] = 1;
    prm[P_IDS] = tok;
  }
}

// stage 2 of a batched decode step: block m merges row m's partials; the token of sequence seq_m (at position pos_m)
// goes to out[m], is logged at tokens[seq_m][pos_m + 1] and becomes token m of the next step at pos_m + 1 (so
// steps can be chained on the device, as k_argmax2 does for one sequence).
static __global__ void k_argmax2_batch(const float* __restrict__ pv, const int* __restrict__ pi, int np,
                                int32_t* __restrict__ prm, int32_t* __restrict__ toklog, int ctx,
                                int32_t* __restrict__ out) {
  const int m = blockIdx.x;
  pv += (size_t)m * np;
  pi += (size_t)m * np;
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < np; i += 32) amax_merge(v, idx, pv[i], pi[i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
    amax_merge(v, idx, v2, i2);
  }
  if (threadIdx.x == 0) {
    const int tok = idx == 0x7fffffff ? 0 : idx;
    const int next_pos = tok_pos(prm, m) + 1;
    out[m] = tok;
    if (next_pos <= ctx) toklog[(size_t)tok_seq(prm, m) * (ctx + 1) + next_pos] = tok;
    prm[P_IDS + m] = tok;
    prm[P_IDS + P_CAP + m] = next_pos;
  }
}

}  // namespace h2
