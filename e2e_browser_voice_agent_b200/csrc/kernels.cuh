// Device kernels of the H2 Qwen2 token loop for sm_100a.
//
// Data layout in HBM (all per engine):
//   Q4_0 matrix [N][K]: values [N][K/32][16] bytes (byte j: low nibble = element j, high = element j+16, as in
//                       GGUF), then scales [N][K/32] fp16 (the GGUF bits; fp16 -> fp32 is exact).
//   Q8_0 matrix [N][K]: values [N][K/32][32] int8, then scales [N][K/32] fp16.
//   activations: x [M][D] f32 residual stream; qkv [M][D + 2*KVH*HD]; att [M][D]; gu [M][2F];
//   int8 activations xq [M][K] with per-32 scales xd [M][K/32] f32 and integer sums xs [M][K/32];
//   KV cache [seq][layer][kv_head][ctx][HD] f32 (the reference's dtype and order, kernels.c:347-348).
//
// Arithmetic follows the reference CPU path (h2-own-inference-engine/engine/kernels.c): matrix inputs are
// quantized to int8 per 32 values with round-to-nearest-even of x * (1 / (amax / 127)) (kernels.c:90-114),
// every block dot product is an exact integer, scaled by f32(dw * dx) and accumulated in f32 (kernels.c:121-139);
// RoPE, SwiGLU, softmax use the reference's own fast_exp (kernels.c:69-78) and its operation order, with IEEE
// round-to-nearest intrinsics so that nvcc does not contract them into fused multiply-adds. Only the order of
// floating-point sums (rmsnorm, matvec rows, attention) differs from the CPU's lane order.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace h2 {

// device-resident parameters of one pass, written by the host with one copy before each pass
enum { P_POS0 = 0, P_M = 1, P_SEQ = 2, P_IDS = 4 };

constexpr int ATT_CH = 64;   // positions per attention split
constexpr int MAXG = 8;      // query heads per KV head handled by one attention CTA

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

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Quantize the 32 values held one per lane (kernels.c:90-114): d = amax / 127, q = nearest-even(x * (1/d)).
// Lane 0 stores the scale and the integer sum of the block (the int8 values the dot products use).
__device__ __forceinline__ void quant_block_warp(float v, int lane, int8_t* q, float* d, int* s) {
  float amax = warp_max(fabsf(v));
  float dd = __fdiv_rn(amax, 127.0f);
  float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
  int qi = __float2int_rn(__fmul_rn(v, id));
  qi = max(-128, min(127, qi));
  q[lane] = (int8_t)qi;
  int sum = warp_sum_i(qi);
  if (lane == 0) { *d = dd; *s = sum; }
}

// x[m] = dequant(embedding row ids[m]) (kernels.c:313-322)
__global__ void k_embed(const int32_t* __restrict__ prm, const uint8_t* __restrict__ qs, const __half* __restrict__ dsc,
                        int D, float* __restrict__ x) {
  const int m = blockIdx.x;
  const int t = prm[P_IDS + m];
  const int nb = D / 32;
  const uint8_t* q = qs + (size_t)t * nb * 16;
  const __half* d = dsc + (size_t)t * nb;
  float* xr = x + (size_t)m * D;
  for (int i = threadIdx.x; i < D / 2; i += blockDim.x) {
    int blk = i >> 4, j = i & 15;
    uint8_t b = q[blk * 16 + j];
    float s = __half2float(d[blk]);
    xr[32 * blk + j] = __fmul_rn((float)((b & 15) - 8), s);
    xr[32 * blk + 16 + j] = __fmul_rn((float)((b >> 4) - 8), s);
  }
}

// RMSNorm (kernels.c:80-86) of row `row` of x, then int8 quantization (kernels.c:90-114) into slot blockIdx.x.
// One CTA per token; blockDim a multiple of 32.
__global__ void k_norm_quant(const float* __restrict__ x, int row0, const float* __restrict__ w, int D, float eps,
                             int8_t* __restrict__ xq, float* __restrict__ xd, int* __restrict__ xs) {
  __shared__ float red[32];
  __shared__ float rs;
  const int slot = blockIdx.x;
  const float* xr = x + (size_t)(row0 + slot) * D;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) { float v = xr[i]; ss = __fadd_rn(ss, __fmul_rn(v, v)); }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < nw; i++) t += red[i];
    rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)D), eps)));
  }
  __syncthreads();
  const float r = rs;
  const int nb = D / 32;
  for (int b = warp; b < nb; b += nw) {
    int i = b * 32 + lane;
    float v = __fmul_rn(__fmul_rn(xr[i], r), w[i]);
    quant_block_warp(v, lane, xq + (size_t)slot * D + b * 32, xd + (size_t)slot * nb + b, xs + (size_t)slot * nb + b);
  }
}

// int8 quantization of M rows of length K (the attention output before the O projection, kernels.c:379):
// one warp per 32-value block.
__global__ void k_quant(const float* __restrict__ x, int K, int M, int8_t* __restrict__ xq, float* __restrict__ xd,
                        int* __restrict__ xs) {
  const int nb = K / 32;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (gw >= M * nb) return;
  const int m = gw / nb, b = gw % nb;
  float v = x[(size_t)m * K + b * 32 + lane];
  quant_block_warp(v, lane, xq + (size_t)m * K + b * 32, xd + (size_t)m * nb + b, xs + (size_t)m * nb + b);
}

// act = silu(gate) * up, then int8 quantization (kernels.c:393-397); one warp per 32-value block of act.
__global__ void k_swiglu_quant(const float* __restrict__ gu, int F, int M, int8_t* __restrict__ xq,
                               float* __restrict__ xd, int* __restrict__ xs) {
  const int nb = F / 32;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (gw >= M * nb) return;
  const int m = gw / nb, b = gw % nb;
  const float* g = gu + (size_t)m * 2 * F;
  float gt = g[b * 32 + lane], up = g[F + b * 32 + lane];
  float v = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, fast_exp_ref(-gt))), up);
  quant_block_warp(v, lane, xq + (size_t)m * F + b * 32, xd + (size_t)m * nb + b, xs + (size_t)m * nb + b);
}

enum { OP_STORE = 0, OP_BIAS = 1, OP_ADD = 2 };

// Exact integer dot of one Q4_0 block (16 bytes of nibbles) with 32 int8 activations: sum((q - 8) * x) computed
// as sum(q * x) - 8 * sum(x). Nibble values 0..15 are the same as signed bytes, so signed dp4a applies.
__device__ __forceinline__ int q4_block_dot(uint4 w, int4 x0, int4 x1, int xsum) {
  int p = 0;
  p = __dp4a((int)(w.x & 0x0f0f0f0fu), x0.x, p);
  p = __dp4a((int)(w.y & 0x0f0f0f0fu), x0.y, p);
  p = __dp4a((int)(w.z & 0x0f0f0f0fu), x0.z, p);
  p = __dp4a((int)(w.w & 0x0f0f0f0fu), x0.w, p);
  p = __dp4a((int)((w.x >> 4) & 0x0f0f0f0fu), x1.x, p);
  p = __dp4a((int)((w.y >> 4) & 0x0f0f0f0fu), x1.y, p);
  p = __dp4a((int)((w.z >> 4) & 0x0f0f0f0fu), x1.z, p);
  p = __dp4a((int)((w.w >> 4) & 0x0f0f0f0fu), x1.w, p);
  return p - 8 * xsum;
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {  // weights are read once per pass: no L1 allocation
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// y[m][n] (op)= sum_b f32(int dot_b) * (dw * dx), for R rows per warp and up to MAXM tokens (matmul_q4,
// kernels.c:200-273). Lanes stride over the K/32 blocks of a row with 16-byte loads (512 contiguous bytes per
// warp and row); lane partial sums are reduced with shuffles.
template <int R, int MAXM, int OP>
__global__ void __launch_bounds__(128) k_matvec_q4(const uint8_t* __restrict__ qs, const __half* __restrict__ dsc,
                                                   int N, int K, const int8_t* __restrict__ xq,
                                                   const float* __restrict__ xd, const int* __restrict__ xs, int M,
                                                   float* __restrict__ y, int ldy, const float* __restrict__ bias) {
  const int nb = K / 32;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int row0 = warp * R;
  if (row0 >= N) return;
  float acc[R][MAXM];
#pragma unroll
  for (int r = 0; r < R; r++)
#pragma unroll
    for (int m = 0; m < MAXM; m++) acc[r][m] = 0.f;
  for (int b = lane; b < nb; b += 32) {
    uint4 w[R];
    float dw[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
      int n = min(row0 + r, N - 1);
      w[r] = ldg_stream(qs + ((size_t)n * nb + b) * 16);
      dw[r] = __half2float(dsc[(size_t)n * nb + b]);
    }
#pragma unroll
    for (int m = 0; m < MAXM; m++) {
      if (m < M) {
        const int4* xp = reinterpret_cast<const int4*>(xq + (size_t)m * K + b * 32);
        int4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
        float dx = __ldg(xd + (size_t)m * nb + b);
        int sx = __ldg(xs + (size_t)m * nb + b);
#pragma unroll
        for (int r = 0; r < R; r++) {
          int p = q4_block_dot(w[r], x0, x1, sx);
          acc[r][m] = __fadd_rn(acc[r][m], __fmul_rn((float)p, __fmul_rn(dw[r], dx)));
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; r++)
#pragma unroll
    for (int m = 0; m < MAXM; m++) acc[r][m] = warp_sum(acc[r][m]);
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < R; r++) {
      const int n = row0 + r;
      if (n >= N) break;
#pragma unroll
      for (int m = 0; m < MAXM; m++) {
        if (m < M) {
          float* o = y + (size_t)m * ldy + n;
          if (OP == OP_ADD) *o = __fadd_rn(*o, acc[r][m]);
          else if (OP == OP_BIAS) *o = __fadd_rn(acc[r][m], bias[n]);
          else *o = acc[r][m];
        }
      }
    }
  }
}

// logits[n] = sum_b f32(int dot_b) * (dw * dx) for a Q8_0 output matrix (dot_q8_q8, kernels.c:157-170).
template <int R>
__global__ void __launch_bounds__(128) k_matvec_q8(const int8_t* __restrict__ qs, const __half* __restrict__ dsc, int N,
                                                   int K, const int8_t* __restrict__ xq, const float* __restrict__ xd,
                                                   float* __restrict__ y) {
  const int nb = K / 32;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int row0 = warp * R;
  if (row0 >= N) return;
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; r++) acc[r] = 0.f;
  for (int b = lane; b < nb; b += 32) {
    const int4* xp = reinterpret_cast<const int4*>(xq + b * 32);
    int4 x0 = __ldg(xp), x1 = __ldg(xp + 1);
    float dx = __ldg(xd + b);
#pragma unroll
    for (int r = 0; r < R; r++) {
      int n = min(row0 + r, N - 1);
      const int8_t* wp = qs + ((size_t)n * nb + b) * 32;
      uint4 w0 = ldg_stream(wp), w1 = ldg_stream(wp + 16);
      int p = 0;
      p = __dp4a((int)w0.x, x0.x, p); p = __dp4a((int)w0.y, x0.y, p);
      p = __dp4a((int)w0.z, x0.z, p); p = __dp4a((int)w0.w, x0.w, p);
      p = __dp4a((int)w1.x, x1.x, p); p = __dp4a((int)w1.y, x1.y, p);
      p = __dp4a((int)w1.z, x1.z, p); p = __dp4a((int)w1.w, x1.w, p);
      acc[r] = __fadd_rn(acc[r], __fmul_rn((float)p, __fmul_rn(__half2float(dsc[(size_t)n * nb + b]), dx)));
    }
  }
#pragma unroll
  for (int r = 0; r < R; r++) acc[r] = warp_sum(acc[r]);
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < R; r++)
      if (row0 + r < N) y[row0 + r] = acc[r];
  }
}

// RoPE on the Q and K heads of each token (pairs (i, i + HD/2), table cos/sin), then K and V appended to the
// cache of (seq, layer) (kernels.c:337-352). One CTA per token.
__global__ void k_rope_kv(const int32_t* __restrict__ prm, float* __restrict__ qkv, int QKV, const float* __restrict__ rope,
                          float* __restrict__ kc, float* __restrict__ vc, int H, int KVH, int HD, int ctx, int layers,
                          int layer) {
  const int m = blockIdx.x;
  const int pos = prm[P_POS0] + m, seq = prm[P_SEQ];
  const int D = H * HD, half = HD / 2;
  float* row = qkv + (size_t)m * QKV;
  const float* cs = rope + (size_t)pos * HD;
  for (int task = threadIdx.x; task < (H + KVH) * half; task += blockDim.x) {
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

// Split-K flash decode (kernels.c:355-377 computes the same softmax(q.K^T / sqrt(HD)) V per (token, head)).
// grid (split, kv_head, token): one CTA takes ATT_CH cached positions of one KV head for all G = H/KVH query
// heads that share it, and writes unnormalised partials (o[HD], max, sum) per head and split.
template <int HD>
__global__ void __launch_bounds__(128) k_attn_split(const int32_t* __restrict__ prm, const float* __restrict__ qkv, int QKV,
                                                    const float* __restrict__ kc, const float* __restrict__ vc, int H,
                                                    int KVH, int ctx, int layers, int layer, float* __restrict__ part,
                                                    int nsplit_max) {
  const int split = blockIdx.x, kh = blockIdx.y, m = blockIdx.z;
  const int pos0 = prm[P_POS0], seq = prm[P_SEQ];
  const int T = pos0 + m + 1;
  const int t0 = split * ATT_CH;
  if (t0 >= T) return;
  const int n = min(ATT_CH, T - t0);
  const int G = H / KVH;
  __shared__ float q_s[MAXG][HD];
  __shared__ float s_s[MAXG][ATT_CH];
  __shared__ float mx_s[MAXG], l_s[MAXG];
  __shared__ float o_s[2][MAXG][HD];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  const float* qrow = qkv + (size_t)m * QKV + (size_t)kh * G * HD;
  for (int i = tid; i < G * HD; i += blockDim.x) q_s[i / HD][i % HD] = qrow[i];
  __syncthreads();
  const size_t cbase = (((size_t)seq * layers + layer) * KVH + kh) * (size_t)ctx * HD;
  const float* kb = kc + cbase;
  const float* vb = vc + cbase;
  // scores: thread = (position p, head parity)
  {
    const int p = tid % ATT_CH, g0 = tid / ATT_CH;
    if (p < n) {
      const float4* kr = reinterpret_cast<const float4*>(kb + (size_t)(t0 + p) * HD);
      float dots[MAXG];
#pragma unroll
      for (int g = 0; g < MAXG; g++) dots[g] = 0.f;
#pragma unroll 4
      for (int i = 0; i < HD / 4; i++) {
        float4 k4 = __ldg(kr + i);
#pragma unroll
        for (int g = 0; g < MAXG; g++) {
          if (g < G && (g & 1) == g0) {
            dots[g] = __fadd_rn(dots[g], __fmul_rn(q_s[g][4 * i], k4.x));
            dots[g] = __fadd_rn(dots[g], __fmul_rn(q_s[g][4 * i + 1], k4.y));
            dots[g] = __fadd_rn(dots[g], __fmul_rn(q_s[g][4 * i + 2], k4.z));
            dots[g] = __fadd_rn(dots[g], __fmul_rn(q_s[g][4 * i + 3], k4.w));
          }
        }
      }
#pragma unroll
      for (int g = 0; g < MAXG; g++)
        if (g < G && (g & 1) == g0) s_s[g][p] = __fmul_rn(dots[g], scale);
    }
  }
  __syncthreads();
  // per head: max and sum of exp over this split's positions
  for (int g = warp; g < G; g += 4) {
    float mx = -1e30f;
    for (int p = lane; p < n; p += 32) mx = fmaxf(mx, s_s[g][p]);
    mx = warp_max(mx);
    float l = 0.f;
    for (int p = lane; p < n; p += 32) {
      float e = fast_exp_ref(__fsub_rn(s_s[g][p], mx));
      s_s[g][p] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) { mx_s[g] = mx; l_s[g] = l; }
  }
  __syncthreads();
  // o[g][d] = sum_p e[g][p] * v[p][d]; thread = (dim d, half of the positions)
  {
    const int halves = 128 / HD;  // 2 for HD=64, 1 for HD=128
    const int d = tid % HD, hf = tid / HD;
    float o[MAXG];
#pragma unroll
    for (int g = 0; g < MAXG; g++) o[g] = 0.f;
    for (int p = hf; p < n; p += halves) {
      float v = __ldg(vb + (size_t)(t0 + p) * HD + d);
#pragma unroll
      for (int g = 0; g < MAXG; g++)
        if (g < G) o[g] = __fadd_rn(o[g], __fmul_rn(s_s[g][p], v));
    }
#pragma unroll
    for (int g = 0; g < MAXG; g++)
      if (g < G) o_s[hf][g][d] = o[g];
  }
  __syncthreads();
  for (int i = tid; i < G * HD; i += blockDim.x) {
    const int g = i / HD, d = i % HD;
    float v = o_s[0][g][d];
    if (128 / HD > 1) v = __fadd_rn(v, o_s[1][g][d]);
    const int h = kh * G + g;
    float* dst = part + (((size_t)m * H + h) * nsplit_max + split) * (HD + 2);
    dst[d] = v;
    if (d == 0) { dst[HD] = mx_s[g]; dst[HD + 1] = l_s[g]; }
  }
}

// Merge the splits of each (token, head): att = sum_s o_s e^(m_s - m) / sum_s l_s e^(m_s - m).
__global__ void k_attn_combine(const int32_t* __restrict__ prm, const float* __restrict__ part, int H, int HD,
                               int nsplit_max, float* __restrict__ att, int D) {
  const int h = blockIdx.x, m = blockIdx.y, d = threadIdx.x;
  const int T = prm[P_POS0] + m + 1;
  const int ns = (T + ATT_CH - 1) / ATT_CH;
  const float* src = part + ((size_t)m * H + h) * nsplit_max * (HD + 2);
  float mx = -1e30f;
  for (int s = 0; s < ns; s++) mx = fmaxf(mx, src[s * (HD + 2) + HD]);
  float l = 0.f, o = 0.f;
  for (int s = 0; s < ns; s++) {
    const float* e = src + s * (HD + 2);
    float f = fast_exp_ref(__fsub_rn(e[HD], mx));
    l = __fadd_rn(l, __fmul_rn(e[HD + 1], f));
    if (d < HD) o = __fadd_rn(o, __fmul_rn(e[d], f));
  }
  if (d < HD) att[(size_t)m * D + h * HD + d] = __fdiv_rn(o, l);
}

// Greedy argmax, stage 1: per-CTA (value, index) with ties to the lowest index (cpu-worker.js:156-157 scans
// with a strict >).
__device__ __forceinline__ void amax_merge(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}
__global__ void k_argmax1(const float* __restrict__ logits, int V, float* __restrict__ pv, int* __restrict__ pi) {
  __shared__ float sv[32];
  __shared__ int si[32];
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) amax_merge(v, idx, logits[i], i);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
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
__global__ void k_argmax2(const float* __restrict__ pv, const int* __restrict__ pi, int np, int32_t* __restrict__ prm,
                          int32_t* __restrict__ toklog, int ctx, int32_t* __restrict__ out) {
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < np; i += 32) amax_merge(v, idx, pv[i], pi[i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    float v2 = __shfl_xor_sync(0xffffffffu, v, o);
    int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
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

}  // namespace h2
