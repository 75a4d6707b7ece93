// Attention of a prompt pass: M tokens of one sequence at positions pos0 .. pos0+M-1, token m attending to positions
// 0 .. pos0+m (kernels.c:355-377, for every token exactly the arithmetic of the one-token form). The per-token form
// (k_attention_gqa: one CTA per (kv head, token), the two ordered sums in a few threads) keeps the SMs busy only at
// small contexts; here the pass runs as three kernels over a score buffer S in global memory, so that the scores and
// the p.v products are register-tiled over many tokens and heads at once. Rows of each kv head kh: r = m G + g
// (token m, query head kh G + g, G = H / KVH); row r attends to T_r = pos0 + r / G + 1 positions.
//
//  k_pf_scores  S[kh][r][t] = ((((s0 + s1) + s2) + s3) * (1 / sqrt(HD)) for t < T_r, where lane l sums q[4i+l] k_t[4i+l]
//               in order i = 0 .. HD/4-1 (products and sums rounded separately, no fused multiply-add; the products
//               two at a time as packed f32x2 multiplies); 64 rows x 64 positions per CTA, 4 x 4 (row, position)
//               pairs per thread, four lane sums each; also each row's maximum over the CTA's 64 positions (PM).
//  k_pf_soft    max over t < T_r (from the partial maxima: max is order-free); e_t = fast_exp(s_t - max) written
//               back over s_t; sum_t e_t in position order. 16 rows per CTA: seven warps compute the exponentials of
//               a 64-position chunk into shared memory (the next chunk's scores already loading) while 16 lanes of
//               warp 0 run the rows' ordered sums over the previous chunk (lane j = row j).
//  k_pf_pv      o[r][d] = sum_t (e_t / sum) v_t[d] in position order; 2 rows x 4 dims per thread, V tiles of 64
//               positions double-buffered through cp.async, the next tile's e values loaded while this one is used;
//               p staged twice per position so that packed multiplies take (p, p) x (v_d, v_d+1) straight from it.
//
// Exactness: every value is formed by the same operations in the same order as the reference's per-token loop;
// only which thread computes it changes. Positions t >= T_r of a row are never added to its sums (the rows of one
// CTA differ in length by a few positions: those tiles take a per-row predicated path).
#pragma once
#include "kernels.cuh"

namespace h2 {

constexpr int PF_RB = 64;  // score rows per CTA
constexpr int PF_TB = 64;  // score positions per CTA
constexpr int PF_SR = 16;  // softmax rows per CTA
constexpr int PF_SC = 64;  // softmax positions per chunk
constexpr int PF_VT = 64;  // p.v positions per V tile

template <int HD>
__host__ __device__ constexpr int pf_scores_smem() { return (PF_RB + PF_TB) * (HD + 4) * 4; }
template <int HD>
__host__ __device__ constexpr int pf_pv_rows() { return 1024 / HD; }  // 128 threads x 2 rows x 4 dims
template <int HD>
__host__ __device__ constexpr int pf_pv_smem() { return (2 * PF_VT * HD + 2 * pf_pv_rows<HD>() * (2 * PF_VT + 4)) * 4; }
// partial maxima per row: one per PF_TB positions of the context
__host__ __device__ constexpr int pf_pm_pitch(int ctx) { return (ctx + PF_TB - 1) / PF_TB; }

// grid (ceil((pos0 + M) / PF_TB), ceil(G M / PF_RB), KVH), 256 threads, dynamic smem pf_scores_smem<HD>().
// q: the pass's qkv rows (row stride QKV; query head h at h HD); S: [KVH][G M][ldS]; PM: [KVH][G M][ldP], entry b
// the row's maximum over positions [64 b, 64 b + 64) below its length.
template <int HD>
__global__ void __launch_bounds__(256) k_pf_scores(const float* __restrict__ qkv, int QKV, const float* __restrict__ kc,
                                                   int H, int KVH, int ctx, int layers, int layer, int seq, int pos0,
                                                   int M, float* __restrict__ S, int ldS, float* __restrict__ PM,
                                                   int ldP) {
  constexpr int LD = HD + 4;  // padded rows: the 16 positions a warp reads fall in distinct banks
  extern __shared__ __align__(16) float pfs[];
  float* qs = pfs;              // [PF_RB][LD]
  float* ks = pfs + PF_RB * LD;  // [PF_TB][LD]
  const int kh = blockIdx.z, G = H / KVH, R = G * M, tid = threadIdx.x;
  const int r0 = blockIdx.y * PF_RB, t0 = blockIdx.x * PF_TB;
  const int Tb = pos0 + (min(R, r0 + PF_RB) - 1) / G + 1;  // positions the block's longest row attends to
  if (r0 >= R || t0 >= Tb) return;
  for (int i = tid; i < PF_RB * (HD / 4); i += 256) {
    const int r = i / (HD / 4), c = i % (HD / 4), rr = r0 + r;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (rr < R)
      v = *reinterpret_cast<const float4*>(qkv + (size_t)(rr / G) * QKV + (size_t)(kh * G + rr % G) * HD + 4 * c);
    *reinterpret_cast<float4*>(qs + r * LD + 4 * c) = v;
  }
  const float* kb = kc + (((size_t)seq * layers + layer) * KVH + kh) * (size_t)ctx * HD;
  for (int i = tid; i < PF_TB * (HD / 4); i += 256) {
    const int r = i / (HD / 4), c = i % (HD / 4), t = t0 + r;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < Tb) v = __ldg(reinterpret_cast<const float4*>(kb + (size_t)t * HD + 4 * c));
    *reinterpret_cast<float4*>(ks + r * LD + 4 * c) = v;
  }
  __syncthreads();
  const int tr = tid >> 4, tc = tid & 15;  // rows 4 tr + a, positions tc + 16 b
  float acc[4][4][4];
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int b = 0; b < 4; b++)
#pragma unroll
      for (int l = 0; l < 4; l++) acc[a][b][l] = 0.f;
#pragma unroll 2
  for (int i = 0; i < HD / 4; i++) {
    float4 q[4], k[4];
#pragma unroll
    for (int a = 0; a < 4; a++) q[a] = *reinterpret_cast<const float4*>(qs + (4 * tr + a) * LD + 4 * i);
#pragma unroll
    for (int b = 0; b < 4; b++) k[b] = *reinterpret_cast<const float4*>(ks + (tc + 16 * b) * LD + 4 * i);
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
      for (int b = 0; b < 4; b++) {  // products packed in pairs, sums as scalars (never fused with the products)
        const unsigned long long p01 = f2_mul(f2(q[a].x, q[a].y), f2(k[b].x, k[b].y));
        const unsigned long long p23 = f2_mul(f2(q[a].z, q[a].w), f2(k[b].z, k[b].w));
        acc[a][b][0] = __fadd_rn(acc[a][b][0], f2_lo(p01));
        acc[a][b][1] = __fadd_rn(acc[a][b][1], f2_hi(p01));
        acc[a][b][2] = __fadd_rn(acc[a][b][2], f2_lo(p23));
        acc[a][b][3] = __fadd_rn(acc[a][b][3], f2_hi(p23));
      }
  }
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  float* Sk = S + (size_t)kh * R * ldS;
#pragma unroll
  for (int a = 0; a < 4; a++) {
    const int r = r0 + 4 * tr + a;
    const int T = r < R ? pos0 + r / G + 1 : 0;
    float mx = -1e30f;
#pragma unroll
    for (int b = 0; b < 4; b++) {
      const int t = t0 + tc + 16 * b;
      if (t < T) {
        const float v =
            __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc[a][b][0], acc[a][b][1]), acc[a][b][2]), acc[a][b][3]), scale);
        Sk[(size_t)r * ldS + t] = v;
        mx = fmaxf(mx, v);
      }
    }
#pragma unroll
    for (int o = 8; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));  // the 16 threads of row r
    if (tc == 0 && r < R) PM[((size_t)kh * R + r) * ldP + blockIdx.x] = mx;
  }
}

// grid ceil(KVH G M / PF_SR), 256 threads. Flattened rows w = kh G M + r of S and PM; sums[w] = the row's ordered
// sum.
__global__ void __launch_bounds__(256) k_pf_soft(float* __restrict__ S, int ldS, const float* __restrict__ PM, int ldP,
                                                 int rows, int R, int G, int pos0, float* __restrict__ sums) {
  constexpr int NEL = PF_SR * PF_SC, EPT = (NEL + 223) / 224;  // exponentials per thread of warps 1..7 per chunk
  __shared__ __align__(16) float eb[2][PF_SR][PF_SC + 4];
  __shared__ float mxs[PF_SR];
  __shared__ int ts[PF_SR];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, row0 = blockIdx.x * PF_SR;
  if (tid < PF_SR) ts[tid] = row0 + tid < rows ? pos0 + ((row0 + tid) % R) / G + 1 : 0;
  __syncthreads();
  for (int j = warp; j < PF_SR; j += 8) {  // the row's maximum from its partial maxima (order-free)
    const int nb = (ts[j] + PF_TB - 1) / PF_TB;
    float mx = -1e30f;
    for (int b = lane; b < nb; b += 32) mx = fmaxf(mx, PM[(size_t)(row0 + j) * ldP + b]);
    mx = warp_max(mx);
    if (lane == 0) mxs[j] = mx;
  }
  int Tc = 0;
#pragma unroll
  for (int j = 0; j < PF_SR; j++) Tc = max(Tc, ts[j]);
  __syncthreads();
  const int nc = (Tc + PF_SC - 1) / PF_SC;
  const int Tl = lane < PF_SR ? ts[lane] : 0;  // warp 0: lane j sums row j
  float sum = 0.f;
  float v[EPT];
  auto load = [&](int c, float* dst) {  // chunk c's scores of this thread's elements
#pragma unroll
    for (int k = 0; k < EPT; k++) {
      const int i = tid - 32 + 224 * k, j = i / PF_SC, t = c * PF_SC + i % PF_SC;
      dst[k] = c < nc && i < NEL && t < ts[j] ? S[(size_t)(row0 + j) * ldS + t] : 0.f;
    }
  };
  if (warp > 0) load(0, v);
  for (int c = 0; c <= nc; c++) {
    if (warp > 0 && c < nc) {
      float nv[EPT];
      load(c + 1, nv);  // in flight while chunk c is used
#pragma unroll
      for (int k = 0; k < EPT; k++) {
        const int i = tid - 32 + 224 * k, j = i / PF_SC, tt = i % PF_SC, t = c * PF_SC + tt;
        if (i < NEL && t < ts[j]) {
          const float e = fast_exp_ref(__fsub_rn(v[k], mxs[j]));
          S[(size_t)(row0 + j) * ldS + t] = e;
          eb[c & 1][j][tt] = e;
        }
        v[k] = nv[k];
      }
    }
    if (warp == 0 && c > 0 && lane < PF_SR) {  // the ordered sums over chunk c - 1 (kernels.c:368)
      const float* b = &eb[(c - 1) & 1][lane][0];
      const int tb = (c - 1) * PF_SC;
#pragma unroll
      for (int q = 0; q < PF_SC / 4; q++) {
        const float4 x = *reinterpret_cast<const float4*>(b + 4 * q);
        const int t = tb + 4 * q;
        if (t < Tl) sum = __fadd_rn(sum, x.x);
        if (t + 1 < Tl) sum = __fadd_rn(sum, x.y);
        if (t + 2 < Tl) sum = __fadd_rn(sum, x.z);
        if (t + 3 < Tl) sum = __fadd_rn(sum, x.w);
      }
    }
    __syncthreads();  // chunk c's buffer is complete; chunk c - 1's buffer is free for chunk c + 1
  }
  if (warp == 0 && lane < PF_SR && row0 + lane < rows) sums[row0 + lane] = sum;
}

// grid (ceil(G M / pf_pv_rows<HD>()), KVH), 128 threads, dynamic smem pf_pv_smem<HD>(). att: row stride D, query
// head h of token m at att[m D + h HD] (the pass's first token at att[0]).
template <int HD>
__global__ void __launch_bounds__(128) k_pf_pv(const float* __restrict__ S, int ldS, const float* __restrict__ sums,
                                               const float* __restrict__ vc, int H, int KVH, int ctx, int layers,
                                               int layer, int seq, int pos0, int M, float* __restrict__ att, int D) {
  constexpr int RB = pf_pv_rows<HD>(), DG = HD / 4, PL = 2 * PF_VT + 4, PF4 = RB * PF_VT / 4 / 128;
  extern __shared__ __align__(16) float pvs[];
  float* vs = pvs;                   // [2][PF_VT][HD]
  float* ps = pvs + 2 * PF_VT * HD;  // [2][RB][PL]: p of position t at 2 t and 2 t + 1
  const int kh = blockIdx.y, G = H / KVH, R = G * M, tid = threadIdx.x;
  const int r0 = blockIdx.x * RB;
  if (r0 >= R) return;
  const int dg = tid % DG, rp = tid / DG;  // dims 4 dg .. 4 dg + 3 of rows 2 rp, 2 rp + 1 (block-local)
  const int ra = r0 + 2 * rp, rb = ra + 1;
  const int Ta = ra < R ? pos0 + ra / G + 1 : 0, Tb = rb < R ? pos0 + rb / G + 1 : 0;
  const int Tlo = pos0 + r0 / G + 1, Thi = pos0 + (min(R, r0 + RB) - 1) / G + 1;
  const int nt = (Thi + PF_VT - 1) / PF_VT;
  const float* vb = vc + (((size_t)seq * layers + layer) * KVH + kh) * (size_t)ctx * HD;
  const float* Sk = S + (size_t)kh * R * ldS;
  // the e values this thread stages: float4 k of a tile is (row pr[k], positions 4 pq[k] .. + 3)
  int pr[PF4], pq[PF4], pT[PF4];
  float psum[PF4];
#pragma unroll
  for (int k = 0; k < PF4; k++) {
    const int i = tid + 128 * k, rr = r0 + i / (PF_VT / 4);
    pr[k] = i / (PF_VT / 4);
    pq[k] = i % (PF_VT / 4);
    pT[k] = rr < R ? pos0 + rr / G + 1 : 0;
    psum[k] = rr < R ? sums[(size_t)kh * R + rr] : 1.f;
  }
  auto stage_v = [&](int c) {  // V rows of tile c into buffer c & 1
    if (c < nt) {
      float* dst = vs + (c & 1) * PF_VT * HD;
      const int t0 = c * PF_VT, tc = min(PF_VT, Thi - t0);
      for (int i = tid; i < tc * DG; i += 128) {
        const int t = i / DG, q = i % DG;
        cp_async16(dst + t * HD + 4 * q, vb + (size_t)(t0 + t) * HD + 4 * q);
      }
    }
    cp_async_commit();
  };
  float4 sv[PF4];
  auto load_e = [&](int c) {
#pragma unroll
    for (int k = 0; k < PF4; k++) {
      const int t = c * PF_VT + 4 * pq[k];
      sv[k] = c < nt && t < pT[k]
                  ? *reinterpret_cast<const float4*>(Sk + (size_t)(r0 + pr[k]) * ldS + t)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto store_p = [&](int c) {  // p = e / sum (kernels.c:369), 0 past the row's length
    if (c >= nt) return;
#pragma unroll
    for (int k = 0; k < PF4; k++) {
      const int t = c * PF_VT + 4 * pq[k];
      float4 p;
      p.x = t < pT[k] ? __fdiv_rn(sv[k].x, psum[k]) : 0.f;
      p.y = t + 1 < pT[k] ? __fdiv_rn(sv[k].y, psum[k]) : 0.f;
      p.z = t + 2 < pT[k] ? __fdiv_rn(sv[k].z, psum[k]) : 0.f;
      p.w = t + 3 < pT[k] ? __fdiv_rn(sv[k].w, psum[k]) : 0.f;
      float* d = ps + (c & 1) * RB * PL + pr[k] * PL + 8 * pq[k];
      *reinterpret_cast<float4*>(d) = make_float4(p.x, p.x, p.y, p.y);
      *reinterpret_cast<float4*>(d + 4) = make_float4(p.z, p.z, p.w, p.w);
    }
  };
  stage_v(0);
  stage_v(1);
  load_e(0);
  store_p(0);
  float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
  for (int c = 0; c < nt; c++) {
    load_e(c + 1);               // in flight while tile c is used
    cp_async_wait_group<1>();    // V tile c has landed
    __syncthreads();             // V tile c and p tile c are visible to every thread
    const float* v = vs + (c & 1) * PF_VT * HD + 4 * dg;
    const float* pa = ps + (c & 1) * RB * PL + (2 * rp) * PL;
    const float* pb = pa + PL;
    const int t0 = c * PF_VT;
    if (t0 + PF_VT <= Tlo) {  // every row of the block attends to the whole tile
#pragma unroll 2
      for (int q = 0; q < PF_VT / 2; q++) {  // positions 2 q, 2 q + 1: (p, p) pairs straight from shared memory
        const ulonglong2 xa = *reinterpret_cast<const ulonglong2*>(pa + 4 * q);
        const ulonglong2 xb = *reinterpret_cast<const ulonglong2*>(pb + 4 * q);
#pragma unroll
        for (int u = 0; u < 2; u++) {
          const ulonglong2 w = *reinterpret_cast<const ulonglong2*>(v + (2 * q + u) * HD);
          const unsigned long long pa2 = u ? xa.y : xa.x, pb2 = u ? xb.y : xb.x;
          const unsigned long long qa01 = f2_mul(pa2, w.x), qa23 = f2_mul(pa2, w.y);
          const unsigned long long qb01 = f2_mul(pb2, w.x), qb23 = f2_mul(pb2, w.y);
          a0[0] = __fadd_rn(a0[0], f2_lo(qa01));
          a0[1] = __fadd_rn(a0[1], f2_hi(qa01));
          a0[2] = __fadd_rn(a0[2], f2_lo(qa23));
          a0[3] = __fadd_rn(a0[3], f2_hi(qa23));
          a1[0] = __fadd_rn(a1[0], f2_lo(qb01));
          a1[1] = __fadd_rn(a1[1], f2_hi(qb01));
          a1[2] = __fadd_rn(a1[2], f2_lo(qb23));
          a1[3] = __fadd_rn(a1[3], f2_hi(qb23));
        }
      }
    } else {  // the rows' last positions: each row adds only t < its length
      const int tn = min(PF_VT, Thi - t0);
      for (int u = 0; u < tn; u++) {
        const int t = t0 + u;
        const float4 w = *reinterpret_cast<const float4*>(v + u * HD);
        const float p0 = pa[2 * u], p1 = pb[2 * u];
        if (t < Ta) {
          a0[0] = __fadd_rn(a0[0], __fmul_rn(p0, w.x));
          a0[1] = __fadd_rn(a0[1], __fmul_rn(p0, w.y));
          a0[2] = __fadd_rn(a0[2], __fmul_rn(p0, w.z));
          a0[3] = __fadd_rn(a0[3], __fmul_rn(p0, w.w));
        }
        if (t < Tb) {
          a1[0] = __fadd_rn(a1[0], __fmul_rn(p1, w.x));
          a1[1] = __fadd_rn(a1[1], __fmul_rn(p1, w.y));
          a1[2] = __fadd_rn(a1[2], __fmul_rn(p1, w.z));
          a1[3] = __fadd_rn(a1[3], __fmul_rn(p1, w.w));
        }
      }
    }
    store_p(c + 1);     // buffer (c + 1) & 1 was last read in tile c - 1, before this tile's barrier
    __syncthreads();    // V buffer c & 1 is free again
    stage_v(c + 2);
  }
  cp_async_wait_all();
  if (ra < R)
    *reinterpret_cast<float4*>(att + (size_t)(ra / G) * D + (size_t)(kh * G + ra % G) * HD + 4 * dg) =
        make_float4(a0[0], a0[1], a0[2], a0[3]);
  if (rb < R)
    *reinterpret_cast<float4*>(att + (size_t)(rb / G) * D + (size_t)(kh * G + rb % G) * HD + 4 * dg) =
        make_float4(a1[0], a1[1], a1[2], a1[3]);
}

}  // namespace h2
