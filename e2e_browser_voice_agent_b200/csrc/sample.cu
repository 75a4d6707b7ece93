// Temperature sampling on the device: the reference's sample() (cpu-worker.js:153-167) without copying the logits
// to the host.
//
// The reference, per token: best = argmax (strict >, ties to the lowest id); if temperature <= 0 the token is best;
// else mx = lg[best] / T, sum = sum_i exp(lg[i] / T - mx), r = mulberry32(seed) * sum, and the token is the first i
// at which r -= exp(lg[i] / T - mx) reaches <= 0 (best if it never does). All in double precision (JavaScript
// numbers), the two sums in index order.
//
// Here the vocabulary is split into SAMPLE_RANGES contiguous ranges, each range into 256 contiguous thread chunks:
//   k_sample_max   (ranges x rows)  per-range argmax;
//   k_sample_sum   (ranges x rows)  every range merges the argmax partials, then sums its exponentials chunk by
//                                   chunk (each chunk in index order) and the chunk sums in order;
//   k_sample_pick  (rows)           the range sums added in order give `sum`; r is walked down range by range, then
//                                   chunk by chunk inside the range where it would reach <= 0 (chunk sums recomputed
//                                   by the same code, so the same values), then element by element, as the
//                                   reference walks it.
// Same operations per element as the reference (double division, subtraction, exp), but the total and the coarse
// steps of the walk are added by range and chunk instead of one element at a time, so each differs from the
// reference's running double sum by a few units in the last place (relative error about 1e-16 x the number of
// terms). The token can therefore differ only when r falls that close to a category boundary; double exp here and
// the host's may also differ by one unit in the last place.
#include "sample.cuh"

#include <cfloat>
#include <cmath>

namespace h2 {
namespace {

constexpr int ST = 256;  // threads per CTA

struct Range {
  int lo, hi, chunk;  // [lo, hi) of the vocabulary; elements per thread chunk
};
__device__ __forceinline__ Range range_of(int c, int V) {
  Range r;
  r.lo = (int)((long long)c * V / SAMPLE_RANGES);
  r.hi = (int)((long long)(c + 1) * V / SAMPLE_RANGES);
  r.chunk = (r.hi - r.lo + ST - 1) / ST;
  return r;
}

__device__ __forceinline__ void amax_merge_s(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

// mulberry32 (cpu-worker.js:159): one draw in [0, 1) from state seed
__device__ __forceinline__ double mulberry32_draw(uint32_t s) {
  s = s + 0x6d2b79f5u;
  uint32_t t = s;
  t = (t ^ (t >> 15)) * (t | 1u);
  t ^= t + (t ^ (t >> 7)) * (t | 61u);
  return (double)(t ^ (t >> 14)) / 4294967296.0;
}

__device__ __forceinline__ double expo(const float* lg, int i, double T, double mx) {
  return exp((double)lg[i] / T - mx);
}

// merge the per-range argmax partials of one row (all threads take part; every thread gets the result)
__device__ int merged_best(const float* pv, const int* pi) {
  __shared__ float sv[ST / 32];
  __shared__ int si[ST / 32];
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int c = threadIdx.x; c < SAMPLE_RANGES; c += ST) amax_merge_s(v, idx, pv[c], pi[c]);
#pragma unroll
  for (int o = 16; o; o >>= 1) amax_merge_s(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = v;
    si[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  v = sv[0];
  idx = si[0];
  for (int w = 1; w < ST / 32; w++) amax_merge_s(v, idx, sv[w], si[w]);
  __syncthreads();
  return idx == 0x7fffffff ? 0 : idx;
}

// chunk sums of range c into cs[ST] (each chunk's exponentials added in index order)
__device__ void chunk_sums(const float* lg, const Range& R, double T, double mx, double* cs) {
  const int a = R.lo + threadIdx.x * R.chunk, b = min(R.hi, a + R.chunk);
  double s = 0.0;
  for (int i = a; i < b; i++) s += expo(lg, i, T, mx);
  cs[threadIdx.x] = s;
  __syncthreads();
}

__global__ void __launch_bounds__(ST) k_sample_max(const float* __restrict__ logits, int V, float* __restrict__ pv,
                                                   int* __restrict__ pi) {
  const int c = blockIdx.x, m = blockIdx.y;
  const float* lg = logits + (size_t)m * V;
  const Range R = range_of(c, V);
  __shared__ float sv[ST / 32];
  __shared__ int si[ST / 32];
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = R.lo + threadIdx.x; i < R.hi; i += ST) amax_merge_s(v, idx, lg[i], i);
#pragma unroll
  for (int o = 16; o; o >>= 1) amax_merge_s(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = v;
    si[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    v = sv[0];
    idx = si[0];
    for (int w = 1; w < ST / 32; w++) amax_merge_s(v, idx, sv[w], si[w]);
    pv[(size_t)m * SAMPLE_RANGES + c] = v;
    pi[(size_t)m * SAMPLE_RANGES + c] = idx;
  }
}

__global__ void __launch_bounds__(ST) k_sample_sum(const float* __restrict__ logits, int V, double T,
                                                   const float* __restrict__ pv, const int* __restrict__ pi,
                                                   double* __restrict__ ps) {
  const int c = blockIdx.x, m = blockIdx.y;
  const float* lg = logits + (size_t)m * V;
  const int best = merged_best(pv + (size_t)m * SAMPLE_RANGES, pi + (size_t)m * SAMPLE_RANGES);
  const double mx = (double)lg[best] / T;
  __shared__ double cs[ST];
  chunk_sums(lg, range_of(c, V), T, mx, cs);
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int t = 0; t < ST; t++) s += cs[t];
    ps[(size_t)m * SAMPLE_RANGES + c] = s;
  }
}

__global__ void __launch_bounds__(ST) k_sample_pick(const float* __restrict__ logits, int V, double T,
                                                    const uint32_t* __restrict__ seeds, uint32_t seed0,
                                                    const float* __restrict__ pv, const int* __restrict__ pi,
                                                    const double* __restrict__ ps, int32_t* __restrict__ out) {
  const int m = blockIdx.x;
  const float* lg = logits + (size_t)m * V;
  const int best = merged_best(pv + (size_t)m * SAMPLE_RANGES, pi + (size_t)m * SAMPLE_RANGES);
  if (!(T > 0.0)) {
    if (threadIdx.x == 0) out[m] = best;
    return;
  }
  const double mx = (double)lg[best] / T;
  const double* psm = ps + (size_t)m * SAMPLE_RANGES;
  __shared__ double cs[ST];
  __shared__ double r_s;
  __shared__ int c_s;
  if (threadIdx.x == 0) {
    double sum = 0.0;
    for (int c = 0; c < SAMPLE_RANGES; c++) sum += psm[c];
    double r = mulberry32_draw(seeds ? seeds[m] : seed0) * sum;
    int c = 0;
    for (; c < SAMPLE_RANGES; c++) {
      const double r2 = r - psm[c];
      if (r2 <= 0.0) break;
      r = r2;
    }
    r_s = r;
    c_s = c;
  }
  __syncthreads();
  const int c = c_s;
  if (c == SAMPLE_RANGES) {  // r stayed above 0 (rounding): the reference's fall-through
    if (threadIdx.x == 0) out[m] = best;
    return;
  }
  const Range R = range_of(c, V);
  chunk_sums(lg, R, T, mx, cs);
  if (threadIdx.x == 0) {
    double r = r_s;
    int t = 0;
    for (; t < ST; t++) {
      const double r2 = r - cs[t];
      if (r2 <= 0.0) break;
      r = r2;
    }
    int tok = best;
    for (int i = t < ST ? R.lo + t * R.chunk : R.hi; i < V; i++) {  // element by element from that chunk on
      r -= expo(lg, i, T, mx);
      if (r <= 0.0) {
        tok = i;
        break;
      }
    }
    out[m] = tok;
  }
}

}  // namespace

size_t sample_scratch_bytes(int M) { return (size_t)M * SAMPLE_RANGES * (sizeof(double) + sizeof(float) + sizeof(int)); }

cudaError_t launch_sample(const float* logits, int V, int M, double temperature, const uint32_t* seeds,
                          uint32_t seed0, int32_t* out, void* scratch, cudaStream_t st) {
  if (V < SAMPLE_RANGES || M < 1) return cudaErrorInvalidValue;
  double* ps = static_cast<double*>(scratch);
  float* pv = reinterpret_cast<float*>(ps + (size_t)M * SAMPLE_RANGES);
  int* pi = reinterpret_cast<int*>(pv + (size_t)M * SAMPLE_RANGES);
  k_sample_max<<<dim3(SAMPLE_RANGES, M), ST, 0, st>>>(logits, V, pv, pi);
  if (temperature > 0.0) k_sample_sum<<<dim3(SAMPLE_RANGES, M), ST, 0, st>>>(logits, V, temperature, pv, pi, ps);
  k_sample_pick<<<M, ST, 0, st>>>(logits, V, temperature, seeds, seed0, pv, pi, ps, out);
  return cudaGetLastError();
}

}  // namespace h2
