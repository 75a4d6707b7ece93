/* Test infrastructure: the CPU parity oracle. Never linked into, loaded by, or called from the product path.
 *
 * A scalar C restatement of the H2 engine's Qwen2 forward pass as the reference computes it in
 * h2-own-inference-engine/engine/kernels.c (SIMD128, non-relaxed build). Every floating-point operation is
 * written in the same order and with the same roundings as the reference's four 32-bit SIMD lanes, so that the
 * results are bit-identical to the reference built natively through oracle/shim (checked by tests). Integer
 * parts (Q4_0 / Q8_0 unpacking, int8 activation quantization, block dot products) are exact by construction.
 *
 * Differences from the reference, all extensions that leave its computation unchanged:
 *   - head_dim is not capped at 64 (the reference's `v128_t acc[16]`, kernels.c:370, limits it);
 *   - no MAXL layer cap (kernels.c:17);
 *   - tensor kind 10 = a Q4_0 output matrix (tied embeddings): logits through the same per-block lane
 *     arithmetic as dot_q4_q8 (kernels.c:121-139), which equals dot_q8_q8 (kernels.c:157-170) on the
 *     Q8_0 expansion of the same blocks;
 *   - rows are split across OpenMP threads; each row is computed by one thread in the reference's order,
 *     so the result does not depend on the thread count (the reference's property, wiki 04:75-77).
 *
 * The exported API mirrors the reference's exports (kernels.c:418-465) with an h2o_ prefix.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define H2O_MAX_LAYERS 256

typedef struct { const uint8_t* qs; const float* d; } q4_mat;  /* qs: 16 B per 32 values, d: one scale per 32 */
typedef struct { const int8_t* qs; const float* d; } q8_mat;
typedef struct { const float *attn_norm, *ffn_norm, *bqkv; q4_mat qkv, o, gu, down; } layer_w;

static struct {
  int dim, layers, ffn, heads, kvh, hd, vocab, ctx, mt;
  float eps;
  q4_mat embd; q8_mat out8; q4_mat out4; int out_is_q4; const float* out_norm;
  layer_w L[H2O_MAX_LAYERS];
  const float* rope;
  float *x, *xn, *qkv, *att, *gu, *act, *logits, *kc, *vc, *scores;
  int8_t* aq; float *ad, *as;
  const int* tokens;
} S;

/* ------------------------------------------------------------------ scalar lane helpers */

/* f32x4.max of the WebAssembly spec for one lane (kernels.c:94 uses it on absolute values). */
static inline float lane_max(float a, float b) {
  if (a != a || b != b) return NAN;
  if (a == 0.0f && b == 0.0f) { uint32_t ua, ub; memcpy(&ua, &a, 4); memcpy(&ub, &b, 4); ua &= ub; memcpy(&a, &ua, 4); return a; }
  return a > b ? a : b;
}

/* i32x4.trunc_sat_f32x4_s for one lane. */
static inline int32_t trunc_sat(float f) {
  if (f != f) return 0;
  if (f >= 2147483648.0f) return INT32_MAX;
  if (f < -2147483648.0f) return INT32_MIN;
  return (int32_t)f;
}
static inline int32_t sat16(int32_t v) { return v > 32767 ? 32767 : v < -32768 ? -32768 : v; }
static inline int8_t sat8(int32_t v) { return (int8_t)(v > 127 ? 127 : v < -128 ? -128 : v); }

/* The four 32-bit lanes of i32x4.dot_i16x8_s applied to (lo-nibble values, x[0..15]) and (hi, x[16..31]), as in
 * q4_bdot (kernels.c:179-185): lane i sums elements {2i, 2i+1, 8+2i, 9+2i} of both halves. */
static inline void block_lanes(const int8_t w[32], const int8_t* x, int32_t p[4]) {
  for (int i = 0; i < 4; i++) {
    int32_t s = 0;
    const int e[4] = { 2 * i, 2 * i + 1, 8 + 2 * i, 9 + 2 * i };
    for (int k = 0; k < 4; k++) s += (int32_t)w[e[k]] * x[e[k]] + (int32_t)w[16 + e[k]] * x[16 + e[k]];
    p[i] = s;
  }
}

static inline void unpack_q4(const uint8_t* qs, int8_t w[32]) {  /* kernels.c:129-130: lo = q & 15, hi = q >> 4, minus 8 */
  for (int j = 0; j < 16; j++) { w[j] = (int8_t)((qs[j] & 15) - 8); w[16 + j] = (int8_t)((qs[j] >> 4) - 8); }
}

static inline float hsum4(const float a[4]) { return a[0] + a[1] + a[2] + a[3]; }  /* kernels.c:116-118 */

/* fast_exp, kernels.c:69-78 (the reference's own e^x). */
static inline float ref_fast_exp(float x) {
  if (x < -87.0f) return 0.0f;
  if (x > 88.0f) x = 88.0f;
  float n = floorf(x * 1.44269504f + 0.5f);
  float r = x - n * 0.693145752f - n * 1.42860677e-6f;
  float p = 1.0f + r * (1.0f + r * (0.5f + r * (0.166666672f + r * (0.0416666679f + r * (0.00833333377f + r * 0.00138888892f)))));
  union { float f; int32_t i; } u = { .f = p };
  u.i += (int32_t)n << 23;
  return u.f;
}

/* ------------------------------------------------------------------ ops */

/* rmsnorm, kernels.c:80-86: sum of squares in 4 lanes (element i goes to lane i mod 4), lanes added 0+1+2+3. */
static void rmsnorm(float* out, const float* x, const float* w, int n, float eps) {
  float s[4] = { 0, 0, 0, 0 };
  for (int i = 0; i < n; i += 4)
    for (int l = 0; l < 4; l++) s[l] = s[l] + x[i + l] * x[i + l];
  float ss = hsum4(s);
  float r = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = 0; i < n; i++) out[i] = (x[i] * r) * w[i];
}

/* quantize_row, kernels.c:90-114: per 32 values, amax over 4 lanes, d = amax/127, q = sat(nearest_even(x / d)). */
static void quantize_row(int8_t* q, float* d, float* s, const float* x, int n) {
  for (int b = 0; b < n / 32; b++) {
    const float* xb = x + 32 * b;
    float mx[4] = { 0, 0, 0, 0 };
    for (int i = 0; i < 32; i += 4)
      for (int l = 0; l < 4; l++) mx[l] = lane_max(mx[l], fabsf(xb[i + l]));
    float amax = mx[0] > mx[1] ? mx[0] : mx[1];
    if (mx[2] > amax) amax = mx[2];
    if (mx[3] > amax) amax = mx[3];
    float dd = amax / 127.0f, id = dd != 0.0f ? 1.0f / dd : 0.0f;
    int32_t sum = 0;
    for (int i = 0; i < 32; i++) {
      int32_t v = trunc_sat(nearbyintf(xb[i] * id));
      q[32 * b + i] = sat8(sat16(v));
      sum += v;
    }
    d[b] = dd;
    s[b] = dd * (float)sum;
  }
}

/* One Q4_0 row against one quantized activation row: dot_q4_q8 / the M=1 rows of matmul_q4 (kernels.c:121-139,
 * 209-229): per block four exact integer lane sums, each lane accumulating f32(p) * (dw * dx) in block order. */
static float dot_q4_row(const uint8_t* wq, const float* wd, const int8_t* xq, const float* xd, int nb) {
  float acc[4] = { 0, 0, 0, 0 };
  int8_t w[32];
  int32_t p[4];
  for (int b = 0; b < nb; b++) {
    unpack_q4(wq + 16 * b, w);
    block_lanes(w, xq + 32 * b, p);
    float sc = wd[b] * xd[b];
    for (int l = 0; l < 4; l++) acc[l] = acc[l] + (float)p[l] * sc;
  }
  return hsum4(acc);
}

/* dot_q8_q8, kernels.c:157-170: the same lane structure on 32 signed bytes (w0 = values 0..15, w1 = 16..31). */
static float dot_q8_row(const int8_t* wq, const float* wd, const int8_t* xq, const float* xd, int nb) {
  float acc[4] = { 0, 0, 0, 0 };
  int32_t p[4];
  for (int b = 0; b < nb; b++) {
    block_lanes(wq + 32 * b, xq + 32 * b, p);
    float sc = wd[b] * xd[b];
    for (int l = 0; l < 4; l++) acc[l] = acc[l] + (float)p[l] * sc;
  }
  return hsum4(acc);
}

enum { OP_STORE, OP_BIAS, OP_ADD };  /* put(), kernels.c:190-194 */

/* matmul_q4, kernels.c:200-273: every branch uses the per-block arithmetic of dot_q4_row, so one loop suffices. */
static void matmul_q4(q4_mat W, int K, int N, int M, const int8_t* xq, const float* xd, float* y, int op,
                      const float* bias, int nth) {
  const int nb = K / 32;
#pragma omp parallel for schedule(static) num_threads(nth)
  for (int n = 0; n < N; n++) {
    const uint8_t* wq = W.qs + (size_t)n * nb * 16;
    const float* wd = W.d + (size_t)n * nb;
    for (int m = 0; m < M; m++) {
      float v = dot_q4_row(wq, wd, xq + (size_t)m * K, xd + (size_t)m * nb, nb);
      float* o = y + (size_t)m * N + n;
      if (op == OP_ADD) *o += v; else if (op == OP_BIAS) *o = v + bias[n]; else *o = v;
    }
  }
}

/* ------------------------------------------------------------------ the forward pass (kernels.c:306-415) */
static void forward_pass(int pos0, int M, int want_logits, int nth) {
  const int D = S.dim, F = S.ffn, H = S.heads, KVH = S.kvh, HD = S.hd, QKV = D + 2 * KVH * HD;

  for (int m = 0; m < M; m++) {  /* embedding rows (kernels.c:313-322) */
    int t = S.tokens[pos0 + m];
    const uint8_t* q = S.embd.qs + (size_t)t * (D / 32) * 16;
    const float* d = S.embd.d + (size_t)t * (D / 32);
    float* xr = S.x + (size_t)m * D;
    for (int blk = 0; blk < D / 32; blk++)
      for (int j = 0; j < 16; j++) {
        xr[32 * blk + j] = (float)((q[16 * blk + j] & 15) - 8) * d[blk];
        xr[32 * blk + 16 + j] = (float)((q[16 * blk + j] >> 4) - 8) * d[blk];
      }
  }

  for (int l = 0; l < S.layers; l++) {
    const layer_w* L = &S.L[l];
    for (int m = 0; m < M; m++) {  /* kernels.c:328-331 */
      rmsnorm(S.xn + (size_t)m * D, S.x + (size_t)m * D, L->attn_norm, D, S.eps);
      quantize_row(S.aq + (size_t)m * D, S.ad + (size_t)m * (D / 32), S.as + (size_t)m * (D / 32), S.xn + (size_t)m * D, D);
    }
    matmul_q4(L->qkv, D, QKV, M, S.aq, S.ad, S.qkv, OP_BIAS, L->bqkv, nth);  /* kernels.c:333-334 */

    for (int m = 0; m < M; m++)  /* RoPE on Q and K heads, then K/V append (kernels.c:337-352) */
      for (int h = 0; h < H + KVH; h++) {
        int pos = pos0 + m;
        float* v = S.qkv + (size_t)m * QKV + (size_t)h * HD;
        const float* cs = S.rope + (size_t)pos * HD;
        for (int i = 0; i < HD / 2; i++) {
          float c = cs[2 * i], s = cs[2 * i + 1], x0 = v[i], x1 = v[i + HD / 2];
          v[i] = x0 * c - x1 * s;
          v[i + HD / 2] = x1 * c + x0 * s;
        }
        if (h >= H) {
          int kh = h - H;
          float* kd = S.kc + (((size_t)l * KVH + kh) * S.ctx + pos) * HD;
          float* vd = S.vc + (((size_t)l * KVH + kh) * S.ctx + pos) * HD;
          const float* vs = S.qkv + (size_t)m * QKV + D + KVH * HD + (size_t)kh * HD;
          for (int i = 0; i < HD; i++) { kd[i] = v[i]; vd[i] = vs[i]; }
        }
      }

#pragma omp parallel for schedule(static) num_threads(nth)
    for (int task = 0; task < M * H; task++) {  /* attention per (token, head), kernels.c:355-377 */
      int m = task / H, h = task % H, T = pos0 + m + 1, kh = h / (H / KVH);
      int tid = 0;
#ifdef _OPENMP
      tid = omp_get_thread_num();
#endif
      const float* q = S.qkv + (size_t)m * QKV + (size_t)h * HD;
      const float* kb = S.kc + ((size_t)l * KVH + kh) * S.ctx * HD;
      const float* vb = S.vc + ((size_t)l * KVH + kh) * S.ctx * HD;
      float* sc = S.scores + (size_t)tid * S.ctx;
      float mx = -1e30f, scale = 1.0f / sqrtf((float)HD);
      for (int t = 0; t < T; t++) {
        float s[4] = { 0, 0, 0, 0 };
        for (int i = 0; i < HD; i += 4)
          for (int ln = 0; ln < 4; ln++) s[ln] = s[ln] + q[i + ln] * kb[(size_t)t * HD + i + ln];
        float v = hsum4(s) * scale;
        sc[t] = v;
        if (v > mx) mx = v;
      }
      float sum = 0;
      for (int t = 0; t < T; t++) { float e = ref_fast_exp(sc[t] - mx); sc[t] = e; sum += e; }
      float* o = S.att + (size_t)m * D + (size_t)h * HD;
      for (int i = 0; i < HD; i++) o[i] = 0.0f;
      for (int t = 0; t < T; t++) {
        float p = sc[t] / sum;
        for (int i = 0; i < HD; i++) o[i] = o[i] + p * vb[(size_t)t * HD + i];
      }
    }

    for (int m = 0; m < M; m++)  /* kernels.c:379 */
      quantize_row(S.aq + (size_t)m * D, S.ad + (size_t)m * (D / 32), S.as + (size_t)m * (D / 32), S.att + (size_t)m * D, D);
    matmul_q4(L->o, D, D, M, S.aq, S.ad, S.x, OP_ADD, 0, nth);  /* kernels.c:381-382 */

    for (int m = 0; m < M; m++) {  /* kernels.c:385-388 */
      rmsnorm(S.xn + (size_t)m * D, S.x + (size_t)m * D, L->ffn_norm, D, S.eps);
      quantize_row(S.aq + (size_t)m * D, S.ad + (size_t)m * (D / 32), S.as + (size_t)m * (D / 32), S.xn + (size_t)m * D, D);
    }
    matmul_q4(L->gu, D, 2 * F, M, S.aq, S.ad, S.gu, OP_STORE, 0, nth);  /* kernels.c:390-391 */
    for (int m = 0; m < M; m++) {  /* silu(gate) * up, then quantize (kernels.c:393-397) */
      float* gu = S.gu + (size_t)m * 2 * F;
      float* ac = S.act + (size_t)m * F;
      for (int i = 0; i < F; i++) { float gt = gu[i]; ac[i] = gt / (1.0f + ref_fast_exp(-gt)) * gu[F + i]; }
      quantize_row(S.aq + (size_t)m * F, S.ad + (size_t)m * (F / 32), S.as + (size_t)m * (F / 32), ac, F);
    }
    matmul_q4(L->down, F, D, M, S.aq, S.ad, S.x, OP_ADD, 0, nth);  /* kernels.c:399-400 */
  }

  if (want_logits) {  /* last token only (kernels.c:404-414) */
    rmsnorm(S.xn, S.x + (size_t)(M - 1) * D, S.out_norm, D, S.eps);
    quantize_row(S.aq, S.ad, S.as, S.xn, D);
    const int nb = D / 32;
#pragma omp parallel for schedule(static) num_threads(nth)
    for (int n = 0; n < S.vocab; n++)
      S.logits[n] = S.out_is_q4
          ? dot_q4_row(S.out4.qs + (size_t)n * nb * 16, S.out4.d + (size_t)n * nb, S.aq, S.ad, nb)
          : dot_q8_row(S.out8.qs + (size_t)n * D, S.out8.d + (size_t)n * nb, S.aq, S.ad, nb);
  }
}

/* ------------------------------------------------------------------ exports (kernels.c:418-465) */
int h2o_set_config(int dim, int layers, int ffn, int heads, int kvh, int vocab, int ctx, int mt, float eps) {
  if (layers > H2O_MAX_LAYERS || dim % 32 || ffn % 32 || heads <= 0 || kvh <= 0 || heads % kvh || dim % heads) return -1;
  S.dim = dim; S.layers = layers; S.ffn = ffn; S.heads = heads; S.kvh = kvh; S.hd = dim / heads;
  S.vocab = vocab; S.ctx = ctx; S.mt = mt; S.eps = eps;
  return 0;
}

/* kind: 0 qkv, 1 o, 2 gu, 3 down (Q4); 4 attn_norm, 5 ffn_norm, 6 bqkv (f32); 7 embd (Q4); 8 output (Q8);
 * 9 output_norm; 10 output (Q4, tied embeddings: an extension of the reference's kinds). */
int h2o_set_tensor(int kind, int layer, const void* qs, const float* d) {
  if (layer < 0 || layer >= H2O_MAX_LAYERS) return -1;
  layer_w* L = &S.L[layer];
  switch (kind) {
    case 0: L->qkv = (q4_mat){ qs, d }; break;
    case 1: L->o = (q4_mat){ qs, d }; break;
    case 2: L->gu = (q4_mat){ qs, d }; break;
    case 3: L->down = (q4_mat){ qs, d }; break;
    case 4: L->attn_norm = d; break;
    case 5: L->ffn_norm = d; break;
    case 6: L->bqkv = d; break;
    case 7: S.embd = (q4_mat){ qs, d }; break;
    case 8: S.out8 = (q8_mat){ qs, d }; S.out_is_q4 = 0; break;
    case 9: S.out_norm = d; break;
    case 10: S.out4 = (q4_mat){ qs, d }; S.out_is_q4 = 1; break;
    default: return -1;
  }
  return 0;
}

void h2o_set_buffers(float* x, float* xn, float* qkv, float* att, float* gu, float* act, float* logits, float* kc,
                     float* vc, float* scores, int8_t* aq, float* ad, float* as, const float* rope, const int* tokens) {
  S.x = x; S.xn = xn; S.qkv = qkv; S.att = att; S.gu = gu; S.act = act; S.logits = logits; S.kc = kc; S.vc = vc;
  S.scores = scores; S.aq = aq; S.ad = ad; S.as = as; S.rope = rope; S.tokens = tokens;
}

/* Run tokens[pos0 .. pos0+M) (kernels.c:454-465). nth = threads for row splits (results do not depend on it). */
void h2o_run(int pos0, int M, int want_logits, int nth) { forward_pass(pos0, M, want_logits, nth < 1 ? 1 : nth); }

/* Stand-alone pieces for kernel-level parity tests. */
void h2o_quantize_row(int8_t* q, float* d, float* s, const float* x, int n) { quantize_row(q, d, s, x, n); }
void h2o_rmsnorm(float* out, const float* x, const float* w, int n, float eps) { rmsnorm(out, x, w, n, eps); }
float h2o_fast_exp(float x) { return ref_fast_exp(x); }

/* y[m][n] (op)= W[n] . quant(x[m]) for a Q4_0 matrix: the Q4_0 matvec microbench of the reference's CPU path
 * (quantize_row then matmul_q4). op: 0 store, 1 bias, 2 add. */
void h2o_matvec_q4(const uint8_t* qs, const float* d, int N, int K, int M, const float* x, float* y, int op,
                   const float* bias, int nth, int8_t* aq, float* ad, float* as) {
  for (int m = 0; m < M; m++)
    quantize_row(aq + (size_t)m * K, ad + (size_t)m * (K / 32), as + (size_t)m * (K / 32), x + (size_t)m * K, K);
  matmul_q4((q4_mat){ qs, d }, K, N, M, aq, ad, y, op, bias, nth < 1 ? 1 : nth);
}

/* The CPU sampler, cpu-worker.js:154-167: greedy argmax (strict >, ties to the lowest index), or softmax of
 * logits / temperature sampled with mulberry32(seed), all in double precision as JavaScript numbers. */
static double mulberry32(uint32_t* s) {
  *s = *s + 0x6d2b79f5u;
  uint32_t t = *s;
  t = (t ^ (t >> 15)) * (t | 1u);
  t ^= t + (t ^ (t >> 7)) * (t | 61u);
  return (double)(t ^ (t >> 14)) / 4294967296.0;
}

int h2o_sample(const float* lg, int n, double temperature, uint32_t seed) {
  int best = 0;
  for (int i = 1; i < n; i++) if (lg[i] > lg[best]) best = i;
  if (!(temperature > 0)) return best;
  uint32_t s = seed;
  double mx = (double)lg[best] / temperature, sum = 0;
  for (int i = 0; i < n; i++) sum += exp((double)lg[i] / temperature - mx);
  double r = mulberry32(&s) * sum;
  for (int i = 0; i < n; i++) { r -= exp((double)lg[i] / temperature - mx); if (r <= 0) return i; }
  return best;
}
