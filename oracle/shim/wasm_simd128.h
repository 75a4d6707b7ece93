/* Test infrastructure (parity oracle), not product code.
 *
 * A native stand-in for clang's <wasm_simd128.h>, so that the reference engine's own CPU kernels
 * (h2-own-inference-engine/engine/kernels.c, built by build.py:12-20 for wasm32 with -msimd128) compile
 * unmodified with gcc on x86-64. Every intrinsic below is written to the WebAssembly SIMD specification's
 * lane semantics, using SSE4.1 only where the x86 instruction has exactly the same result on every input:
 *
 *   i32x4.dot_i16x8_s            == pmaddwd (signed 16x16 products, pairwise wrapping add)
 *   i16x8.narrow_i32x4_s         == packssdw (signed saturation)
 *   i8x16.narrow_i16x8_s         == packsswb (signed saturation)
 *   i16x8.extend_{low,high}      == pmovsxbw
 *   f32x4.add / mul / convert    == addps / mulps / cvtdq2ps (IEEE binary32, round-to-nearest-even)
 *   f32x4.nearest                == roundps with _MM_FROUND_TO_NEAREST_INT (ties to even)
 *
 * and with explicit fix-ups where x86 differs from WebAssembly:
 *   f32x4.max                    NaN in either lane gives NaN; max(-0, +0) = +0 (maxps returns its 2nd operand)
 *   i32x4.trunc_sat_f32x4_s      NaN gives 0 and positive overflow gives INT32_MAX (cvttps2dq gives INT32_MIN)
 *   u8x16.shr                    per-byte logical shift (x86 has no 8-bit shift)
 *
 * The relaxed-SIMD build (-DRELAXED) is not supported: its dot product is implementation-defined, so the
 * oracle uses the deterministic SIMD128 variant, as the survey of the reference prescribes.
 *
 * Threading builtins of the MT build (memory.atomic.wait32 / notify, kernels.c:52-55, 445, 460) map to Linux
 * futexes implemented in oracle/ref_host.c. The export_name / import_* attributes are ignored by gcc
 * (-Wno-attributes), and the imported clock js_now (kernels.c:20) is defined in ref_host.c.
 */
#ifndef H2_ORACLE_WASM_SIMD128_SHIM_H
#define H2_ORACLE_WASM_SIMD128_SHIM_H

#if !defined(__x86_64__) || !defined(__SSE4_1__)
#error "the wasm_simd128 shim needs x86-64 with SSE4.1 (compile with -msse4.1 or -march=x86-64-v2 or later)"
#endif
#ifdef RELAXED
#error "the relaxed-SIMD variant is implementation-defined and is not part of the oracle"
#endif

#include <stdint.h>
#include <string.h>
#include <smmintrin.h>

typedef __m128i v128_t;

static inline __m128 h2s_ps(v128_t v) { return _mm_castsi128_ps(v); }
static inline v128_t h2s_si(__m128 v) { return _mm_castps_si128(v); }

static inline v128_t wasm_v128_load(const void* p) { return _mm_loadu_si128((const __m128i*)p); }
static inline void wasm_v128_store(void* p, v128_t v) { _mm_storeu_si128((__m128i*)p, v); }
static inline v128_t wasm_v128_and(v128_t a, v128_t b) { return _mm_and_si128(a, b); }
static inline v128_t wasm_v128_xor(v128_t a, v128_t b) { return _mm_xor_si128(a, b); }

static inline v128_t wasm_f32x4_splat(float x) { return h2s_si(_mm_set1_ps(x)); }
static inline v128_t wasm_i32x4_splat(int32_t x) { return _mm_set1_epi32(x); }
static inline v128_t wasm_i8x16_splat(int8_t x) { return _mm_set1_epi8(x); }

static inline v128_t wasm_f32x4_add(v128_t a, v128_t b) { return h2s_si(_mm_add_ps(h2s_ps(a), h2s_ps(b))); }
static inline v128_t wasm_f32x4_mul(v128_t a, v128_t b) { return h2s_si(_mm_mul_ps(h2s_ps(a), h2s_ps(b))); }
static inline v128_t wasm_f32x4_abs(v128_t a) { return _mm_and_si128(a, _mm_set1_epi32(0x7fffffff)); }

static inline v128_t wasm_f32x4_max(v128_t a, v128_t b) {
  __m128 fa = h2s_ps(a), fb = h2s_ps(b);
  /* For ordered, unequal inputs both orders agree; for (+0,-0) the AND keeps -0 only when both are -0. */
  __m128 r = _mm_and_ps(_mm_max_ps(fa, fb), _mm_max_ps(fb, fa));
  __m128 nan = _mm_cmpunord_ps(fa, fb);
  r = _mm_blendv_ps(r, _mm_castsi128_ps(_mm_set1_epi32(0x7fc00000)), nan);
  return h2s_si(r);
}

static inline v128_t wasm_f32x4_nearest(v128_t a) {
  return h2s_si(_mm_round_ps(h2s_ps(a), _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC));
}
static inline v128_t wasm_f32x4_convert_i32x4(v128_t a) { return h2s_si(_mm_cvtepi32_ps(a)); }

static inline v128_t wasm_i32x4_trunc_sat_f32x4(v128_t a) {
  __m128 f = h2s_ps(a);
  __m128i t = _mm_cvttps_epi32(f);
  __m128i pos_over = _mm_castps_si128(_mm_cmpge_ps(f, _mm_set1_ps(2147483648.0f)));
  t = _mm_blendv_epi8(t, _mm_set1_epi32(0x7fffffff), pos_over);
  __m128i is_nan = _mm_castps_si128(_mm_cmpunord_ps(f, f));
  return _mm_andnot_si128(is_nan, t);
}

static inline v128_t wasm_i32x4_add(v128_t a, v128_t b) { return _mm_add_epi32(a, b); }
static inline v128_t wasm_i32x4_dot_i16x8(v128_t a, v128_t b) { return _mm_madd_epi16(a, b); }
static inline v128_t wasm_i16x8_extend_low_i8x16(v128_t a) { return _mm_cvtepi8_epi16(a); }
static inline v128_t wasm_i16x8_extend_high_i8x16(v128_t a) { return _mm_cvtepi8_epi16(_mm_srli_si128(a, 8)); }
static inline v128_t wasm_i16x8_narrow_i32x4(v128_t a, v128_t b) { return _mm_packs_epi32(a, b); }
static inline v128_t wasm_i8x16_narrow_i16x8(v128_t a, v128_t b) { return _mm_packs_epi16(a, b); }
static inline v128_t wasm_i8x16_sub(v128_t a, v128_t b) { return _mm_sub_epi8(a, b); }
static inline v128_t wasm_u8x16_shr(v128_t a, uint32_t n) {
  n &= 7;
  return _mm_and_si128(_mm_srl_epi16(a, _mm_cvtsi32_si128((int)n)), _mm_set1_epi8((char)(0xffu >> n)));
}

static inline float h2s_f32_lane(v128_t v, int i) { float f[4]; memcpy(f, &v, 16); return f[i]; }
static inline int32_t h2s_i32_lane(v128_t v, int i) { int32_t x[4]; memcpy(x, &v, 16); return x[i]; }
#define wasm_f32x4_extract_lane(v, i) h2s_f32_lane((v), (i))
#define wasm_i32x4_extract_lane(v, i) h2s_i32_lane((v), (i))

/* memory.atomic.wait32 / notify of the threaded build, on futexes (oracle/ref_host.c). */
int h2shim_wait32(int* addr, int expected, long long timeout_ns);
int h2shim_notify(int* addr, int count);
#define __builtin_wasm_memory_atomic_wait32(p, v, t) h2shim_wait32((p), (v), (long long)(t))
#define __builtin_wasm_memory_atomic_notify(p, n) h2shim_notify((p), (int)(n))

#endif
