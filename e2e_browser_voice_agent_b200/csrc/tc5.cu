// The multi-token Q4_0 matmul on the Blackwell tensor cores: tcgen05.mma (kind::i8) with TMEM accumulators, TMA
// for the activations, a warp-specialized pipeline. Bit-identical to the reference's matmul_q4 (kernels.c:200-273):
// the integer block dots are exact on the tensor cores and the float epilogue is the reference's, in its order.
//
// Arithmetic. For weight row n, token m and block b the reference forms four exact integer "lane" dots
// p_l = sum over lane l's 8 elements of (q - 8) x (lane l of the wasm i32x4 dot owns elements {2l, 2l+1, 8+2l, 9+2l}
// of each 16-value half, kernels.c:121-155, 173-188) and accumulates acc_l += f32(p_l) * (dw * dx) in block order,
// then returns ((acc_0 + acc_1) + acc_2) + acc_3 (kernels.c:230-267). In the device layout the 16 bytes of a Q4_0
// block are permuted so that 32-bit word l holds lane l's bytes (low nibbles: lane l's elements of the first half,
// high nibbles: of the second), and the int8 activations of a block are permuted the same way per half. So with
// K ordered as the activation bytes (32 per block), an A row that keeps only word l of weight row r, as signed bytes
// q - 8 (low nibbles at K = 4l..4l+3, high nibbles at K = 16+4l..16+4l+3, zeros elsewhere), dotted with a token's
// 32 activation bytes gives exactly p_l. One MMA (M = 128 = 32 weight rows x 4 lanes, N = tokens, K = 32 = one
// block) yields every lane dot of 32 rows x N tokens for one block, in its own TMEM columns. The columns are preset
// to the bit pattern 0x4B400000 (the float 12582912), so the accumulated result is the bit pattern of the float
// 12582912 + p_l, and subtracting 12582912 gives f32(p_l) exactly (|p_l| <= 8192). The epilogue then adds
// f32(p) * (dw * dx) into per-(row, lane, token) running sums in block order, with IEEE round-to-nearest multiplies
// and adds (packed f32x2 for the products; the running sums added as scalars, so no multiply-add is ever fused).
//
// CTA = 4 warps + 4 warps per epilogue warpgroup, one token group of NT = EW x NW tokens, a list of 32-row tiles:
//   warp 0 (lane 0)   producer: per chunk of 4 blocks, one TMA load of the token group's activation bytes (NT rows x
//                     128 B, 128-byte swizzle), one TMA load of their transposed block scales (4 x NT floats) and two
//                     bulk copies of the tile's 4 x 512 raw weight bytes and 4 x 32 fp16 scales, all completing on the
//                     chunk's mbarrier;
//   warp 1 (lane 0)   MMA issuer: one tcgen05.mma per block into a rotating TMEM slot, tcgen05.commit to release the
//                     A tile, signal the epilogue and (per chunk) release the stage; warp 1 also owns the TMEM
//                     allocation;
//   warps 2-3         converters: expand each block's nibbles into the lane-masked signed-byte A tile (the zero bytes
//                     of every A slot are written once at start);
//   warps 4..         epilogue warpgroups (NW tokens each): tcgen05.ld of the slot, re-arm it with the constant,
//                     release it, then the float chains; at the end of a tile ((l0 + l1) + l2) + l3 across the four
//                     lane threads of a row and the put() op (kernels.c:190-194).
// Every wait is bounded (%globaltimer, 1 s) and watches a CTA abort flag: on expiry the CTA records the failure in
// `err`, drains its copies and MMAs, frees its TMEM and returns.
#include "tc5.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

namespace h2 {
namespace {

constexpr int CB = 4;         // Q4_0 blocks per chunk (128 activation bytes per token: one 128-byte swizzle row)
constexpr int NA = 16;        // A-tile slots (4 chunks)
constexpr int ATILE = 4096;   // one A tile: 128 rows x 32 bytes, no swizzle (core matrices 8 rows x 16 B)
constexpr uint32_t FMAGIC = 0x4B400000u;
constexpr unsigned long long TIMEOUT_NS = 1000000000ull;

// Every hand-off between the roles is per chunk of 4 blocks (one mbarrier wait per role per chunk: a wait costs
// about 0.1 us even when the phase has completed, which per block was the pipeline's whole budget), and the rings are
// deep enough to cover one chunk's trip through the pipe (HBM load, conversion, MMA, epilogue: 4-5 us).
template <int NT>
struct Cfg {
  static constexpr int B_BYTES = NT * 128;
  static constexpr int RAW_BYTES = CB * 512 + CB * 64;  // values, then the fp16 scales of the 32 rows
  static constexpr int DX_BYTES = CB * NT * 4;
  static constexpr int STG = (B_BYTES + RAW_BYTES + DX_BYTES + 1023) / 1024 * 1024;
  static constexpr int NS = 8;                   // chunk stages
  static constexpr int NAC = NA / CB;            // A chunk slots
  static constexpr int NTC = NT <= 32 ? 4 : 2;   // TMEM chunk slots (CB blocks x NT columns each)
  static constexpr int COLS = NTC * CB * NT;     // 256, 512, 512: powers of two >= 32
  static constexpr int OFF_A = NS * STG;
  static constexpr int OFF_BAR = OFF_A + NA * ATILE;
  static constexpr int NBAR = 2 * NS + 2 * NAC + 2 * NTC + 1;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + alignment slack of the dynamic base
  static_assert(COLS <= 512 && SMEM <= 227 * 1024, "TMEM or shared memory budget");
};

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void bar_init(uint64_t* b, unsigned n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n));
}
__device__ __forceinline__ void bar_expect(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
// (with a suspend-time hint: a waiting thread sleeps in hardware until the phase completes, or at most ~20 us,
// instead of polling; polling warps crowd the shared-memory pipe that the working warps need)
__device__ __forceinline__ bool bar_try(uint64_t* b, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

struct Abort {
  volatile int* flag;  // shared: any role of the CTA raised it
  int* err;            // global: {code, CTA, role, 0}
};
__device__ __noinline__ void raise_abort(const Abort& a, int role) {
  if (atomicCAS(a.err, 0, 1) == 0) {
    a.err[1] = blockIdx.x;
    a.err[2] = role;
  }
  *a.flag = 1;
}
// bounded wait for the completion of the phase with this parity; false (abort raised) on expiry or abort
__device__ __forceinline__ bool wait_phase(uint64_t* b, unsigned parity, const Abort& a, int role) {
  if (bar_try(b, parity)) return true;
  const unsigned long long t0 = now_ns();
  for (unsigned it = 0;; it++) {
    if (bar_try(b, parity)) return true;
    if ((it & 3) == 3) {
      if (*a.flag) return false;
      if (now_ns() - t0 > TIMEOUT_NS) {
        raise_abort(a, role);
        return false;
      }
    }
  }
}
// the same for a whole warp: lane 0 polls (32 lanes polling one mbarrier serialize on it) and the warp follows;
// false on every lane if it failed
__device__ __forceinline__ bool wait_phase_warp(uint64_t* b, unsigned parity, const Abort& a, int role) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = wait_phase(b, parity, a, role);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}
// the same, ignoring the abort flag (teardown: copies or MMAs that were issued must complete)
__device__ __forceinline__ void drain_phase(uint64_t* b, unsigned parity) {
  const unsigned long long t0 = now_ns();
  while (!bar_try(b, parity))
    if (now_ns() - t0 > TIMEOUT_NS) return;
}

__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          su32(dst)),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(su32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk1d(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(su32(dst)),
               "l"(src), "r"(bytes), "r"(su32(bar))
               : "memory");
}

// shared-memory matrix descriptors (tcgen05): start address, leading / stride byte offsets (16-byte units), version 1
__device__ __forceinline__ uint64_t desc_plain(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) |
         (2ull << 61);
}

__device__ __forceinline__ void mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 columns of 32-bit words (lane = the thread's TMEM lane) into v[0..16)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
// every one of the NW columns of the warp's 32 lanes set to w
template <int NW>
__device__ __forceinline__ void tmem_fill(uint32_t taddr, uint32_t w);
template <>
__device__ __forceinline__ void tmem_fill<16>(uint32_t taddr, uint32_t w) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
      "%1};" ::"r"(taddr),
      "r"(w)
      : "memory");
}
template <>
__device__ __forceinline__ void tmem_fill<32>(uint32_t taddr, uint32_t w) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
      "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
      "r"(w)
      : "memory");
}

__device__ __forceinline__ unsigned long long pk(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ unsigned long long pk_add(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long pk_mul(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float lo_f(unsigned long long v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_f(unsigned long long v) { return __uint_as_float((uint32_t)(v >> 32)); }

enum { OPS = 0, OPB = 1, OPA = 2 };
enum { ROLE_PRODUCER = 1, ROLE_MMA = 2, ROLE_CONVERT = 3, ROLE_EPILOGUE = 4 };

template <int EW, int NW, int OP>
__global__ void __launch_bounds__(128 + 128 * EW, EW * NW <= 16 ? 2 : 1)
    k_matmul_tc5(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmD,
                 const uint8_t* __restrict__ qs, const __half* __restrict__ dsc, int N, int nb, int M,
                 float* __restrict__ y, int ldy, const float* __restrict__ bias, int* __restrict__ err,
                 int ctas_per_tg) {
  constexpr int NT = EW * NW;
  using C = Cfg<NT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (su32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);  // stage loaded (TMA / bulk copies)
  uint64_t* empty = full + C::NS;                                  // stage consumed by every role
  uint64_t* afull = empty + C::NS;                                 // A chunk written (converters)
  uint64_t* aempty = afull + C::NAC;                               // A chunk read (MMA commit)
  uint64_t* tfull = aempty + C::NAC;                               // TMEM chunk computed (MMA commit)
  uint64_t* tempty = tfull + C::NTC;                               // TMEM chunk read and re-armed (epilogue)
  uint64_t* done = tempty + C::NTC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* abort_s = reinterpret_cast<int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NS; s++) {
      bar_init(full + s, 1);
      bar_init(empty + s, 2 + 1 + 4 * EW);
    }
    for (int a = 0; a < C::NAC; a++) {
      bar_init(afull + a, 2);
      bar_init(aempty + a, 1);
    }
    for (int t = 0; t < C::NTC; t++) {
      bar_init(tfull + t, 1);
      bar_init(tempty + t, 4 * EW);
    }
    bar_init(done, 1);
    *abort_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "n"(C::COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == 2 || warp == 3) {  // the zero bytes of the lane-masked A tiles, once
    int4* a = reinterpret_cast<int4*>(sm + C::OFF_A);
    for (int i = threadIdx.x - 64; i < NA * ATILE / 16; i += 64) a[i] = make_int4(0, 0, 0, 0);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const Abort ab{abort_s, err};

  const int ntg = (M + NT - 1) / NT;
  const int tg = blockIdx.x % ntg, first_tile = blockIdx.x / ntg;
  const int m0 = tg * NT;
  const int ntiles = (N + 31) / 32;
  const int nchunk = (nb + CB - 1) / CB;

  if (warp == 0) {
    if (lane == 0) {  // ---------------- producer
      uint32_t ci = 0;
      for (int tile = first_tile; tile < ntiles; tile += ctas_per_tg) {
        for (int c = 0; c < nchunk; c++, ci++) {
          const int s = ci % C::NS;
          if (!wait_phase(empty + s, ((ci / C::NS) & 1) ^ 1, ab, ROLE_PRODUCER)) goto producer_done;
          const int b0 = c * CB, nbk = min(CB, nb - b0);
          uint8_t* stg = sm + s * C::STG;
          bar_expect(full + s, C::B_BYTES + nbk * (512 + 64) + C::DX_BYTES);
          tma2d(stg, &tmB, 32 * b0, m0, full + s);
          bulk1d(stg + C::B_BYTES, qs + ((size_t)tile * nb + b0) * 512, nbk * 512, full + s);
          bulk1d(stg + C::B_BYTES + CB * 512, dsc + ((size_t)tile * nb + b0) * 32, nbk * 64, full + s);
          tma2d(stg + C::B_BYTES + C::RAW_BYTES, &tmD, m0, b0, full + s);
        }
      }
    producer_done:
      for (uint32_t k = ci > C::NS ? ci - C::NS : 0; k < ci; k++) drain_phase(full + k % C::NS, (k / C::NS) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer
      const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NT >> 3) << 17) | (8u << 24);
      uint32_t ci = 0;
      for (int tile = first_tile; tile < ntiles; tile += ctas_per_tg) {
        for (int c = 0; c < nchunk; c++, ci++) {
          const int s = ci % C::NS, ac = ci % C::NAC, tc = ci % C::NTC;
          if (!wait_phase(full + s, (ci / C::NS) & 1, ab, ROLE_MMA)) goto mma_done;
          if (!wait_phase(afull + ac, (ci / C::NAC) & 1, ab, ROLE_MMA)) goto mma_done;
          if (!wait_phase(tempty + tc, (ci / C::NTC) & 1, ab, ROLE_MMA)) goto mma_done;
          tc_fence_after();
          const int nbk = min(CB, nb - c * CB);
          const uint32_t bbase = su32(sm + s * C::STG), abase = su32(sm + C::OFF_A + ac * CB * ATILE);
          for (int j = 0; j < nbk; j++)
            mma_i8(tmem + (tc * CB + j) * NT, desc_plain(abase + j * ATILE, 128, 256), desc_sw128(bbase + 32 * j, 1024),
                   idesc, 1);
          mma_commit(aempty + ac);
          mma_commit(tfull + tc);
          mma_commit(empty + s);
        }
      }
    mma_done:
      mma_commit(done);
      drain_phase(done, 0);
    }
  } else if (warp < 4) {  // ---------------- converters (warps 2, 3): 2 A rows of every block per thread
    const int t64 = threadIdx.x - 64;
    uint32_t ci = 0;
    for (int tile = first_tile; tile < ntiles; tile += ctas_per_tg) {
      for (int c = 0; c < nchunk; c++, ci++) {
        const int s = ci % C::NS, ac = ci % C::NAC;
        if (!wait_phase_warp(full + s, (ci / C::NS) & 1, ab, ROLE_CONVERT)) goto convert_done;
        if (!wait_phase_warp(aempty + ac, ((ci / C::NAC) & 1) ^ 1, ab, ROLE_CONVERT)) goto convert_done;
        const int nbk = min(CB, nb - c * CB);
        const uint32_t* raw = reinterpret_cast<const uint32_t*>(sm + s * C::STG + C::B_BYTES);
        uint32_t w[CB][2];
#pragma unroll
        for (int j = 0; j < CB; j++)  // every load of the chunk first
#pragma unroll
          for (int h = 0; h < 2; h++) w[j][h] = j < nbk ? raw[j * 128 + t64 + 64 * h] : 0u;  // row r word l = 4r + l
        uint8_t* A = sm + C::OFF_A + ac * CB * ATILE;
#pragma unroll
        for (int j = 0; j < CB; j++) {
          if (j < nbk) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
              const int i = t64 + 64 * h, l = i & 3;
              const uint32_t lo = ((w[j][h] & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;  // q - 8 as signed bytes
              const uint32_t hi = (((w[j][h] >> 4) & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
              const int o = j * ATILE + (i >> 3) * 256 + (i & 7) * 16 + 4 * l;
              *reinterpret_cast<uint32_t*>(A + o) = lo;
              *reinterpret_cast<uint32_t*>(A + o + 128) = hi;
            }
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          bar_arrive(afull + ac);
          bar_arrive(empty + s);
        }
      }
    }
  convert_done:;
  } else {  // ---------------- epilogue warpgroups
    const int ew = (warp - 4) >> 2, q = warp & 3;
    const int i = 32 * q + lane, r = i >> 2, l = i & 3;
    const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16) + ew * NW;
    for (int k = 0; k < C::NTC * CB; k++) tmem_fill<NW>(tl + k * NT, FMAGIC);
    tc_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int t = 0; t < C::NTC; t++) bar_arrive(tempty + t);
    const unsigned long long magic2 = pk(-12582912.0f, -12582912.0f);
    uint32_t ci = 0;
    for (int tile = first_tile; tile < ntiles; tile += ctas_per_tg) {
      float acc[NW];
#pragma unroll
      for (int t = 0; t < NW; t++) acc[t] = 0.f;
      for (int c = 0; c < nchunk; c++, ci++) {
        const int s = ci % C::NS, tc = ci % C::NTC;
        if (!wait_phase_warp(full + s, (ci / C::NS) & 1, ab, ROLE_EPILOGUE)) goto epi_done;
        if (!wait_phase_warp(tfull + tc, (ci / C::NTC) & 1, ab, ROLE_EPILOGUE)) goto epi_done;
        tc_fence_after();
        const int nbk = min(CB, nb - c * CB);
        const float* dxs = reinterpret_cast<const float*>(sm + s * C::STG + C::B_BYTES + C::RAW_BYTES);
        const __half* dws = reinterpret_cast<const __half*>(sm + s * C::STG + C::B_BYTES + CB * 512) + r;
#pragma unroll
        for (int jj = 0; jj < CB; jj += 2) {  // two blocks' columns in flight
          if (jj < nbk) {
            uint32_t u[2][NW];
#pragma unroll
            for (int e = 0; e < 2; e++)
              if (jj + e < nbk)
#pragma unroll
                for (int hh = 0; hh < NW / 16; hh++)
                  tmem_ld16(tl + (tc * CB + jj + e) * NT + 16 * hh, &u[e][16 * hh]);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 2; e++) {
              if (jj + e < nbk) {
                const int j = jj + e;
                const float dw = __half2float(dws[j * 32]);
                const unsigned long long dw2 = pk(dw, dw);
                const float* dxr = dxs + j * NT + ew * NW;
#pragma unroll
                for (int k = 0; k < NW / 4; k++) {
                  const float4 d4 = *reinterpret_cast<const float4*>(dxr + 4 * k);
                  const unsigned long long s01 = pk_mul(dw2, pk(d4.x, d4.y)), s23 = pk_mul(dw2, pk(d4.z, d4.w));
                  const unsigned long long p01 =
                      pk_add(pk(__uint_as_float(u[e][4 * k]), __uint_as_float(u[e][4 * k + 1])), magic2);
                  const unsigned long long p23 =
                      pk_add(pk(__uint_as_float(u[e][4 * k + 2]), __uint_as_float(u[e][4 * k + 3])), magic2);
                  const unsigned long long q01 = pk_mul(p01, s01), q23 = pk_mul(p23, s23);
                  acc[4 * k] = __fadd_rn(acc[4 * k], lo_f(q01));
                  acc[4 * k + 1] = __fadd_rn(acc[4 * k + 1], hi_f(q01));
                  acc[4 * k + 2] = __fadd_rn(acc[4 * k + 2], lo_f(q23));
                  acc[4 * k + 3] = __fadd_rn(acc[4 * k + 3], hi_f(q23));
                }
              }
            }
          }
        }
#pragma unroll
        for (int j = 0; j < CB; j++) tmem_fill<NW>(tl + (tc * CB + j) * NT, FMAGIC);  // re-arm the chunk's columns
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          bar_arrive(tempty + tc);
          bar_arrive(empty + s);
        }
      }
      {  // the tile is complete: ((l0 + l1) + l2) + l3 across the row's four lane threads, then put()
        const int n = tile * 32 + r;
#pragma unroll
        for (int t = 0; t < NW; t++) {
          const float v0 = acc[t];
          const float v1 = __shfl_down_sync(0xffffffffu, v0, 1), v2 = __shfl_down_sync(0xffffffffu, v0, 2),
                      v3 = __shfl_down_sync(0xffffffffu, v0, 3);
          const int m = m0 + ew * NW + t;
          if (l == 0 && n < N && m < M) {
            const float v = __fadd_rn(__fadd_rn(__fadd_rn(v0, v1), v2), v3);
            float* o = y + (size_t)m * ldy + n;
            if (OP == OPA) *o = __fadd_rn(*o, v);
            else if (OP == OPB) *o = __fadd_rn(v, bias[n]);
            else *o = v;
          }
        }
      }
    }
  epi_done:;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(C::COLS) : "memory");
  }
}

// ---------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// The tensor maps of one launch, cached by their arguments (the engine's buffers repeat from call to call).
struct MapKey {
  const void* ptr;
  uint64_t d0, d1, stride;
  uint32_t b0, b1;
  int kind;
  bool operator==(const MapKey& o) const { return memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapEntry {
  MapKey k;
  CUtensorMap m;
};

bool make_map(CUtensorMap* out, int kind, const void* ptr, uint64_t d0, uint64_t d1, uint64_t stride, uint32_t b0,
              uint32_t b1) {
  thread_local MapEntry cache[32];
  thread_local int next = 0;
  MapKey key;
  memset(&key, 0, sizeof key);
  key.ptr = ptr; key.d0 = d0; key.d1 = d1; key.stride = stride; key.b0 = b0; key.b1 = b1; key.kind = kind;
  for (auto& e : cache)
    if (e.k == key) {
      *out = e.m;
      return true;
    }
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {d0, d1};
  const cuuint64_t strides[1] = {stride};
  const cuuint32_t box[2] = {b0, b1};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(out, kind == 0 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  kind == 0 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  cache[next].k = key;
  cache[next].m = *out;
  next = (next + 1) % 32;
  return true;
}

template <int EW, int NW>
cudaError_t launch_inst(int op, const CUtensorMap& mb, const CUtensorMap& md, const uint8_t* qs, const __half* dsc,
                        int N, int nb, int M, float* y, int ldy, const float* bias, int* err, cudaStream_t st) {
  constexpr int NT = EW * NW;
  const int ntg = (M + NT - 1) / NT, ntiles = (N + 31) / 32;
  const int per_sm = NT <= 16 ? 2 : 1;
  const int ctas = std::max(1, std::min(ntiles, 148 * per_sm / ntg));
  const dim3 grid(ntg * ctas), block(128 + 128 * EW);
  const size_t smem = Cfg<NT>::SMEM;
  if (op == OPS) k_matmul_tc5<EW, NW, OPS><<<grid, block, smem, st>>>(mb, md, qs, dsc, N, nb, M, y, ldy, bias, err, ctas);
  else if (op == OPB) k_matmul_tc5<EW, NW, OPB><<<grid, block, smem, st>>>(mb, md, qs, dsc, N, nb, M, y, ldy, bias, err, ctas);
  else k_matmul_tc5<EW, NW, OPA><<<grid, block, smem, st>>>(mb, md, qs, dsc, N, nb, M, y, ldy, bias, err, ctas);
  return cudaGetLastError();
}

template <int EW, int NW>
cudaError_t attrs_inst() {
  const int smem = Cfg<EW * NW>::SMEM;
  cudaError_t c = cudaFuncSetAttribute(k_matmul_tc5<EW, NW, OPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_matmul_tc5<EW, NW, OPB>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_matmul_tc5<EW, NW, OPA>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  return c;
}

}  // namespace

int tc5_tokens_per_cta(int M, int N) {  // (16, 32 or 64)
  // the widest token group (fewest passes over the weights) that still gives every SM a CTA; the narrowest otherwise
  const int ntiles = (N + 31) / 32;
  for (int nt = 64; nt >= 16; nt /= 2) {
    if (nt > 16 && (M + nt / 2 - 1) / (nt / 2) == 1) continue;  // a narrower group already holds every token
    if ((long long)ntiles * ((M + nt - 1) / nt) >= 148) return nt;
  }
  return 16;
}

cudaError_t tc5_set_attrs() {
  cudaError_t c = attrs_inst<1, 16>();
  if (c == cudaSuccess) c = attrs_inst<1, 32>();
  if (c == cudaSuccess) c = attrs_inst<2, 32>();
  return c;
}

cudaError_t launch_tc5(int op, const uint8_t* qs, const __half* dsc, int N, int K, const int8_t* xq, int xq_rows,
                       const float* xdT, int ldT, int M, float* y, int ldy, const float* bias, int* err,
                       cudaStream_t st) {
  if (N < 1 || K < 32 || K % 32 || M < 1 || xq_rows < M || ldT < M || ldT % 4 || !err) return cudaErrorInvalidValue;
  if (((uintptr_t)xq | (uintptr_t)xdT | (uintptr_t)qs) & 15) return cudaErrorInvalidValue;
  const int NT = tc5_tokens_per_cta(M, N), nb = K / 32;
  CUtensorMap mb, md;
  if (!make_map(&mb, 0, xq, (uint64_t)K, (uint64_t)xq_rows, (uint64_t)K, 128, (uint32_t)NT) ||
      !make_map(&md, 1, xdT, (uint64_t)ldT, (uint64_t)nb, (uint64_t)ldT * 4, (uint32_t)NT, CB))
    return cudaErrorInvalidValue;
  switch (NT) {
    case 16: return launch_inst<1, 16>(op, mb, md, qs, dsc, N, nb, M, y, ldy, bias, err, st);
    case 32: return launch_inst<1, 32>(op, mb, md, qs, dsc, N, nb, M, y, ldy, bias, err, st);
    default: return launch_inst<2, 32>(op, mb, md, qs, dsc, N, nb, M, y, ldy, bias, err, st);
  }
}

}  // namespace h2
