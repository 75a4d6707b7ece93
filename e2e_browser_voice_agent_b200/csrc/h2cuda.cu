// h2cuda: C-ABI implementation (include/h2cuda.h). The engine owns device weights, KV cache, scratch and the
// CUDA graph of one decode step; callers pass host pointers only.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <atomic>
#include <mutex>
#include <chrono>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "../../include/h2cuda.h"
#include "decode_mk.cuh"
#include "kernels.cuh"
#include "prompt_att.cuh"
#include "sample.cuh"
#include "tc5.cuh"

using namespace h2;

namespace {

thread_local std::string g_create_error;

// The multi-token matmul kernel (h2c_set_matmul_kernel): H2C_MATMUL_TCGEN05 takes the tcgen05 form (tc5.cu) for
// Q4_0 matrices, H2C_MATMUL_MMA_SYNC the warp-level int8 mma.sync form (k_matmul_tc); H2C_MATMUL_AUTO the tcgen05 form
// for passes of TC5_MIN_TOKENS or more tokens and the mma.sync form below (measured on B200: at 32 tokens the
// mma.sync form is 1.2-2x faster, from 64 tokens on the tcgen05 form is as fast or up to 1.8x faster).
constexpr int TC5_MIN_TOKENS = 64;
// Prompt passes of this many tokens or more (one sequence) take the tiled prompt attention (prompt_att.cuh).
constexpr int PF_MIN_TOKENS = 32;
std::atomic<int> g_mm_kind{H2C_MATMUL_AUTO};
bool use_tc5(int M) {
  const int k = g_mm_kind.load(std::memory_order_relaxed);
  return k == H2C_MATMUL_TCGEN05 || (k == H2C_MATMUL_AUTO && M >= TC5_MIN_TOKENS);
}

// NCCL for tensor-parallel engines (h2c_create_tp), resolved at run time from the libnccl.so.2 the process has (a
// PyTorch host has already loaded its own) or the system's, so single-GPU users need none. Communicators are created
// non-blocking: every call that answers ncclInProgress is polled to completion against a deadline, and a peer that
// never joins or stops answering ends in ncclCommAbort and an error instead of a wait without end.
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*finalize)(ncclComm_t) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  std::string why;  // empty when every entry point resolved
};
const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* d = dlerror();
      api.why = std::string("libnccl.so.2 not found: ") + (d ? d : "");
      return;
    }
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (!fn && api.why.empty()) api.why = std::string("libnccl.so.2 lacks ") + name;
    };
    sym(api.get_unique_id, "ncclGetUniqueId");
    sym(api.init_rank_config, "ncclCommInitRankConfig");
    sym(api.all_gather, "ncclAllGather");
    sym(api.group_start, "ncclGroupStart");
    sym(api.group_end, "ncclGroupEnd");
    sym(api.async_error, "ncclCommGetAsyncError");
    sym(api.finalize, "ncclCommFinalize");
    sym(api.destroy, "ncclCommDestroy");
    sym(api.abort, "ncclCommAbort");
    sym(api.error_string, "ncclGetErrorString");
  });
  return api;
}

// What the tcgen05 matmul needs besides the activations: the transposed block scales, the rows of the activation
// buffer, and the device word its bounded waits report into.
struct MmCtx {
  const float* xdT;
  int ldT;
  int xq_rows;
  int* err;
  bool* used;  // set when a launch took the tcgen05 form
};

struct Q4Mat {
  uint8_t* qs = nullptr;
  __half* d = nullptr;
  int N = 0, K = 0;
};
struct Q8Mat {
  int8_t* qs = nullptr;
  __half* d = nullptr;
  int N = 0, K = 0;
};
struct LayerW {
  Q4Mat qkv, o, gu, down;
  float *attn_norm = nullptr, *ffn_norm = nullptr, *bqkv = nullptr;
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

struct h2c_engine {
  h2c_config cfg{};
  int dev = 0, HD = 0, QKV = 0;
  std::vector<LayerW> L;
  Q4Mat embd;
  Q4Mat out4;
  Q8Mat out8;
  int out_type = -1;  // -1 tied to embd, 2 Q4_0, 8 Q8_0
  float* out_norm = nullptr;
  float* rope = nullptr;
  float *kc = nullptr, *vc = nullptr;
  float *x = nullptr, *qkv = nullptr, *att = nullptr, *gu = nullptr, *logits = nullptr;
  int8_t* xq = nullptr;
  float* xd = nullptr;
  int4* xs = nullptr;
  float* xdT = nullptr;         // block scales transposed, [max(D, F) / 32][ldT] (tcgen05 matmul)
  int ldT = 0;
  float* pf_s = nullptr;        // prompt attention: scores / exponentials of a pass (prompt_att.cuh), pf_bytes
  float* pf_sum = nullptr;      // and the rows' sums, [heads x max_chunk]
  float* pf_pm = nullptr;       // and the rows' maxima per 64 positions, [heads x max_chunk][pf_pm_pitch(ctx)]
  size_t pf_bytes = 0;          // 0: prompt passes take the per-token attention
  int* tc5_err = nullptr;       // device: the tcgen05 matmul's failure record
  int32_t* tc5_err_h = nullptr; // pinned copy
  bool tc5_used = false;        // a pass of the current call took the tcgen05 matmul (its record is copied back)
  float* am_v = nullptr;
  int* am_i = nullptr;
  int am_np = 0;
  int32_t* prm = nullptr;      // device params [P_WORDS]
  int32_t* next_d = nullptr;   // device next token
  int32_t* toklog = nullptr;   // device token log [max_seqs][ctx + 1]
  int graph_kernels = 0;       // kernel nodes in the decode-step graph
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  int32_t* prm_h = nullptr;    // pinned host params, one slot per chunk of a forward
  int prm_slots = 0;
  int32_t* next_h = nullptr;   // pinned
  cudaStream_t st = nullptr;
  cudaGraphExec_t gexec = nullptr;
  cudaGraph_t graph = nullptr;
  // batched decode steps (h2c_forward_batch): logits of every token, per-token argmax partials, the tokens, and
  // one CUDA graph per batch size
  float* logits_b = nullptr;
  float* am_vb = nullptr;
  int* am_ib = nullptr;
  int32_t* next_b = nullptr;
  int32_t* prm_bh = nullptr;   // pinned [P_WORDS]
  // temperature sampling on the device (sample.cu): scratch for up to P_CAP rows, per-token seeds
  void* samp = nullptr;
  uint32_t* seeds_d = nullptr;  // [P_CAP]
  uint32_t* seeds_h = nullptr;  // pinned [P_CAP]
  int32_t* next_bh = nullptr;  // pinned [P_CAP]
  std::vector<cudaGraphExec_t> bexec;
  std::vector<int> bkernels;   // kernel nodes of each batch graph
  std::vector<char> btc5;      // the batch graph of that size contains tcgen05 matmuls
  std::string err;
  int64_t dev_bytes = 0;
  std::vector<void*> dallocs;
  std::vector<int> layer_set;  // bit mask of kinds 0..6 set per layer
  bool embd_set = false, out_norm_set = false;
  std::vector<int> last_logits_valid;
  // persistent decode kernel (decode_mk.cuh)
  int decode_mode = H2C_DECODE_AUTO;
  bool mk_built = false, mk_ok = false;
  std::string mk_why;
  int mk_ncta = 0, mk_tile_stride = 0, mk_prod_items = 0, mk_kv_stage = 0;
  size_t mk_smem = 0;
  uint8_t* mk_stream = nullptr;
  MkTile* mk_tiles = nullptr;
  float *mk_attn_norm = nullptr, *mk_ffn_norm = nullptr, *mk_bqkv = nullptr;
  unsigned long long *mk_xw = nullptr, *mk_qw = nullptr, *mk_kvw = nullptr, *mk_attw = nullptr, *mk_actw = nullptr,
                     *mk_lmw = nullptr, *mk_kvdone = nullptr, *mk_rawact = nullptr, *mk_lcmax = nullptr,
                     *mk_lce = nullptr, *mk_lcsum = nullptr;
  int mk_nsplit = 0;
  uint32_t mk_epoch = 0, mk_lm_epoch = 0;  // tag epochs used by earlier launches
  bool mk_io_dirty = true;                   // error words must be cleared before the next launch
  int mk_stall_cta = -1;                          // h2c_set_decode_fault
  unsigned long long mk_timeout_ns = 2000000000ull;
  void* mk_kernel = nullptr;        // the k_decode_persistent instance for this model's shape
  void* mk_kernel_trace = nullptr;  // the same with the timestamp trace compiled in
  void* mk_kernel_lc = nullptr;     // for launches that reach positions beyond mk_kv_stage (long-context attention)
  size_t mk_tagged_words = 0;  // mk_xw .. mk_kvdone are one allocation of this many words
  int32_t* mk_io = nullptr;   // device: [0] next token, [4..7] error words
  int* mk_tile_count = nullptr;
  int32_t* mk_io_h = nullptr; // pinned
  int32_t* mk_done_h = nullptr;  // mapped pinned record CTA 0 writes when a single-token launch finishes
  int32_t* mk_done_d = nullptr;  // its device alias
  int32_t mk_launch_seq = 0;
  bool mk_pending = false;    // the last pass of the current forward ran on the persistent kernel
  // tensor parallelism (h2c_create_tp). Every matrix is split by output rows, so each row is computed whole, in the
  // reference's order, by one rank: this rank holds its heads' q/k/v rows (Hl query and KVHl kv heads) and their
  // KV cache, Dl = D / G rows of O and of down, Fl = F / G rows of gate and of up, and Vl rows of the lm_head
  // (rank r from row r * Vp). NCCL all-gathers give every rank the full vectors between the matrices; the
  // normalisations and quantizations of full vectors run on every rank. Without TP: G = 1 and the full sizes.
  int tp_rank = 0, tp_world = 1;
  ncclComm_t comm = nullptr;
  bool comm_dead = false;        // aborted after a failure: passes are refused
  int64_t tp_timeout_ms = 0;     // deadline of NCCL set-up, of enqueueing and of a pass's completion
  std::string tp_fail;           // first NCCL failure inside an enqueue (reported after it)
  int Hl = 0, KVHl = 0, Dl = 0, Fl = 0, Vp = 0, Vl = 0;
  // one-token passes exchange over peer memory instead: each rank's buffers that receive other ranks' slices are
  // mapped into every rank (CUDA IPC), a copy kernel writes this rank's slice into each peer's buffer and counts
  // its arrival there, and waits (bounded) until every peer's slice has arrived here (k_xch)
  bool xch = false;
  void* xtab_d = nullptr;                 // XchTab on the device: every rank's buffer bases
  std::vector<void*> ipc_open;            // peer mappings (closed on destroy)
  unsigned long long* xcnt = nullptr;     // [0] pass epoch, [1 + slot] arrivals, [4 L + 2] logits epoch
  int32_t* xerr_h = nullptr;              // mapped pinned: {1, slot, 0, 0} when a wait expired
  int32_t* xerr_d = nullptr;
  int8_t* actq = nullptr;                 // the FFN activation received for the down matrix (one token)
  float* actd = nullptr;
  int4* acts = nullptr;
  uint8_t* tp_send = nullptr;    // passes of several tokens: this rank's columns, packed, before a gather
  uint8_t* tp_recv = nullptr;    // ... and the gathered [G][M][columns], before they are unpacked into [M][full row]
  size_t tp_stage = 0;           // bytes of tp_send (tp_recv has G times as many)

  int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    err = buf;
    return code;
  }
};

#define CUDA_TRY(e, call)                                                                          \
  do {                                                                                             \
    cudaError_t _c = (call);                                                                       \
    if (_c != cudaSuccess) return (e)->fail(H2C_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(_c)); \
  } while (0)

namespace {

int dalloc(h2c_engine* e, void** p, size_t bytes) {
  cudaError_t c = cudaMalloc(p, bytes);
  if (c != cudaSuccess) {
    *p = nullptr;
    return e->fail(c == cudaErrorMemoryAllocation ? H2C_ERR_NO_MEMORY : H2C_ERR_CUDA, "cudaMalloc(%zu): %s", bytes,
                   cudaGetErrorString(c));
  }
  e->dallocs.push_back(*p);
  e->dev_bytes += (int64_t)bytes;
  c = cudaMemset(*p, 0, bytes);
  if (c != cudaSuccess) return e->fail(H2C_ERR_CUDA, "cudaMemset: %s", cudaGetErrorString(c));
  return H2C_OK;
}

template <typename T>
int dalloc_t(h2c_engine* e, T** p, size_t count) {
  return dalloc(e, reinterpret_cast<void**>(p), count * sizeof(T));
}

// GGUF blocks -> device layout (kernels.cuh): rows in groups of 32, [group][block][32 rows][BB bytes] with each
// 16-byte half permuted so that 32-bit word l holds lane l's bytes, and fp16 scales [group][block][32 rows].
// Rows past N (padding to a multiple of 32) are zero. src_block_bytes: 18 (Q4_0) or 34 (Q8_0).
void pack_blocks_host(const uint8_t* src, int N, int K, int src_block_bytes, uint8_t* dst_qs, uint16_t* dst_d) {
  const int nb = K / 32, BB = src_block_bytes - 2, Np = (N + 31) / 32 * 32;
  memset(dst_qs, 0, (size_t)Np * nb * BB);
  memset(dst_d, 0, (size_t)Np * nb * 2);
  for (int n = 0; n < N; n++) {
    const int g = n >> 5, r = n & 31;
    for (int b = 0; b < nb; b++) {
      const uint8_t* s = src + ((size_t)n * nb + b) * src_block_bytes;
      const size_t e = ((size_t)g * nb + b) * 32 + r;
      dst_d[e] = (uint16_t)(s[0] | (s[1] << 8));
      uint8_t* d = dst_qs + e * BB;
      for (int h = 0; h < BB; h += 16)
        for (int p = 0; p < 16; p++) d[h + p] = s[2 + h + perm16(p)];
    }
  }
}

size_t padded_rows(int N) { return (size_t)(N + 31) / 32 * 32; }

int upload_q4(h2c_engine* e, Q4Mat* m, int N, int K, const void* data, uint64_t nbytes) {
  const int64_t nb = (int64_t)N * (K / 32);
  if ((uint64_t)nb * 18 != nbytes) return e->fail(H2C_ERR_INVALID, "Q4_0 tensor %dx%d: %llu bytes, expected %lld", N, K,
                                                  (unsigned long long)nbytes, (long long)(nb * 18));
  const size_t nbp = padded_rows(N) * (K / 32);
  if (!m->qs) {
    int r = dalloc_t(e, &m->qs, nbp * 16);
    if (r) return r;
    r = dalloc_t(e, &m->d, nbp);
    if (r) return r;
  }
  std::vector<uint8_t> qs(nbp * 16);
  std::vector<uint16_t> d(nbp);
  pack_blocks_host((const uint8_t*)data, N, K, 18, qs.data(), d.data());
  CUDA_TRY(e, cudaMemcpy(m->qs, qs.data(), qs.size(), cudaMemcpyHostToDevice));
  CUDA_TRY(e, cudaMemcpy(m->d, d.data(), d.size() * 2, cudaMemcpyHostToDevice));
  m->N = N;
  m->K = K;
  return H2C_OK;
}

int upload_q8(h2c_engine* e, Q8Mat* m, int N, int K, const void* data, uint64_t nbytes) {
  const int64_t nb = (int64_t)N * (K / 32);
  if ((uint64_t)nb * 34 != nbytes) return e->fail(H2C_ERR_INVALID, "Q8_0 tensor %dx%d: %llu bytes, expected %lld", N, K,
                                                  (unsigned long long)nbytes, (long long)(nb * 34));
  const size_t nbp = padded_rows(N) * (K / 32);
  if (!m->qs) {
    int r = dalloc_t(e, &m->qs, nbp * 32);
    if (r) return r;
    r = dalloc_t(e, &m->d, nbp);
    if (r) return r;
  }
  std::vector<uint8_t> qs(nbp * 32);
  std::vector<uint16_t> d(nbp);
  pack_blocks_host((const uint8_t*)data, N, K, 34, qs.data(), d.data());
  CUDA_TRY(e, cudaMemcpy(m->qs, qs.data(), qs.size(), cudaMemcpyHostToDevice));
  CUDA_TRY(e, cudaMemcpy(m->d, d.data(), d.size() * 2, cudaMemcpyHostToDevice));
  m->N = N;
  m->K = K;
  return H2C_OK;
}

int upload_f32(h2c_engine* e, float** p, int64_t count, const void* data, uint64_t nbytes) {
  if ((uint64_t)count * 4 != nbytes)
    return e->fail(H2C_ERR_INVALID, "F32 tensor: %llu bytes, expected %lld", (unsigned long long)nbytes, (long long)count * 4);
  if (!*p) {
    int r = dalloc_t(e, p, (size_t)count);
    if (r) return r;
  }
  CUDA_TRY(e, cudaMemcpy(*p, data, nbytes, cudaMemcpyHostToDevice));
  return H2C_OK;
}

// ---------------------------------------------------------------- launch helpers

// Launch shapes: one token (the graph decode step) runs k_matvec on 32-row tiles (16 for long rows, to bound
// shared memory); passes of several tokens run k_matmul (below).
template <int WT, int ROWS, int MB>
void launch_mv_t(int op, const uint8_t* qs, const __half* d, int N, int K, const int8_t* xq, const float* xd,
                 const int4* xs, int M, float* y, int ldy, const float* bias, cudaStream_t st) {
  const int blocks = (int)(padded_rows(N) / ROWS);
  const size_t smem = (size_t)MB * (K / 32) * ROWS * 16;
  if (op == OP_STORE) k_matvec<WT, ROWS, MB, OP_STORE><<<blocks, 256, smem, st>>>(qs, d, N, K, xq, xd, xs, M, y, ldy, bias);
  else if (op == OP_BIAS) k_matvec<WT, ROWS, MB, OP_BIAS><<<blocks, 256, smem, st>>>(qs, d, N, K, xq, xd, xs, M, y, ldy, bias);
  else k_matvec<WT, ROWS, MB, OP_ADD><<<blocks, 256, smem, st>>>(qs, d, N, K, xq, xd, xs, M, y, ldy, bias);
}

// One token: k_mv with 32-row CTAs when the matrix has enough rows for two CTAs per SM and rows of at most 256
// blocks, else 8-row CTAs (more CTAs for short matrices, shorter chunks of long rows). Returns false for matrices
// of many short rows (fewer than 64 blocks, e.g. the 0.5B output matrix: 24.6 us on k_matvec against 35.7 us here,
// where each CTA's few chunks leave its pipeline unfilled); k_matvec then takes the call.
constexpr size_t MV_SMEM = 227 * 1024;
template <int WT, int R>
void launch_mv_r(int op, const uint8_t* qs, const __half* d, int N, int K, const int8_t* xq, const float* xd,
                 const int4* xs, float* y, const float* bias, cudaStream_t st) {
  const int blocks = (int)(padded_rows(N) / R);
  const size_t smem = mv_smem_bytes<WT, R>();
  if (op == OP_STORE) k_mv<WT, R, OP_STORE><<<blocks, 256, smem, st>>>(qs, d, N, K, xq, xd, xs, y, bias);
  else if (op == OP_BIAS) k_mv<WT, R, OP_BIAS><<<blocks, 256, smem, st>>>(qs, d, N, K, xq, xd, xs, y, bias);
  else k_mv<WT, R, OP_ADD><<<blocks, 256, smem, st>>>(qs, d, N, K, xq, xd, xs, y, bias);
}
template <int WT>
bool launch_mv(int op, const uint8_t* qs, const __half* d, int N, int K, const int8_t* xq, const float* xd,
               const int4* xs, float* y, const float* bias, cudaStream_t st) {
  const bool many = padded_rows(N) / 32 >= 296;
  if (many && K / 32 < 64) return false;
  const bool wide = many && K / 32 <= 256;
  if (wide) launch_mv_r<WT, 32>(op, qs, d, N, K, xq, xd, xs, y, bias, st);
  else launch_mv_r<WT, 8>(op, qs, d, N, K, xq, xd, xs, y, bias, st);
  return true;
}
// One token on the tensor cores (k_mvt) for matrices of at least 296 groups of 32 rows (gate/up, the output matrix):
// CTAs of 2 warps x 32 rows with 5-chunk rings of 8 blocks (four CTAs per SM, 18 KB of weights in flight per warp).
// Returns false for the other matrices (k_mv takes them: their few rows need the blocks of a row spread over many
// threads) and when the staging does not fit.
template <int WT, int W, int RG, int NSTG, int CK>
void launch_mvt_w(int op, const uint8_t* qs, const __half* d, int N, int K, const int8_t* xq, const float* xd,
                  const int4* xs, float* y, const float* bias, cudaStream_t st) {
  const int blocks = (int)((padded_rows(N) / (8 * RG) + W - 1) / W);
  const size_t smem = mt_smem_bytes<WT, W, RG, NSTG, CK>(K);
  if (op == OP_STORE) k_mvt<WT, W, RG, NSTG, CK, OP_STORE><<<blocks, W * 32, smem, st>>>(qs, d, N, K, xq, xd, xs, y, bias);
  else if (op == OP_BIAS) k_mvt<WT, W, RG, NSTG, CK, OP_BIAS><<<blocks, W * 32, smem, st>>>(qs, d, N, K, xq, xd, xs, y, bias);
  else k_mvt<WT, W, RG, NSTG, CK, OP_ADD><<<blocks, W * 32, smem, st>>>(qs, d, N, K, xq, xd, xs, y, bias);
}
template <int WT>
bool launch_mvt(int op, const uint8_t* qs, const __half* d, int N, int K, const int8_t* xq, const float* xd,
                const int4* xs, float* y, const float* bias, cudaStream_t st) {
  // (rows of fewer than 64 blocks, e.g. the 0.5B output matrix, are faster on k_matvec: 24.6 against 32.6 us)
  const bool wide = padded_rows(N) / 32 >= 296 && K / 32 >= 64;
  if (!wide || mt_smem_bytes<WT, 2, 4, 5, 8>(K) > MV_SMEM) return false;
  launch_mvt_w<WT, 2, 4, 5, 8>(op, qs, d, N, K, xq, xd, xs, y, bias, st);
  return true;
}
template <int WT, int W, int RG, int NSTG, int CK>
cudaError_t mvt_attr() {
  const int smem = (int)MV_SMEM;
  cudaError_t c = cudaFuncSetAttribute(k_mvt<WT, W, RG, NSTG, CK, OP_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_mvt<WT, W, RG, NSTG, CK, OP_BIAS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_mvt<WT, W, RG, NSTG, CK, OP_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  return c;
}

template <int WT, int R>
cudaError_t mv2_attr() {
  const int smem = (int)MV_SMEM;
  cudaError_t c = cudaFuncSetAttribute(k_mv<WT, R, OP_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_mv<WT, R, OP_BIAS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_mv<WT, R, OP_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  return c;
}

// Several tokens (prompt chunks, batched decode steps): k_matmul with token groups of 32, 16 or 8 (the largest whose
// activations fit next to the weight ring in a third of an SM's shared memory, so three CTAs share an SM) and row
// ranges that give about four CTAs per SM.
constexpr size_t MM_SMEM = 160 * 1024;   // attribute limit (long rows)
constexpr size_t MM_SMEM_FAST = 72 * 1024;
template <int WT, int TG, int RT>
size_t mm_smem(int nb) { return (size_t)mm_act_bytes(TG, nb) + 2 * (size_t)mm_chunk_bytes(WT, (256 / (4 * TG)) * RT); }

template <int WT, int TG, int RT>
void launch_mm_t(int op, const uint8_t* qs, const __half* d, int N, int K, const int8_t* xq, const float* xd,
                 const int4* xs, int M, float* y, int ldy, const float* bias, cudaStream_t st) {
  constexpr int SR = (256 / (4 * TG)) * RT;
  const int ntg = (M + TG - 1) / TG;
  const int nrr = std::max(1, 4 * 148 / ntg);
  const int rows = std::max(SR, N / nrr / SR * SR);
  const int grid = ntg * ((N + rows - 1) / rows);
  const size_t smem = mm_smem<WT, TG, RT>(K / 32);
  if (op == OP_STORE) k_matmul<WT, TG, RT, OP_STORE><<<grid, 256, smem, st>>>(qs, d, N, K, xq, xd, xs, M, rows, y, ldy, bias);
  else if (op == OP_BIAS) k_matmul<WT, TG, RT, OP_BIAS><<<grid, 256, smem, st>>>(qs, d, N, K, xq, xd, xs, M, rows, y, ldy, bias);
  else k_matmul<WT, TG, RT, OP_ADD><<<grid, 256, smem, st>>>(qs, d, N, K, xq, xd, xs, M, rows, y, ldy, bias);
}

// 8 rows per thread when the matrix is tall enough to keep every SM busy with them, else 2
template <int WT, int TG>
void launch_mm(int op, const uint8_t* qs, const __half* d, int N, int K, const int8_t* xq, const float* xd,
               const int4* xs, int M, float* y, int ldy, const float* bias, cudaStream_t st) {
  const int ntg = (M + TG - 1) / TG;
  if ((size_t)N * ntg >= (size_t)4 * 148 * (256 / (4 * TG)) * 8)
    launch_mm_t<WT, TG, 8>(op, qs, d, N, K, xq, xd, xs, M, y, ldy, bias, st);
  else
    launch_mm_t<WT, TG, 2>(op, qs, d, N, K, xq, xd, xs, M, y, ldy, bias, st);
}

// The tensor-core form: 32-row sub-ranges; token groups of 32, 16 or 8, the largest that still gives one CTA per SM
// and fits two CTAs' shared memory per SM.
constexpr size_t MMTC_SMEM_FAST = 110 * 1024;
template <int WT, int TG>
size_t mmtc_smem(int nb) { return (size_t)mt_smem_bytes(WT, TG, nb); }

template <int WT, int TG>
void launch_mmtc(int op, const uint8_t* qs, const __half* d, int N, int K, const int8_t* xq, const float* xd,
                 const int4* xs, int M, float* y, int ldy, const float* bias, cudaStream_t st) {
  const int ntg = (M + TG - 1) / TG;
  const int groups = (N + 31) / 32;
  const int nrr = std::max(1, 4 * 148 / ntg);
  const int rows = 32 * std::max(1, groups / nrr);
  const int grid = ntg * ((N + rows - 1) / rows);
  const size_t smem = mmtc_smem<WT, TG>(K / 32);
  if (op == OP_STORE) k_matmul_tc<WT, TG, OP_STORE><<<grid, 256, smem, st>>>(qs, d, N, K, xq, xd, xs, M, rows, y, ldy, bias);
  else if (op == OP_BIAS) k_matmul_tc<WT, TG, OP_BIAS><<<grid, 256, smem, st>>>(qs, d, N, K, xq, xd, xs, M, rows, y, ldy, bias);
  else k_matmul_tc<WT, TG, OP_ADD><<<grid, 256, smem, st>>>(qs, d, N, K, xq, xd, xs, M, rows, y, ldy, bias);
}

// (st null: only report whether a token group of the mma.sync form fits the row length)
template <int WT>
bool matmul_tc(int op, const uint8_t* qs, const __half* d, int N, int K, const int8_t* xq, const float* xd,
               const int4* xs, int M, float* y, int ldy, const float* bias, cudaStream_t st, bool dry = false) {
  const int nb = K / 32, groups = (N + 31) / 32;
  auto enough = [&](int tg) { return (size_t)((M + tg - 1) / tg) * groups >= 148; };
  if (M > 16 && enough(32) && mmtc_smem<WT, 32>(nb) <= MMTC_SMEM_FAST) {
    if (!dry) launch_mmtc<WT, 32>(op, qs, d, N, K, xq, xd, xs, M, y, ldy, bias, st);
  } else if (M > 8 && enough(16) && mmtc_smem<WT, 16>(nb) <= MMTC_SMEM_FAST) {
    if (!dry) launch_mmtc<WT, 16>(op, qs, d, N, K, xq, xd, xs, M, y, ldy, bias, st);
  } else if (mmtc_smem<WT, 8>(nb) <= MM_SMEM) {
    if (!dry) launch_mmtc<WT, 8>(op, qs, d, N, K, xq, xd, xs, M, y, ldy, bias, st);
  } else {
    return false;
  }
  return true;
}

template <int WT>
void matvec_w(int op, const uint8_t* qs, const __half* d, int N, int K, const int8_t* xq, const float* xd,
              const int4* xs, int M, float* y, int ldy, const float* bias, cudaStream_t st, const MmCtx* mc = nullptr) {
  const int nb = K / 32;
  // several tokens on the tcgen05 tensor cores (tc5.cu): from TC5_MIN_TOKENS, or whenever the mma.sync form's resident
  // activations do not fit (long rows, e.g. the 7B down projection: it streams them)
  if (WT == WQ4 && M > 1 && mc &&
      (use_tc5(M) || (g_mm_kind.load(std::memory_order_relaxed) == H2C_MATMUL_AUTO &&
                      !matmul_tc<WT>(op, qs, d, N, K, xq, xd, xs, M, y, ldy, bias, st, true)))) {
    launch_tc5(op, qs, d, N, K, xq, mc->xq_rows, mc->xdT, mc->ldT, M, y, ldy, bias, mc->err, st);
    if (mc->used) *mc->used = true;
    return;
  }
  if (M == 1) {
    if (launch_mvt<WT>(op, qs, d, N, K, xq, xd, xs, y, bias, st)) return;
    if (launch_mv<WT>(op, qs, d, N, K, xq, xd, xs, y, bias, st)) return;
    // rows per CTA: the product buffer (rows x blocks x 16 B) small enough for several CTAs per SM
    if (nb <= 64) launch_mv_t<WT, 32, 1>(op, qs, d, N, K, xq, xd, xs, 1, y, ldy, bias, st);
    else if (nb <= 256) launch_mv_t<WT, 16, 1>(op, qs, d, N, K, xq, xd, xs, 1, y, ldy, bias, st);
    else launch_mv_t<WT, 8, 1>(op, qs, d, N, K, xq, xd, xs, 1, y, ldy, bias, st);
    return;
  }
  if (matmul_tc<WT>(op, qs, d, N, K, xq, xd, xs, M, y, ldy, bias, st)) return;
  // (token groups too large for the tensor-core form's shared memory: the CUDA-core form below)
  if (M > 16 && mm_smem<WT, 32, 8>(nb) <= MM_SMEM_FAST) return launch_mm<WT, 32>(op, qs, d, N, K, xq, xd, xs, M, y, ldy, bias, st);
  if (M > 8 && mm_smem<WT, 16, 8>(nb) <= MM_SMEM_FAST) return launch_mm<WT, 16>(op, qs, d, N, K, xq, xd, xs, M, y, ldy, bias, st);
  if (mm_smem<WT, 8, 8>(nb) <= MM_SMEM) return launch_mm<WT, 8>(op, qs, d, N, K, xq, xd, xs, M, y, ldy, bias, st);
  for (int m0 = 0; m0 < M; m0++)  // rows too long for a staged token group: one token per launch
    launch_mv_t<WT, 16, 1>(op, qs, d, N, K, xq + (size_t)m0 * K, xd + (size_t)m0 * nb, xs + (size_t)m0 * nb, 1,
                           y + (size_t)m0 * ldy, ldy, bias, st);
}

void matvec(int op, const Q4Mat& W, const int8_t* xq, const float* xd, const int4* xs, int M, float* y, int ldy,
            const float* bias, cudaStream_t st, const MmCtx* mc = nullptr) {
  matvec_w<WQ4>(op, W.qs, W.d, W.N, W.K, xq, xd, xs, M, y, ldy, bias, st, mc);
}

// Opt every kernel that takes more than 48 KB of dynamic shared memory into the larger carve-out.
template <int WT, int ROWS, int MB>
cudaError_t mv_attr(int max_smem) {
  cudaError_t c = cudaFuncSetAttribute(k_matvec<WT, ROWS, MB, OP_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_matvec<WT, ROWS, MB, OP_BIAS>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_matvec<WT, ROWS, MB, OP_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  return c;
}

template <int WT, int TG, int RT>
cudaError_t mm_attr() {
  const int smem = (int)MM_SMEM;
  cudaError_t c = cudaFuncSetAttribute(k_matmul<WT, TG, RT, OP_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_matmul<WT, TG, RT, OP_BIAS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_matmul<WT, TG, RT, OP_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  return c;
}
template <int WT, int TG>
cudaError_t mm_attr_mt() {
  cudaError_t c = mm_attr<WT, TG, 8>();
  if (c == cudaSuccess) c = mm_attr<WT, TG, 2>();
  const int smem = (int)MM_SMEM;
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_matmul_tc<WT, TG, OP_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_matmul_tc<WT, TG, OP_BIAS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_matmul_tc<WT, TG, OP_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  return c;
}

// the grouped attention kernel holds G score rows of ctx floats: usable up to ATTG_SMEM bytes
constexpr size_t ATTG_SMEM = 100 * 1024;
bool attg_ok(int G, int HD, int ctx) {
  if (G > 16 || G * HD > 1024) return false;
  return (HD == 64 ? attg_smem_bytes<64>(G, ctx) : attg_smem_bytes<128>(G, ctx)) <= ATTG_SMEM;
}

// The largest context h2c_create accepts: k_attention keeps one float score per position in shared memory, next to
// its V staging ring (16 KB at head_dim 64, 32 KB at 128), within the 227 KB a CTA can have.
constexpr int MAX_CTX = 49152;
// The largest hidden size: k_norm_quant keeps a row, its weights and its squares in shared memory.
constexpr int MAX_DIM = 8192;

// The attributes are per device and only ever raised to fixed maxima (a launch's own size decides its occupancy),
// so engines with different contexts on one device never lower each other's limits.
cudaError_t set_kernel_attrs() {
  const int big = 200 * 1024;
  cudaError_t c = mv_attr<WQ4, 32, 1>(big);
  if (c == cudaSuccess) c = mv_attr<WQ4, 16, 1>(big);
  if (c == cudaSuccess) c = mv_attr<WQ4, 8, 1>(big);
  if (c == cudaSuccess) c = mv_attr<WQ8, 8, 1>(big);
  if (c == cudaSuccess) c = mv_attr<WQ8, 32, 1>(big);
  if (c == cudaSuccess) c = mv_attr<WQ8, 16, 1>(big);
  if (c == cudaSuccess) c = mm_attr_mt<WQ4, 8>();
  if (c == cudaSuccess) c = mm_attr_mt<WQ4, 16>();
  if (c == cudaSuccess) c = mm_attr_mt<WQ4, 32>();
  if (c == cudaSuccess) c = mm_attr_mt<WQ8, 8>();
  if (c == cudaSuccess) c = mm_attr_mt<WQ8, 16>();
  if (c == cudaSuccess) c = mm_attr_mt<WQ8, 32>();
  if (c == cudaSuccess)
    c = cudaFuncSetAttribute(k_attention<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)at_smem_bytes<64>(MAX_CTX));
  if (c == cudaSuccess)
    c = cudaFuncSetAttribute(k_attention_gqa<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATTG_SMEM);
  if (c == cudaSuccess)
    c = cudaFuncSetAttribute(k_attention_gqa<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATTG_SMEM);
  if (c == cudaSuccess)
    c = cudaFuncSetAttribute(k_attention<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)at_smem_bytes<128>(MAX_CTX));
  if (c == cudaSuccess)
    c = cudaFuncSetAttribute(k_att_cl<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)ac_smem_bytes<64>(MAX_CTX));
  if (c == cudaSuccess)
    c = cudaFuncSetAttribute(k_att_cl<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)ac_smem_bytes<64>(MAX_CTX));
  if (c == cudaSuccess)
    c = cudaFuncSetAttribute(k_att_cl<128, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)ac_smem_bytes<128>(MAX_CTX));
  if (c == cudaSuccess)
    c = cudaFuncSetAttribute(k_att_cl<128, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)ac_smem_bytes<128>(MAX_CTX));
  if (c == cudaSuccess)
    c = cudaFuncSetAttribute(k_norm_quant, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)nq_smem_bytes(MAX_DIM));
  if (c == cudaSuccess) c = mvt_attr<WQ4, 2, 4, 5, 8>();
  if (c == cudaSuccess) c = mvt_attr<WQ8, 2, 4, 5, 8>();
  if (c == cudaSuccess) c = mv2_attr<WQ4, 32>();
  if (c == cudaSuccess) c = mv2_attr<WQ4, 8>();
  if (c == cudaSuccess) c = mv2_attr<WQ8, 32>();
  if (c == cudaSuccess) c = mv2_attr<WQ8, 8>();
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_pf_scores<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, pf_scores_smem<64>());
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_pf_scores<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, pf_scores_smem<128>());
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_pf_pv<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, pf_pv_smem<64>());
  if (c == cudaSuccess) c = cudaFuncSetAttribute(k_pf_pv<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, pf_pv_smem<128>());
  if (c == cudaSuccess) c = tc5_set_attrs();
  return c;
}

// set_kernel_attrs once per device, for the device current on the calling thread (any thread may call).
constexpr int ATTR_MAX_DEVICES = 64;
bool g_attrs_done[ATTR_MAX_DEVICES];
std::mutex g_attrs_mutex;
bool kernel_attrs_on_current_device(std::string* why) {
  int dev = -1;
  cudaError_t c = cudaGetDevice(&dev);
  if (c != cudaSuccess || dev < 0 || dev >= ATTR_MAX_DEVICES) {
    *why = std::string("cudaGetDevice: ") + (c != cudaSuccess ? cudaGetErrorString(c) : "device index out of range");
    return false;
  }
  std::lock_guard<std::mutex> lock(g_attrs_mutex);
  if (!g_attrs_done[dev]) {
    c = set_kernel_attrs();
    if (c != cudaSuccess) {
      *why = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(c);
      return false;
    }
    g_attrs_done[dev] = true;
  }
  return true;
}

struct Prof {
  cudaEvent_t ev[64];
  int op[64];
  int n = 0;
  bool on = false;
};

inline void mark(Prof* p, int op, cudaStream_t st) {
  if (p && p->on && p->n < 64) {
    p->op[p->n] = op;
    cudaEventRecord(p->ev[p->n++], st);
  }
}

// ---------------------------------------------------------------- tensor parallelism: the all-gathers

// Gathered columns [G][M][w] (32-bit words) -> rows of ld words with rank g's columns at g * w.
static __global__ void k_tp_unpack(const uint32_t* __restrict__ src, int G, int M, int w, uint32_t* __restrict__ dst,
                                   int ld) {
  const size_t total = (size_t)G * M * w;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % w);
    const size_t gm = i / w;
    const int m = (int)(gm % M), g = (int)(gm / M);
    dst[(size_t)m * ld + (size_t)g * w + j] = src[i];
  }
}

int64_t steady_ms() {
  return std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

// Settle a call on the non-blocking communicator: poll its state while it answers ncclInProgress, up to the engine's
// deadline. Records the first failure in e->tp_fail; returns whether the call succeeded.
bool nccl_settle(h2c_engine* e, ncclResult_t res, const char* what) {
  const NcclApi& nc = nccl();
  bool late = false;
  if (res == ncclInProgress) {
    const int64_t t0 = steady_ms();
    while (res == ncclInProgress) {
      if (nc.async_error(e->comm, &res) != ncclSuccess) break;
      if (res == ncclInProgress && steady_ms() - t0 > e->tp_timeout_ms) {
        late = true;
        break;
      }
      if (res == ncclInProgress) std::this_thread::yield();
    }
  }
  if (res == ncclSuccess) return true;
  if (e->tp_fail.empty())
    e->tp_fail = std::string(what) + (late ? ": no answer within the deadline" : std::string(": ") + nc.error_string(res));
  return false;
}

// One column range of a buffer that every rank fills in part: rows of ld bytes, this rank's cols bytes of each row at
// tp_rank * cols. rows == 1: a contiguous range, gathered in place.
struct TpPart {
  uint8_t* full;
  size_t cols, ld;
  int rows;
};

size_t tp_stage_bytes(const TpPart* p, int n) {
  size_t o = 0;
  for (int i = 0; i < n; i++)
    if (p[i].rows > 1) o += align_up(p[i].cols * p[i].rows, 256);
  return o;
}

// All-gather the parts in one NCCL group so that every rank's buffers hold every rank's columns. Rows of several
// tokens are packed first (their columns are not contiguous) and unpacked after.
void tp_gather(h2c_engine* e, cudaStream_t st, const TpPart* p, int n) {
  if (e->tp_world == 1 || !e->tp_fail.empty()) return;
  const NcclApi& nc = nccl();
  const int G = e->tp_world, r = e->tp_rank;
  size_t off[4], o = 0;
  for (int i = 0; i < n; i++) {
    off[i] = o;
    if (p[i].rows > 1) {
      cudaMemcpy2DAsync(e->tp_send + o, p[i].cols, p[i].full + (size_t)r * p[i].cols, p[i].ld, p[i].cols, p[i].rows,
                        cudaMemcpyDeviceToDevice, st);
      o += align_up(p[i].cols * p[i].rows, 256);
    }
  }
  if (o > e->tp_stage) {
    e->tp_fail = "gather staging too small";
    return;
  }
  if (!nccl_settle(e, nc.group_start(), "ncclGroupStart")) return;
  for (int i = 0; i < n; i++) {
    const ncclResult_t res =
        p[i].rows > 1 ? nc.all_gather(e->tp_send + off[i], e->tp_recv + off[i] * G, p[i].cols * p[i].rows, ncclUint8,
                                      e->comm, st)
                      : nc.all_gather(p[i].full + (size_t)r * p[i].cols, p[i].full, p[i].cols, ncclUint8, e->comm, st);
    if (!nccl_settle(e, res, "ncclAllGather")) {
      nc.group_end();
      return;
    }
  }
  if (!nccl_settle(e, nc.group_end(), "ncclGroupEnd")) return;
  for (int i = 0; i < n; i++) {
    if (p[i].rows == 1) continue;
    const size_t words = (size_t)G * p[i].rows * (p[i].cols / 4);
    const int grid = (int)std::min<size_t>((words + 255) / 256, 148 * 8);
    k_tp_unpack<<<grid, 256, 0, st>>>(reinterpret_cast<const uint32_t*>(e->tp_recv + off[i] * G), G, p[i].rows,
                                      (int)(p[i].cols / 4), reinterpret_cast<uint32_t*>(p[i].full), (int)(p[i].ld / 4));
  }
}

// ---------------------------------------------------------------- tensor parallelism: the peer-memory exchange

// Buffers of each rank that receive the other ranks' slices in a one-token pass (mapped into every rank).
enum { XB_X, XB_ATT, XB_ACTQ, XB_ACTD, XB_ACTS, XB_LOGITS, XB_CNT, XB_N };
constexpr int XCH_MAX_RANKS = 8;
struct XchTab {
  uint8_t* base[XB_N][XCH_MAX_RANKS];
};
struct XchPart {
  int buf, bytes;
  long long off;
};
struct XchArgs {
  const XchTab* tab;
  XchPart part[3];
  int nparts, rank, world, slot, epoch_idx;
  int* err;
  unsigned long long timeout_ns;
};
constexpr unsigned long long XCH_TIMEOUT_NS = 2000000000ull;

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// A new epoch for the exchanges of one one-token pass, or of its logits (every rank runs the same passes, so epochs
// agree; the logits slot has its own epoch since not every pass computes logits).
static __global__ void k_xch_step(unsigned long long* epoch) { *epoch += 1; }

// All-gather of this rank's slices over peer memory: every CTA copies its share of the slices into each peer's
// buffers (the same offsets), then, after a system-scope fence, adds one arrival to each peer's counter of the slot;
// CTA 0 waits until every peer's CTAs have arrived here for this epoch (acquire), with a time limit: on expiry it
// records {1, slot} in err and returns (the host reports the failure; no trap).
static __global__ void __launch_bounds__(256) k_xch(XchArgs a) {
  const XchTab* t = a.tab;
  unsigned long long* cnt = reinterpret_cast<unsigned long long*>(t->base[XB_CNT][a.rank]);
  const unsigned long long epoch = reinterpret_cast<volatile unsigned long long*>(cnt)[a.epoch_idx];
  for (int p = 0; p < a.world; p++) {
    if (p == a.rank) continue;
    for (int q = 0; q < a.nparts; q++) {
      const XchPart& x = a.part[q];
      const uint8_t* src = t->base[x.buf][a.rank] + x.off;
      uint8_t* dst = t->base[x.buf][p] + x.off;
      if (((x.off | x.bytes) & 15) == 0) {
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < x.bytes / 16; i += gridDim.x * blockDim.x)
          reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
      } else {
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < x.bytes / 4; i += gridDim.x * blockDim.x)
          reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(src)[i];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < a.world; p++)
      if (p != a.rank) atomicAdd_system(reinterpret_cast<unsigned long long*>(t->base[XB_CNT][p]) + 1 + a.slot, 1ull);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const unsigned long long want = epoch * (unsigned long long)(a.world - 1) * gridDim.x;
    const unsigned long long t0 = now_ns();
    while (ld_acquire_sys(cnt + 1 + a.slot) < want) {
      if (now_ns() - t0 > a.timeout_ns) {
        *reinterpret_cast<volatile int*>(a.err + 1) = a.slot;
        *reinterpret_cast<volatile int*>(a.err) = 1;
        break;
      }
      __nanosleep(64);
    }
  }
}

// Enqueue the peer-memory exchange of up to three contiguous slices (this rank's range of one token's vector).
void tp_xch(h2c_engine* e, cudaStream_t st, std::initializer_list<XchPart> parts, int slot, int epoch_idx = 0) {
  XchArgs a{};
  a.tab = reinterpret_cast<const XchTab*>(e->xtab_d);
  a.nparts = 0;
  long long total = 0;
  for (const XchPart& p : parts) {
    a.part[a.nparts++] = p;
    total += p.bytes;
  }
  a.rank = e->tp_rank;
  a.world = e->tp_world;
  a.slot = slot;
  a.epoch_idx = epoch_idx;
  a.err = e->xerr_d;
  a.timeout_ns = XCH_TIMEOUT_NS;
  const int grid = (int)std::min<long long>(32, std::max<long long>(1, (total + 16383) / 16384));
  k_xch<<<grid, 256, 0, st>>>(a);
}

int sync_stream(h2c_engine* e);

// Set up the peer exchange after the communicator: map every rank's receive buffers (IPC handles all-gathered
// through NCCL) and build the device table. Returns false (the engine keeps NCCL for every pass) when a step fails.
bool tp_setup_xch(h2c_engine* e, std::string* why) {
  const int G = e->tp_world, rk = e->tp_rank;
  const h2c_config& c = e->cfg;
  if (G > XCH_MAX_RANKS) {
    *why = "too many ranks";
    return false;
  }
  const int slots = 4 * c.layers + 1;
  int r = 0;
  if ((r = dalloc_t(e, &e->xcnt, (size_t)slots + 2)) || (r = dalloc_t(e, &e->actq, (size_t)c.ffn)) ||
      (r = dalloc_t(e, &e->actd, (size_t)c.ffn / 32 + 4)) || (r = dalloc_t(e, &e->acts, (size_t)c.ffn / 32)) ||
      (r = dalloc(e, &e->xtab_d, sizeof(XchTab)))) {
    *why = e->err;
    return false;
  }
  if (cudaHostAlloc(&e->xerr_h, 4 * sizeof(int32_t), cudaHostAllocMapped) != cudaSuccess ||
      cudaHostGetDevicePointer(reinterpret_cast<void**>(&e->xerr_d), e->xerr_h, 0) != cudaSuccess) {
    *why = "mapped pinned allocation";
    return false;
  }
  memset(e->xerr_h, 0, 4 * sizeof(int32_t));
  void* mine[XB_N] = {e->x, e->att, e->actq, e->actd, e->acts, e->logits, e->xcnt};
  std::vector<cudaIpcMemHandle_t> h((size_t)G * XB_N);
  for (int b = 0; b < XB_N; b++)
    if (cudaIpcGetMemHandle(&h[(size_t)rk * XB_N + b], mine[b]) != cudaSuccess) {
      *why = "cudaIpcGetMemHandle";
      return false;
    }
  // every rank's handles to every rank
  uint8_t* hd = nullptr;
  const size_t hb = sizeof(cudaIpcMemHandle_t) * XB_N;
  if (dalloc(e, reinterpret_cast<void**>(&hd), hb * G) ||
      cudaMemcpy(hd + hb * rk, &h[(size_t)rk * XB_N], hb, cudaMemcpyHostToDevice) != cudaSuccess) {
    *why = "handle buffer";
    return false;
  }
  const TpPart hp{hd, hb, 0, 1};
  tp_gather(e, e->st, &hp, 1);
  if (!e->tp_fail.empty() || sync_stream(e) != H2C_OK ||
      cudaMemcpy(h.data(), hd, hb * G, cudaMemcpyDeviceToHost) != cudaSuccess) {
    *why = "handle exchange: " + (e->tp_fail.empty() ? e->err : e->tp_fail);
    return false;
  }
  XchTab tab{};
  for (int b = 0; b < XB_N; b++) tab.base[b][rk] = static_cast<uint8_t*>(mine[b]);
  for (int p = 0; p < G; p++) {
    if (p == rk) continue;
    for (int b = 0; b < XB_N; b++) {
      void* ptr = nullptr;
      const cudaError_t ce = cudaIpcOpenMemHandle(&ptr, h[(size_t)p * XB_N + b], cudaIpcMemLazyEnablePeerAccess);
      if (ce != cudaSuccess) {
        *why = std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(ce);
        return false;
      }
      e->ipc_open.push_back(ptr);
      tab.base[b][p] = static_cast<uint8_t*>(ptr);
    }
  }
  if (cudaMemcpy(e->xtab_d, &tab, sizeof(tab), cudaMemcpyHostToDevice) != cudaSuccess) {
    *why = "exchange table upload";
    return false;
  }
  e->xch = true;
  return true;
}

// Attention of a prompt pass of M tokens of sequence seq at positions pos0 .. pos0+M-1 (prompt_att.cuh): scores,
// softmax and p.v over e->pf_s, in query blocks whose score rows fit the buffer. Output rows at att_r (stride D).
void launch_prompt_attention(h2c_engine* e, int M, int pos0, int seq, int layer, float* att_r, cudaStream_t st) {
  const h2c_config& c = e->cfg;
  const int H = e->Hl, KVH = e->KVHl, HD = e->HD, G = H / KVH, QKV = e->QKV, NL = c.layers, D = c.dim;
  for (int q0 = 0; q0 < M;) {
    const int P0 = pos0 + q0, left = M - q0;
    const size_t per = (size_t)H * 4 * (size_t)((P0 + left + 3) & ~3);
    const int Mq = (int)std::min<size_t>((size_t)left, e->pf_bytes / per);  // >= 1: the buffer holds one full row
    const int ldS = (P0 + Mq + 3) & ~3, R = G * Mq;
    const float* q = e->qkv + (size_t)q0 * QKV;
    float* o = att_r + (size_t)q0 * D;
    const dim3 gs((P0 + Mq + PF_TB - 1) / PF_TB, (R + PF_RB - 1) / PF_RB, KVH);
    const int soft_grid = (KVH * R + PF_SR - 1) / PF_SR, ldP = pf_pm_pitch(c.ctx);
    if (HD == 64) {
      k_pf_scores<64><<<gs, 256, pf_scores_smem<64>(), st>>>(q, QKV, e->kc, H, KVH, c.ctx, NL, layer, seq, P0, Mq,
                                                              e->pf_s, ldS, e->pf_pm, ldP);
      k_pf_soft<<<soft_grid, 256, 0, st>>>(e->pf_s, ldS, e->pf_pm, ldP, KVH * R, R, G, P0, e->pf_sum);
      k_pf_pv<64><<<dim3((R + pf_pv_rows<64>() - 1) / pf_pv_rows<64>(), KVH), 128, pf_pv_smem<64>(), st>>>(
          e->pf_s, ldS, e->pf_sum, e->vc, H, KVH, c.ctx, NL, layer, seq, P0, Mq, o, D);
    } else {
      k_pf_scores<128><<<gs, 256, pf_scores_smem<128>(), st>>>(q, QKV, e->kc, H, KVH, c.ctx, NL, layer, seq, P0, Mq,
                                                               e->pf_s, ldS, e->pf_pm, ldP);
      k_pf_soft<<<soft_grid, 256, 0, st>>>(e->pf_s, ldS, e->pf_pm, ldP, KVH * R, R, G, P0, e->pf_sum);
      k_pf_pv<128><<<dim3((R + pf_pv_rows<128>() - 1) / pf_pv_rows<128>(), KVH), 128, pf_pv_smem<128>(), st>>>(
          e->pf_s, ldS, e->pf_sum, e->vc, H, KVH, c.ctx, NL, layer, seq, P0, Mq, o, D);
    }
    q0 += Mq;
  }
}

// Enqueue one pass of M tokens (positions and ids are read from e->prm on the device). logits: compute the
// last token's logits and the greedy next token into e->next_d. Under tensor parallelism every matrix product
// computes this rank's rows and an all-gather completes the vector (QKV and attention stay per head: only the
// attention output is gathered). pos0 / seq: the pass's first position and its sequence when the host knows them
// (prompt passes), else -1.
void enqueue_pass(h2c_engine* e, int M, bool logits, Prof* pf, bool batch = false, int pos0 = -1, int seq = -1) {
  const h2c_config& c = e->cfg;
  const int D = c.dim, F = c.ffn, H = e->Hl, KVH = e->KVHl, HD = e->HD, QKV = e->QKV, NL = c.layers;
  const int rk = e->tp_rank, Dl = e->Dl, Fl = e->Fl, nbf = F / 32, nbl = Fl / 32;
  cudaStream_t st = e->st;
  const MmCtx mcv{e->xdT, e->ldT, c.max_chunk, e->tc5_err, &e->tc5_used};
  const MmCtx* mc = M > 1 ? &mcv : nullptr;
  float* xdT = M > 1 ? e->xdT : nullptr;
  float* att_r = e->att + (size_t)rk * H * HD;  // this rank's heads' columns of the attention output
  float* x_r = e->x + (size_t)rk * Dl;          // this rank's rows of O and down
  const TpPart g_att{reinterpret_cast<uint8_t*>(e->att), (size_t)H * HD * 4, (size_t)D * 4, M};
  const TpPart g_x{reinterpret_cast<uint8_t*>(e->x), (size_t)Dl * 4, (size_t)D * 4, M};
  const TpPart g_act[4] = {{reinterpret_cast<uint8_t*>(e->xq), (size_t)Fl, (size_t)F, M},
                           {reinterpret_cast<uint8_t*>(e->xd), (size_t)nbl * 4, (size_t)nbf * 4, M},
                           {reinterpret_cast<uint8_t*>(e->xs), (size_t)nbl * 16, (size_t)nbf * 16, M},
                           {reinterpret_cast<uint8_t*>(e->xdT), (size_t)nbl * e->ldT * 4, 0, 1}};
  // one token under tensor parallelism: the exchanges go through peer memory (k_xch), slots 4 l + {0 attention, 1 x
  // after O, 2 FFN activation, 3 x after down} and 4 L (logits), under a new epoch
  const bool px = e->xch && M == 1 && !pf && !batch;
  if (px) k_xch_step<<<1, 1, 0, st>>>(e->xcnt);
  mark(pf, -1, st);
  k_embed<<<M, 128, 0, st>>>(e->prm, e->embd.qs, e->embd.d, D, e->x);
  mark(pf, 0, st);
  for (int l = 0; l < NL; l++) {
    const LayerW& W = e->L[l];
    k_norm_quant<<<M, NQ_THREADS, nq_smem_bytes(D), st>>>(e->x, 0, W.attn_norm, D, c.eps, e->xq, e->xd, e->xs, xdT,
                                                         e->ldT);
    mark(pf, 1, st);
    matvec(OP_BIAS, W.qkv, e->xq, e->xd, e->xs, M, e->qkv, QKV, W.bqkv, st, mc);
    mark(pf, 2, st);
    k_rope_kv<<<dim3(((H + KVH) * (HD / 2) + 127) / 128, M), 128, 0, st>>>(e->prm, e->qkv, QKV, e->rope, e->kc, e->vc,
                                                                            H, KVH, HD, c.ctx, NL, l);
    mark(pf, 3, st);
    // one token: a cluster of CTAs per head (scores shared through distributed shared memory); on one GPU it also
    // quantizes its output for the O matrix (k_quant below is then skipped)
    const bool fq = M == 1 && e->tp_world == 1;
    if (M == 1) {
      if (HD == 64 && fq)
        k_att_cl<64, true><<<H * AC_CL, 128, ac_smem_bytes<64>(c.ctx), st>>>(e->prm, e->qkv, e->kc, e->vc, H, KVH, c.ctx,
                                                                            NL, l, att_r, e->xq, e->xd, e->xs);
      else if (HD == 64)
        k_att_cl<64, false><<<H * AC_CL, 128, ac_smem_bytes<64>(c.ctx), st>>>(e->prm, e->qkv, e->kc, e->vc, H, KVH,
                                                                             c.ctx, NL, l, att_r, nullptr, nullptr,
                                                                             nullptr);
      else if (fq)
        k_att_cl<128, true><<<H * AC_CL, 128, ac_smem_bytes<128>(c.ctx), st>>>(e->prm, e->qkv, e->kc, e->vc, H, KVH,
                                                                              c.ctx, NL, l, att_r, e->xq, e->xd, e->xs);
      else
        k_att_cl<128, false><<<H * AC_CL, 128, ac_smem_bytes<128>(c.ctx), st>>>(e->prm, e->qkv, e->kc, e->vc, H, KVH,
                                                                               c.ctx, NL, l, att_r, nullptr, nullptr,
                                                                               nullptr);
    } else if (!batch && pos0 >= 0 && M >= PF_MIN_TOKENS && e->pf_bytes) {  // a prompt pass: tiled over tokens
      launch_prompt_attention(e, M, pos0, seq, l, att_r, st);
    } else if (attg_ok(H / KVH, HD, c.ctx)) {  // several tokens: one CTA per (kv head, token)
      if (HD == 64)
        k_attention_gqa<64><<<dim3(KVH, M), 256, attg_smem_bytes<64>(H / KVH, c.ctx), st>>>(
            e->prm, e->qkv, QKV, e->kc, e->vc, H, KVH, c.ctx, NL, l, att_r, D);
      else
        k_attention_gqa<128><<<dim3(KVH, M), 256, attg_smem_bytes<128>(H / KVH, c.ctx), st>>>(
            e->prm, e->qkv, QKV, e->kc, e->vc, H, KVH, c.ctx, NL, l, att_r, D);
    } else if (HD == 64) {
      k_attention<64><<<dim3(H, M), 128, at_smem_bytes<64>(c.ctx), st>>>(e->prm, e->qkv, QKV, e->kc, e->vc, H, KVH, c.ctx, NL, l, att_r, D);
    } else {
      k_attention<128><<<dim3(H, M), 128, at_smem_bytes<128>(c.ctx), st>>>(e->prm, e->qkv, QKV, e->kc, e->vc, H, KVH, c.ctx, NL, l, att_r, D);
    }
    if (px) tp_xch(e, st, {{XB_ATT, H * HD * 4, (long long)rk * H * HD * 4}}, 4 * l);
    else tp_gather(e, st, &g_att, 1);
    mark(pf, 4, st);
    if (!fq) {
      const int warps = M * (D / 32);
      k_quant<<<(warps + 7) / 8, 256, 0, st>>>(e->att, D, M, e->xq, e->xd, e->xs, xdT, e->ldT);
    }
    mark(pf, 5, st);
    matvec(OP_ADD, W.o, e->xq, e->xd, e->xs, M, x_r, D, nullptr, st, mc);
    if (px) tp_xch(e, st, {{XB_X, Dl * 4, (long long)rk * Dl * 4}}, 4 * l + 1);
    else tp_gather(e, st, &g_x, 1);
    mark(pf, 6, st);
    k_norm_quant<<<M, NQ_THREADS, nq_smem_bytes(D), st>>>(e->x, 0, W.ffn_norm, D, c.eps, e->xq, e->xd, e->xs, xdT,
                                                         e->ldT);
    mark(pf, 1, st);
    matvec(OP_STORE, W.gu, e->xq, e->xd, e->xs, M, e->gu, 2 * Fl, nullptr, st, mc);
    mark(pf, 7, st);
    {
      const int warps = M * nbl;
      int8_t* aq = px ? e->actq : e->xq;  // (the received activation must not share the buffer other stages use)
      float* ad = px ? e->actd : e->xd;
      int4* as = px ? e->acts : e->xs;
      k_swiglu_quant<<<(warps + 7) / 8, 256, 0, st>>>(e->gu, Fl, M, aq + (size_t)rk * Fl, ad + (size_t)rk * nbl,
                                                      as + (size_t)rk * nbl,
                                                      xdT ? xdT + (size_t)rk * nbl * e->ldT : nullptr, e->ldT, F);
    }
    if (px)
      tp_xch(e, st, {{XB_ACTQ, Fl, (long long)rk * Fl}, {XB_ACTD, nbl * 4, (long long)rk * nbl * 4},
                     {XB_ACTS, nbl * 16, (long long)rk * nbl * 16}}, 4 * l + 2);
    else
      tp_gather(e, st, g_act, M > 1 ? 4 : 3);
    mark(pf, 8, st);
    if (px) matvec(OP_ADD, W.down, e->actq, e->actd, e->acts, M, x_r, D, nullptr, st, mc);
    else matvec(OP_ADD, W.down, e->xq, e->xd, e->xs, M, x_r, D, nullptr, st, mc);
    if (px) tp_xch(e, st, {{XB_X, Dl * 4, (long long)rk * Dl * 4}}, 4 * l + 3);
    else tp_gather(e, st, &g_x, 1);
    mark(pf, 9, st);
  }
  if (batch) {  // every token of a batched decode step is the last of its sequence: logits and a token for each
    k_norm_quant<<<M, NQ_THREADS, nq_smem_bytes(D), st>>>(e->x, 0, e->out_norm, D, c.eps, e->xq, e->xd, e->xs, xdT,
                                                         e->ldT);
    if (e->out_type == 8) {
      matvec_w<WQ8>(OP_STORE, (const uint8_t*)e->out8.qs, e->out8.d, c.vocab, D, e->xq, e->xd, e->xs, M, e->logits_b,
                    c.vocab, nullptr, st);
    } else {
      matvec(OP_STORE, e->out_type == 2 ? e->out4 : e->embd, e->xq, e->xd, e->xs, M, e->logits_b, c.vocab, nullptr, st,
             mc);
    }
    k_argmax1<<<dim3(e->am_np, M), 256, 0, st>>>(e->logits_b, c.vocab, e->am_vb, e->am_ib);
    k_argmax2_batch<<<M, 32, 0, st>>>(e->am_vb, e->am_ib, e->am_np, e->prm, e->toklog, e->cfg.ctx, e->next_b);
    mark(pf, 10, st);
  } else if (logits) {
    k_norm_quant<<<1, NQ_THREADS, nq_smem_bytes(D), st>>>(e->x, M - 1, e->out_norm, D, c.eps, e->xq, e->xd, e->xs);
    // this rank's lm_head rows [rk * Vp, rk * Vp + Vl) straight into their place in the logits, then gathered
    float* lg = e->logits + (size_t)rk * e->Vp;
    if (e->out_type == 8) {
      matvec_w<WQ8>(OP_STORE, (const uint8_t*)e->out8.qs, e->out8.d, e->Vl, D, e->xq, e->xd, e->xs, 1, lg, e->Vl,
                    nullptr, st);
    } else if (e->out_type == 2) {
      matvec(OP_STORE, e->out4, e->xq, e->xd, e->xs, 1, lg, e->Vl, nullptr, st);
    } else {  // tied: this rank's rows of the embedding (groups of 32 rows from row rk * Vp)
      const size_t g0 = (size_t)rk * e->Vp / 32, nb = (size_t)D / 32;
      matvec_w<WQ4>(OP_STORE, e->embd.qs + g0 * nb * 32 * 16, e->embd.d + g0 * nb * 32, e->Vl, D, e->xq, e->xd, e->xs,
                    1, lg, e->Vl, nullptr, st);
    }
    const TpPart g_lg{reinterpret_cast<uint8_t*>(e->logits), (size_t)e->Vp * 4, 0, 1};
    if (px) {
      k_xch_step<<<1, 1, 0, st>>>(e->xcnt + 4 * NL + 2);
      tp_xch(e, st, {{XB_LOGITS, e->Vp * 4, (long long)rk * e->Vp * 4}}, 4 * NL, 4 * NL + 2);
    }
    else tp_gather(e, st, &g_lg, 1);
    k_argmax1<<<e->am_np, 256, 0, st>>>(e->logits, c.vocab, e->am_v, e->am_i);
    k_argmax2<<<1, 32, 0, st>>>(e->am_v, e->am_i, e->am_np, e->prm, e->toklog, e->cfg.ctx, e->next_d);
    mark(pf, 10, st);
  }
}

// Wait for the stream. Under tensor parallelism the wait has the engine's deadline: a peer that stops answering
// leaves this rank's collective waiting, so on expiry the communicator is aborted (its kernels return) and the
// engine refuses further passes.
int sync_stream(h2c_engine* e) {
  if (e->tp_world == 1) {
    CUDA_TRY(e, cudaStreamSynchronize(e->st));
    return H2C_OK;
  }
  const int64_t t0 = steady_ms();
  for (;;) {
    const cudaError_t q = cudaStreamQuery(e->st);
    if (q == cudaSuccess) {
      if (e->xch && e->xerr_h[0]) {  // a peer-exchange wait expired: a peer stopped answering
        const int slot = e->xerr_h[1];
        e->comm_dead = true;
        return e->fail(H2C_ERR_TIMEOUT, "peer exchange %d: a peer's slice did not arrive within %llu ms (engine "
                       "closed for passes)", slot, (unsigned long long)(XCH_TIMEOUT_NS / 1000000));
      }
      return H2C_OK;
    }
    if (q != cudaErrorNotReady) return e->fail(H2C_ERR_CUDA, "stream: %s", cudaGetErrorString(q));
    ncclResult_t a = ncclSuccess;
    if (nccl().async_error(e->comm, &a) == ncclSuccess && a != ncclSuccess && a != ncclInProgress) {
      nccl().abort(e->comm);
      e->comm = nullptr;
      e->comm_dead = true;
      cudaStreamSynchronize(e->st);
      return e->fail(H2C_ERR_CUDA, "NCCL: %s (communicator aborted)", nccl().error_string(a));
    }
    if (steady_ms() - t0 > e->tp_timeout_ms) {
      nccl().abort(e->comm);  // the collectives in flight see the abort and return
      e->comm = nullptr;
      e->comm_dead = true;
      cudaStreamSynchronize(e->st);
      return e->fail(H2C_ERR_TIMEOUT, "tensor-parallel pass not finished within %lld ms: a peer stopped answering "
                     "(communicator aborted)", (long long)e->tp_timeout_ms);
    }
    std::this_thread::yield();
  }
}

// After enqueueing passes: an NCCL failure while enqueueing aborts the communicator.
int tp_enqueue_status(h2c_engine* e) {
  if (e->tp_fail.empty()) return H2C_OK;
  const std::string why = e->tp_fail;
  e->tp_fail.clear();
  if (e->comm) {
    nccl().abort(e->comm);
    e->comm = nullptr;
  }
  e->comm_dead = true;
  cudaStreamSynchronize(e->st);
  return e->fail(H2C_ERR_CUDA, "%s (communicator aborted)", why.c_str());
}

int check_ready(h2c_engine* e) {
  for (int l = 0; l < e->cfg.layers; l++)
    if (e->layer_set[l] != 0x7f) return e->fail(H2C_ERR_NOT_READY, "layer %d: tensor kinds missing (mask 0x%x)", l, e->layer_set[l]);
  if (!e->embd_set) return e->fail(H2C_ERR_NOT_READY, "token embedding not set");
  if (!e->out_norm_set) return e->fail(H2C_ERR_NOT_READY, "output norm not set");
  return H2C_OK;
}

int build_graph(h2c_engine* e) {
  if (e->gexec) return H2C_OK;
  // (relaxed under tensor parallelism: NCCL may set up a connection on the first use of a collective's algorithm)
  CUDA_TRY(e, cudaStreamBeginCapture(e->st, e->tp_world > 1 ? cudaStreamCaptureModeRelaxed
                                                              : cudaStreamCaptureModeThreadLocal));
  enqueue_pass(e, 1, true, nullptr);
  cudaError_t c = cudaStreamEndCapture(e->st, &e->graph);
  if (!e->tp_fail.empty()) {
    if (e->graph) cudaGraphDestroy(e->graph);
    e->graph = nullptr;
    return tp_enqueue_status(e);
  }
  if (c != cudaSuccess) return e->fail(H2C_ERR_CUDA, "graph capture: %s", cudaGetErrorString(c));
  CUDA_TRY(e, cudaGraphInstantiate(&e->gexec, e->graph, 0));
  size_t nn = 0;
  CUDA_TRY(e, cudaGraphGetNodes(e->graph, nullptr, &nn));
  std::vector<cudaGraphNode_t> nodes(nn);
  CUDA_TRY(e, cudaGraphGetNodes(e->graph, nodes.data(), &nn));
  int k = 0;
  for (auto n : nodes) {
    cudaGraphNodeType t;
    CUDA_TRY(e, cudaGraphNodeGetType(n, &t));
    if (t == cudaGraphNodeTypeKernel) k++;
  }
  e->graph_kernels = k;
  return H2C_OK;
}

// ---------------------------------------------------------------- persistent decode kernel: layout and launch

struct TileSpec {
  const uint8_t* qs;  // grouped layout on the host copy
  const uint16_t* d;
  int nb;
  std::vector<int> rows;
  bool chain;         // chain layout (QKV, O, gate/up, lm_head) or row-major (down)
};

size_t tile_bytes(int nb, int R, bool chain) {
  if (chain) return (size_t)R * mk_nbp(nb) * 16 + align_up((size_t)R * mk_nbp(nb) * 2, 16);
  return align_up((size_t)nb * R * 16, 16) + align_up((size_t)nb * R * 2, 16);
}

// Gather rows of a grouped-layout matrix into one tile. Row-major: values [R][nb][16 B], then fp16 scales [R][nb].
// Chain: values [R][4][nbp] 32-bit words (word l of every block of the row, lane by lane), then fp16 scales
// [R][nbp]; the padding blocks up to nbp are zero.
void gather_tile(const TileSpec& t, uint8_t* dst) {
  const int R = (int)t.rows.size(), nb = t.nb, nbp = mk_nbp(nb);
  memset(dst, 0, tile_bytes(nb, R, t.chain));
  uint16_t* dd = reinterpret_cast<uint16_t*>(dst + (t.chain ? (size_t)R * nbp * 16 : align_up((size_t)nb * R * 16, 16)));
  for (int j = 0; j < R; j++)
    for (int b = 0; b < nb; b++) {
      const int n = t.rows[j], g = n >> 5, r = n & 31;
      const size_t e = ((size_t)g * nb + b) * 32 + r;
      if (t.chain) {
        for (int l = 0; l < 4; l++) memcpy(dst + (((size_t)j * 4 + l) * nbp + b) * 4, t.qs + e * 16 + 4 * l, 4);
        dd[(size_t)j * nbp + b] = t.d[e];
      } else {
        memcpy(dst + ((size_t)j * nb + b) * 16, t.qs + e * 16, 16);
        dd[(size_t)j * nb + b] = t.d[e];
      }
    }
}

int mk_unsupported(h2c_engine* e, const char* why) {
  e->mk_ok = false;
  e->mk_why = why;
  return H2C_OK;
}

// Decide whether the persistent kernel applies to this model and, if so, lay out the weight stream.
int mk_build(h2c_engine* e) {
  if (e->mk_built) return H2C_OK;
  e->mk_built = true;
  if (e->tp_world > 1) return mk_unsupported(e, "tensor parallelism (steps run on the CUDA graph path)");
  const h2c_config& c = e->cfg;
  const int D = c.dim, F = c.ffn, H = c.heads, KVH = c.kv_heads, HD = e->HD, QKV = e->QKV, NL = c.layers,
            V = c.vocab;
  const int nbd = D / 32, nbf = F / 32;
  int dev_sms = 0, coop = 0;
  CUDA_TRY(e, cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, e->dev));
  CUDA_TRY(e, cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, e->dev));
  if (!coop) return mk_unsupported(e, "device without cooperative launch");
  if (e->out_type == 8) return mk_unsupported(e, "Q8_0 output matrix (the persistent kernel streams Q4_0 tiles)");
  if (HD % MK_TILE_ROWS) return mk_unsupported(e, "head_dim not a multiple of 64");
  if (F < D) return mk_unsupported(e, "ffn narrower than the hidden size");
  if (tile_bytes(nbd, MK_TILE_ROWS, true) > (size_t)MK_SLOT) return mk_unsupported(e, "rows too long for 64-row tiles");
  const int nh = std::min(dev_sms - H, D / 4);  // CTAs owning O / down rows
  if (nh < 1) return mk_unsupported(e, "not enough SMs");
  const int ncta = H + nh;
  if (V < ncta) return mk_unsupported(e, "vocabulary smaller than the grid");
  const int o_max = (D + nh - 1) / nh;
  if (o_max > 64 || tile_bytes(nbf, o_max, false) > (size_t)MK_SLOT)
    return mk_unsupported(e, "per-CTA O/down tiles larger than a ring slot");
  if (o_max > 16) return mk_unsupported(e, "more than 16 O/down rows per CTA");
  const int nsplit = mk_nsplit(nbf, ncta, nh);
  const int npair = QKV / 2, pr_max = (npair + ncta - 1) / ncta;
  if (2 * pr_max > 64) return mk_unsupported(e, "more than 64 QKV rows per CTA");
  if (nbf > MK_NT) return mk_unsupported(e, "rows longer than the tile kernel's thread count");
  // product buffer (float4 units) of the row-major (down) tiles: 4 lane rows per row; it also holds the squares of
  // the RMSNorm (4 lane rows of D / 4 + 4 floats)
  const int prod_items = std::max(o_max * mk_prod_lane_stride(nbf), D / 4 + 4);
  const size_t base = mk_smem_base(D, F, HD, c.ctx, prod_items);
  int max_optin = 0;
  CUDA_TRY(e, cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, e->dev));
  const size_t budget = (size_t)max_optin - 1024;  // static shared memory of the kernel is far below 1 KB
  if (base > budget) return mk_unsupported(e, "context too long for the shared-memory score buffer");
  // K rows are staged with 4 floats of padding (conflict-free dot products), V rows unpadded
  const int kv_stage = (int)std::min<size_t>((size_t)c.ctx, (budget - base) / ((size_t)(2 * HD + 4) * 4));
  // beyond kv_stage positions attention streams the V columns through the same area: it must hold a few rows
  if (kv_stage < std::min(16, c.ctx)) return mk_unsupported(e, "context too long for the shared-memory budget");
  const size_t smem = base + (size_t)kv_stage * (2 * HD + 4) * 4;
  // the Qwen2.5-0.5B shape on a 148-SM B200 has its own instance with the shape and grid compiled in (and without
  // the chain-tile fallback of the QKV and O tiles, so its QKV and O tiles must fit the two-phase form); other shapes
  // and grids take the generic one
  const bool fixed = D == 896 && F == 4864 && H == 14 && KVH == 2 && HD == 64 && ncta == 148 &&
                     mk_small_tile_fits(2 * pr_max, nbd, prod_items) && mk_small_tile_fits(o_max, nbd, prod_items);
  // (the generic instance keeps the trace and long-context code: it serves every launch)
  e->mk_kernel = fixed ? (void*)k_decode_persistent<896, 4864, 14, 2, 64, 148, false, false>
                       : (void*)k_decode_persistent<0, 0, 0, 0, 0, 0, true, true>;
  e->mk_kernel_lc = fixed ? (void*)k_decode_persistent<896, 4864, 14, 2, 64, 148, false, true> : e->mk_kernel;
  e->mk_kernel_trace = fixed ? (void*)k_decode_persistent<896, 4864, 14, 2, 64, 148, true, true> : e->mk_kernel;
  for (void* kern : {e->mk_kernel, e->mk_kernel_lc, e->mk_kernel_trace}) {
    CUDA_TRY(e, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int occ = 0;
    CUDA_TRY(e, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, MK_THREADS, smem));
    if (occ < 1) return mk_unsupported(e, "persistent kernel does not fit on an SM");
  }

  // host copies of the packed (grouped) matrices
  auto fetch = [&](const Q4Mat& m, std::vector<uint8_t>& qs, std::vector<uint16_t>& d) -> int {
    const size_t nbp = padded_rows(m.N) * (m.K / 32);
    qs.resize(nbp * 16);
    d.resize(nbp);
    CUDA_TRY(e, cudaMemcpy(qs.data(), m.qs, qs.size(), cudaMemcpyDeviceToHost));
    CUDA_TRY(e, cudaMemcpy(d.data(), m.d, d.size() * 2, cudaMemcpyDeviceToHost));
    return H2C_OK;
  };
  std::vector<std::vector<uint8_t>> hq(4 * NL + 1);
  std::vector<std::vector<uint16_t>> hd(4 * NL + 1);
  int r = 0;
  for (int l = 0; l < NL; l++) {
    const LayerW& W = e->L[l];
    if ((r = fetch(W.qkv, hq[4 * l], hd[4 * l])) || (r = fetch(W.o, hq[4 * l + 1], hd[4 * l + 1])) ||
        (r = fetch(W.gu, hq[4 * l + 2], hd[4 * l + 2])) || (r = fetch(W.down, hq[4 * l + 3], hd[4 * l + 3])))
      return r;
  }
  if ((r = fetch(e->out_type == 2 ? e->out4 : e->embd, hq[4 * NL], hd[4 * NL]))) return r;

  // per-CTA tile lists, in consumption order (must match k_decode_persistent)
  std::vector<std::vector<TileSpec>> specs(ncta);
  const int half = HD / 2;
  auto rows_tile = [&](int mat, int nb, int first, int count, bool chain) {
    TileSpec t{hq[mat].data(), hd[mat].data(), nb, {}, chain};
    for (int n = first; n < first + count; n++) t.rows.push_back(n);
    return t;
  };
  for (int cta = 0; cta < ncta; cta++) {
    const bool head = cta < H;
    const int jj = cta - H;
    const int o_lo = head ? 0 : (int)((long long)jj * D / nh), o_hi = head ? 0 : (int)((long long)(jj + 1) * D / nh);
    const int v_lo = (int)((long long)cta * V / ncta), v_hi = (int)((long long)(cta + 1) * V / ncta);
    const int pr_lo = (int)((long long)cta * npair / ncta), pr_hi = (int)((long long)(cta + 1) * npair / ncta);
    auto& Lst = specs[cta];
    for (int l = 0; l < NL; l++) {
      TileSpec a{hq[4 * l].data(), hd[4 * l].data(), nbd, {}, true};
      for (int pi = pr_lo; pi < pr_hi; pi++) {  // QKV rows in RoPE pairs (i, i + HD/2) of a head
        const int hh = pi / half, i = pi % half;
        a.rows.push_back(hh * HD + i);
        a.rows.push_back(hh * HD + i + half);
      }
      Lst.push_back(a);
      if (!head) Lst.push_back(rows_tile(4 * l + 1, nbd, o_lo, o_hi - o_lo, true));
      for (int ab = cta; ab < (nsplit ? ncta : nbf); ab += ncta) {
        TileSpec g{hq[4 * l + 2].data(), hd[4 * l + 2].data(), nbd, {}, true};
        for (int q = 0; q < 32; q++) g.rows.push_back(32 * ab + q);
        for (int q = 0; q < 32; q++) g.rows.push_back(F + 32 * ab + q);
        Lst.push_back(g);
      }
      if (nsplit && cta >= ncta - 4 * nsplit) {  // piece q: act values 8 (q % 4) .. + 7 of block ncta + q / 4
        const int q = cta - (ncta - 4 * nsplit), ab = ncta + q / 4;
        TileSpec g{hq[4 * l + 2].data(), hd[4 * l + 2].data(), nbd, {}, true};
        for (int j = 0; j < 8; j++) g.rows.push_back(32 * ab + 8 * (q % 4) + j);
        for (int j = 0; j < 8; j++) g.rows.push_back(F + 32 * ab + 8 * (q % 4) + j);
        Lst.push_back(g);
      }
      if (!head) Lst.push_back(rows_tile(4 * l + 3, nbf, o_lo, o_hi - o_lo, false));
    }
    for (int r0 = v_lo; r0 < v_hi; r0 += MK_TILE_ROWS)
      Lst.push_back(rows_tile(4 * NL, nbd, r0, std::min(v_hi, r0 + MK_TILE_ROWS) - r0, true));
  }
  size_t maxt = 0, total = 0;
  for (auto& Lst : specs) {
    maxt = std::max(maxt, Lst.size());
    for (auto& t : Lst) total += tile_bytes(t.nb, (int)t.rows.size(), t.chain);
  }
  if (maxt > (size_t)MK_MAX_TILES) return mk_unsupported(e, "more tiles per token than the shared-memory table holds");
  std::vector<uint8_t> stream(total);
  std::vector<MkTile> table((size_t)ncta * maxt);
  std::vector<int> counts(ncta);
  size_t off = 0;
  for (int cta = 0; cta < ncta; cta++) {
    counts[cta] = (int)specs[cta].size();
    for (size_t i = 0; i < specs[cta].size(); i++) {
      const TileSpec& t = specs[cta][i];
      const size_t b = tile_bytes(t.nb, (int)t.rows.size(), t.chain);
      if (b > (size_t)MK_SLOT) return mk_unsupported(e, "tile larger than a ring slot");
      gather_tile(t, stream.data() + off);
      table[(size_t)cta * maxt + i] = MkTile{(uint64_t)off, (uint32_t)b, (uint16_t)t.rows.size(), (uint16_t)t.nb};
      off += b;
    }
  }
  // tagged-word regions, each starting on a 4-word (32-byte) boundary for the quad reads, plus one spare quad
  auto q4w = [](size_t n) { return (n + 3) & ~(size_t)3; };
  const size_t lm_words = q4w((size_t)ncta * 2), kvd_words = q4w((size_t)ncta);
  const size_t raw_words = q4w((size_t)nsplit * 32), lcm_words = (size_t)H * q4w((size_t)ncta),
               lce_words = (size_t)H * q4w((size_t)c.ctx), lcs_words = q4w((size_t)H);
  const size_t words = (size_t)D * 3 + (size_t)2 * KVH * HD + (size_t)nbf * MK_ACT_WORDS + lm_words + kvd_words +
                       raw_words + lcm_words + lce_words + lcs_words + 4;
  unsigned long long* tagged = nullptr;
  if ((r = dalloc_t(e, &e->mk_stream, total)) || (r = dalloc_t(e, &e->mk_tiles, table.size())) ||
      (r = dalloc_t(e, &e->mk_attn_norm, (size_t)NL * D)) || (r = dalloc_t(e, &e->mk_ffn_norm, (size_t)NL * D)) ||
      (r = dalloc_t(e, &e->mk_bqkv, (size_t)NL * QKV)) || (r = dalloc_t(e, &tagged, words)) ||
      (r = dalloc_t(e, &e->mk_io, 8)) || (r = dalloc_t(e, &e->mk_tile_count, (size_t)ncta)))
    return r;
  e->mk_xw = tagged;
  e->mk_qw = tagged + D;
  e->mk_attw = tagged + 2 * D;
  e->mk_kvw = tagged + 3 * D;
  e->mk_actw = e->mk_kvw + (size_t)2 * KVH * HD;
  e->mk_lmw = e->mk_actw + (size_t)nbf * MK_ACT_WORDS;
  e->mk_kvdone = e->mk_lmw + lm_words;
  e->mk_rawact = e->mk_kvdone + kvd_words;
  e->mk_lcmax = e->mk_rawact + raw_words;
  e->mk_lce = e->mk_lcmax + lcm_words;
  e->mk_lcsum = e->mk_lce + lce_words;
  e->mk_nsplit = nsplit;
  e->mk_tagged_words = words;
  CUDA_TRY(e, cudaMemset(tagged, 0, words * sizeof(unsigned long long)));  // epoch 0: nothing published yet
  CUDA_TRY(e, cudaMallocHost(&e->mk_io_h, 8 * sizeof(int32_t)));
  CUDA_TRY(e, cudaHostAlloc((void**)&e->mk_done_h, 8 * sizeof(int32_t), cudaHostAllocMapped));
  CUDA_TRY(e, cudaHostGetDevicePointer((void**)&e->mk_done_d, e->mk_done_h, 0));
  memset(e->mk_done_h, 0, 8 * sizeof(int32_t));
  CUDA_TRY(e, cudaMemcpy(e->mk_tile_count, counts.data(), counts.size() * sizeof(int), cudaMemcpyHostToDevice));
  CUDA_TRY(e, cudaMemcpy(e->mk_stream, stream.data(), total, cudaMemcpyHostToDevice));
  CUDA_TRY(e, cudaMemcpy(e->mk_tiles, table.data(), table.size() * sizeof(MkTile), cudaMemcpyHostToDevice));
  for (int l = 0; l < NL; l++) {
    CUDA_TRY(e, cudaMemcpy(e->mk_attn_norm + (size_t)l * D, e->L[l].attn_norm, D * 4, cudaMemcpyDeviceToDevice));
    CUDA_TRY(e, cudaMemcpy(e->mk_ffn_norm + (size_t)l * D, e->L[l].ffn_norm, D * 4, cudaMemcpyDeviceToDevice));
    CUDA_TRY(e, cudaMemcpy(e->mk_bqkv + (size_t)l * QKV, e->L[l].bqkv, (size_t)QKV * 4, cudaMemcpyDeviceToDevice));
  }
  e->mk_ncta = ncta;
  e->mk_tile_stride = (int)maxt;
  e->mk_prod_items = prod_items;
  e->mk_kv_stage = kv_stage;
  e->mk_smem = smem;
  e->mk_ok = true;
  return H2C_OK;
}

bool use_persistent(h2c_engine* e) {
  if (e->decode_mode == H2C_DECODE_GRAPH) return false;
  return e->mk_ok;
}

// Launch `steps` decode steps of the persistent kernel (parameters already in e->prm on the stream).
// args (seq, pos, token) given: the first step's parameters travel in the launch's own parameter block and CTA 0
// reports the outcome in the mapped host record (mk_wait_done polls it), so no copy is enqueued on either side.
// last_pos: the last position the launch decodes (it selects the instance with or without long-context attention)
int mk_launch(h2c_engine* e, int steps, int last_pos, unsigned long long* trace = nullptr,
              const int32_t* args = nullptr) {
  const h2c_config& c = e->cfg;
  MkParams p{};
  p.D = c.dim; p.F = c.ffn; p.H = c.heads; p.KVH = c.kv_heads; p.HD = e->HD; p.QKV = e->QKV; p.L = c.layers;
  p.V = c.vocab; p.ctx = c.ctx; p.ncta = e->mk_ncta; p.eps = c.eps;
  p.stream = e->mk_stream; p.tiles = e->mk_tiles; p.tile_count = e->mk_tile_count; p.tile_stride = e->mk_tile_stride;
  p.prod_items = e->mk_prod_items; p.kv_stage = e->mk_kv_stage;
  p.attn_norm = e->mk_attn_norm; p.ffn_norm = e->mk_ffn_norm; p.bqkv = e->mk_bqkv; p.out_norm = e->out_norm;
  p.rope = e->rope; p.embd_qs = e->embd.qs; p.embd_d = e->embd.d; p.kc = e->kc; p.vc = e->vc; p.logits = e->logits;
  p.xw = e->mk_xw; p.qw = e->mk_qw; p.kvw = e->mk_kvw; p.attw = e->mk_attw; p.actw = e->mk_actw; p.lmw = e->mk_lmw;
  p.kvdone = e->mk_kvdone;
  p.rawact = e->mk_rawact;
  p.lcmax = e->mk_lcmax; p.lce = e->mk_lce; p.lcsum = e->mk_lcsum;
  p.nsplit = e->mk_nsplit;
  p.err = e->mk_io + 4; p.prm = e->prm; p.toklog = e->toklog; p.next = e->mk_io;
  p.steps = steps;
  if (args) {
    p.args_given = 1; p.arg_seq = args[0]; p.arg_pos = args[1]; p.arg_tok = args[2];
    if (++e->mk_launch_seq <= 0) e->mk_launch_seq = 1;
    p.done = e->mk_done_d;
    p.launch_seq = e->mk_launch_seq;
  }
  p.timeout_ns = e->mk_timeout_ns;
  p.stall_cta = e->mk_stall_cta;
  p.trace = trace;
  // Tags grow across launches (epoch0, lm0), so the exchange words are cleared only when the epoch counter nears
  // its range (2^30 layers) and the error words only after a failed launch (they are written only on failure).
  if (e->mk_epoch > (1u << 30) || e->mk_lm_epoch > (1u << 30)) {
    CUDA_TRY(e, cudaMemsetAsync(e->mk_xw, 0, e->mk_tagged_words * sizeof(unsigned long long), e->st));
    e->mk_epoch = e->mk_lm_epoch = 0;
  }
  if (e->mk_io_dirty) {
    CUDA_TRY(e, cudaMemsetAsync(e->mk_io, 0, 8 * sizeof(int32_t), e->st));
    e->mk_io_dirty = false;
  }
  p.epoch0 = e->mk_epoch;
  p.lm0 = e->mk_lm_epoch;
  e->mk_io_dirty = true;  // until mk_status reads this launch's error words back clean
  e->mk_epoch += (uint32_t)steps * (uint32_t)c.layers;
  e->mk_lm_epoch += (uint32_t)steps;
  void* kargs[] = {&p};
  void* kern = trace ? e->mk_kernel_trace : last_pos > e->mk_kv_stage ? e->mk_kernel_lc : e->mk_kernel;
  CUDA_TRY(e, cudaLaunchCooperativeKernel(kern, dim3(e->mk_ncta), dim3(MK_THREADS), kargs, e->mk_smem, e->st));
  return H2C_OK;
}

// After a persistent launch has completed (stream synchronised): turn its error words into a status.
int mk_status(h2c_engine* e) {
  const int32_t* io = e->mk_io_h;
  e->mk_io_dirty = io[4] != 0;  // a launch whose status read back clean leaves the error words zero
  if (io[4] != 0)
    return e->fail(H2C_ERR_TIMEOUT, "persistent decode kernel: bounded wait expired (code %d, CTA %d, stage %d)", io[4],
                   io[5], io[6]);
  return H2C_OK;
}

// After a single-token launch with its arguments given: spin on the mapped record CTA 0 writes when the launch's
// token is known (no device-to-host copy, no stream synchronisation). The spin ends when the record appears or the
// stream reports the kernel finished (its own waits are bounded), so it cannot outlast the kernel.
int mk_wait_done(h2c_engine* e, int32_t* next) {
  volatile int32_t* d = e->mk_done_h;
  const int32_t want = e->mk_launch_seq;
  for (unsigned it = 1; d[0] != want; it++) {
    if (it % 4096) continue;
    const cudaError_t q = cudaStreamQuery(e->st);
    if (q == cudaErrorNotReady) continue;
    if (q != cudaSuccess) return e->fail(H2C_ERR_CUDA, "CUDA: %s", cudaGetErrorString(q));
    if (d[0] == want) break;
    // the kernel ended without writing its record (it cannot, short of a fault): read the device words instead
    CUDA_TRY(e, cudaMemcpy(e->mk_io_h, e->mk_io, 8 * sizeof(int32_t), cudaMemcpyDeviceToHost));
    int r = mk_status(e);
    if (r) return r;
    *next = e->mk_io_h[0];
    return H2C_OK;
  }
  std::atomic_thread_fence(std::memory_order_acquire);
  const int32_t code = d[2];
  e->mk_io_dirty = code != 0;
  if (code)
    return e->fail(H2C_ERR_TIMEOUT, "persistent decode kernel: bounded wait expired (code %d, CTA %d, stage %d)", code,
                   d[3], d[4]);
  *next = d[1];
  return H2C_OK;
}

// The tcgen05 matmul records a bounded wait that expired in e->tc5_err: copy it back after the passes that used it
// (enqueued right behind them) and turn it into a status once the stream has reached the copy.
int tc5_enqueue_check(h2c_engine* e) {
  if (e->tc5_used)
    CUDA_TRY(e, cudaMemcpyAsync(e->tc5_err_h, e->tc5_err, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost, e->st));
  return H2C_OK;
}
int tc5_status(h2c_engine* e) {
  if (!e->tc5_used) return H2C_OK;
  e->tc5_used = false;
  if (e->tc5_err_h[0] == 0) return H2C_OK;
  const int cta = e->tc5_err_h[1], role = e->tc5_err_h[2];
  memset(e->tc5_err_h, 0, 4 * sizeof(int32_t));
  CUDA_TRY(e, cudaMemsetAsync(e->tc5_err, 0, 4 * sizeof(int32_t), e->st));
  return e->fail(H2C_ERR_TIMEOUT, "tcgen05 matmul: bounded wait expired (CTA %d, role %d)", cta, role);
}

int run_forward(h2c_engine* e, int seq, const int32_t* ids, int32_t n, int32_t pos, Prof* pf) {
  const h2c_config& c = e->cfg;
  if (!ids || n < 1) return e->fail(H2C_ERR_INVALID, "forward needs at least one token");
  if (seq < 0 || seq >= c.max_seqs) return e->fail(H2C_ERR_INVALID, "sequence %d out of range [0, %d)", seq, c.max_seqs);
  if (pos < 0) return e->fail(H2C_ERR_INVALID, "negative position");
  if ((int64_t)pos + n >= c.ctx) return e->fail(H2C_ERR_CONTEXT_FULL, "context full");
  for (int i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= c.vocab) return e->fail(H2C_ERR_INVALID, "token id %d out of range", ids[i]);
  int r = check_ready(e);
  if (r) return r;
  if (e->comm_dead) return e->fail(H2C_ERR_INVALID, "tensor-parallel communicator aborted after a failure");
  const int MT = c.max_chunk;
  const int nchunks = (n + MT - 1) / MT;
  if (nchunks > e->prm_slots) return e->fail(H2C_ERR_INVALID, "too many chunks");
  const int stride = P_IDS + MT;
  e->mk_pending = false;
  for (int ci = 0; ci < nchunks; ci++) {
    e->mk_pending = false;
    const int c0 = ci * MT, mlen = n - c0 < MT ? n - c0 : MT;
    const bool last = ci == nchunks - 1;
    int32_t* h = e->prm_h + (size_t)ci * stride;
    h[P_POS0] = pos + c0;
    h[P_M] = mlen;
    h[P_SEQ] = seq;
    h[3] = 0;
    memcpy(h + P_IDS, ids + c0, sizeof(int32_t) * mlen);
    if (mlen == 1 && !pf) {
      if (e->decode_mode != H2C_DECODE_GRAPH && (r = mk_build(e))) return r;
      if (use_persistent(e)) {  // the token's parameters travel with the launch: nothing to copy first
        const int32_t args[3] = {seq, pos + c0, ids[c0]};
        if ((r = mk_launch(e, 1, pos + c0, nullptr, args))) return r;
        e->mk_pending = true;
        continue;
      }
    }
    CUDA_TRY(e, cudaMemcpyAsync(e->prm, h, sizeof(int32_t) * (P_IDS + mlen), cudaMemcpyHostToDevice, e->st));
    if (mlen == 1 && !pf) {
      if (!e->gexec) {
        r = build_graph(e);
        if (r) return r;
      }
      CUDA_TRY(e, cudaGraphLaunch(e->gexec, e->st));
    } else {
      enqueue_pass(e, mlen, last, pf, false, pos + c0, seq);
      if ((r = tp_enqueue_status(e))) return r;
      CUDA_TRY(e, cudaGetLastError());
      if ((r = tc5_enqueue_check(e))) return r;
    }
  }
  return H2C_OK;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

// Create an engine for one rank of a tensor-parallel group of G (G = 1: the whole model on this device).
int create_engine(int device, const h2c_config* cfg, int G, int rk, h2c_engine** out) {
  if (!out || !cfg) {
    g_create_error = "null argument";
    return H2C_ERR_INVALID;
  }
  *out = nullptr;
  const h2c_config& c = *cfg;
  if (c.dim <= 0 || c.dim % 32 || c.ffn <= 0 || c.ffn % 32 || c.heads <= 0 || c.kv_heads <= 0 || c.heads % c.kv_heads ||
      c.dim % c.heads || c.dim > MAX_DIM || c.layers <= 0 || c.vocab <= 0 || c.ctx < 2 || c.max_chunk < 1 ||
      c.max_chunk > 256 || c.max_seqs < 1) {
    g_create_error = "invalid configuration";
    return H2C_ERR_INVALID;
  }
  const int HD = c.dim / c.heads;
  if (HD != 64 && HD != 128) {
    g_create_error = "head_dim must be 64 or 128";
    return H2C_ERR_INVALID;
  }
  if (G > 1 && (c.kv_heads % G || c.dim % (32 * G) || c.ffn % (32 * G))) {
    g_create_error = "tensor parallelism needs kv_heads, dim / 32 and ffn / 32 divisible by the group size";
    return H2C_ERR_INVALID;
  }
  const int Vp = G == 1 ? c.vocab : (c.vocab + 32 * G - 1) / (32 * G) * 32;
  if (G > 1 && c.vocab <= (G - 1) * Vp) {
    g_create_error = "vocabulary too small for the group size";
    return H2C_ERR_INVALID;
  }
  h2c_engine* e = new h2c_engine();
  e->cfg = c;
  e->dev = device;
  e->HD = HD;
  e->tp_world = G;
  e->tp_rank = rk;
  e->Hl = c.heads / G;
  e->KVHl = c.kv_heads / G;
  e->Dl = c.dim / G;
  e->Fl = c.ffn / G;
  e->Vp = Vp;
  e->Vl = std::min(Vp, c.vocab - rk * Vp);
  e->QKV = (e->Hl + 2 * e->KVHl) * HD;
  e->L.resize(c.layers);
  e->layer_set.assign(c.layers, 0);
  e->last_logits_valid.assign(c.max_seqs, 0);
  auto bail = [&](int code) {
    g_create_error = e->err;
    h2c_destroy(e);
    return code;
  };
  cudaError_t ce = cudaSetDevice(device);
  if (ce != cudaSuccess) {
    e->err = std::string("cudaSetDevice: ") + cudaGetErrorString(ce);
    return bail(H2C_ERR_CUDA);
  }
  ce = cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking);
  if (ce != cudaSuccess) {
    e->err = std::string("cudaStreamCreate: ") + cudaGetErrorString(ce);
    return bail(H2C_ERR_CUDA);
  }
  const int MT = c.max_chunk, D = c.dim, F = c.ffn;
  const size_t kv = (size_t)c.max_seqs * c.layers * e->KVHl * c.ctx * HD;
  e->am_np = 296;
  if (c.ctx > MAX_CTX) {
    e->err = "ctx above 49152 positions (attention keeps one score per position in shared memory)";
    return bail(H2C_ERR_INVALID);
  }
  if (!kernel_attrs_on_current_device(&e->err)) return bail(H2C_ERR_CUDA);
  int r = 0;
  const int KQ = F > D ? F : D;
  if ((r = dalloc_t(e, &e->kc, kv)) || (r = dalloc_t(e, &e->vc, kv)) || (r = dalloc_t(e, &e->x, (size_t)MT * D)) ||
      (r = dalloc_t(e, &e->qkv, (size_t)MT * e->QKV)) || (r = dalloc_t(e, &e->att, (size_t)MT * D)) ||
      (r = dalloc_t(e, &e->gu, (size_t)MT * 2 * e->Fl)) || (r = dalloc_t(e, &e->logits, (size_t)G * Vp)) ||
      (r = dalloc_t(e, &e->xq, (size_t)MT * KQ)) || (r = dalloc_t(e, &e->xd, (size_t)MT * KQ / 32)) ||
      (r = dalloc_t(e, &e->xs, (size_t)MT * KQ / 32)) ||
      (r = dalloc_t(e, &e->am_v, (size_t)e->am_np)) || (r = dalloc_t(e, &e->am_i, (size_t)e->am_np)) ||
      (r = dalloc_t(e, &e->prm, (size_t)P_WORDS)) || (r = dalloc_t(e, &e->next_d, 1)) ||
      (r = dalloc_t(e, &e->toklog, (size_t)c.max_seqs * (c.ctx + 1))) ||
      (r = dalloc_t(e, &e->rope, (size_t)c.ctx * HD)) || (r = dalloc(e, &e->samp, sample_scratch_bytes(P_CAP))) ||
      (r = dalloc_t(e, &e->seeds_d, (size_t)P_CAP)) ||
      (r = dalloc_t(e, &e->xdT, (size_t)(KQ / 32) * ((MT + 3) / 4 * 4))) || (r = dalloc_t(e, &e->tc5_err, 4)))
    return bail(r);
  e->ldT = (MT + 3) / 4 * 4;
  // prompt attention (prompt_att.cuh) for passes of PF_MIN_TOKENS or more: scores of up to max_chunk tokens x all
  // positions, within a cap (H2C_PROMPT_SCORES_MB, default 256 MB); longer passes run in several query blocks
  if (MT >= PF_MIN_TOKENS && (HD == 64 || HD == 128)) {
    size_t cap = (size_t)256 << 20;
    if (const char* v = getenv("H2C_PROMPT_SCORES_MB")) {
      const long mb = atol(v);
      if (mb > 0) cap = (size_t)mb << 20;
    }
    const size_t row = (size_t)e->Hl * 4 * (size_t)((c.ctx + 3) & ~3);  // one token's score rows at full context
    e->pf_bytes = std::min(row * MT, cap);
    if (e->pf_bytes < row) e->pf_bytes = 0;
    if (e->pf_bytes && ((r = dalloc(e, reinterpret_cast<void**>(&e->pf_s), e->pf_bytes)) ||
                        (r = dalloc_t(e, &e->pf_sum, (size_t)e->Hl * MT)) ||
                        (r = dalloc_t(e, &e->pf_pm, (size_t)e->Hl * MT * pf_pm_pitch(c.ctx)))))
      return bail(r);
  }
  if (G > 1 && MT > 1) {  // staging of the gathers of passes of several tokens (the largest of them)
    const size_t nbl = (size_t)e->Fl / 32;
    const TpPart act[3] = {{nullptr, (size_t)e->Fl, 0, MT}, {nullptr, nbl * 4, 0, MT}, {nullptr, nbl * 16, 0, MT}};
    const TpPart xp{nullptr, (size_t)e->Dl * 4, 0, MT};
    e->tp_stage = std::max(tp_stage_bytes(act, 3), tp_stage_bytes(&xp, 1));
    if ((r = dalloc_t(e, &e->tp_send, e->tp_stage)) || (r = dalloc_t(e, &e->tp_recv, e->tp_stage * G))) return bail(r);
  }
  // RoPE table in double precision, cpu-worker.js:131-135
  {
    std::vector<float> t((size_t)c.ctx * HD);
    for (int i = 0; i < HD / 2; i++) {
      const double inv = std::pow(c.rope_theta, (2.0 * i) / HD);
      for (int p = 0; p < c.ctx; p++) {
        const double a = p / inv;
        t[(size_t)p * HD + 2 * i] = (float)std::cos(a);
        t[(size_t)p * HD + 2 * i + 1] = (float)std::sin(a);
      }
    }
    ce = cudaMemcpy(e->rope, t.data(), t.size() * 4, cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
      e->err = std::string("rope upload: ") + cudaGetErrorString(ce);
      return bail(H2C_ERR_CUDA);
    }
  }
  e->prm_slots = (c.ctx + MT - 1) / MT + 1;
  ce = cudaMallocHost(&e->prm_h, sizeof(int32_t) * (size_t)(P_IDS + MT) * e->prm_slots);
  if (ce == cudaSuccess) ce = cudaMallocHost(&e->next_h, sizeof(int32_t) * P_CAP);
  if (ce == cudaSuccess) ce = cudaMallocHost(&e->seeds_h, sizeof(uint32_t) * P_CAP);
  if (ce == cudaSuccess) ce = cudaMallocHost(&e->tc5_err_h, sizeof(int32_t) * 4);
  if (ce == cudaSuccess) memset(e->tc5_err_h, 0, sizeof(int32_t) * 4);
  if (ce != cudaSuccess) {
    e->err = std::string("pinned allocation: ") + cudaGetErrorString(ce);
    return bail(H2C_ERR_NO_MEMORY);
  }
  ce = cudaEventCreate(&e->ev0);
  if (ce == cudaSuccess) ce = cudaEventCreate(&e->ev1);
  if (ce != cudaSuccess) {
    e->err = std::string("cudaEventCreate: ") + cudaGetErrorString(ce);
    return bail(H2C_ERR_CUDA);
  }
  *out = e;
  return H2C_OK;
}

}  // namespace

extern "C" {

int h2c_create(int device, const h2c_config* cfg, h2c_engine** out) { return create_engine(device, cfg, 1, 0, out); }

int h2c_tp_unique_id(uint8_t* id) {
  if (!id) return H2C_ERR_INVALID;
  const NcclApi& nc = nccl();
  if (!nc.why.empty()) {
    g_create_error = nc.why;
    return H2C_ERR_UNSUPPORTED;
  }
  ncclUniqueId u;
  const ncclResult_t res = nc.get_unique_id(&u);
  if (res != ncclSuccess) {
    g_create_error = std::string("ncclGetUniqueId: ") + nc.error_string(res);
    return H2C_ERR_CUDA;
  }
  static_assert(sizeof(u.internal) == H2C_TP_ID_BYTES, "NCCL unique id size");
  memcpy(id, u.internal, H2C_TP_ID_BYTES);
  return H2C_OK;
}

int h2c_create_tp(int device, const h2c_config* cfg, int32_t world, int32_t rank, const uint8_t* id,
                  int32_t timeout_ms, h2c_engine** out) {
  if (out) *out = nullptr;
  if (!id || world < 1 || world > 8 || rank < 0 || rank >= world) {
    g_create_error = "tensor parallelism: world in [1, 8], rank in [0, world) and an id are required";
    return H2C_ERR_INVALID;
  }
  const NcclApi& nc = nccl();
  if (world > 1 && !nc.why.empty()) {
    g_create_error = nc.why;
    return H2C_ERR_UNSUPPORTED;
  }
  h2c_engine* e = nullptr;
  int r = create_engine(device, cfg, world, rank, &e);
  if (r) return r;
  e->tp_timeout_ms = timeout_ms > 0 ? timeout_ms : 120000;
  if (world == 1) {
    *out = e;
    return H2C_OK;
  }
  ncclUniqueId u;
  memcpy(u.internal, id, H2C_TP_ID_BYTES);
  ncclConfig_t conf = NCCL_CONFIG_INITIALIZER;
  conf.blocking = 0;  // every call returns at once; nccl_settle polls it against the deadline
  ncclResult_t res = nc.init_rank_config(&e->comm, world, u, rank, &conf);
  if (res != ncclSuccess && res != ncclInProgress) {
    e->comm = nullptr;
    g_create_error = std::string("ncclCommInitRankConfig: ") + nc.error_string(res);
    h2c_destroy(e);
    return H2C_ERR_CUDA;
  }
  if (!nccl_settle(e, res, "ncclCommInitRankConfig")) {  // a peer that never joined: abort, then report
    nc.abort(e->comm);
    e->comm = nullptr;
    const bool late = e->tp_fail.find("deadline") != std::string::npos;
    g_create_error = e->tp_fail + " (communicator aborted)";
    h2c_destroy(e);
    return late ? H2C_ERR_TIMEOUT : H2C_ERR_CUDA;
  }
  // first collectives outside any graph capture (connections are set up on first use): a small and a large gather
  for (size_t bytes : {(size_t)e->Dl * 4, (size_t)e->Vp * 4}) {
    const TpPart warm{reinterpret_cast<uint8_t*>(e->logits), bytes, 0, 1};
    tp_gather(e, e->st, &warm, 1);
    if ((r = tp_enqueue_status(e)) || (r = sync_stream(e))) {
      g_create_error = e->err;
      h2c_destroy(e);
      return r;
    }
  }
  std::string why;
  if (!tp_setup_xch(e, &why)) {
    g_create_error = "tensor parallelism: peer exchange set-up failed: " + why;
    h2c_destroy(e);
    return H2C_ERR_CUDA;
  }
  *out = e;
  return H2C_OK;
}

int32_t h2c_tp_rank(const h2c_engine* e) { return e ? e->tp_rank : -1; }
int32_t h2c_tp_world(const h2c_engine* e) { return e ? e->tp_world : 0; }

int h2c_set_tensor(h2c_engine* e, int kind, int layer, int ggml_type, const void* data, uint64_t nbytes) {
  if (!e || !data) return H2C_ERR_INVALID;
  const h2c_config& c = e->cfg;
  CUDA_TRY(e, cudaSetDevice(e->dev));
  if (kind < 0 || kind > 9) return e->fail(H2C_ERR_INVALID, "unknown tensor kind %d", kind);
  if (kind <= 6 && (layer < 0 || layer >= c.layers)) return e->fail(H2C_ERR_INVALID, "layer %d out of range", layer);
  const int D = c.dim, F = c.ffn, HD = e->HD, rk = e->tp_rank;
  const int Hl = e->Hl, KVHl = e->KVHl, Dl = e->Dl, Fl = e->Fl;
  int r = H2C_OK;
  auto need = [&](int t) { return ggml_type == t; };
  // Under tensor parallelism the caller passes the full tensor (full_rows rows of row_bytes): keep this rank's rows,
  // the ranges {first row, rows}, in that order.
  std::vector<uint8_t> part;
  auto keep = [&](int full_rows, size_t row_bytes, std::initializer_list<std::pair<int, int>> ranges) {
    if (e->tp_world == 1) return true;
    if (nbytes != (uint64_t)full_rows * row_bytes) {
      e->fail(H2C_ERR_INVALID, "kind %d: %llu bytes, expected the full tensor of %lld", kind, (unsigned long long)nbytes,
              (long long)full_rows * (long long)row_bytes);
      return false;
    }
    size_t n = 0;
    for (auto& g : ranges) n += (size_t)g.second * row_bytes;
    part.resize(n);
    size_t o = 0;
    for (auto& g : ranges) {
      memcpy(part.data() + o, (const uint8_t*)data + (size_t)g.first * row_bytes, (size_t)g.second * row_bytes);
      o += (size_t)g.second * row_bytes;
    }
    data = part.data();
    nbytes = n;
    return true;
  };
  const int qkv_full = D + 2 * c.kv_heads * HD;
  // q rows of this rank's heads, then the k and v rows of its kv heads
  const std::initializer_list<std::pair<int, int>> qkv_rows = {
      {rk * Hl * HD, Hl * HD}, {D + rk * KVHl * HD, KVHl * HD}, {D + (c.kv_heads + rk * KVHl) * HD, KVHl * HD}};
  const size_t q4_row_d = (size_t)(D / 32) * 18;
  switch (kind) {
    case H2C_KIND_QKV:
    case H2C_KIND_O:
    case H2C_KIND_GATE_UP:
    case H2C_KIND_DOWN: {
      if (!need(H2C_GGML_Q4_0)) return e->fail(H2C_ERR_BAD_TYPE, "layer %d kind %d: expected Q4_0", layer, kind);
      LayerW& W = e->L[layer];
      bool ok = true;
      if (kind == 0) ok = keep(qkv_full, q4_row_d, qkv_rows);
      if (kind == 1) ok = keep(D, q4_row_d, {{rk * Dl, Dl}});
      if (kind == 2) ok = keep(2 * F, q4_row_d, {{rk * Fl, Fl}, {F + rk * Fl, Fl}});
      if (kind == 3) ok = keep(D, (size_t)(F / 32) * 18, {{rk * Dl, Dl}});
      if (!ok) return H2C_ERR_INVALID;
      if (kind == 0) r = upload_q4(e, &W.qkv, e->QKV, D, data, nbytes);
      if (kind == 1) r = upload_q4(e, &W.o, Dl, D, data, nbytes);
      if (kind == 2) r = upload_q4(e, &W.gu, 2 * Fl, D, data, nbytes);
      if (kind == 3) r = upload_q4(e, &W.down, Dl, F, data, nbytes);
      break;
    }
    case H2C_KIND_ATTN_NORM:
    case H2C_KIND_FFN_NORM:
    case H2C_KIND_QKV_BIAS: {
      if (!need(H2C_GGML_F32)) return e->fail(H2C_ERR_BAD_TYPE, "layer %d kind %d: expected F32", layer, kind);
      LayerW& W = e->L[layer];
      if (kind == 4) r = upload_f32(e, &W.attn_norm, D, data, nbytes);
      if (kind == 5) r = upload_f32(e, &W.ffn_norm, D, data, nbytes);
      if (kind == 6) {
        if (!keep(qkv_full, 4, qkv_rows)) return H2C_ERR_INVALID;
        r = upload_f32(e, &W.bqkv, e->QKV, data, nbytes);
      }
      break;
    }
    case H2C_KIND_EMBED:  // every rank keeps the whole table (token lookups; the tied lm_head uses its rows)
      if (!need(H2C_GGML_Q4_0)) return e->fail(H2C_ERR_BAD_TYPE, "token_embd: expected Q4_0");
      r = upload_q4(e, &e->embd, c.vocab, D, data, nbytes);
      if (!r) e->embd_set = true;
      return r;
    case H2C_KIND_OUTPUT:
      if (need(H2C_GGML_Q8_0)) {
        if (!keep(c.vocab, (size_t)(D / 32) * 34, {{rk * e->Vp, e->Vl}})) return H2C_ERR_INVALID;
        r = upload_q8(e, &e->out8, e->Vl, D, data, nbytes);
        if (!r) e->out_type = 8;
      } else if (need(H2C_GGML_Q4_0)) {
        if (!keep(c.vocab, q4_row_d, {{rk * e->Vp, e->Vl}})) return H2C_ERR_INVALID;
        r = upload_q4(e, &e->out4, e->Vl, D, data, nbytes);
        if (!r) e->out_type = 2;
      } else {
        return e->fail(H2C_ERR_BAD_TYPE, "output.weight: expected Q8_0 or Q4_0");
      }
      return r;
    case H2C_KIND_OUTPUT_NORM:
      if (!need(H2C_GGML_F32)) return e->fail(H2C_ERR_BAD_TYPE, "output_norm: expected F32");
      r = upload_f32(e, &e->out_norm, D, data, nbytes);
      if (!r) e->out_norm_set = true;
      return r;
  }
  if (!r) e->layer_set[layer] |= 1 << kind;
  return r;
}

int h2c_forward(h2c_engine* e, int seq, const int32_t* ids, int32_t n, int32_t pos, double temperature, uint32_t seed,
                int32_t* next) {
  if (!e || !next) return H2C_ERR_INVALID;
  CUDA_TRY(e, cudaSetDevice(e->dev));
  int r = run_forward(e, seq, ids, n, pos, nullptr);
  if (r) return r;
  if (temperature > 0) {  // the draw runs on the device (sample.cu) over the logits of the last token
    CUDA_TRY(e, launch_sample(e->logits, e->cfg.vocab, 1, temperature, nullptr, seed + (uint32_t)pos, e->next_d,
                              e->samp, e->st));
    CUDA_TRY(e, cudaMemcpyAsync(e->next_h, e->next_d, 4, cudaMemcpyDeviceToHost, e->st));
    if (e->mk_pending)
      CUDA_TRY(e, cudaMemcpyAsync(e->mk_io_h, e->mk_io, 8 * sizeof(int32_t), cudaMemcpyDeviceToHost, e->st));
    if ((r = sync_stream(e))) return r;
    if (e->mk_pending && (r = mk_status(e))) return r;
    *next = *e->next_h;
  } else if (e->mk_pending) {
    if ((r = mk_wait_done(e, next))) return r;
  } else {
    CUDA_TRY(e, cudaMemcpyAsync(e->next_h, e->next_d, 4, cudaMemcpyDeviceToHost, e->st));
    if ((r = sync_stream(e))) return r;
    *next = *e->next_h;
  }
  if ((r = tc5_status(e))) return r;
  e->last_logits_valid.assign(e->cfg.max_seqs, 0);
  e->last_logits_valid[seq] = 1;
  return H2C_OK;
}

// Validate a batch, allocate the batch buffers on first use, write the pass parameters (mode 1) and launch the
// batch graph for n tokens `steps` times (each launch's argmax feeds the next).
int batch_launch(h2c_engine* e, int32_t n, const int32_t* seqs, const int32_t* ids, const int32_t* pos, int steps,
                 cudaEvent_t before = nullptr) {
  const h2c_config& c = e->cfg;
  if (e->tp_world > 1) return e->fail(H2C_ERR_INVALID, "batched steps are not available with tensor parallelism");
  const int cap = c.max_chunk < P_CAP ? c.max_chunk : P_CAP;
  if (n < 1 || n > cap) return e->fail(H2C_ERR_INVALID, "batch of %d sequences (1 .. %d per step)", n, cap);
  std::vector<char> seen(c.max_seqs, 0);
  for (int m = 0; m < n; m++) {
    if (seqs[m] < 0 || seqs[m] >= c.max_seqs) return e->fail(H2C_ERR_INVALID, "sequence %d out of range [0, %d)", seqs[m], c.max_seqs);
    if (seen[seqs[m]]) return e->fail(H2C_ERR_INVALID, "sequence %d appears twice in one batch", seqs[m]);
    seen[seqs[m]] = 1;
    if (pos[m] < 0) return e->fail(H2C_ERR_INVALID, "negative position");
    if ((int64_t)pos[m] + steps >= c.ctx) return e->fail(H2C_ERR_CONTEXT_FULL, "context full (sequence %d)", seqs[m]);
    if (ids[m] < 0 || ids[m] >= c.vocab) return e->fail(H2C_ERR_INVALID, "token id %d out of range", ids[m]);
  }
  CUDA_TRY(e, cudaSetDevice(e->dev));
  int r = check_ready(e);
  if (r) return r;
  if (!e->logits_b) {
    if ((r = dalloc_t(e, &e->logits_b, (size_t)cap * c.vocab)) || (r = dalloc_t(e, &e->am_vb, (size_t)cap * e->am_np)) ||
        (r = dalloc_t(e, &e->am_ib, (size_t)cap * e->am_np)) || (r = dalloc_t(e, &e->next_b, (size_t)P_CAP)))
      return r;
    CUDA_TRY(e, cudaMallocHost(&e->prm_bh, sizeof(int32_t) * P_WORDS));
    CUDA_TRY(e, cudaMallocHost(&e->next_bh, sizeof(int32_t) * P_CAP));
    memset(e->prm_bh, 0, sizeof(int32_t) * P_WORDS);
    e->bexec.assign(cap + 1, nullptr);
    e->bkernels.assign(cap + 1, 0);
    e->btc5.assign(cap + 1, 0);
  }
  int32_t* h = e->prm_bh;
  h[P_POS0] = 0; h[P_M] = n; h[P_SEQ] = 0; h[P_MODE] = 1;
  for (int m = 0; m < n; m++) {
    h[P_IDS + m] = ids[m];
    h[P_IDS + P_CAP + m] = pos[m];
    h[P_IDS + 2 * P_CAP + m] = seqs[m];
  }
  CUDA_TRY(e, cudaMemcpyAsync(e->prm, h, sizeof(int32_t) * P_WORDS, cudaMemcpyHostToDevice, e->st));
  if (!e->bexec[n]) {  // one graph per batch size, captured on first use
    cudaGraph_t g = nullptr;
    CUDA_TRY(e, cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
    const bool used_before = e->tc5_used;
    e->tc5_used = false;
    enqueue_pass(e, n, false, nullptr, true);
    e->btc5[n] = e->tc5_used;
    e->tc5_used = used_before;
    cudaError_t ce = cudaStreamEndCapture(e->st, &g);
    if (ce != cudaSuccess) return e->fail(H2C_ERR_CUDA, "graph capture: %s", cudaGetErrorString(ce));
    ce = cudaGraphInstantiate(&e->bexec[n], g, 0);
    size_t nn = 0;
    if (ce == cudaSuccess) ce = cudaGraphGetNodes(g, nullptr, &nn);
    std::vector<cudaGraphNode_t> nodes(nn);
    if (ce == cudaSuccess && nn) ce = cudaGraphGetNodes(g, nodes.data(), &nn);
    for (size_t i = 0; ce == cudaSuccess && i < nn; i++) {
      cudaGraphNodeType ty;
      ce = cudaGraphNodeGetType(nodes[i], &ty);
      if (ce == cudaSuccess && ty == cudaGraphNodeTypeKernel) e->bkernels[n]++;
    }
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return e->fail(H2C_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(ce));
  }
  if (before) CUDA_TRY(e, cudaEventRecord(before, e->st));
  for (int i = 0; i < steps; i++) CUDA_TRY(e, cudaGraphLaunch(e->bexec[n], e->st));
  if (e->btc5[n]) {
    e->tc5_used = true;
    if ((r = tc5_enqueue_check(e))) return r;
  }
  return H2C_OK;
}

int h2c_forward_batch(h2c_engine* e, int32_t n, const int32_t* seqs, const int32_t* ids, const int32_t* pos,
                      double temperature, uint32_t seed, int32_t* next) {
  if (!e || !seqs || !ids || !pos || !next) return H2C_ERR_INVALID;
  const h2c_config& c = e->cfg;
  int r = batch_launch(e, n, seqs, ids, pos, 1);
  if (r) return r;
  if (temperature > 0) {  // each token's draw on the device, seeded by seed + its position
    for (int m = 0; m < n; m++) e->seeds_h[m] = seed + (uint32_t)pos[m];
    CUDA_TRY(e, cudaMemcpyAsync(e->seeds_d, e->seeds_h, sizeof(uint32_t) * n, cudaMemcpyHostToDevice, e->st));
    CUDA_TRY(e, launch_sample(e->logits_b, c.vocab, n, temperature, e->seeds_d, 0, e->next_b, e->samp, e->st));
    CUDA_TRY(e, cudaMemcpyAsync(e->next_bh, e->next_b, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, e->st));
    CUDA_TRY(e, cudaStreamSynchronize(e->st));
    memcpy(next, e->next_bh, sizeof(int32_t) * n);
  } else {
    CUDA_TRY(e, cudaMemcpyAsync(e->next_bh, e->next_b, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, e->st));
    CUDA_TRY(e, cudaStreamSynchronize(e->st));
    memcpy(next, e->next_bh, sizeof(int32_t) * n);
  }
  if ((r = tc5_status(e))) return r;
  e->last_logits_valid.assign(c.max_seqs, 0);
  for (int m = 0; m < n; m++) e->last_logits_valid[seqs[m]] = 2 + m;  // row m of the batch logits
  return H2C_OK;
}

int h2c_generate_batch(h2c_engine* e, int32_t n, const int32_t* seqs, const int32_t* ids, const int32_t* pos,
                       int32_t steps, int32_t* out_tokens, float* device_ms) {
  if (!e || !seqs || !ids || !pos || steps < 1) return H2C_ERR_INVALID;
  const h2c_config& c = e->cfg;
  CUDA_TRY(e, cudaSetDevice(e->dev));
  int r = batch_launch(e, n, seqs, ids, pos, steps, e->ev0);  // ev0: after the parameter copy and graph build
  if (r) return r;
  CUDA_TRY(e, cudaEventRecord(e->ev1, e->st));
  if (out_tokens)
    for (int m = 0; m < n; m++)
      CUDA_TRY(e, cudaMemcpyAsync(out_tokens + (size_t)m * steps, e->toklog + (size_t)seqs[m] * (c.ctx + 1) + pos[m] + 1,
                                  sizeof(int32_t) * steps, cudaMemcpyDeviceToHost, e->st));
  CUDA_TRY(e, cudaStreamSynchronize(e->st));
  if ((r = tc5_status(e))) return r;
  if (device_ms) CUDA_TRY(e, cudaEventElapsedTime(device_ms, e->ev0, e->ev1));
  e->last_logits_valid.assign(c.max_seqs, 0);
  for (int m = 0; m < n; m++) e->last_logits_valid[seqs[m]] = 2 + m;
  return H2C_OK;
}

int h2c_generate(h2c_engine* e, int seq, int32_t first_id, int32_t pos, int32_t steps, int32_t* out_tokens,
                 float* device_ms) {
  if (!e || steps < 1) return H2C_ERR_INVALID;
  const h2c_config& c = e->cfg;
  if (seq < 0 || seq >= c.max_seqs) return e->fail(H2C_ERR_INVALID, "sequence %d out of range", seq);
  if (pos < 0 || (int64_t)pos + steps >= c.ctx) return e->fail(H2C_ERR_CONTEXT_FULL, "context full");
  if (first_id < 0 || first_id >= c.vocab) return e->fail(H2C_ERR_INVALID, "token id %d out of range", first_id);
  CUDA_TRY(e, cudaSetDevice(e->dev));
  int r = check_ready(e);
  if (r) return r;
  if (e->comm_dead) return e->fail(H2C_ERR_INVALID, "tensor-parallel communicator aborted after a failure");
  if (e->decode_mode != H2C_DECODE_GRAPH && (r = mk_build(e))) return r;
  if (!use_persistent(e) && !e->gexec && (r = build_graph(e))) return r;
  int32_t* h = e->prm_h;
  h[P_POS0] = pos;
  h[P_M] = 1;
  h[P_SEQ] = seq;
  h[3] = 0;
  h[P_IDS] = first_id;
  CUDA_TRY(e, cudaMemcpyAsync(e->prm, h, sizeof(int32_t) * (P_IDS + 1), cudaMemcpyHostToDevice, e->st));
  const bool mk = use_persistent(e);
  CUDA_TRY(e, cudaEventRecord(e->ev0, e->st));
  if (mk) {
    if ((r = mk_launch(e, steps, pos + steps - 1))) return r;
  } else {
    for (int i = 0; i < steps; i++) CUDA_TRY(e, cudaGraphLaunch(e->gexec, e->st));
  }
  CUDA_TRY(e, cudaEventRecord(e->ev1, e->st));
  if (mk) CUDA_TRY(e, cudaMemcpyAsync(e->mk_io_h, e->mk_io, 8 * sizeof(int32_t), cudaMemcpyDeviceToHost, e->st));
  if (out_tokens)
    CUDA_TRY(e, cudaMemcpyAsync(out_tokens, e->toklog + (size_t)seq * (c.ctx + 1) + pos + 1, sizeof(int32_t) * steps,
                                cudaMemcpyDeviceToHost, e->st));
  if ((r = sync_stream(e))) return r;
  if (mk && (r = mk_status(e))) return r;
  if (device_ms) CUDA_TRY(e, cudaEventElapsedTime(device_ms, e->ev0, e->ev1));
  e->last_logits_valid.assign(c.max_seqs, 0);
  e->last_logits_valid[seq] = 1;
  return H2C_OK;
}

int h2c_trace_decode(h2c_engine* e, int seq, int32_t first_id, int32_t pos, int32_t steps, uint64_t* out, int64_t n) {
  if (!e || !out || steps < 1) return H2C_ERR_INVALID;
  const h2c_config& c = e->cfg;
  if (seq < 0 || seq >= c.max_seqs || pos < 0 || (int64_t)pos + steps >= c.ctx || first_id < 0 || first_id >= c.vocab)
    return e->fail(H2C_ERR_INVALID, "bad trace arguments");
  CUDA_TRY(e, cudaSetDevice(e->dev));
  int r = check_ready(e);
  if (r) return r;
  if ((r = mk_build(e))) return r;
  if (!e->mk_ok) return e->fail(H2C_ERR_INVALID, "persistent decode kernel unavailable: %s", e->mk_why.c_str());
  const int64_t need = (int64_t)e->mk_ncta * steps * (c.layers + 1) * MK_TRACE_PTS;
  if (n < need) return e->fail(H2C_ERR_INVALID, "trace needs %lld entries", (long long)need);
  unsigned long long* d = nullptr;
  CUDA_TRY(e, cudaMalloc(&d, need * 8));
  CUDA_TRY(e, cudaMemsetAsync(d, 0, need * 8, e->st));
  int32_t* h = e->prm_h;
  h[P_POS0] = pos; h[P_M] = 1; h[P_SEQ] = seq; h[3] = 0; h[P_IDS] = first_id;
  CUDA_TRY(e, cudaMemcpyAsync(e->prm, h, sizeof(int32_t) * (P_IDS + 1), cudaMemcpyHostToDevice, e->st));
  r = mk_launch(e, steps, pos + steps - 1, d);
  if (!r) {
    CUDA_TRY(e, cudaMemcpyAsync(e->mk_io_h, e->mk_io, 8 * sizeof(int32_t), cudaMemcpyDeviceToHost, e->st));
    CUDA_TRY(e, cudaMemcpyAsync(out, d, need * 8, cudaMemcpyDeviceToHost, e->st));
    CUDA_TRY(e, cudaStreamSynchronize(e->st));
    r = mk_status(e);
  }
  cudaFree(d);
  return r;
}

int h2c_set_decode_fault(h2c_engine* e, int stall_cta, int64_t timeout_ns) {
  if (!e || stall_cta < -1 || timeout_ns < 1000000 || timeout_ns > 10000000000ll)
    return e ? e->fail(H2C_ERR_INVALID, "stall_cta must be >= -1 and timeout_ns in [1 ms, 10 s]") : H2C_ERR_INVALID;
  e->mk_stall_cta = stall_cta;
  e->mk_timeout_ns = (unsigned long long)timeout_ns;
  return H2C_OK;
}

int h2c_decode_ctas(h2c_engine* e) {
  if (!e) return H2C_ERR_INVALID;
  CUDA_TRY(e, cudaSetDevice(e->dev));
  int r = check_ready(e);
  if (r) return r;
  if ((r = mk_build(e))) return r;
  return e->mk_ok ? e->mk_ncta : 0;
}

int h2c_batch_kernels(h2c_engine* e, int32_t n) {
  if (!e) return H2C_ERR_INVALID;
  if (n < 1 || n >= (int)e->bexec.size() || !e->bexec[n]) return 0;
  return e->bkernels[n];
}

int h2c_decode_kernels(h2c_engine* e) {
  if (!e) return H2C_ERR_INVALID;
  CUDA_TRY(e, cudaSetDevice(e->dev));
  {
    int r = check_ready(e);
    if (r) return r;
    if (e->decode_mode != H2C_DECODE_GRAPH && (r = mk_build(e))) return r;
    if (use_persistent(e)) return 1;
  }
  if (!e->gexec) {
    int r = check_ready(e);
    if (r) return r;
    if ((r = build_graph(e))) return r;
  }
  return e->graph_kernels;
}

int h2c_set_decode_mode(h2c_engine* e, int mode) {
  if (!e || mode < H2C_DECODE_AUTO || mode > H2C_DECODE_PERSISTENT) return H2C_ERR_INVALID;
  if (mode == H2C_DECODE_PERSISTENT) {
    CUDA_TRY(e, cudaSetDevice(e->dev));
    int r = check_ready(e);
    if (r) return r;
    if ((r = mk_build(e))) return r;
    if (!e->mk_ok) return e->fail(H2C_ERR_INVALID, "persistent decode kernel unavailable: %s", e->mk_why.c_str());
  }
  e->decode_mode = mode;
  return H2C_OK;
}

int h2c_decode_path(h2c_engine* e) {
  if (!e) return H2C_ERR_INVALID;
  CUDA_TRY(e, cudaSetDevice(e->dev));
  int r = check_ready(e);
  if (r) return r;
  if (e->decode_mode != H2C_DECODE_GRAPH && (r = mk_build(e))) return r;
  return use_persistent(e) ? H2C_DECODE_PERSISTENT : H2C_DECODE_GRAPH;
}

int h2c_read_logits(h2c_engine* e, int seq, float* out, int64_t n) {
  if (!e || !out) return H2C_ERR_INVALID;
  if (seq < 0 || seq >= e->cfg.max_seqs || !e->last_logits_valid[seq])
    return e->fail(H2C_ERR_INVALID, "no logits for sequence %d (its last forward was not the latest)", seq);
  if (n < e->cfg.vocab) return e->fail(H2C_ERR_INVALID, "output holds %lld floats, vocab is %d", (long long)n, e->cfg.vocab);
  CUDA_TRY(e, cudaSetDevice(e->dev));
  const int v = e->last_logits_valid[seq];
  const float* src = v >= 2 ? e->logits_b + (size_t)(v - 2) * e->cfg.vocab : e->logits;
  CUDA_TRY(e, cudaMemcpyAsync(out, src, (size_t)e->cfg.vocab * 4, cudaMemcpyDeviceToHost, e->st));
  return sync_stream(e);
}

int h2c_profile(h2c_engine* e, int seq, const int32_t* ids, int32_t n, int32_t pos, double* ms) {
  if (!e || !ms) return H2C_ERR_INVALID;
  CUDA_TRY(e, cudaSetDevice(e->dev));
  Prof pf;
  for (int i = 0; i < 64; i++) CUDA_TRY(e, cudaEventCreate(&pf.ev[i]));
  pf.on = true;
  int r = run_forward(e, seq, ids, n, pos, &pf);
  if (!r) r = sync_stream(e);
  if (!r) r = tc5_status(e);
  for (int i = 0; i < H2C_NPROF; i++) ms[i] = 0;
  if (!r) {
    // events are reused in a ring when more than 64 marks are recorded: fold only the final window
    for (int i = 1; i < pf.n; i++) {
      float t = 0;
      cudaEventElapsedTime(&t, pf.ev[i - 1], pf.ev[i]);
      if (pf.op[i] >= 0 && pf.op[i] < H2C_NPROF) ms[pf.op[i]] += t;
    }
  }
  for (int i = 0; i < 64; i++) cudaEventDestroy(pf.ev[i]);
  if (!r) {
    e->last_logits_valid.assign(e->cfg.max_seqs, 0);
    e->last_logits_valid[seq] = 1;
  }
  return r;
}

int h2c_destroy(h2c_engine* e) {
  if (!e) return H2C_OK;
  cudaSetDevice(e->dev);
  if (e->st) cudaStreamSynchronize(e->st);
  if (e->gexec) cudaGraphExecDestroy(e->gexec);
  for (cudaGraphExec_t g : e->bexec)
    if (g) cudaGraphExecDestroy(g);
  if (e->prm_bh) cudaFreeHost(e->prm_bh);
  if (e->next_bh) cudaFreeHost(e->next_bh);
  if (e->graph) cudaGraphDestroy(e->graph);
  for (void* p : e->ipc_open) cudaIpcCloseMemHandle(p);
  if (e->xerr_h) cudaFreeHost(e->xerr_h);
  if (e->comm) {  // after the graphs that hold its collectives; a finalize that does not settle ends in an abort
    const NcclApi& nc = nccl();
    ncclResult_t res = nc.finalize(e->comm);
    const int64_t t0 = steady_ms();
    while (res == ncclInProgress && steady_ms() - t0 < std::max<int64_t>(e->tp_timeout_ms, 1000)) {
      std::this_thread::yield();
      if (nc.async_error(e->comm, &res) != ncclSuccess) break;
    }
    if (res == ncclSuccess) nc.destroy(e->comm);
    else nc.abort(e->comm);
    e->comm = nullptr;
  }
  for (void* p : e->dallocs) cudaFree(p);
  if (e->prm_h) cudaFreeHost(e->prm_h);
  if (e->mk_io_h) cudaFreeHost(e->mk_io_h);
  if (e->mk_done_h) cudaFreeHost(e->mk_done_h);
  if (e->next_h) cudaFreeHost(e->next_h);
  if (e->seeds_h) cudaFreeHost(e->seeds_h);
  if (e->tc5_err_h) cudaFreeHost(e->tc5_err_h);
  if (e->ev0) cudaEventDestroy(e->ev0);
  if (e->ev1) cudaEventDestroy(e->ev1);
  if (e->st) cudaStreamDestroy(e->st);
  delete e;
  return H2C_OK;
}

const char* h2c_last_error(const h2c_engine* e) { return e ? e->err.c_str() : g_create_error.c_str(); }

int64_t h2c_device_bytes(const h2c_engine* e) { return e ? e->dev_bytes : 0; }

uint64_t h2c_q4_matrix_bytes(int32_t n_rows, int32_t k) {
  if (n_rows <= 0 || k <= 0) return 0;
  const uint64_t nbp = padded_rows(n_rows) * (uint64_t)(k / 32);
  return align_up(nbp * 16, 256) + align_up(nbp * 2, 16);
}

int h2c_q4_pack(const void* gguf_blocks, int32_t n_rows, int32_t k, void* packed_host) {
  if (!gguf_blocks || !packed_host || n_rows <= 0 || k <= 0 || k % 32) return H2C_ERR_INVALID;
  const size_t nbp = padded_rows(n_rows) * (k / 32);
  uint8_t* dst = (uint8_t*)packed_host;
  memset(dst, 0, h2c_q4_matrix_bytes(n_rows, k));
  pack_blocks_host((const uint8_t*)gguf_blocks, n_rows, k, 18, dst, (uint16_t*)(dst + align_up(nbp * 16, 256)));
  return H2C_OK;
}

uint64_t h2c_q4_matvec_scratch_bytes(int32_t m, int32_t k) {
  if (m <= 0 || k <= 0) return 0;
  const uint64_t nb = (uint64_t)m * (uint64_t)(k / 32);
  return align_up((uint64_t)m * k, 256) + align_up(nb * 4, 256) + align_up(nb * 16, 256);
}

}  // extern "C"

namespace {
// The failure record of tcgen05 matmuls launched by h2c_q4_matvec (no engine to hold one): a small __device__
// array, its address looked up once per device.
__device__ int g_tc5_err_words[4];
int* g_tc5_err_ptr[ATTR_MAX_DEVICES];
std::mutex g_tc5_err_mutex;
int* tc5_standalone_err(std::string* why) {
  int dev = -1;
  cudaError_t c = cudaGetDevice(&dev);
  if (c != cudaSuccess || dev < 0 || dev >= ATTR_MAX_DEVICES) {
    *why = "cudaGetDevice failed";
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_tc5_err_mutex);
  if (!g_tc5_err_ptr[dev]) {
    void* p = nullptr;
    c = cudaGetSymbolAddress(&p, g_tc5_err_words);
    if (c != cudaSuccess || !p) {
      *why = std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(c);
      return nullptr;
    }
    g_tc5_err_ptr[dev] = static_cast<int*>(p);
  }
  return g_tc5_err_ptr[dev];
}
}  // namespace

extern "C" {

int h2c_set_matmul_kernel(int kind) {
  if (kind < H2C_MATMUL_AUTO || kind > H2C_MATMUL_TCGEN05) return H2C_ERR_INVALID;
  g_mm_kind.store(kind);
  return H2C_OK;
}

int h2c_matmul_kernel(void) { return g_mm_kind.load(); }

int h2c_q4_matvec(const void* w, int32_t n_rows, int32_t k, const float* x, int32_t m, float* y, int32_t op,
                  const float* bias, void* scratch, void* stream) {
  if (!w || !x || !y || !scratch || n_rows <= 0 || k <= 0 || k % 32 || m < 1 || op < 0 || op > 2 || (op == 1 && !bias)) {
    g_create_error = "h2c_q4_matvec: invalid argument";
    return H2C_ERR_INVALID;
  }
  if (((uintptr_t)w | (uintptr_t)scratch | (uintptr_t)x) & 15) {
    g_create_error = "h2c_q4_matvec: w, x and scratch must be 16-byte aligned";
    return H2C_ERR_INVALID;
  }
  std::string why;
  if (!kernel_attrs_on_current_device(&why)) {
    g_create_error = "h2c_q4_matvec: " + why;
    return H2C_ERR_CUDA;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const size_t nbp = padded_rows(n_rows) * (k / 32);
  Q4Mat W;
  W.qs = (uint8_t*)w;
  W.d = (__half*)((uint8_t*)w + align_up(nbp * 16, 256));
  W.N = n_rows;
  W.K = k;
  uint8_t* s = (uint8_t*)scratch;
  const size_t mb = (size_t)m * (k / 32);
  int8_t* xq = (int8_t*)s;
  float* xd = (float*)(s + align_up((size_t)m * k, 256));
  int4* xs = (int4*)(s + align_up((size_t)m * k, 256) + align_up(mb * 4, 256));
  const int warps = (int)mb;
  if (m > 1 && use_tc5(m)) {  // the tcgen05 form reads the scales transposed, kept where the lane sums would go
    int* err = tc5_standalone_err(&why);
    if (!err) {
      g_create_error = "h2c_q4_matvec: " + why;
      return H2C_ERR_CUDA;
    }
    const int ldT = (m + 3) / 4 * 4;
    float* xdT = reinterpret_cast<float*>(xs);
    k_quant<<<(warps + 7) / 8, 256, 0, st>>>(x, k, m, xq, xd, nullptr, xdT, ldT);
    const MmCtx mc{xdT, ldT, m, err, nullptr};
    matvec(op, W, xq, xd, nullptr, m, y, n_rows, bias, st, &mc);
  } else {
    k_quant<<<(warps + 7) / 8, 256, 0, st>>>(x, k, m, xq, xd, xs);
    matvec(op, W, xq, xd, xs, m, y, n_rows, bias, st);
  }
  cudaError_t c = cudaGetLastError();
  if (c != cudaSuccess) {
    g_create_error = std::string("h2c_q4_matvec: launch failed: ") + cudaGetErrorString(c);
    return H2C_ERR_CUDA;
  }
  return H2C_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- Q4_0 matvec without any allocation
//
// Some callers cannot call cudaMalloc: a host application that owns all device memory through its own pool and
// forbids side allocations, or code on a latency-critical thread (a voice pipeline's audio callback, say), where
// cudaMalloc can block and synchronize the device. For them h2c_q4_matvec_noalloc takes its scratch (the int8
// activations, their scales and lane sums) from this fixed array instead of from the caller.
//
// The array is a file-scope __device__ variable: every GPU that loads this library holds its 256 KiB until the
// process exits. On the host, its name is only a stand-in, not a device address, so the address the kernels get
// comes from cudaGetSymbolAddress, looked up once per device with that device current (the first call of
// h2c_q4_matvec_noalloc on a device does it; make that first call before any stream capture). Every call shares
// the array and it keeps the last call's contents: nothing has to start at zero, because each call writes every
// scratch byte it reads before reading it, but calls that overlap on the GPU (concurrent streams or threads) race
// on it and must be serialised by the caller.

namespace {
constexpr uint64_t NOALLOC_SCRATCH_BYTES = 256 * 1024;
constexpr int NOALLOC_MAX_DEVICES = 64;
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];
void* g_noalloc_ptr[NOALLOC_MAX_DEVICES];
std::mutex g_noalloc_mutex;

// The device address of g_noalloc_scratch on the current device (looked up once per device); nullptr on error.
void* noalloc_scratch(std::string* why) {
  int dev = -1;
  cudaError_t c = cudaGetDevice(&dev);
  if (c != cudaSuccess || dev < 0 || dev >= NOALLOC_MAX_DEVICES) {
    *why = std::string("cudaGetDevice: ") + (c != cudaSuccess ? cudaGetErrorString(c) : "device index out of range");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    c = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (c != cudaSuccess || !ptr) {
      *why = std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(c);
      return nullptr;
    }
    g_noalloc_ptr[dev] = ptr;
  }
  return g_noalloc_ptr[dev];
}
}  // namespace

extern "C" int h2c_q4_matvec_noalloc(const void* w, int32_t n_rows, int32_t k, const float* x, int32_t m, float* y,
                                     int32_t op, const float* bias, void* stream) {
  if (!w || !x || !y || n_rows <= 0 || k <= 0 || k % 32 || m < 1 || op < 0 || op > 2 || (op == 1 && !bias)) {
    g_create_error = "h2c_q4_matvec_noalloc: invalid argument";
    return H2C_ERR_INVALID;
  }
  const uint64_t need = h2c_q4_matvec_scratch_bytes(m, k);
  if (need > NOALLOC_SCRATCH_BYTES) {
    char buf[200];
    snprintf(buf, sizeof buf,
             "h2c_q4_matvec_noalloc: %d x %d inputs need %llu bytes of scratch, above the %llu-byte static buffer",
             m, k, (unsigned long long)need, (unsigned long long)NOALLOC_SCRATCH_BYTES);
    g_create_error = buf;
    return H2C_ERR_INVALID;
  }
  std::string why;
  void* scratch = noalloc_scratch(&why);
  if (!scratch) {
    g_create_error = "h2c_q4_matvec_noalloc: " + why;
    return H2C_ERR_CUDA;
  }
  const int r = h2c_q4_matvec(w, n_rows, k, x, m, y, op, bias, scratch, stream);
  if (r != H2C_OK) g_create_error = "h2c_q4_matvec_noalloc: " + g_create_error;  // (the inner call's message)
  return r;
}

// ---------------------------------------------------------------- self-test of the fast correctly rounded forms

namespace {
__global__ void k_selftest_math(unsigned long long* bad) {
  unsigned long long n[4] = {0, 0, 0, 0};
  const uint64_t step = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (1ull << 32); i += step) {
    const float x = __uint_as_float((uint32_t)i);
    n[0] += __float_as_uint(h2::div127_rn(x)) != __float_as_uint(__fdiv_rn(x, 127.0f));
    n[1] += __float_as_uint(h2::div896_rn(x)) != __float_as_uint(__fdiv_rn(x, 896.0f));
    n[2] += __float_as_uint(h2::rcp_rn(x)) != __float_as_uint(__fdiv_rn(1.0f, x));
    n[3] += __float_as_uint(h2::sqrt_rn(x)) != __float_as_uint(__fsqrt_rn(x));
  }
  for (int k = 0; k < 4; k++)
    if (n[k]) atomicAdd(bad + k, n[k]);
}
}  // namespace

extern "C" int h2c_selftest_math(int device, uint64_t* mismatches) {
  if (!mismatches) return H2C_ERR_INVALID;
  if (cudaSetDevice(device) != cudaSuccess) return H2C_ERR_CUDA;
  unsigned long long* d = nullptr;
  if (cudaMalloc(&d, 4 * sizeof(unsigned long long)) != cudaSuccess) return H2C_ERR_NO_MEMORY;
  cudaError_t c = cudaMemset(d, 0, 4 * sizeof(unsigned long long));
  if (c == cudaSuccess) {
    k_selftest_math<<<148 * 8, 256>>>(d);
    c = cudaGetLastError();
  }
  if (c == cudaSuccess) c = cudaMemcpy(mismatches, d, 4 * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  cudaFree(d);
  return c == cudaSuccess ? H2C_OK : H2C_ERR_CUDA;
}
