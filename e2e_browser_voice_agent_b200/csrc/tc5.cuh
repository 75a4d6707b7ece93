// The multi-token Q4_0 matmul on the Blackwell tensor cores (tcgen05.mma with TMEM accumulators), host interface.
// Used for passes of several tokens (prompt chunks, batched decode steps); results are bit-identical to the
// reference's matmul_q4 (kernels.c:200-273), like every other matmul of this library.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace h2 {

// Tokens per CTA the kernel takes for M tokens and N weight rows (16, 32, 64 or 128).
int tc5_tokens_per_cta(int M, int N);

// y[m][n] (op)= W[n] . x[m] for m < M, n < N (op: 0 store, 1 add bias[n], 2 accumulate: put(), kernels.c:190-194).
//   qs, dsc : the Q4_0 matrix in the grouped device layout (rows in groups of 32, [group][block][32 rows][16 B] with
//             permuted bytes; fp16 scales [group][block][32 rows]);
//   xq      : int8 activations [xq_rows][K] (each 32-value block permuted like the weights), xq_rows >= M;
//   xdT     : their block scales transposed, [K/32][ldT] floats (token m of block b at b * ldT + m), ldT a multiple of
//             4 and >= M;
//   err     : 4 device ints; on a bounded wait that expires the kernel writes {1, CTA, role, 0} there and returns
//             (no trap), so the caller can report it.
// Every pointer 16-byte aligned. Returns the launch status (cudaErrorInvalidValue when the shapes do not fit).
cudaError_t launch_tc5(int op, const uint8_t* qs, const __half* dsc, int N, int K, const int8_t* xq, int xq_rows,
                       const float* xdT, int ldT, int M, float* y, int ldy, const float* bias, int* err,
                       cudaStream_t st);

// Opt the kernel instances into the shared memory they use (once per device, before the first launch there).
cudaError_t tc5_set_attrs();

}  // namespace h2
