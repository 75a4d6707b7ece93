// Temperature sampling on the device (the reference's sample(), cpu-worker.js:153-167), host interface.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace h2 {

// CTAs per row of the sampler's first two kernels (the vocabulary is split into this many contiguous ranges).
constexpr int SAMPLE_RANGES = 148;

// Device scratch of launch_sample for M rows, in bytes.
size_t sample_scratch_bytes(int M);

// For each row m < M of logits ([M][V] floats on the device) choose the next token as cpu-worker.js:153-167 does:
// the argmax (strict >, ties to the lowest id) when temperature <= 0, else a draw from softmax(logits / temperature)
// with mulberry32 seeded by seeds[m] (device array of M) or, when seeds is null, by seed0. The token goes to out[m]
// (device). scratch: sample_scratch_bytes(M) bytes of device memory. Launches three kernels on `st`.
cudaError_t launch_sample(const float* logits, int V, int M, double temperature, const uint32_t* seeds,
                          uint32_t seed0, int32_t* out, void* scratch, cudaStream_t st);

}  // namespace h2
