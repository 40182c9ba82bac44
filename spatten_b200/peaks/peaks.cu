// Throughput microbenchmark of the special-function unit (MUFU ex2), the
// resource that bounds the progressive-attention kernel at long sequences
// (every score costs one exp2 per pass). Used by bench.py to measure the
// denominator of the kernel's exp2 roofline; not part of the attention API.
//
// Each thread runs kChains independent dependency chains x <- exp2(-x), so
// the unit, not the latency of one chain, limits the rate. Values stay in
// (0, 1]; the sum is written out so nothing is optimised away.
#include <cuda_runtime.h>
#include <stdint.h>

namespace {

constexpr int kChains = 8;

__global__ void __launch_bounds__(256) ex2_rate_kernel(float* out, int iters) {
  float x[kChains];
#pragma unroll
  for (int c = 0; c < kChains; ++c) x[c] = 0.001f * (float)((threadIdx.x + c) & 63);
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int c = 0; c < kChains; ++c) asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(x[c]) : "f"(-x[c]));
  }
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < kChains; ++c) s += x[c];
  out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

}  // namespace

extern "C" {

// Launch blocks x 256 threads, each doing iters * 8 exp2; `out` holds
// blocks * 256 floats. Returns the number of exp2 evaluated (0 on a launch
// error); time it with events on `stream`.
long long spatten_peak_ex2(int blocks, int iters, float* out, void* stream) {
  if (blocks <= 0 || iters <= 0 || out == nullptr) return 0;
  ex2_rate_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(out, iters);
  if (cudaGetLastError() != cudaSuccess) return 0;
  return (long long)blocks * 256 * (long long)iters * kChains;
}

}  // extern "C"
