// SPDX-License-Identifier: MIT OR Apache-2.0
//
// Measurement tooling (not product code): the fp32 FMA throughput of one B200, issued as scalar
// FFMA (fmaf) or as the packed sm_100 form fma.rn.f32x2 (two single-rounding FMAs per lane per
// instruction). Every thread runs 16 independent accumulator chains, so the FMA pipe, not latency,
// is the bound. baseline/ffma_peak.py times it with CUDA events and reports TFLOP/s.
#include <cstdint>
#include <cuda_runtime.h>

namespace {

constexpr int kChains = 16;

__global__ void __launch_bounds__(256) ffma_scalar(float* out, int iters, float a, float b) {
  float acc[kChains];
#pragma unroll
  for (int c = 0; c < kChains; ++c) acc[c] = threadIdx.x * 1e-3f + c;
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int c = 0; c < kChains; ++c) acc[c] = fmaf(acc[c], a, b);
  }
  float s = 0.0f;
#pragma unroll
  for (int c = 0; c < kChains; ++c) s += acc[c];
  out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

__device__ __forceinline__ uint64_t fma2(uint64_t x, uint64_t y, uint64_t z) {
  uint64_t d;
  asm volatile("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(x), "l"(y), "l"(z));
  return d;
}

__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__global__ void __launch_bounds__(256) ffma_packed(float* out, int iters, float a, float b) {
  uint64_t acc[kChains / 2];
#pragma unroll
  for (int c = 0; c < kChains / 2; ++c) acc[c] = pack2(threadIdx.x * 1e-3f + 2 * c, 2 * c + 1.0f);
  const uint64_t aa = pack2(a, a), bb = pack2(b, b);
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int c = 0; c < kChains / 2; ++c) acc[c] = fma2(acc[c], aa, bb);
  }
  float s = 0.0f;
#pragma unroll
  for (int c = 0; c < kChains / 2; ++c) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(acc[c]));
    s += lo + hi;
  }
  out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

}  // namespace

// Runs `reps` launches of `blocks` x 256 threads, each thread `iters` x 16 FMAs; returns the
// elapsed milliseconds (CUDA events), or a negative value on a CUDA error.
extern "C" float ffma_peak_run(int packed, float* out, int blocks, int iters, int reps) {
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  for (int w = 0; w < 2; ++w) {
    if (packed) ffma_packed<<<blocks, 256>>>(out, iters, 0.999f, 1e-3f);
    else ffma_scalar<<<blocks, 256>>>(out, iters, 0.999f, 1e-3f);
  }
  cudaEventRecord(e0);
  for (int r = 0; r < reps; ++r) {
    if (packed) ffma_packed<<<blocks, 256>>>(out, iters, 0.999f, 1e-3f);
    else ffma_scalar<<<blocks, 256>>>(out, iters, 0.999f, 1e-3f);
  }
  cudaEventRecord(e1);
  cudaEventSynchronize(e1);
  float ms = -1.0f;
  if (cudaGetLastError() == cudaSuccess) cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return ms;
}
