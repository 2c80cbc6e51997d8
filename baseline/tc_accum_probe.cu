// SPDX-License-Identifier: MIT OR Apache-2.0
//
// Measurement tooling (not product code): how does the sm_100a tensor core accumulate in fp32?
// D[128][N] = C0 + sum over MMA steps of A_step * B_step^T with tcgen05.mma (bf16: kind::f16,
// tf32: kind::tf32), fp32 accumulator in TMEM; baseline/tc_accum_probe.py compares D on the CPU
// against round-to-nearest and truncating accumulation models. The answer decides whether a
// split-precision tensor-core attention can match plain-FFMA fp32 accuracy.
#include <cstdint>
#include "cfa_tc.cuh"  // candle-fused-attn_b200/csrc
using namespace cfa::tc;

template <int KIND>
__global__ void __launch_bounds__(128, 1) probe(const void* A, const void* B, const float* C0, float* D, int K, int N, int use_c, int* status) {
  extern __shared__ __align__(1024) unsigned char sm[];
  constexpr int ES = KIND == 1 ? 2 : 4;
  constexpr int EPC = 16 / ES;
  constexpr int KSTEP = KIND == 1 ? 16 : 8;
  const int nkc = K / EPC;
  unsigned char* As = sm;
  unsigned char* Bs = sm + 128 * K * ES;
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, w = tid / 32;
  for (int idx = tid; idx < 128 * nkc; idx += 128) {
    int row = idx / nkc, kc = idx % nkc;
    *(uint4*)(As + ((row / 8) * nkc + kc) * 128 + (row % 8) * 16) = *(const uint4*)((const unsigned char*)A + (size_t)(row * K + kc * EPC) * ES);
  }
  for (int idx = tid; idx < N * nkc; idx += 128) {
    int row = idx / nkc, kc = idx % nkc;
    *(uint4*)(Bs + ((row / 8) * nkc + kc) * 128 + (row % 8) * 16) = *(const uint4*)((const unsigned char*)B + (size_t)(row * K + kc * EPC) * ES);
  }
  const uint32_t ncols = N <= 32 ? 32 : (N <= 64 ? 64 : (N <= 128 ? 128 : 256));
  if (tid == 0) { mbar_init(&bar, 1); fence_mbar_init(); }
  if (w == 0) { tmem_alloc(&tbase, ncols); tmem_relinquish(); }
  fence_async_smem();
  fence_before_sync(); __syncthreads(); fence_after_sync();
  const uint32_t t = tbase;
  const uint32_t lane_base = t + ((uint32_t)(32 * w) << 16);
  if (use_c) {
    for (int c0 = 0; c0 < N; c0 += 16) { float v[16]; for (int i = 0; i < 16; ++i) v[i] = C0[tid * N + c0 + i]; tmem_st16(lane_base + c0, v); }
    tmem_wait_st();
  }
  fence_before_sync(); __syncthreads(); fence_after_sync();
  if (tid == 0) {
    const uint32_t idesc = idesc_f32acc(KIND, 128, N);
    for (int ks = 0; ks < K / KSTEP; ++ks) {
      uint64_t ad = desc_kmajor(smem_u32(As) + 2 * ks * 128, 128, nkc * 128);
      uint64_t bd = desc_kmajor(smem_u32(Bs) + 2 * ks * 128, 128, nkc * 128);
      if (KIND == 1) mma_bf16(t, ad, bd, idesc, (ks > 0 || use_c) ? 1u : 0u);
      else mma_tf32(t, ad, bd, idesc, (ks > 0 || use_c) ? 1u : 0u);
    }
    commit(&bar);
  }
  bool ok = mbar_wait(&bar, 0, 1000000000ull);
  if (!ok) { atomicExch(status, 1); ok = mbar_wait(&bar, 0, 1000000000ull); }
  fence_after_sync();
  if (ok) {
    for (int c0 = 0; c0 < N; c0 += 16) { float v[16]; tmem_ld16(lane_base + c0, v); tmem_wait_ld(); for (int i = 0; i < 16; ++i) D[tid * N + c0 + i] = v[i]; }
  }
  fence_before_sync(); __syncthreads(); fence_after_sync();
  if (w == 0 && ok) tmem_dealloc(t, ncols);
}

extern "C" int run_probe(int kind, const void* A, const void* B, const float* C0, float* D, int K, int N, int use_c, int* status) {
  int smem = 128 * K * (kind == 1 ? 2 : 4) + N * K * (kind == 1 ? 2 : 4);
  if (kind == 1) { cudaFuncSetAttribute(probe<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); probe<1><<<1, 128, smem>>>(A, B, C0, D, K, N, use_c, status); }
  else { cudaFuncSetAttribute(probe<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); probe<2><<<1, 128, smem>>>(A, B, C0, D, K, N, use_c, status); }
  cudaError_t e = cudaDeviceSynchronize();
  return (int)e;
}
