// SPDX-License-Identifier: MIT OR Apache-2.0
//
// Measurement tooling (B200): cycles per tcgen05.mma (kind::f16, fp32 accumulate in TMEM) by shape
// and operand placement, issued by one converged warp (warp 16 of a 544-thread block, as in the
// tensor-core attention kernels) with one elected lane, 96 MMAs per measurement; and the same
// M128 N64 K16 stream (A in TMEM) while warps 0-15 run background work. One block per SM (120 KB
// of shared memory), 148 blocks, block 0 reported, second of two launches. Operand values are
// bf16 1.0 (timing only). Every wait is bounded.
//
//   make -C baseline mma_rate && baseline/_ref/mma_rate_probe
#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>

#include "cfa_common.cuh"
#include "cfa_tc.cuh"

using namespace cfa;

namespace {

constexpr int SMEM = 120 * 1024;
__device__ long long g_cycles[16][2];
__device__ float g_sink[544];
__device__ float g_src[1 << 22];

// Shape / operand variants of the MMA stream (background: none).
//  0 M128 N64, A and B in shared memory   1 M128 N64, A in TMEM   2 M64 N64, shared memory
//  3 M128 N128, shared memory              4 M128 N256, shared memory
//  5 M128 N16, A in TMEM (issue cost)      6 the kernels' window pattern (24 MMAs per window, six
//  part pairs x 4 K-steps, two alternating part buffers), A in TMEM, B K-major
//  7 the same, B read MN-major
// Background variants (stream 1): 8 expf, 9 TMEM loads and stores, 10 cp.async global -> shared,
// 11 shared-memory loads and stores, 12 FMA chains.
template <int V>
__global__ void __launch_bounds__(544, 1) probe() {
  extern __shared__ __align__(1024) unsigned char sm[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tb;
  const int tid = threadIdx.x, w = tid >> 5;
  for (int i = tid; i < SMEM / 4; i += 544) reinterpret_cast<uint32_t*>(sm)[i] = 0x3f803f80u;
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
  }
  if (w == 0) {
    tc::tmem_alloc(&tb, 512);
    tc::tmem_relinquish();
  }
  tc::fence_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tb;
  const uint32_t s0 = tc::smem_u32(sm);
  constexpr int S = V >= 8 ? 1 : V;  // the stream's shape variant
  if (w == 16) {
    constexpr int M = S == 2 ? 64 : 128;
    constexpr int N = S == 3 ? 128 : (S == 4 ? 256 : (S == 5 ? 16 : 64));
    constexpr bool A_TMEM = S == 1 || S == 5 || S == 6 || S == 7;
    constexpr bool B_MN = S == 7;
    const uint32_t id = tc::idesc_f32acc(1, M, N) | (B_MN ? (1u << 16) : 0u);
    const tc::Desc ad = tc::split_desc(tc::desc_kmajor(s0, 128, 1024));
    const tc::Desc bd =
        tc::split_desc(tc::desc_kmajor(s0 + 32768, B_MN ? 1024 : 128, B_MN ? 128 : 1024));
    if (V >= 8)
      for (int spin = 0; spin < 200; ++spin) __nanosleep(0);  // the background is under way
    const long long t0 = clock64();
    const uint32_t alo = tc::opaque(ad.lo), blo = tc::opaque(bd.lo);
    constexpr int PA[6] = {0, 0, 1, 0, 1, 2};
    constexpr int PB[6] = {0, 1, 0, 2, 1, 0};
#pragma unroll
    for (int i = 0; i < 96; ++i) {
      const int win = i / 24, j = i % 24, ks = j % 4, p = j / 4;
      uint32_t acol = 8 * (i & 3), boff = 256 * (i & 3), d = tbase + 256;
      bool acc = i > 0;
      if (S == 6 || S == 7) {
        acol = 32 * PA[p] + 8 * ks;
        boff = PB[p] * 8192 + (B_MN ? 2048 : 256) * ks + 24576 * (win & 1);
        d = tbase + 256 + 64 * (win & 1);
        acc = j > 0;
      }
      if (A_TMEM)
        tc::mma_bf16_tmem_a_warp(S == 4 ? tbase : d, tbase + acol, blo + (boff >> 4), bd.hi, id, acc);
      else
        tc::mma_bf16_warp(S == 4 ? tbase : d, alo + (boff >> 4), ad.hi, blo + (boff >> 4), bd.hi, id,
                          acc);
    }
    const long long t1 = clock64();
    tc::commit_warp(&bar);
    const bool ok = tc::mbar_wait(&bar, 0, 1000000000ull);
    const long long t2 = clock64();
    if ((tid & 31) == 0 && blockIdx.x == 0) {
      g_cycles[V][0] = t1 - t0;
      g_cycles[V][1] = ok ? t2 - t0 : -1;
    }
    tc::fence_after_sync();
  } else if (V == 8) {
    float x[16];
    for (int i = 0; i < 16; ++i) x[i] = 0.01f * (tid + i);
    for (int it = 0; it < 300; ++it)
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = expf(x[i] * -0.5f);
    float t = 0.f;
    for (int i = 0; i < 16; ++i) t += x[i];
    g_sink[tid] = t;
  } else if (V == 9) {
    const uint32_t lane_sel = static_cast<uint32_t>(32 * (w & 3)) << 16;
    float s2 = 0.f;
    for (int it = 0; it < 300; ++it) {
      float v[16];
      tc::tmem_ld16(tbase + lane_sel + 384 + 16 * (w >> 2), v);
      tc::tmem_wait_ld();
      v[0] += 1.0f;
      tc::tmem_st16(tbase + lane_sel + 448 + 16 * (w >> 2), v);
      tc::tmem_wait_st();
      s2 += v[3];
    }
    g_sink[tid] = s2;
  } else if (V == 10) {
    for (int it = 0; it < 40; ++it) {
      const int i = (tid + it * 512) & 2047;
      const int64_t base = (static_cast<int64_t>(blockIdx.x) * 40 + it) * 2048;
      cp_async16(sm + 65536 + 16 * i, g_src + ((base + i) * 4) % (1 << 22), 16);
      cp_async16(sm + 65536 + 16 * ((i + 1024) & 2047), g_src + ((base + i + 1024) * 4) % (1 << 22),
                 16);
      cp_async_commit();
      if ((it & 3) == 3) cp_async_wait_all();
    }
    cp_async_wait_all();
  } else if (V == 11) {
    float4* p = reinterpret_cast<float4*>(sm + 65536);
    float4 acc = make_float4(0, 0, 0, 0);
    for (int it = 0; it < 400; ++it) {
      const int i = (tid + it * 544) % 3072;
      const float4 v = p[i];
      acc.x += v.x;
      acc.y += v.y;
      p[(i + 1) % 3072] = acc;
    }
    g_sink[tid] = acc.x;
  } else if (V == 12) {
    float a0 = tid, a1 = tid + 1, a2 = tid + 2, a3 = tid + 3;
    for (int it = 0; it < 3000; ++it) {
      a0 = fmaf(a0, 1.0001f, 0.5f);
      a1 = fmaf(a1, 1.0001f, 0.5f);
      a2 = fmaf(a2, 1.0001f, 0.5f);
      a3 = fmaf(a3, 1.0001f, 0.5f);
    }
    g_sink[tid] = a0 + a1 + a2 + a3;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (w == 0) tc::tmem_dealloc(tbase, 512);
}

template <int V>
bool run() {
  if (cudaFuncSetAttribute(probe<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
    return false;
  for (int rep = 0; rep < 2; ++rep) probe<V><<<148, 544, SMEM>>>();
  return cudaGetLastError() == cudaSuccess;
}

}  // namespace

int main() {
  bool ok = run<0>() && run<1>() && run<2>() && run<3>() && run<4>() && run<5>() && run<6>() &&
            run<7>() && run<8>() && run<9>() && run<10>() && run<11>() && run<12>();
  const cudaError_t e = cudaDeviceSynchronize();
  if (!ok || e != cudaSuccess) {
    printf("error: %s\n", cudaGetErrorString(e));
    return 1;
  }
  long long c[16][2];
  cudaMemcpyFromSymbol(c, g_cycles, sizeof(c));
  const char* names[13] = {"M128 N64, A+B smem", "M128 N64, A TMEM", "M64 N64, A+B smem",
                           "M128 N128, A+B smem", "M128 N256, A+B smem", "M128 N16, A TMEM",
                           "window pattern, B K-major", "window pattern, B MN-major",
                           "M128 N64 A TMEM + expf warps", "  + TMEM ld/st warps",
                           "  + cp.async warps", "  + smem ld/st warps", "  + FMA warps"};
  printf("96 tcgen05.mma from one warp (cycles: issue, done; per MMA)\n");
  for (int v = 0; v < 13; ++v)
    printf("  %-30s %6lld %6lld  %6.1f\n", names[v], c[v][0], c[v][1], c[v][1] / 96.0);
  return 0;
}
