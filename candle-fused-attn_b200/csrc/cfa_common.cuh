// SPDX-License-Identifier: MIT OR Apache-2.0
//
// Device helpers shared by the sm_100a attention kernels: asynchronous 16-byte global->shared
// copies, padded tile loads, row reductions over 16 lanes, the bounded GPU-scope wait that
// orders the backward's dQ accumulation, and programmatic dependent launch.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "cfa_internal.h"

namespace cfa {

// Programmatic dependent launch. Every kernel here is launched with programmatic stream
// serialization, so it may be scheduled while the previous kernel on the stream drains its last
// blocks, and it lets its own successor do the same (griddep_launch_dependents). Each kernel calls
// griddep_wait() before its first global-memory access: that blocks until the previous kernel has
// completed and its writes are visible, so the results are those of plain stream order. (After a
// predecessor that does not take part -- a copy, another library's kernel -- the wait returns at
// once: the stream already ordered the launch after it.) Measured at the canvas shape: -5 us per
// forward + backward step, the launch gaps between the three kernels.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Shared-memory row strides, in floats. LD pads a 64-float row to 68: rows stay 16-byte aligned
// for float4 reads and consecutive rows start 4 banks apart, so the two rows read by the two
// half-warps of one float4 load never share a bank. LDP = 80 pads the probability / dS tiles so
// that the scalar stores of two half-warps (rows r and r + 1, 16 consecutive columns each) land
// in disjoint bank halves.
constexpr int LD = 68;
constexpr int LDP = 80;

__device__ __forceinline__ float4 ld4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

// acc + a.b over four products, in x, y, z, w order (one fixed order: the bitwise gate).
__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
  acc = fmaf(a.x, b.x, acc);
  acc = fmaf(a.y, b.y, acc);
  acc = fmaf(a.z, b.z, acc);
  return fmaf(a.w, b.w, acc);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem),
               "r"(src_bytes)
               : "memory");
}

// 4-byte asynchronous copy (L1-allocating), zero-filled when src_bytes == 0.
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, int src_bytes) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem),
               "r"(src_bytes)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

// ROWS rows of a strided [seq, 64] slice, starting at row `row0`, into a [ROWS][LD] tile by
// NTHREADS threads, 16 bytes per copy. Rows at or past `seq` are zero-filled (source size 0; the
// address given is row0's, which the caller guarantees is < seq, so no copy reads out of range).
template <int ROWS, int NTHREADS>
__device__ __forceinline__ void load_tile_async(float* dst, const float* __restrict__ src,
                                                int64_t s_stride, int row0, int seq) {
#pragma unroll
  for (int idx = threadIdx.x; idx < ROWS * 16; idx += NTHREADS) {
    const int r = idx >> 4, c4 = idx & 15;
    const int row = row0 + r;
    const bool ok = row < seq;
    const float* g = src + static_cast<int64_t>(ok ? row : row0) * s_stride + 4 * c4;
    cp_async16(dst + r * LD + 4 * c4, g, ok ? 16 : 0);
  }
}

// Max / sum over the 16 lanes that share bits 4.. of the lane index (one half-warp), by the xor
// butterfly 1, 2, 4, 8: the max is order-free and the sum's order is fixed.
__device__ __forceinline__ float half_warp_max(float x) {
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 4));
  return fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 8));
}

__device__ __forceinline__ float half_warp_sum(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  x += __shfl_xor_sync(0xffffffffu, x, 4);
  return x + __shfl_xor_sync(0xffffffffu, x, 8);
}

// log2(e) split into a float head and tail (head + tail = log2(e) to 4e-16).
constexpr float LOG2E_HI = 1.4426950216293335f;
constexpr float LOG2E_LO = 1.925963033500011e-08f;

// 2^x by the SFU (ex2.approx.ftz.f32: max relative error about 2^-22 per the PTX ISA;
// 2^-inf = +0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// e^d for an argument d <= 0 already formed in natural units: d * log2(e) is taken with the
// split constant (the product's own rounding only, no systematic error from rounding log2(e)),
// then one SFU exp2. -inf gives +0. (Kept for comparison; the kernels use CUDA's expf, whose
// smaller error keeps the outputs at or below the reference kernel's error against fp64.)
__device__ __forceinline__ float exp_nat(float d) {
  return ex2(fmaf(d, LOG2E_HI, d * LOG2E_LO));
}

__device__ __forceinline__ float f4c(const float4& v, int c) {
  return c == 0 ? v.x : (c == 1 ? v.y : (c == 2 ? v.z : v.w));
}

// Packed fp32 pairs (sm_100 fma.rn.f32x2: two single-rounding FMAs per lane per instruction).
// A float4 loaded from shared memory as ulonglong2 holds the pairs (x, y) and (z, w).
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__device__ __forceinline__ ulonglong2 ld2x2(const float* p) {
  return *reinterpret_cast<const ulonglong2*>(p);
}

__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// (x, x): one value in both halves of a pair (the broadcast operand of an outer product).
__device__ __forceinline__ uint64_t dup2(float x) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(x));
  return r;
}

// The two halves of a pair.
__device__ __forceinline__ float2 split2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}

// The sum of a pair's two halves: lo + hi.
__device__ __forceinline__ float sum2(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo + hi;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int ld_relaxed_gpu(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Records that a bounded wait expired: CFA_ERR_TIMEOUT into the device flag `err` (the first
// writer wins) and, when the caller registered one with cfa_error_sink, into that host-visible
// flag -- a plain system-scope store (no atomic on host memory), so the host reads it without a
// synchronisation and without the kernel depending on host atomics.
__device__ __forceinline__ void flag_timeout(int* err, int* sink) {
  if (err != nullptr) atomicCAS(err, 0, CFA_ERR_TIMEOUT);
  if (sink != nullptr) {
    asm volatile("st.relaxed.sys.global.b32 [%0], %1;" ::"l"(sink), "r"(int(CFA_ERR_TIMEOUT))
                 : "memory");
    __threadfence_system();
  }
}

// Wait (one thread) until *turn == want, at most `timeout_ns` of GPU time. Returns true when the
// turn came. On expiry it records CFA_ERR_TIMEOUT (flag_timeout) and returns false; it also
// returns false as soon as any other waiter has recorded an error, so one expired wait ends every
// chain quickly instead of each waiter spending its own full limit.
// ORDER: the acquire pairs with the release in pass_turn by the previous contributor: once this
// returns true, that block's dQ stores are visible to the caller (extended to the whole block by
// the caller's fence + barrier).
__device__ __forceinline__ bool wait_turn_bounded(const int* turn, int want, int* err,
                                                  uint64_t timeout_ns, int* sink) {
  if (ld_acquire_gpu(turn) == want) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t spin = 1;; ++spin) {
    __nanosleep(64);
    if (ld_acquire_gpu(turn) == want) return true;
    if ((spin & 15u) == 0u) {
      if (ld_relaxed_gpu(err) != 0) return false;
      if (global_timer_ns() - t0 > timeout_ns) {
        flag_timeout(err, sink);
        return false;
      }
    }
  }
}

}  // namespace cfa
