// SPDX-License-Identifier: MIT OR Apache-2.0
//
// The reference's own CUDA kernels (kernels/fused_attn.cu of candle-fused-attn v0.4.0), compiled
// from their source file where it lies (the include path points at the read-only reference tree;
// nothing is copied) for sm_100a, and launched exactly as the reference's Rust launch layer does:
//   ref_fwd  mirrors cuda::forward   (src/cuda.rs:140-185): grid (ceil(S/64), H, B) x 256 threads,
//            69,632 B of dynamic shared memory (src/cuda.rs:51), arguments in the kernel's order.
//   ref_bwd  mirrors cuda::backward  (src/cuda.rs:190-260): fattn_bwd_dot_f32_d64 on
//            ceil(B*H*S / 8) x 256 (src/cuda.rs:225-231), then fattn_bwd_f32_d64 on
//            (ceil(S/64), H, B) x 256 with 87,552 B (src/cuda.rs:57-58), on one stream.
// It is the same-GPU speed bar for bench.py and a second check in tests/. The build recipe is
// baseline/Makefile; the library goes to baseline/_ref/ (git-ignored, shipped with the tree).
#include <cstddef>
#include <cstdint>
#include <mutex>

#include "fused_attn.cu"

namespace {
constexpr int kThreads = 256;                                     // src/cuda.rs:32
constexpr unsigned kFwdSmem = (2 * 64 + 2 * 64) * 68 * 4;         // src/cuda.rs:51
constexpr unsigned kBwdSmem = ((2 * 64 + 6 * 32) * 68 + 4 * 32) * 4;  // src/cuda.rs:57-58
std::once_flag g_once[64];
cudaError_t g_once_err[64];

int set_attributes() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  std::call_once(g_once[dev], [dev] {
    cudaError_t e = cudaFuncSetAttribute(fattn_fwd_f32_d64,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(fattn_bwd_f32_d64, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kBwdSmem);
    g_once_err[dev] = e;
  });
  return g_once_err[dev] == cudaSuccess ? 0 : 2;
}
}  // namespace

extern "C" {

// Scratch of ref_bwd in bytes: D [B*H*S] floats, then the turn counters [B*H*ceil(S/32)] ints
// (src/cuda.rs:203-209), each 256-byte aligned.
size_t ref_bwd_workspace_bytes(int B, int H, int S) {
  const size_t d = ((size_t)B * H * S * 4 + 255) & ~(size_t)255;
  const size_t t = ((size_t)B * H * ((S + 31) / 32) * 4 + 255) & ~(size_t)255;
  return d + t;
}

int ref_fwd(const float* q, const float* k, const float* v, float* o, float* lse, int B, int H,
            int S, float scale, int causal, const int64_t* qs, const int64_t* ks,
            const int64_t* vs, void* stream) {
  if (set_attributes() != 0) return 2;
  const dim3 grid((S + 63) / 64, H, B);
  fattn_fwd_f32_d64<<<grid, kThreads, kFwdSmem, (cudaStream_t)stream>>>(
      q, k, v, o, lse, B, H, S, scale, causal, qs[0], qs[1], qs[2], ks[0], ks[1], ks[2], vs[0],
      vs[1], vs[2]);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

int ref_bwd(const float* q, const float* k, const float* v, const float* o, const float* lse,
            const float* d_o, float* dqkv, void* ws, int B, int H, int S, float scale, int causal,
            const int64_t* qs, const int64_t* ks, const int64_t* vs, const int64_t* dos,
            void* stream) {
  if (set_attributes() != 0) return 2;
  float* dsum = (float*)ws;
  int* turn = (int*)((char*)ws + (((size_t)B * H * S * 4 + 255) & ~(size_t)255));
  const cudaStream_t s = (cudaStream_t)stream;
  const unsigned dot_blocks = (unsigned)(((long long)B * H * S + 7) / 8);
  fattn_bwd_dot_f32_d64<<<dot_blocks, kThreads, 0, s>>>(o, d_o, dsum, turn, B, H, S, dos[0],
                                                         dos[1], dos[2]);
  if (cudaGetLastError() != cudaSuccess) return 3;
  const dim3 grid((S + 63) / 64, H, B);
  fattn_bwd_f32_d64<<<grid, kThreads, kBwdSmem, s>>>(
      q, k, v, d_o, lse, dsum, dqkv, turn, B, H, S, scale, causal, qs[0], qs[1], qs[2], ks[0],
      ks[1], ks[2], vs[0], vs[1], vs[2], dos[0], dos[1], dos[2]);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

}  // extern "C"
