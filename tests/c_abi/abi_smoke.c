/* SPDX-License-Identifier: MIT OR Apache-2.0
 *
 * A C caller of the ABI in include/cfa.h, as a Rust / Go / C host would bind it: no Python, no
 * torch. Reads qkv [B, S, 3*H*64] and dO [B, S, H*64] (float32, raw files), runs the forward and
 * the backward on the GPU through cfa_fwd_f32_d64 / cfa_bwd_f32_d64 (and the no-allocation entry
 * point), and writes O [B, S, H*64] and dqkv [B, S, 3*H*64] back. Built and run by
 * tests/test_c_abi_gpu.py, which checks the outputs against the CPU oracle.
 *
 *   abi_smoke B H S causal qkv.bin dout.bin o.bin dqkv.bin dqkv_noalloc.bin
 */
#include <stdio.h>
#include <stdlib.h>

#include <cuda_runtime.h>

#include "cfa.h"

#define CK(x)                                                                  \
  do {                                                                         \
    cudaError_t e_ = (x);                                                      \
    if (e_ != cudaSuccess) {                                                   \
      fprintf(stderr, "%s:%d %s\n", __FILE__, __LINE__, cudaGetErrorString(e_)); \
      return 2;                                                                \
    }                                                                          \
  } while (0)

#define CFA(x)                                                                 \
  do {                                                                         \
    int s_ = (x);                                                              \
    if (s_ != CFA_OK) {                                                        \
      fprintf(stderr, "%s:%d %s\n", __FILE__, __LINE__, cfa_strerror(s_));     \
      return 3;                                                                \
    }                                                                          \
  } while (0)

static int read_file(const char* path, void* dst, size_t n) {
  FILE* f = fopen(path, "rb");
  if (!f) return 1;
  size_t got = fread(dst, 1, n, f);
  fclose(f);
  return got == n ? 0 : 1;
}

static int write_file(const char* path, const void* src, size_t n) {
  FILE* f = fopen(path, "wb");
  if (!f) return 1;
  size_t put = fwrite(src, 1, n, f);
  fclose(f);
  return put == n ? 0 : 1;
}

int main(int argc, char** argv) {
  if (argc != 10) {
    fprintf(stderr, "usage: %s B H S causal qkv dout o dqkv dqkv_noalloc\n", argv[0]);
    return 1;
  }
  const int64_t B = atoll(argv[1]), H = atoll(argv[2]), S = atoll(argv[3]);
  const int causal = atoi(argv[4]);
  const int64_t hd = H * 64;
  const size_t n_qkv = (size_t)(B * S * 3 * hd), n_o = (size_t)(B * S * hd);
  float* h_qkv = (float*)malloc(n_qkv * 4);
  float* h_do = (float*)malloc(n_o * 4);
  float* h_o = (float*)malloc(n_o * 4);
  float* h_dqkv = (float*)malloc(n_qkv * 4);
  if (!h_qkv || !h_do || !h_o || !h_dqkv) return 1;
  if (read_file(argv[5], h_qkv, n_qkv * 4) || read_file(argv[6], h_do, n_o * 4)) return 1;

  float *qkv, *d_o, *o, *lse, *dqkv;
  void* ws;
  const size_t ws_bytes = cfa_bwd_workspace_bytes_fast(B, H, S);
  CK(cudaMalloc((void**)&qkv, n_qkv * 4));
  CK(cudaMalloc((void**)&d_o, n_o * 4));
  CK(cudaMalloc((void**)&o, n_o * 4));
  CK(cudaMalloc((void**)&lse, (size_t)(B * H * S) * 4));
  CK(cudaMalloc((void**)&dqkv, n_qkv * 4));
  CK(cudaMalloc(&ws, ws_bytes));
  cudaStream_t st;
  CK(cudaStreamCreate(&st));
  CK(cudaMemcpyAsync(qkv, h_qkv, n_qkv * 4, cudaMemcpyHostToDevice, st));
  CK(cudaMemcpyAsync(d_o, h_do, n_o * 4, cudaMemcpyHostToDevice, st));

  /* the q / k / v views of the fused projection: (batch, head, seq) strides in floats */
  const int64_t s3[3] = {S * 3 * hd, 64, 3 * hd};
  const int64_t g3[3] = {S * hd, 64, hd};
  CFA(cfa_fwd_f32_d64(qkv, s3, qkv + hd, s3, qkv + 2 * hd, s3, o, lse, B, H, S, 64, 0.125f,
                      causal, st));
  CFA(cfa_bwd_f32_d64(qkv, s3, qkv + hd, s3, qkv + 2 * hd, s3, o, lse, d_o, g3, dqkv, ws, ws_bytes,
                      B, H, S, 64, 0.125f, causal, st));
  CFA(cfa_bwd_status(ws, st));
  CK(cudaMemcpyAsync(h_o, o, n_o * 4, cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(h_dqkv, dqkv, n_qkv * 4, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  if (write_file(argv[7], h_o, n_o * 4) || write_file(argv[8], h_dqkv, n_qkv * 4)) return 1;

  CK(cudaMemsetAsync(dqkv, 0, n_qkv * 4, st));
  CFA(cfa_bwd_f32_d64_noalloc(qkv, s3, qkv + hd, s3, qkv + 2 * hd, s3, o, lse, d_o, g3, dqkv, B, H,
                              S, 64, 0.125f, causal, st));
  CK(cudaMemcpyAsync(h_dqkv, dqkv, n_qkv * 4, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  if (write_file(argv[9], h_dqkv, n_qkv * 4)) return 1;

  CK(cudaStreamDestroy(st));
  cudaFree(qkv);
  cudaFree(d_o);
  cudaFree(o);
  cudaFree(lse);
  cudaFree(dqkv);
  cudaFree(ws);
  free(h_qkv);
  free(h_do);
  free(h_o);
  free(h_dqkv);
  printf("abi_smoke ok: B=%lld H=%lld S=%lld causal=%d\n", (long long)B, (long long)H,
         (long long)S, causal);
  return 0;
}
