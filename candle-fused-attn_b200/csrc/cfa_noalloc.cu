// SPDX-License-Identifier: MIT OR Apache-2.0
//
// cfa_bwd_f32_d64_noalloc: the backward for callers that cannot allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits -- under a framework whose
// allocator owns all device memory and gives plugins no scratch, in a real-time or embedded loop
// where an allocation's latency or failure is not acceptable, or behind an FFI that only passes
// the tensors it was given. Such a caller
// can still supply the inputs and outputs of the backward, but not the scratch that
// cfa_bwd_f32_d64 asks for (D = rowsum(dO o O), the dQ turn counters, the work ticket and the
// error flag). This entry point keeps that scratch in a file-scope static device array instead.
//
// Limits and rules:
//  - The array holds CFA_NOALLOC_SCRATCH_BYTES (4 MiB). Every GPU that loads this library holds
//    it until the process exits. A problem that needs more (cfa_bwd_workspace_bytes(b, h, s) >
//    4 MiB, i.e. b*h*s above about one million rows) is rejected with CFA_ERR_WORKSPACE before
//    anything runs; use cfa_bwd_f32_d64 with your own workspace for those.
//  - The first call on each device looks up the array's device address (cudaGetSymbolAddress)
//    with that device current and caches it; a failed lookup is returned as CFA_ERR_CUDA, on
//    that call and every later one on that device. The cache lives as long as the process: a
//    caller that resets the device (cudaDeviceReset, or anything else that destroys the primary
//    context) must not call this entry point on that device afterwards, since the array may then
//    sit at another address.
//  - Every call on a device shares the one array, which keeps the last call's contents. The
//    backward's first kernel clears the ticket, error flag and turn counters itself, and writes
//    all of D, so no state carries over between calls. Calls whose kernels can overlap on the
//    GPU (different streams without ordering between them) race on the array: order them.
//  - No cudaMalloc, cudaFree or allocating library routine is called.
//  - The bounded-wait error flag lives in the array and is not exposed; a caller that needs
//    cfa_bwd_status must use cfa_bwd_f32_d64 with its own workspace.
#include <mutex>

#include "cfa_internal.h"

namespace {

// The scratch. In host code this name is a host-side stand-in, not a device address: kernels
// get the address cfa_bwd_f32_d64_noalloc looks up with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[CFA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

struct ScratchAddress {
  std::once_flag once;
  void* ptr = nullptr;
  cudaError_t err = cudaSuccess;
};
ScratchAddress g_addr[kMaxDevices];

// The checks of cfa_bwd_f32_d64 that do not need the workspace, in its order, so that a bad head
// dim, an empty or oversized problem or a null pointer is reported as such and not as a
// workspace shortage. The size bound keeps cfa_bwd_workspace_bytes's arithmetic in range.
int precheck(const float* q, const float* k, const float* v, const float* o, const float* lse,
             const float* d_o, float* dqkv, const int64_t* qs, const int64_t* ks,
             const int64_t* vs, const int64_t* dos, int64_t batch, int64_t heads, int64_t seq,
             int64_t head_dim, bool* empty) {
  *empty = false;
  if (batch < 0 || heads < 0 || seq < 0 || head_dim < 0) return CFA_ERR_SHAPE;
  if (head_dim != CFA_HEAD_DIM) return CFA_ERR_HEAD_DIM;
  if (batch == 0 || heads == 0 || seq == 0) {
    *empty = true;
    return CFA_OK;
  }
  const int64_t lim = (int64_t(1) << 31) - 1;
  if (batch > lim || heads > lim || seq > lim || batch > lim / heads || batch * heads > lim / seq)
    return CFA_ERR_OVERFLOW;
  if (!q || !k || !v || !o || !lse || !d_o || !dqkv || !qs || !ks || !vs || !dos)
    return CFA_ERR_NULL;
  return CFA_OK;
}

int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CFA_ERR_CUDA;
  ScratchAddress& a = g_addr[dev];
  std::call_once(a.once, [&a] {
    a.err = cudaGetSymbolAddress(&a.ptr, g_noalloc_scratch);
  });
  if (a.err != cudaSuccess || a.ptr == nullptr) return CFA_ERR_CUDA;
  *out = a.ptr;
  return CFA_OK;
}

}  // namespace

extern "C" int cfa_bwd_f32_d64_noalloc(const float* q, const int64_t q_strides[3],
                                       const float* k, const int64_t k_strides[3],
                                       const float* v, const int64_t v_strides[3],
                                       const float* o, const float* lse, const float* d_o,
                                       const int64_t do_strides[3], float* dqkv, int64_t batch,
                                       int64_t heads, int64_t seq, int64_t head_dim, float scale,
                                       int causal, void* stream) {
  bool empty = false;
  const int st = precheck(q, k, v, o, lse, d_o, dqkv, q_strides, k_strides, v_strides,
                          do_strides, batch, heads, seq, head_dim, &empty);
  if (st != CFA_OK || empty) return st;
  if (cfa_bwd_workspace_bytes(batch, heads, seq) > CFA_NOALLOC_SCRATCH_BYTES)
    return CFA_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int sa = scratch_address(&scratch);
  if (sa != CFA_OK) return sa;
  return cfa_bwd_f32_d64(q, q_strides, k, k_strides, v, v_strides, o, lse, d_o, do_strides, dqkv,
                         scratch, CFA_NOALLOC_SCRATCH_BYTES, batch, heads, seq, head_dim, scale,
                         causal, stream);
}

extern "C" int cfa_bwd_noalloc_status(void* stream) {
  void* scratch = nullptr;
  const int sa = scratch_address(&scratch);
  if (sa != CFA_OK) return sa;
  return cfa_bwd_status(scratch, stream);
}
