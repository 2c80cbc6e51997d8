// SPDX-License-Identifier: MIT OR Apache-2.0
//
// The C++ host layer (host/candle_fused_attn.hpp): src/lib.rs's checks, geometry and custom ops
// over the C ABI (include/cfa.h) -- the role candle's CustomOp glue plays for the Rust crate.
#include "candle_fused_attn.hpp"

#include <algorithm>
#include <cstdint>
#include <sstream>
#include <string>

#include "cfa.h"

namespace candle_fused_attn {

namespace {

std::string fmt_dims(const std::vector<size_t>& v) {
  std::ostringstream os;
  os << "[";
  for (size_t i = 0; i < v.size(); ++i) os << (i ? ", " : "") << v[i];
  os << "]";
  return os.str();
}

void check_status(int st) {
  if (st != CFA_OK) throw Error(cfa_strerror(st));
}

// The host-visible error flag (cfa_error_sink): page-locked, registered once per process, never
// freed (kernels of any later call may write it).
volatile int* error_flag() {
  static volatile int* flag = [] {
    void* p = nullptr;
    check_cuda(cudaHostAlloc(&p, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable),
               "cudaHostAlloc");
    *static_cast<volatile int*>(p) = 0;
    check_status(cfa_error_sink(static_cast<int*>(p)));
    return static_cast<volatile int*>(p);
  }();
  return flag;
}

// Throws (once) for a bounded wait that expired in a kernel launched earlier; no synchronisation,
// so kernels still running are not covered.
void raise_if_expired() {
  volatile int* flag = error_flag();
  const int code = *flag;
  if (code != 0) {
    *flag = 0;
    throw Error(cfa_strerror(code));
  }
}

// src/lib.rs:302-315: the forward's L, kept for the backward.
void save(std::mutex& mu, std::optional<Tensor>& slot, const Tensor& l) {
  std::lock_guard<std::mutex> g(mu);
  slot = l;
}

Tensor saved(std::mutex& mu, std::optional<Tensor>& slot) {
  std::lock_guard<std::mutex> g(mu);
  if (!slot) throw Error("fused_attention: backward before forward");
  return *slot;
}

bool head_dim_ok(size_t d) {
  return std::find(HEAD_DIMS.begin(), HEAD_DIMS.end(), d) != HEAD_DIMS.end();
}

// One forward through the C ABI (the role of src/cuda.rs:140-185): O [b, s, h, d] and
// L [b, h, s] for operands given as (device pointer, (sb, sh, ss)).
std::pair<Tensor, Tensor> forward(float scale, bool causal, const Dims& dims,
                                  const std::array<const float*, 3>& ptr,
                                  const std::array<std::array<int64_t, 3>, 3>& st) {
  const auto [b, h, s, d] = dims;
  if (!head_dim_ok(d))
    throw Error("fused_attention: the CUDA kernels take head_dim 64 (and 32 or 128), got " +
                std::to_string(d));
  raise_if_expired();
  Tensor o = Tensor::empty({b, s, h, d});
  Tensor l = Tensor::empty({b, h, s});
  check_status(cfa_fwd_f32(ptr[0], st[0].data(), ptr[1], st[1].data(), ptr[2], st[2].data(),
                           o.mutable_data(), l.mutable_data(), static_cast<int64_t>(b),
                           static_cast<int64_t>(h), static_cast<int64_t>(s),
                           static_cast<int64_t>(d), scale, causal ? 1 : 0, current_stream()));
  return {o, l};
}

// src/lib.rs:329-366 (with src/cuda.rs:190-260): dqkv [b, s, 3, h, d] from the operands, the
// output O (contiguous [b, s, h, d] or [b, s, h*d]), dO through (gb, gh, gs) strides, and L.
Tensor cuda_backward(float scale, bool causal, const Dims& dims,
                     const std::array<const float*, 3>& ptr,
                     const std::array<std::array<int64_t, 3>, 3>& st, const Tensor& o,
                     const Tensor& grad, const std::array<int64_t, 3>& g, const Tensor& l) {
  if (!o.layout().is_contiguous() || !l.layout().is_contiguous())
    throw Error("fused_attention: O and L must be contiguous");
  const auto [b, h, s, d] = dims;
  raise_if_expired();
  Tensor dqkv = Tensor::empty({b, s, 3, h, d});
  const size_t ws_bytes = cfa_bwd_workspace_bytes_fast_hd(
      static_cast<int64_t>(b), static_cast<int64_t>(h), static_cast<int64_t>(s),
      static_cast<int64_t>(d));
  // Stream-ordered scratch (the role of the three `dev.alloc` calls of src/cuda.rs:203-209): it
  // is released after the kernels that use it, on the same stream, without a host sync. The ABI
  // wants 256-byte alignment; the pool's is not promised, so the pointer is rounded up.
  const cudaStream_t stream = current_stream();
  void* raw = nullptr;
  check_cuda(cudaMallocAsync(&raw, ws_bytes + 256, stream), "cudaMallocAsync");
  void* ws = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(raw) + 255) & ~uintptr_t{255});
  const int rc = cfa_bwd_f32(ptr[0], st[0].data(), ptr[1], st[1].data(), ptr[2], st[2].data(),
                             o.data(), l.data(), grad.data(), g.data(), dqkv.mutable_data(), ws,
                             ws_bytes, static_cast<int64_t>(b), static_cast<int64_t>(h),
                             static_cast<int64_t>(s), static_cast<int64_t>(d), scale,
                             causal ? 1 : 0, stream);
  check_cuda(cudaFreeAsync(raw, stream), "cudaFreeAsync");
  check_status(rc);
  return dqkv;
}

std::array<int64_t, 3> i64(const std::array<size_t, 3>& a) {
  return {static_cast<int64_t>(a[0]), static_cast<int64_t>(a[1]), static_cast<int64_t>(a[2])};
}

}  // namespace

void check_status() {
  check_cuda(cudaStreamSynchronize(current_stream()), "cudaStreamSynchronize");
  raise_if_expired();
}

bool float4_aligned(const Layout& l) {
  return l.rank() == 4 && l.start_offset % 4 == 0 && l.stride[3] == 1 && l.stride[0] % 4 == 0 &&
         l.stride[1] % 4 == 0 && l.stride[2] % 4 == 0;
}

Tensor float4_rows(const Tensor& t) { return float4_aligned(t.layout()) ? t : t.contiguous(); }

std::array<size_t, 3> bhs_strides(const Layout& l) {
  if (l.rank() != 4 || l.stride[3] != 1)
    throw Error("fused_attention: [b, h, s, d] with d contiguous expected, strides " +
                fmt_dims(l.stride));
  return {l.stride[0], l.stride[1], l.stride[2]};
}

QkvGeometry qkv_geometry(const Layout& l, size_t heads) {
  if (l.rank() != 3)
    throw Error("fused_attention_qkv: rank-3 qkv expected, shape " + fmt_dims(l.shape));
  const size_t b = l.shape[0], s = l.shape[1], three_hd = l.shape[2];
  if (heads == 0 || three_hd % (3 * heads) != 0)
    throw Error("fused_attention_qkv: last dimension " + std::to_string(three_hd) + " is not 3 x " +
                std::to_string(heads) + " heads x head_dim");
  const size_t hd = three_hd / 3, d = hd / heads;
  if (l.stride[2] != 1)
    throw Error("fused_attention_qkv: the last dimension must be contiguous, strides " +
                fmt_dims(l.stride));
  return {Dims{b, heads, s, d}, {l.stride[0], d, l.stride[1]}, {0, hd, 2 * hd}};
}

Dims check_shapes(const Layout& q, const Layout& k, const Layout& v) {
  if (q.rank() != 4 || k.shape != q.shape || v.shape != q.shape)
    throw Error("fused_attention: q, k, v must share one [b, h, s, d] shape, got " +
                fmt_dims(q.shape) + " " + fmt_dims(k.shape) + " " + fmt_dims(v.shape));
  return Dims{q.shape[0], q.shape[1], q.shape[2], q.shape[3]};
}

Tensor aligned_grad(const Tensor& grad) {
  const Layout& l = grad.layout();
  bool ok = l.start_offset % 4 == 0 && l.rank() > 0 && l.stride.back() == 1;
  for (size_t st : l.stride) ok = ok && (st == 1 || st % 4 == 0);
  return ok ? grad : grad.contiguous();
}

// ---- FusedAttention (CustomOp3) -------------------------------------------------------------

Tensor FusedAttention::cuda_fwd(const Tensor& q, const Tensor& k, const Tensor& v) {
  const Dims dims = check_shapes(q.layout(), k.layout(), v.layout());
  if (!float4_aligned(q.layout()) || !float4_aligned(k.layout()) || !float4_aligned(v.layout()))
    throw Error("fused_attention: rows must be 16-byte aligned");
  auto [o, l] = forward(scale_, causal_, dims, {q.data(), k.data(), v.data()},
                        {i64(bhs_strides(q.layout())), i64(bhs_strides(k.layout())),
                         i64(bhs_strides(v.layout()))});
  save(mu_, lse_, l);
  return o;  // [b, s, h, d]
}

std::array<Tensor, 3> FusedAttention::bwd(const Tensor& q, const Tensor& k, const Tensor& v,
                                          const Tensor& res, const Tensor& grad_res) {
  const Tensor l = saved(mu_, lse_);
  const Tensor grad = aligned_grad(grad_res);
  const Dims dims = check_shapes(q.layout(), k.layout(), v.layout());
  if (grad.rank() != 4) throw Error("fused_attention: rank-4 gradient expected");
  const auto& gst = grad.stride();  // grad is [b, s, h, d] like res
  const std::array<int64_t, 3> g = {static_cast<int64_t>(gst[0]), static_cast<int64_t>(gst[2]),
                                    static_cast<int64_t>(gst[1])};
  const Tensor dqkv = cuda_backward(
      scale_, causal_, dims, {q.data(), k.data(), v.data()},
      {i64(bhs_strides(q.layout())), i64(bhs_strides(k.layout())), i64(bhs_strides(v.layout()))},
      res, grad, g, l);
  auto part = [&](size_t i) { return dqkv.narrow(2, i, 1).squeeze(2).transpose(1, 2); };
  return {part(0), part(1), part(2)};
}

// ---- FusedAttentionQkv (CustomOp1) ----------------------------------------------------------

Tensor FusedAttentionQkv::cuda_fwd(const Tensor& qkv) {
  const QkvGeometry g = qkv_geometry(qkv.layout(), heads_);
  if (qkv.layout().start_offset % 4 != 0 ||
      std::any_of(g.strides.begin(), g.strides.end(), [](size_t s) { return s % 4 != 0; }))
    throw Error("fused_attention_qkv: rows must be 16-byte aligned");
  const float* base = qkv.data();
  const auto st = i64(g.strides);
  auto [o, l] = forward(scale_, causal_, g.dims,
                        {base + g.offsets[0], base + g.offsets[1], base + g.offsets[2]},
                        {st, st, st});
  save(mu_, lse_, l);
  const auto [b, h, s, d] = g.dims;
  return o.reshape({b, s, h * d});
}

Tensor FusedAttentionQkv::bwd(const Tensor& qkv, const Tensor& res, const Tensor& grad_res) {
  const Tensor l = saved(mu_, lse_);
  const Tensor grad = aligned_grad(grad_res);
  const QkvGeometry geo = qkv_geometry(qkv.layout(), heads_);
  const auto [b, h, s, d] = geo.dims;
  if (grad.rank() != 3) throw Error("fused_attention_qkv: rank-3 gradient expected");
  const std::array<int64_t, 3> g = {static_cast<int64_t>(grad.stride()[0]),
                                    static_cast<int64_t>(d),
                                    static_cast<int64_t>(grad.stride()[1])};
  const float* base = qkv.data();
  const auto st = i64(geo.strides);
  const Tensor dqkv =
      cuda_backward(scale_, causal_, geo.dims,
                    {base + geo.offsets[0], base + geo.offsets[1], base + geo.offsets[2]},
                    {st, st, st}, res, grad, g, l);
  return dqkv.reshape({b, s, 3 * h * d});
}

// ---- the public functions --------------------------------------------------------------------

Tensor QkvAttention::backward(const Tensor& grad) const { return op->bwd(qkv, out, grad); }

std::array<Tensor, 3> Attention::backward(const Tensor& grad) const {
  // out = res.transpose(1, 2), so the gradient reaching the op is grad.transpose(1, 2).
  return op->bwd(q, k, v, res, grad.transpose(1, 2));
}

QkvAttention fused_attention_qkv(const Tensor& qkv, size_t heads, float scale, bool causal) {
  const Layout& l = qkv.layout();
  const bool aligned = l.start_offset % 4 == 0 && l.rank() == 3 && l.stride[2] == 1 &&
                       l.stride[0] % 4 == 0 && l.stride[1] % 4 == 0;
  const Tensor x = aligned ? qkv : qkv.contiguous();
  auto op = std::make_shared<FusedAttentionQkv>(heads, scale, causal);
  Tensor out = op->cuda_fwd(x);
  return QkvAttention{out, x, op};
}

Attention fused_attention(const Tensor& q, const Tensor& k, const Tensor& v, float scale,
                          bool causal) {
  const Tensor q4 = float4_rows(q), k4 = float4_rows(k), v4 = float4_rows(v);
  auto op = std::make_shared<FusedAttention>(scale, causal);
  Tensor res = op->cuda_fwd(q4, k4, v4);
  return Attention{res.transpose(1, 2), q4, k4, v4, res, op};
}

}  // namespace candle_fused_attn
