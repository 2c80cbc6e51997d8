// SPDX-License-Identifier: MIT OR Apache-2.0
//
// candle-fused-attn's public API in C++, over the C ABI of include/cfa.h: the host layer a
// compiled caller links (libcfa_host.so), mirroring src/lib.rs name for name -- the two public
// functions, the layout predicates and geometry, the two custom ops with their saved L, and the
// `fused_attention:` error messages. The Rust crate itself keeps src/lib.rs and swaps only its
// launch layer (src/cuda.rs) for an `extern "C"` binding of include/cfa.h; this file is the same
// contract for C++ hosts.
//
// Failure detection: the kernels' device-side waits are bounded. An expired wait (results
// invalid) reaches a page-locked host flag this layer registers with the C ABI (cfa_error_sink)
// on its first call, so the next call of any function here throws Error without synchronising;
// check_status() synchronises the current stream first.
//
// What differs from candle, by necessity: there is no autograd graph, so the public functions
// return the output together with the op that made it, and `backward(grad)` runs the op's `bwd`
// exactly as candle's backprop would (src/lib.rs:449-490, :554-589). Tensors are f32 on CUDA by
// construction (host/tensor.hpp), so the dtype and device errors of the Rust ops cannot arise.
// The CPU composed path (src/lib.rs:241-299) is the test oracle (oracle/), not part of this layer.
#pragma once

#include <array>
#include <cstddef>
#include <memory>
#include <mutex>
#include <optional>
#include <tuple>

#include "tensor.hpp"

namespace candle_fused_attn {

// src/lib.rs:91. The CUDA kernels of the reference take this head dim only; these also take 32
// and 128 (HEAD_DIMS), the reference's listed next step.
constexpr size_t CUDA_HEAD_DIM = 64;
constexpr std::array<size_t, 3> HEAD_DIMS = {32, 64, 128};

// (batch, heads, seq, head_dim)
using Dims = std::tuple<size_t, size_t, size_t, size_t>;

// src/lib.rs:165-168: the offset and the (batch, head, seq) strides are multiples of 4 floats and
// head_dim is contiguous -- the kernels read rows as float4.
bool float4_aligned(const Layout& l);

// src/lib.rs:172-178: `t` itself when float4_aligned, else a contiguous copy.
Tensor float4_rows(const Tensor& t);

// src/lib.rs:181-188: (sb, sh, ss) of a rank-4 [b, h, s, d] layout with d contiguous.
std::array<size_t, 3> bhs_strides(const Layout& l);

// src/lib.rs:191-206: dims, the (batch, head, seq) strides shared by q, k, v, and their offsets
// in a fused projection [b, s, 3*heads*d].
struct QkvGeometry {
  Dims dims;
  std::array<size_t, 3> strides;
  std::array<size_t, 3> offsets;
};
QkvGeometry qkv_geometry(const Layout& l, size_t heads);

// src/lib.rs:209-220: the common [b, h, s, d] of q, k, v.
Dims check_shapes(const Layout& q, const Layout& k, const Layout& v);

// src/lib.rs:370-380: the gradient itself when its rows are float4-aligned, else a copy.
Tensor aligned_grad(const Tensor& grad);

// CustomOp3 `FusedAttention` (src/lib.rs:383-491): q, k, v [b, h, s, d] -> O [b, s, h, d].
class FusedAttention {
 public:
  FusedAttention(float scale, bool causal) : scale_(scale), causal_(causal) {}
  static const char* name() { return "fused-attention"; }
  // src/lib.rs:420-447: checks, one forward, L saved for the backward.
  Tensor cuda_fwd(const Tensor& q, const Tensor& k, const Tensor& v);
  // src/lib.rs:449-490: dq, dk, dv [b, h, s, d] (views of one [b, s, 3, h, d] buffer).
  std::array<Tensor, 3> bwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& res,
                            const Tensor& grad_res);

 private:
  float scale_;
  bool causal_;
  std::mutex mu_;
  std::optional<Tensor> lse_;
};

// CustomOp1 `FusedAttentionQkv` (src/lib.rs:494-590): qkv [b, s, 3hd] -> [b, s, hd].
class FusedAttentionQkv {
 public:
  FusedAttentionQkv(size_t heads, float scale, bool causal)
      : heads_(heads), scale_(scale), causal_(causal) {}
  static const char* name() { return "fused-attention-qkv"; }
  Tensor cuda_fwd(const Tensor& qkv);
  // dqkv [b, s, 3hd], laid out like qkv.
  Tensor bwd(const Tensor& qkv, const Tensor& res, const Tensor& grad_res);

 private:
  size_t heads_;
  float scale_;
  bool causal_;
  std::mutex mu_;
  std::optional<Tensor> lse_;
};

// The results of the two public functions: the output and the op that made it (the op keeps the
// saved L), with its backward as candle's backprop applies it.
struct QkvAttention {
  Tensor out;  // [b, s, h*d]
  Tensor qkv;  // the op's input as it saw it (possibly a contiguous copy)
  std::shared_ptr<FusedAttentionQkv> op;
  // d(sum(out * grad)) / d(qkv): [b, s, 3*h*d].
  Tensor backward(const Tensor& grad) const;
};

struct Attention {
  Tensor out;  // [b, h, s, d], a transposed view of a dense [b, s, h, d] buffer
  Tensor q, k, v, res;
  std::shared_ptr<FusedAttention> op;
  // d(sum(out * grad)) / d(q, k, v): three [b, h, s, d] views.
  std::array<Tensor, 3> backward(const Tensor& grad) const;
};

// src/lib.rs:110-125.
QkvAttention fused_attention_qkv(const Tensor& qkv, size_t heads, float scale, bool causal);

// src/lib.rs:143-161.
// Synchronises the current stream and throws Error if a bounded device-side wait of any earlier
// call expired (their results are then invalid). Has no counterpart in the reference.
void check_status();

Attention fused_attention(const Tensor& q, const Tensor& k, const Tensor& v, float scale,
                          bool causal);

}  // namespace candle_fused_attn
