// SPDX-License-Identifier: MIT OR Apache-2.0
//
// The C++ host layer's tensor (host/tensor.hpp): device storage, layouts, views and the
// strided-to-contiguous device copy behind `contiguous()` (candle's `Tensor::contiguous`).
#include "tensor.hpp"

#include <algorithm>
#include <numeric>

namespace candle_fused_attn {

namespace {

thread_local cudaStream_t g_stream = nullptr;

constexpr int kMaxRank = 6;

struct CopyArgs {
  const float* src;
  float* dst;
  int rank;
  int64_t n;
  int64_t dims[kMaxRank];
  int64_t src_stride[kMaxRank];
};

// dst[i] = src[offset of logical element i], i in row-major order of `dims`.
__global__ void strided_copy_kernel(CopyArgs a) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < a.n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t rem = i, off = 0;
    for (int r = a.rank - 1; r >= 0; --r) {
      const int64_t c = rem % a.dims[r];
      rem /= a.dims[r];
      off += c * a.src_stride[r];
    }
    a.dst[i] = a.src[off];
  }
}

void copy_to_contiguous(const Tensor& src, float* dst) {
  const Layout& l = src.layout();
  if (l.rank() > static_cast<size_t>(kMaxRank)) throw Error("fused_attention: rank above 6");
  CopyArgs a{};
  a.src = src.data();
  a.dst = dst;
  a.rank = static_cast<int>(l.rank());
  a.n = static_cast<int64_t>(l.elem_count());
  for (size_t r = 0; r < l.rank(); ++r) {
    a.dims[r] = static_cast<int64_t>(l.shape[r]);
    a.src_stride[r] = static_cast<int64_t>(l.stride[r]);
  }
  if (a.n == 0) return;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((a.n + threads - 1) / threads, 148 * 8);
  strided_copy_kernel<<<static_cast<unsigned>(blocks), threads, 0, current_stream()>>>(a);
  check_cuda(cudaGetLastError(), "strided copy");
}

}  // namespace

cudaStream_t current_stream() { return g_stream; }
void set_current_stream(cudaStream_t stream) { g_stream = stream; }

void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw Error(std::string("fused_attention: CUDA runtime error (") + what +
                "): " + cudaGetErrorString(e));
}

Storage::Storage(size_t elems) : elems_(elems) {
  if (elems_ > 0) check_cuda(cudaMalloc(&ptr_, elems_ * sizeof(float)), "cudaMalloc");
}

Storage::~Storage() {
  if (ptr_) cudaFree(ptr_);
}

size_t Layout::elem_count() const {
  return std::accumulate(shape.begin(), shape.end(), size_t{1}, std::multiplies<size_t>());
}

bool Layout::is_contiguous() const {
  size_t expect = 1;
  for (size_t r = rank(); r-- > 0;) {
    if (shape[r] != 1 && stride[r] != expect) return false;
    expect *= shape[r];
  }
  return true;
}

Layout Layout::contiguous(const std::vector<size_t>& shape, size_t offset) {
  Layout l;
  l.shape = shape;
  l.stride.assign(shape.size(), 1);
  for (size_t r = shape.size(); r-- > 1;) l.stride[r - 1] = l.stride[r] * shape[r];
  l.start_offset = offset;
  return l;
}

Tensor Tensor::empty(const std::vector<size_t>& shape) {
  Tensor t;
  t.layout_ = Layout::contiguous(shape);
  t.storage_ = std::make_shared<Storage>(t.layout_.elem_count());
  return t;
}

Tensor Tensor::zeros(const std::vector<size_t>& shape) {
  Tensor t = empty(shape);
  if (t.elem_count() > 0)
    check_cuda(cudaMemsetAsync(t.mutable_data(), 0, t.elem_count() * sizeof(float),
                               current_stream()),
               "cudaMemsetAsync");
  return t;
}

Tensor Tensor::from_host(const std::vector<float>& data, const std::vector<size_t>& shape) {
  Tensor t = empty(shape);
  if (data.size() != t.elem_count()) throw Error("fused_attention: host data size mismatch");
  if (!data.empty()) {
    check_cuda(cudaMemcpyAsync(t.mutable_data(), data.data(), data.size() * sizeof(float),
                               cudaMemcpyHostToDevice, current_stream()),
               "cudaMemcpyAsync");
    check_cuda(cudaStreamSynchronize(current_stream()), "cudaStreamSynchronize");
  }
  return t;
}

Tensor Tensor::view(const Tensor& base, const Layout& layout) {
  Tensor t;
  t.storage_ = base.storage_;
  t.layout_ = layout;
  return t;
}

std::vector<float> Tensor::to_host() const {
  const Tensor c = contiguous();
  std::vector<float> out(c.elem_count());
  if (!out.empty()) {
    check_cuda(cudaMemcpyAsync(out.data(), c.data(), out.size() * sizeof(float),
                               cudaMemcpyDeviceToHost, current_stream()),
               "cudaMemcpyAsync");
  }
  check_cuda(cudaStreamSynchronize(current_stream()), "cudaStreamSynchronize");
  return out;
}

Tensor Tensor::contiguous() const {
  if (layout_.is_contiguous()) return *this;
  Tensor t = empty(layout_.shape);
  copy_to_contiguous(*this, t.mutable_data());
  return t;
}

Tensor Tensor::transpose(size_t a, size_t b) const {
  if (a >= rank() || b >= rank()) throw Error("fused_attention: transpose out of range");
  Tensor t = *this;
  std::swap(t.layout_.shape[a], t.layout_.shape[b]);
  std::swap(t.layout_.stride[a], t.layout_.stride[b]);
  return t;
}

Tensor Tensor::narrow(size_t dim, size_t start, size_t len) const {
  if (dim >= rank() || start + len > layout_.shape[dim])
    throw Error("fused_attention: narrow out of range");
  Tensor t = *this;
  t.layout_.start_offset += start * layout_.stride[dim];
  t.layout_.shape[dim] = len;
  return t;
}

Tensor Tensor::reshape(const std::vector<size_t>& shape) const {
  const Layout want = Layout::contiguous(shape);
  if (want.elem_count() != elem_count()) throw Error("fused_attention: reshape size mismatch");
  const Tensor c = contiguous();
  Tensor t = c;
  t.layout_ = Layout::contiguous(shape, c.layout_.start_offset);
  return t;
}

Tensor Tensor::squeeze(size_t dim) const {
  if (dim >= rank() || layout_.shape[dim] != 1) throw Error("fused_attention: squeeze of a non-1 dim");
  Tensor t = *this;
  t.layout_.shape.erase(t.layout_.shape.begin() + static_cast<std::ptrdiff_t>(dim));
  t.layout_.stride.erase(t.layout_.stride.begin() + static_cast<std::ptrdiff_t>(dim));
  return t;
}

}  // namespace candle_fused_attn
