// SPDX-License-Identifier: MIT OR Apache-2.0
//
// A minimal f32 CUDA tensor for the C++ host layer: the part of candle's `Tensor` / `Layout` /
// `CudaStorage` that the crate's attention path touches (src/lib.rs: layouts with a start offset
// and strides in elements, views by transpose / narrow / reshape / squeeze, `contiguous()` copies
// on the device). Views share one device allocation, freed with the last view.
//
// Everything runs on one CUDA stream per thread (`current_stream`, default: the legacy default
// stream), as candle runs everything on its device's stream (src/cuda.rs:4-7).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace candle_fused_attn {

// The crate's `candle_core::Error::Msg` (messages start with "fused_attention").
class Error : public std::runtime_error {
 public:
  explicit Error(const std::string& msg) : std::runtime_error(msg) {}
};

// The stream this thread's tensor operations and kernels run on.
cudaStream_t current_stream();
void set_current_stream(cudaStream_t stream);

// f32 device memory (cudaMalloc: 256-byte aligned).
class Storage {
 public:
  explicit Storage(size_t elems);
  ~Storage();
  Storage(const Storage&) = delete;
  Storage& operator=(const Storage&) = delete;
  float* data() const { return ptr_; }
  size_t size() const { return elems_; }

 private:
  float* ptr_ = nullptr;
  size_t elems_ = 0;
};

// candle's Layout: dims, strides (in elements) and the start offset into the storage.
struct Layout {
  std::vector<size_t> shape;
  std::vector<size_t> stride;
  size_t start_offset = 0;

  size_t rank() const { return shape.size(); }
  size_t elem_count() const;
  bool is_contiguous() const;
  static Layout contiguous(const std::vector<size_t>& shape, size_t offset = 0);
};

class Tensor {
 public:
  Tensor() = default;
  static Tensor zeros(const std::vector<size_t>& shape);
  static Tensor empty(const std::vector<size_t>& shape);
  static Tensor from_host(const std::vector<float>& data, const std::vector<size_t>& shape);
  // A view of `base` with an explicit layout (used for strided / offset views in tests).
  static Tensor view(const Tensor& base, const Layout& layout);

  std::vector<float> to_host() const;  // row-major copy of the logical elements
  const Layout& layout() const { return layout_; }
  const std::vector<size_t>& dims() const { return layout_.shape; }
  const std::vector<size_t>& stride() const { return layout_.stride; }
  size_t rank() const { return layout_.rank(); }
  size_t elem_count() const { return layout_.elem_count(); }
  bool defined() const { return storage_ != nullptr; }

  // Device pointer to the first element (start offset applied).
  const float* data() const { return storage_->data() + layout_.start_offset; }
  float* mutable_data() const { return storage_->data() + layout_.start_offset; }
  const std::shared_ptr<Storage>& storage() const { return storage_; }

  Tensor contiguous() const;  // this tensor if contiguous, else a device copy
  Tensor transpose(size_t a, size_t b) const;
  Tensor narrow(size_t dim, size_t start, size_t len) const;
  Tensor reshape(const std::vector<size_t>& shape) const;  // a view when contiguous, else a copy
  Tensor squeeze(size_t dim) const;

 private:
  std::shared_ptr<Storage> storage_;
  Layout layout_;
};

// Throws Error("fused_attention: CUDA runtime error: ...") on a CUDA error.
void check_cuda(cudaError_t e, const char* what);

}  // namespace candle_fused_attn
