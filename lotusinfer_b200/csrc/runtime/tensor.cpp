#include "tensor.hpp"

#include <stdexcept>

namespace lotus {

void CudaCheck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

static std::shared_ptr<void> device_alloc(size_t bytes) {
  void* p = nullptr;
  CudaCheck(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc");
  return std::shared_ptr<void>(p, [](void* q) { cudaFree(q); });
}

size_t Tensor::StorageBytes(const std::vector<uint32_t>& shape, Format fmt) {
  size_t n = 1;
  if (fmt == Format::kNHWC_F16) {
    // logical [N, C, H, W] (or [N, C]) stored as [N, H, W, Cs] fp16
    if (shape.size() < 2) throw std::runtime_error("NHWC tensor needs at least [N, C]");
    for (size_t i = 0; i < shape.size(); ++i) n *= (i == 1) ? ((shape[1] + 7u) / 8u * 8u) : shape[i];
    return n * 2;
  }
  for (uint32_t d : shape) n *= d;
  return n * 4;
}

Tensor::Tensor(const std::vector<uint32_t>& shape, Format fmt) : shape_(shape), fmt_(fmt) {
  bytes_ = StorageBytes(shape, fmt);
  data_ = device_alloc(bytes_);
}

Tensor::Tensor(const std::vector<uint32_t>& shape, const std::vector<char>& data) : shape_(shape) {
  bytes_ = StorageBytes(shape, Format::kNCHW_F32);
  if (data.size() != bytes_) throw std::runtime_error("Tensor: data size does not match shape");
  data_ = device_alloc(bytes_);
  CudaCheck(cudaMemcpy(data_.get(), data.data(), bytes_, cudaMemcpyHostToDevice), "Tensor upload");
  // a pageable-host cudaMemcpy may return before its DMA lands; kernels on
  // non-blocking streams must not read the buffer before it does
  CudaCheck(cudaDeviceSynchronize(), "Tensor upload");
}

void Tensor::AssignData(const std::vector<float>& data) {
  if (fmt_ != Format::kNCHW_F32) throw std::runtime_error("AssignData needs an fp32 NCHW tensor");
  if (data.size() * 4 != bytes_) throw std::runtime_error("AssignData: size mismatch");
  CudaCheck(cudaMemcpy(Data(), data.data(), bytes_, cudaMemcpyHostToDevice), "AssignData");
  CudaCheck(cudaDeviceSynchronize(), "AssignData");
}

void Tensor::Reshape(const std::vector<uint32_t>& shape) {
  if (StorageBytes(shape, fmt_) != bytes_) throw std::runtime_error("Reshape: size mismatch");
  shape_ = shape;
}

uint32_t Tensor::Size() const {
  uint64_t n = 1;
  for (uint32_t d : shape_) n *= d;
  return static_cast<uint32_t>(n);
}

uint32_t Tensor::ChannelStride() const {
  if (shape_.size() < 2) return 0;
  return fmt_ == Format::kNHWC_F16 ? (shape_[1] + 7u) / 8u * 8u : shape_[1];
}

Tensor Tensor::Element(uint32_t i) const {
  if (shape_.empty() || i >= shape_[0]) throw std::runtime_error("Element: index out of range");
  if (!Dense()) throw std::runtime_error("Element: not supported on a channel slice");
  Tensor t;
  t.shape_ = shape_;
  t.shape_[0] = 1;
  t.fmt_ = fmt_;
  t.data_ = data_;
  t.bytes_ = bytes_ / shape_[0];
  t.offset_ = offset_ + t.bytes_ * i;
  return t;
}

Tensor Tensor::View(const std::vector<uint32_t>& shape, Format fmt) const {
  if (!Dense()) throw std::runtime_error("View: not supported on a channel slice");
  Tensor t;
  t.shape_ = shape;
  t.fmt_ = fmt;
  t.data_ = data_;
  t.offset_ = offset_;
  t.bytes_ = StorageBytes(shape, fmt);
  if (t.bytes_ > bytes_) throw std::runtime_error("View larger than storage");
  return t;
}

Tensor Tensor::ChannelSlice(uint32_t c0, uint32_t c) const {
  if (fmt_ != Format::kNHWC_F16 || shape_.size() != 4) throw std::runtime_error("ChannelSlice: needs a 4-D NHWC tensor");
  if (c0 % 8 != 0 || c == 0 || c0 + c > shape_[1]) throw std::runtime_error("ChannelSlice: bad channel range");
  Tensor t;
  t.shape_ = {shape_[0], c, shape_[2], shape_[3]};
  t.fmt_ = fmt_;
  t.data_ = data_;
  t.offset_ = offset_ + static_cast<size_t>(c0) * 2;
  t.bytes_ = StorageBytes(t.shape_, fmt_);  // the slice's own (dense-equivalent) bytes
  t.pixel_stride_ = PixelStride();
  return t;
}

Tensor Tensor::Unallocated(const std::vector<uint32_t>& shape, Format fmt) {
  Tensor t;
  t.shape_ = shape;
  t.fmt_ = fmt;
  t.bytes_ = StorageBytes(shape, fmt);
  return t;
}

void Tensor::BindStorage(std::shared_ptr<void> data, size_t offset) {
  data_ = std::move(data);
  offset_ = offset;
}

}  // namespace lotus
