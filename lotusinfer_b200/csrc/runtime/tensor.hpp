// lotus::Tensor - device tensor of the runtime.
//
// Keeps the reference's Tensor API (include/tensor.hpp:13-40: shape vector,
// Dim/DimSize/Size/Data, Reshape, AssignData, Element(i) batch sub-view) and
// adds the two storage formats this runtime uses:
//   kNCHW_F32  - the reference's own format (graph inputs/outputs, fp32 rows);
//   kNHWC_F16  - activations between layers, channel stride Cs = roundup(C, 8),
//                pad channels zero.
// Shapes are always reported in the reference's logical NCHW order.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

namespace lotus {

enum class Format { kNCHW_F32 = 0, kNHWC_F16 = 1 };

// Throws std::runtime_error with the CUDA error text (the reference aborts
// through glog CHECK, include/lotus_utils.hpp:28-32).
void CudaCheck(cudaError_t e, const char* what);

class Tensor {
 public:
  Tensor() = default;
  // Uninitialised device tensor on the current device.
  explicit Tensor(const std::vector<uint32_t>& shape, Format fmt = Format::kNCHW_F32);
  // fp32 tensor initialised from raw little-endian float bytes (weights;
  // reference source/tensor.cpp:13-26).
  Tensor(const std::vector<uint32_t>& shape, const std::vector<char>& data);

  void AssignData(const std::vector<float>& data);  // H2D of an fp32 NCHW tensor
  void Reshape(const std::vector<uint32_t>& shape);
  size_t DimSize() const { return shape_.size(); }
  uint32_t Dim(size_t i) const { return shape_.at(i); }
  const std::vector<uint32_t>& Shape() const { return shape_; }
  // Logical element count (C, not Cs).
  uint32_t Size() const;
  // Bytes held (includes channel padding).
  size_t Bytes() const { return bytes_; }
  Format Fmt() const { return fmt_; }
  uint32_t ChannelStride() const;  // Cs for kNHWC_F16, C otherwise
  void* Data() const { return data_ ? static_cast<char*>(data_.get()) + offset_ : nullptr; }
  float* DataF32() const { return static_cast<float*>(Data()); }
  bool Empty() const { return !data_; }
  // Sub-view of batch element i (reference source/tensor.cpp:79-88).
  Tensor Element(uint32_t i) const;
  // Alias with a different logical shape and format (no copy).
  Tensor View(const std::vector<uint32_t>& shape, Format fmt) const;
  // Channels [c0, c0 + c) of a 4-D NHWC fp16 tensor as a tensor of its own:
  // same storage, the slice's first channel as its start, consecutive pixels
  // PixelStride() elements apart (c0 must be a multiple of 8).
  Tensor ChannelSlice(uint32_t c0, uint32_t c) const;
  // Elements between consecutive pixels of an NHWC fp16 tensor: the channel
  // stride of a dense tensor, the parent's for a channel slice.
  uint32_t PixelStride() const { return pixel_stride_ ? pixel_stride_ : ChannelStride(); }
  bool Dense() const { return pixel_stride_ == 0 || pixel_stride_ == ChannelStride(); }

  // A tensor with a shape but no storage yet (the graph's memory planner binds
  // it), and the binding: `bytes` of `data` starting at byte `offset` must
  // cover StorageBytes(shape, fmt).
  static Tensor Unallocated(const std::vector<uint32_t>& shape, Format fmt);
  void BindStorage(std::shared_ptr<void> data, size_t offset);

  static size_t StorageBytes(const std::vector<uint32_t>& shape, Format fmt);

 private:
  std::vector<uint32_t> shape_;
  Format fmt_ = Format::kNCHW_F32;
  std::shared_ptr<void> data_;
  size_t offset_ = 0;
  size_t bytes_ = 0;
  uint32_t pixel_stride_ = 0;  // 0: dense
};

}  // namespace lotus
