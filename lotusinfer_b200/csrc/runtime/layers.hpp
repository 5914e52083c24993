// Layer classes: one per PNNX operator type of the hot path, each a thin
// caller of the C ABI (include/lotus_ops.h), launched once per layer for the
// whole batch on the graph's stream.
//
// Mirrors the reference's Layer hierarchy (include/layer/layer.hpp:9-27 and
// include/layer/*.hpp): name, input/output operand names and operands, a
// fused ActivationFunction, and Forward().  Differences: Forward takes the
// stream (no per-Forward StreamPool, no per-layer device sync), weights are
// prepacked to fp16 at construction, Conv2dLayer can fold a residual add.
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../../include/lotus_ops.h"
#include "pnnx.hpp"
#include "tensor.hpp"

namespace lotus {

// Same values as the reference enum (include/lotus_utils.hpp:44-48).
enum ActivationFunction { NONE = 0, RELU = 1, SIGMOID = 2 };

struct Operand {
  Tensor tensor_;
  std::string name_;
  std::string producer_;
  std::vector<std::string> consumers_;
};

using OperandMap = std::map<std::string, std::shared_ptr<Operand>>;

// Throws std::runtime_error with lotus_last_error_string() on a non-zero status.
void LotusCheck(int status, const std::string& where);

class Layer {
 public:
  virtual ~Layer() = default;
  const std::string& Name() const { return name_; }
  const std::string& Type() const { return type_; }
  const std::vector<std::string>& InputsName() const { return inputs_name_; }
  const std::vector<std::string>& OutputsName() const { return outputs_name_; }
  ActivationFunction Activation() const { return af_; }
  // Binds operand tensors (after allocation) and validates shapes.
  virtual void Bind(const OperandMap& operands);
  virtual void Forward(cudaStream_t stream) = 0;
  // Algorithmic work of one Forward over the whole batch.
  virtual double Flops() const { return 0.0; }
  virtual double Bytes() const;
  // Number of library kernel launches one Forward issues.
  virtual int Launches() const { return 1; }
  // Split-K workspace this layer's kernels want (0 = none) and the shared
  // graph workspace it may use (layers run one after another on one stream).
  virtual size_t WorkspaceBytes() const { return 0; }
  void SetWorkspace(void* ws, size_t bytes) {
    workspace_ = ws;
    workspace_bytes_ = bytes;
  }
  // Prepacked weight (device) and its size; null when the layer has none.
  virtual const void* Weight(size_t* bytes) const {
    if (bytes) *bytes = 0;
    return nullptr;
  }

 protected:
  std::string name_, type_;
  std::vector<std::string> inputs_name_, outputs_name_;
  std::vector<std::shared_ptr<Operand>> inputs_, outputs_;
  ActivationFunction af_ = NONE;
  void* workspace_ = nullptr;
  size_t workspace_bytes_ = 0;
  friend class Graph;
};

// NCHW fp32 graph input -> NHWC fp16 activation, optionally as the
// space-to-depth (factor f, zero padding) of the input for a rewritten stem.
class InputConvertLayer : public Layer {
 public:
  InputConvertLayer(const std::string& in, const std::string& out);
  void SetSpaceToDepth(int factor, int pad_h, int pad_w) {
    s2d_ = factor;
    pad_h_ = pad_h;
    pad_w_ = pad_w;
  }
  void Forward(cudaStream_t stream) override;

 private:
  int s2d_ = 1, pad_h_ = 0, pad_w_ = 0;
};

// NHWC fp16 activation -> NCHW fp32 graph output.
class OutputConvertLayer : public Layer {
 public:
  OutputConvertLayer(const std::string& in, const std::string& out);
  void Forward(cudaStream_t stream) override;
};

class Conv2dLayer : public Layer {
 public:
  // s2d > 1 rewrites a stride-s2d conv as a stride-1 conv over the
  // space-to-depth input: Cin*s2d^2 channels, kernel ceil(k/s2d), no padding
  // (the padding moves into the input conversion).
  Conv2dLayer(const pnnx::Operator& op, int c_in, int c_out, int kh, int kw, int sh, int sw, int ph, int pw,
              cudaStream_t stream, int s2d = 1);
  void SetResidual(const std::string& operand) {
    residual_name_ = operand;
    inputs_name_.push_back(operand);
  }
  const std::string& Residual() const { return residual_name_; }
  // Fold the max pool that consumes this conv's output into the conv's
  // epilogue (lotus_conv2d_maxpool_fwd); the output operand becomes the
  // pool's.
  void SetPool(const lotus_pool2d_desc& pool) {
    pool_ = pool;
    has_pool_ = true;
  }
  bool HasPool() const { return has_pool_; }
  void Bind(const OperandMap& operands) override;
  void Forward(cudaStream_t stream) override;
  double Flops() const override;
  size_t WorkspaceBytes() const override;
  int Launches() const override;
  lotus_conv2d_desc Desc() const { return desc_; }
  const void* Weight(size_t* bytes) const override {
    if (bytes) *bytes = w_bytes_;
    return w_packed_.get();
  }

 private:
  double flops_per_pixel_ = 0.0;  // 2*Cout*Cin*kh*kw of the model's own conv
  size_t w_bytes_ = 0;
  std::shared_ptr<void> w_packed_;
  std::shared_ptr<void> bias_;
  std::string residual_name_;
  lotus_conv2d_desc desc_{};
  lotus_pool2d_desc pool_{};
  bool has_pool_ = false;
};

class TransposedConv2dLayer : public Layer {
 public:
  TransposedConv2dLayer(const pnnx::Operator& op, int c_in, int c_out, int kh, int kw, int sh, int sw, int ph, int pw,
                        int oph, int opw, cudaStream_t stream);
  void Bind(const OperandMap& operands) override;
  void Forward(cudaStream_t stream) override;
  double Flops() const override;
  int Launches() const override;
  const void* Weight(size_t* bytes) const override {
    if (bytes) *bytes = w_bytes_;
    return w_packed_.get();
  }

 private:
  size_t w_bytes_ = 0;
  std::shared_ptr<void> w_packed_;
  std::shared_ptr<void> bias_;
  lotus_tconv2d_desc desc_{};
};

class LinearLayer : public Layer {
 public:
  // fc_chw: the flattened spatial input's (C, H, W) when the weight columns
  // must be permuted to NHWC order, else all zero.
  LinearLayer(const pnnx::Operator& op, int in_f, int out_f, int fc_c, int fc_h, int fc_w, cudaStream_t stream);
  void Bind(const OperandMap& operands) override;
  void Forward(cudaStream_t stream) override;
  double Flops() const override;
  size_t WorkspaceBytes() const override;
  int Launches() const override;
  const void* Weight(size_t* bytes) const override {
    if (bytes) *bytes = w_bytes_;
    return w_packed_.get();
  }

 private:
  size_t w_bytes_ = 0;
  std::shared_ptr<void> w_packed_;
  std::shared_ptr<void> bias_;
  int in_f_ = 0, out_f_ = 0, m_ = 0;
  bool out_f32_ = false;
};

class Maxpool2dLayer : public Layer {
 public:
  Maxpool2dLayer(const pnnx::Operator& op, int kh, int kw, int sh, int sw, int ph, int pw);
  void Bind(const OperandMap& operands) override;
  void Forward(cudaStream_t stream) override;
  // Window, stride, padding and folded activation (sizes are set at Bind).
  lotus_pool2d_desc Desc() const {
    lotus_pool2d_desc d = desc_;
    d.act = af_;
    return d;
  }

 private:
  lotus_pool2d_desc desc_{};
};

class AdaptiveAvgpool2dLayer : public Layer {
 public:
  AdaptiveAvgpool2dLayer(const pnnx::Operator& op, int oh, int ow);
  void Bind(const OperandMap& operands) override;
  void Forward(cudaStream_t stream) override;

 private:
  int oh_, ow_;
  bool out_f32_ = false;
};

// pnnx.Expression add(@0,@1) not folded into a convolution.
class ExpressionLayer : public Layer {
 public:
  explicit ExpressionLayer(const pnnx::Operator& op);
  void Forward(cudaStream_t stream) override;
};

// torch.flatten: the output operand aliases the input (no kernel).
class FlattenLayer : public Layer {
 public:
  explicit FlattenLayer(const pnnx::Operator& op);
  void Bind(const OperandMap& operands) override;
  void Forward(cudaStream_t) override {}
  int Launches() const override { return 0; }
  double Bytes() const override { return 0.0; }
};

class CatLayer : public Layer {
 public:
  explicit CatLayer(const pnnx::Operator& op);
  void Forward(cudaStream_t stream) override;
  // Both halves are written in place by their producers: nothing to launch.
  void SetFused() { fused_ = true; }
  bool Fused() const { return fused_; }
  int Launches() const override { return fused_ ? 0 : 1; }
  double Bytes() const override { return fused_ ? 0.0 : Layer::Bytes(); }

 private:
  bool fused_ = false;
};

}  // namespace lotus
