#include "layers.hpp"

#include <stdexcept>

namespace lotus {

void LotusCheck(int status, const std::string& where) {
  if (status != LOTUS_OK) throw std::runtime_error(where + ": " + lotus_last_error_string());
}

static std::shared_ptr<void> device_buffer(size_t bytes) {
  void* p = nullptr;
  CudaCheck(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc");
  return std::shared_ptr<void>(p, [](void* q) { cudaFree(q); });
}

// Uploads an fp32 attribute on `stream` and waits for it; returns an empty
// pointer when the attribute is absent.  The copy must be ordered before the
// prepack kernel on the same (non-blocking) stream: a plain cudaMemcpy from
// pageable memory may return before its DMA lands and runs on the legacy
// stream, which a non-blocking stream does not wait for.
static std::shared_ptr<void> upload_f32(const pnnx::Operator& op, const std::string& key, size_t expect_elems,
                                        cudaStream_t stream) {
  auto it = op.attrs.find(key);
  if (it == op.attrs.end() || it->second.data.empty()) return nullptr;
  if (it->second.type != "f32") throw std::runtime_error(op.name + "." + key + ": only f32 weights are supported");
  if (it->second.data.size() != expect_elems * 4)
    throw std::runtime_error(op.name + "." + key + ": unexpected size");
  auto buf = device_buffer(it->second.data.size());
  CudaCheck(cudaMemcpyAsync(buf.get(), it->second.data.data(), it->second.data.size(), cudaMemcpyHostToDevice, stream),
            "weight upload");
  CudaCheck(cudaStreamSynchronize(stream), "weight upload");
  return buf;
}

static std::shared_ptr<void> upload_host(const std::vector<float>& v, cudaStream_t stream) {
  auto buf = device_buffer(v.size() * 4);
  CudaCheck(cudaMemcpyAsync(buf.get(), v.data(), v.size() * 4, cudaMemcpyHostToDevice, stream), "weight upload");
  CudaCheck(cudaStreamSynchronize(stream), "weight upload");
  return buf;
}

static bool param_bool(const pnnx::Operator& op, const std::string& k, bool dflt) {
  auto it = op.params.find(k);
  return it == op.params.end() ? dflt : it->second.b;
}

void Layer::Bind(const OperandMap& operands) {
  inputs_.clear();
  outputs_.clear();
  for (auto& n : inputs_name_) {
    auto it = operands.find(n);
    if (it == operands.end()) throw std::runtime_error(name_ + ": missing input operand " + n);
    inputs_.push_back(it->second);
  }
  for (auto& n : outputs_name_) {
    auto it = operands.find(n);
    if (it == operands.end()) throw std::runtime_error(name_ + ": missing output operand " + n);
    outputs_.push_back(it->second);
  }
}

double Layer::Bytes() const {
  double b = 0;
  for (auto& o : inputs_) b += static_cast<double>(o->tensor_.Bytes());
  for (auto& o : outputs_) b += static_cast<double>(o->tensor_.Bytes());
  return b;
}

// ------------------------------------------------------------------ convert
InputConvertLayer::InputConvertLayer(const std::string& in, const std::string& out) {
  name_ = "input_to_nhwc";
  type_ = "lotus.InputConvert";
  inputs_name_ = {in};
  outputs_name_ = {out};
}

void InputConvertLayer::Forward(cudaStream_t stream) {
  const Tensor& x = inputs_[0]->tensor_;
  if (s2d_ > 1) {
    const Tensor& y = outputs_[0]->tensor_;
    LotusCheck(lotus_space_to_depth_f16(x.DataF32(), y.Data(), x.Dim(0), x.Dim(1), x.Dim(2), x.Dim(3), s2d_, pad_h_,
                                        pad_w_, y.Dim(2), y.Dim(3), stream),
               name_);
    return;
  }
  LotusCheck(lotus_nchw_f32_to_nhwc_f16(x.DataF32(), outputs_[0]->tensor_.Data(), x.Dim(0), x.Dim(1), x.Dim(2),
                                        x.Dim(3), stream),
             name_);
}

OutputConvertLayer::OutputConvertLayer(const std::string& in, const std::string& out) {
  name_ = "output_to_nchw";
  type_ = "lotus.OutputConvert";
  inputs_name_ = {in};
  outputs_name_ = {out};
}

void OutputConvertLayer::Forward(cudaStream_t stream) {
  const Tensor& x = inputs_[0]->tensor_;
  const auto& s = x.Shape();
  const int h = s.size() > 2 ? static_cast<int>(s[2]) : 1;
  const int w = s.size() > 3 ? static_cast<int>(s[3]) : 1;
  LotusCheck(lotus_nhwc_f16_to_nchw_f32(x.Data(), outputs_[0]->tensor_.DataF32(), s[0], s[1], h, w, stream), name_);
}

// ------------------------------------------------------------------ conv
Conv2dLayer::Conv2dLayer(const pnnx::Operator& op, int c_in, int c_out, int kh, int kw, int sh, int sw, int ph,
                         int pw, cudaStream_t stream, int s2d) {
  name_ = op.name;
  type_ = op.type;
  inputs_name_ = {op.inputs.at(0)};
  outputs_name_ = {op.outputs.at(0)};
  flops_per_pixel_ = 2.0 * c_out * c_in * kh * kw;
  const size_t w_elems = static_cast<size_t>(c_out) * c_in * kh * kw;
  std::shared_ptr<void> w32;
  if (s2d > 1) {
    // W'[co][(a*f + b)*Cin + c][r'][s'] = W[co][c][f*r' + a][f*s' + b] (0 past the kernel)
    auto it = op.attrs.find("weight");
    if (it == op.attrs.end() || it->second.data.size() != w_elems * 4)
      throw std::runtime_error(name_ + ": missing or mis-sized weight");
    const float* w = reinterpret_cast<const float*>(it->second.data.data());
    const int f = s2d, kh2 = (kh + f - 1) / f, kw2 = (kw + f - 1) / f, c2 = c_in * f * f;
    std::vector<float> w2(static_cast<size_t>(c_out) * c2 * kh2 * kw2, 0.f);
    for (int co = 0; co < c_out; ++co)
      for (int c = 0; c < c_in; ++c)
        for (int r = 0; r < kh; ++r)
          for (int q = 0; q < kw; ++q) {
            const int a = r % f, r2 = r / f, b = q % f, q2 = q / f;
            const int cc = (a * f + b) * c_in + c;
            w2[((static_cast<size_t>(co) * c2 + cc) * kh2 + r2) * kw2 + q2] =
                w[((static_cast<size_t>(co) * c_in + c) * kh + r) * kw + q];
          }
    w32 = upload_host(w2, stream);
    c_in = c2;
    kh = kh2;
    kw = kw2;
    sh = sw = 1;
    ph = pw = 0;
  } else {
    w32 = upload_f32(op, "weight", w_elems, stream);
    if (!w32) throw std::runtime_error(name_ + ": missing weight");
  }
  desc_.c_in = c_in;
  desc_.c_out = c_out;
  desc_.kh = kh;
  desc_.kw = kw;
  desc_.stride_h = sh;
  desc_.stride_w = sw;
  desc_.pad_h = ph;
  desc_.pad_w = pw;
  desc_.out_kind = LOTUS_OUT_NHWC_F16;
  // weights: OIHW fp32 (source/layer/layer_conv2d.cu:21) -> packed fp16
  desc_.n = 1;
  desc_.h = kh;
  desc_.w = kw;
  w_bytes_ = lotus_conv2d_packed_weight_bytes(&desc_);
  w_packed_ = device_buffer(w_bytes_);
  LotusCheck(lotus_conv2d_prepack(static_cast<const float*>(w32.get()), w_packed_.get(), &desc_, stream), name_);
  CudaCheck(cudaStreamSynchronize(stream), "prepack sync");
  if (param_bool(op, "bias", true)) bias_ = upload_f32(op, "bias", c_out, stream);
}

void Conv2dLayer::Bind(const OperandMap& operands) {
  Layer::Bind(operands);
  const Tensor& x = inputs_[0]->tensor_;
  const Tensor& y = outputs_[0]->tensor_;
  if (x.Fmt() != Format::kNHWC_F16 || y.Fmt() != Format::kNHWC_F16 || x.DimSize() != 4 || y.DimSize() != 4)
    throw std::runtime_error(name_ + ": conv expects NHWC fp16 4-D operands");
  if (!x.Dense()) throw std::runtime_error(name_ + ": conv input must be a dense tensor");
  if (!y.Dense() && (has_pool_ || !residual_name_.empty()))
    throw std::runtime_error(name_ + ": a pooled or residual conv cannot write a channel slice");
  desc_.n = x.Dim(0);
  desc_.h = x.Dim(2);
  desc_.w = x.Dim(3);
  desc_.act = af_;
  if (static_cast<int>(x.Dim(1)) != desc_.c_in) throw std::runtime_error(name_ + ": input channel mismatch");
  int oh = 0, ow = 0;
  LotusCheck(lotus_conv2d_out_hw(&desc_, &oh, &ow), name_);
  if (has_pool_) {
    pool_.n = desc_.n;
    pool_.c = desc_.c_out;
    pool_.h = oh;
    pool_.w = ow;
    LotusCheck(lotus_maxpool2d_out_hw(&pool_, &oh, &ow), name_);
    LotusCheck(lotus_conv2d_maxpool_supported(&desc_, &pool_), name_);
  }
  if (y.Dim(0) != x.Dim(0) || static_cast<int>(y.Dim(1)) != desc_.c_out || static_cast<int>(y.Dim(2)) != oh ||
      static_cast<int>(y.Dim(3)) != ow)
    throw std::runtime_error(name_ + ": output shape mismatch");
  if (!residual_name_.empty() && inputs_.back()->tensor_.Shape() != y.Shape())
    throw std::runtime_error(name_ + ": residual shape mismatch");
}

void Conv2dLayer::Forward(cudaStream_t stream) {
  if (has_pool_) {
    LotusCheck(lotus_conv2d_maxpool_fwd(inputs_[0]->tensor_.Data(), w_packed_.get(),
                                        static_cast<const float*>(bias_.get()), outputs_[0]->tensor_.Data(), &desc_,
                                        &pool_, stream),
               name_);
    return;
  }
  const void* res = residual_name_.empty() ? nullptr : inputs_.back()->tensor_.Data();
  const Tensor& y = outputs_[0]->tensor_;
  if (!y.Dense()) {  // a channel slice of a concat buffer
    LotusCheck(lotus_conv2d_fwd_slice(inputs_[0]->tensor_.Data(), w_packed_.get(),
                                      static_cast<const float*>(bias_.get()), res, y.Data(),
                                      static_cast<int>(y.PixelStride()), &desc_, workspace_, workspace_bytes_, stream),
               name_);
    return;
  }
  LotusCheck(lotus_conv2d_fwd_ws(inputs_[0]->tensor_.Data(), w_packed_.get(), static_cast<const float*>(bias_.get()),
                                 res, y.Data(), &desc_, workspace_, workspace_bytes_, stream),
             name_);
}

size_t Conv2dLayer::WorkspaceBytes() const {
  return has_pool_ ? 0 : lotus_conv2d_workspace_bytes_max(&desc_);
}

int Conv2dLayer::Launches() const {
  if (has_pool_) return 1;
  const size_t need = WorkspaceBytes();
  return (need > 0 && workspace_ != nullptr && need <= workspace_bytes_) ? 2 : 1;  // conv + split-K reduction
}

double Conv2dLayer::Flops() const {
  int oh = 0, ow = 0;
  lotus_conv2d_out_hw(&desc_, &oh, &ow);
  return static_cast<double>(desc_.n) * oh * ow * flops_per_pixel_;
}

// ------------------------------------------------------------------ tconv
TransposedConv2dLayer::TransposedConv2dLayer(const pnnx::Operator& op, int c_in, int c_out, int kh, int kw, int sh,
                                             int sw, int ph, int pw, int oph, int opw, cudaStream_t stream) {
  name_ = op.name;
  type_ = op.type;
  inputs_name_ = {op.inputs.at(0)};
  outputs_name_ = {op.outputs.at(0)};
  desc_ = lotus_tconv2d_desc{1, c_in, kh, kw, c_out, kh, kw, sh, sw, ph, pw, oph, opw, 0};
  desc_.h = desc_.w = 4;  // any valid size for the prepack validation
  auto w32 = upload_f32(op, "weight", static_cast<size_t>(c_in) * c_out * kh * kw, stream);
  if (!w32) throw std::runtime_error(name_ + ": missing weight");
  w_bytes_ = lotus_tconv2d_packed_weight_bytes(&desc_);
  w_packed_ = device_buffer(w_bytes_);
  LotusCheck(lotus_tconv2d_prepack(static_cast<const float*>(w32.get()), w_packed_.get(), &desc_, stream), name_);
  CudaCheck(cudaStreamSynchronize(stream), "prepack sync");
  if (param_bool(op, "bias", true)) bias_ = upload_f32(op, "bias", c_out, stream);
}

void TransposedConv2dLayer::Bind(const OperandMap& operands) {
  Layer::Bind(operands);
  const Tensor& x = inputs_[0]->tensor_;
  const Tensor& y = outputs_[0]->tensor_;
  if (!x.Dense()) throw std::runtime_error(name_ + ": transposed conv input must be a dense tensor");
  desc_.n = x.Dim(0);
  desc_.h = x.Dim(2);
  desc_.w = x.Dim(3);
  desc_.act = af_;
  int oh = 0, ow = 0;
  LotusCheck(lotus_tconv2d_out_hw(&desc_, &oh, &ow), name_);
  if (static_cast<int>(y.Dim(2)) != oh || static_cast<int>(y.Dim(3)) != ow ||
      static_cast<int>(y.Dim(1)) != desc_.c_out)
    throw std::runtime_error(name_ + ": output shape mismatch");
}

void TransposedConv2dLayer::Forward(cudaStream_t stream) {
  const Tensor& y = outputs_[0]->tensor_;
  if (!y.Dense()) {  // a channel slice of a concat buffer
    LotusCheck(lotus_tconv2d_fwd_slice(inputs_[0]->tensor_.Data(), w_packed_.get(),
                                       static_cast<const float*>(bias_.get()), y.Data(),
                                       static_cast<int>(y.PixelStride()), &desc_, stream),
               name_);
    return;
  }
  LotusCheck(lotus_tconv2d_fwd(inputs_[0]->tensor_.Data(), w_packed_.get(), static_cast<const float*>(bias_.get()),
                               y.Data(), &desc_, stream),
             name_);
}

double TransposedConv2dLayer::Flops() const {
  return 2.0 * desc_.n * desc_.h * desc_.w * static_cast<double>(desc_.c_in) * desc_.c_out * desc_.kh * desc_.kw;
}

int TransposedConv2dLayer::Launches() const {
  const bool full = desc_.stride_h == desc_.kh && desc_.stride_w == desc_.kw && desc_.out_pad_h == 0 &&
                    desc_.out_pad_w == 0 && (desc_.c_out % 8) == 0;
  return full ? 1 : 2;
}

// ------------------------------------------------------------------ linear
LinearLayer::LinearLayer(const pnnx::Operator& op, int in_f, int out_f, int fc_c, int fc_h, int fc_w,
                         cudaStream_t stream)
    : in_f_(in_f), out_f_(out_f) {
  name_ = op.name;
  type_ = op.type;
  inputs_name_ = {op.inputs.at(0)};
  outputs_name_ = {op.outputs.at(0)};
  auto w32 = upload_f32(op, "weight", static_cast<size_t>(in_f) * out_f, stream);
  if (!w32) throw std::runtime_error(name_ + ": missing weight");
  w_bytes_ = lotus_linear_packed_weight_bytes(in_f, out_f);
  w_packed_ = device_buffer(w_bytes_);
  LotusCheck(lotus_linear_prepack(static_cast<const float*>(w32.get()), w_packed_.get(), in_f, out_f, fc_c, fc_h, fc_w,
                                  stream),
             name_);
  CudaCheck(cudaStreamSynchronize(stream), "prepack sync");
  if (param_bool(op, "bias", true)) bias_ = upload_f32(op, "bias", out_f, stream);
}

void LinearLayer::Bind(const OperandMap& operands) {
  Layer::Bind(operands);
  const Tensor& x = inputs_[0]->tensor_;
  const Tensor& y = outputs_[0]->tensor_;
  m_ = static_cast<int>(x.Dim(0));
  out_f32_ = y.Fmt() == Format::kNCHW_F32;
  if (x.Fmt() != Format::kNHWC_F16) throw std::runtime_error(name_ + ": linear input must be fp16 rows");
  if (static_cast<int>(y.Dim(1)) != out_f_) throw std::runtime_error(name_ + ": output features mismatch");
}

void LinearLayer::Forward(cudaStream_t stream) {
  LotusCheck(lotus_linear_fwd_ws(inputs_[0]->tensor_.Data(), w_packed_.get(), static_cast<const float*>(bias_.get()),
                                 outputs_[0]->tensor_.Data(), m_, in_f_, out_f_, af_,
                                 out_f32_ ? LOTUS_OUT_ROWS_F32 : LOTUS_OUT_NHWC_F16, workspace_, workspace_bytes_,
                                 stream),
             name_);
}

size_t LinearLayer::WorkspaceBytes() const { return lotus_linear_workspace_bytes(m_, in_f_, out_f_); }

int LinearLayer::Launches() const {
  // GEMV, or GEMM (+ the split-K reduction)
  if (m_ <= 8) return 1;
  const size_t need = WorkspaceBytes();
  return (need > 0 && workspace_ != nullptr && need <= workspace_bytes_) ? 2 : 1;
}

double LinearLayer::Flops() const { return 2.0 * m_ * static_cast<double>(in_f_) * out_f_; }

// ------------------------------------------------------------------ pooling
Maxpool2dLayer::Maxpool2dLayer(const pnnx::Operator& op, int kh, int kw, int sh, int sw, int ph, int pw) {
  name_ = op.name;
  type_ = op.type;
  inputs_name_ = {op.inputs.at(0)};
  outputs_name_ = {op.outputs.at(0)};
  desc_ = lotus_pool2d_desc{0, 0, 0, 0, kh, kw, sh, sw, ph, pw, 0};
}

void Maxpool2dLayer::Bind(const OperandMap& operands) {
  Layer::Bind(operands);
  const Tensor& x = inputs_[0]->tensor_;
  desc_.n = x.Dim(0);
  desc_.c = x.Dim(1);
  desc_.h = x.Dim(2);
  desc_.w = x.Dim(3);
  desc_.act = af_;
  int oh = 0, ow = 0;
  LotusCheck(lotus_maxpool2d_out_hw(&desc_, &oh, &ow), name_);
  const Tensor& y = outputs_[0]->tensor_;
  if (static_cast<int>(y.Dim(2)) != oh || static_cast<int>(y.Dim(3)) != ow)
    throw std::runtime_error(name_ + ": output shape mismatch");
}

void Maxpool2dLayer::Forward(cudaStream_t stream) {
  const Tensor& x = inputs_[0]->tensor_;
  if (!x.Dense()) {  // the encoder half of a concat buffer
    LotusCheck(lotus_maxpool2d_fwd_strided(x.Data(), static_cast<int>(x.PixelStride()), outputs_[0]->tensor_.Data(),
                                           &desc_, stream),
               name_);
    return;
  }
  LotusCheck(lotus_maxpool2d_fwd(x.Data(), outputs_[0]->tensor_.Data(), &desc_, stream), name_);
}

AdaptiveAvgpool2dLayer::AdaptiveAvgpool2dLayer(const pnnx::Operator& op, int oh, int ow) : oh_(oh), ow_(ow) {
  name_ = op.name;
  type_ = op.type;
  inputs_name_ = {op.inputs.at(0)};
  outputs_name_ = {op.outputs.at(0)};
}

void AdaptiveAvgpool2dLayer::Bind(const OperandMap& operands) {
  Layer::Bind(operands);
  out_f32_ = outputs_[0]->tensor_.Fmt() == Format::kNCHW_F32;
  if (out_f32_ && (oh_ != 1 || ow_ != 1))
    throw std::runtime_error(name_ + ": fp32 output of a spatial pooling must go through the output layer");
}

void AdaptiveAvgpool2dLayer::Forward(cudaStream_t stream) {
  const Tensor& x = inputs_[0]->tensor_;
  LotusCheck(lotus_adaptive_avgpool2d_fwd(x.Data(), outputs_[0]->tensor_.Data(), x.Dim(0), x.Dim(1), x.Dim(2),
                                          x.Dim(3), oh_, ow_, af_, out_f32_ ? 1 : 0, stream),
             name_);
}

// ------------------------------------------------------------------ eltwise
ExpressionLayer::ExpressionLayer(const pnnx::Operator& op) {
  name_ = op.name;
  type_ = op.type;
  auto it = op.params.find("expr");
  if (it == op.params.end() || it->second.s.rfind("add(", 0) != 0 || op.inputs.size() != 2)
    throw std::runtime_error(name_ + ": only expr=add(@0,@1) is supported");
  inputs_name_ = op.inputs;
  outputs_name_ = {op.outputs.at(0)};
}

void ExpressionLayer::Forward(cudaStream_t stream) {
  const Tensor& a = inputs_[0]->tensor_;
  size_t pixels = a.Dim(0);
  for (size_t i = 2; i < a.DimSize(); ++i) pixels *= a.Dim(i);
  LotusCheck(lotus_add_act_fwd(a.Data(), inputs_[1]->tensor_.Data(), outputs_[0]->tensor_.Data(), pixels, a.Dim(1),
                               af_, stream),
             name_);
}

FlattenLayer::FlattenLayer(const pnnx::Operator& op) {
  name_ = op.name;
  type_ = op.type;
  inputs_name_ = {op.inputs.at(0)};
  outputs_name_ = {op.outputs.at(0)};
}

void FlattenLayer::Bind(const OperandMap& operands) {
  Layer::Bind(operands);
  const Tensor& x = inputs_[0]->tensor_;
  uint32_t feat = 1;
  for (size_t i = 1; i < x.DimSize(); ++i) feat *= x.Dim(i);
  const bool spatial = x.DimSize() == 4 && (x.Dim(2) != 1 || x.Dim(3) != 1);
  if (spatial && (x.Dim(1) % 8) != 0)
    throw std::runtime_error(name_ + ": flatten of a spatial map needs a channel count divisible by 8");
  // NHWC storage flattened in (h, w, c) order; the consuming Linear permutes its weights to match.
  outputs_[0]->tensor_ = x.View({x.Dim(0), feat}, Format::kNHWC_F16);
}

CatLayer::CatLayer(const pnnx::Operator& op) {
  name_ = op.name;
  type_ = op.type;
  auto it = op.params.find("dim");
  if (op.inputs.size() != 2 || it == op.params.end() || it->second.i != 1)
    throw std::runtime_error(name_ + ": only two-input torch.cat along dim 1 is supported");
  inputs_name_ = op.inputs;
  outputs_name_ = {op.outputs.at(0)};
}

void CatLayer::Forward(cudaStream_t stream) {
  if (fused_) return;
  const Tensor& a = inputs_[0]->tensor_;
  const Tensor& b = inputs_[1]->tensor_;
  LotusCheck(lotus_concat_channels_fwd(a.Data(), a.Dim(1), b.Data(), b.Dim(1), outputs_[0]->tensor_.Data(), a.Dim(0),
                                       a.Dim(2), a.Dim(3), stream),
             name_);
}

}  // namespace lotus
