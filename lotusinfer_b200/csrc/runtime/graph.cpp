#include "graph.hpp"

#include <algorithm>
#include <functional>
#include <queue>
#include <set>
#include <stdexcept>
#include <string>

namespace lotus_impl {
int read_device_error();  // conv_tc.cu: returns and clears the device error word (-1: unreadable)
}

namespace lotus {

namespace {

const pnnx::Parameter& need(const pnnx::Operator& op, const std::string& key) {
  auto it = op.params.find(key);
  if (it == op.params.end()) throw std::runtime_error(op.name + ": missing parameter '" + key + "'");
  return it->second;
}

int pair0(const pnnx::Parameter& p) { return p.ai.empty() ? p.i : p.ai.at(0); }
int pair1(const pnnx::Parameter& p) { return p.ai.size() < 2 ? pair0(p) : p.ai.at(1); }

bool is_act(const std::string& t) { return t == "nn.ReLU" || t == "F.sigmoid"; }

}  // namespace

Graph::Graph(const std::string& param_path, const std::string& bin_path, uint32_t batch_size)
    : Graph(param_path, bin_path, batch_size, Options()) {}

Graph::Graph(const std::string& param_path, const std::string& bin_path, uint32_t batch_size, const Options& opt)
    : batch_(batch_size), opt_(opt) {
  if (batch_size == 0) throw std::runtime_error("batch size must be positive");
  if (opt_.device >= 0) CudaCheck(cudaSetDevice(opt_.device), "cudaSetDevice");
  CudaCheck(cudaGetDevice(&device_), "cudaGetDevice");
  CudaCheck(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
  try {
    Build(param_path, bin_path);
  } catch (...) {
    cudaStreamDestroy(stream_);
    throw;
  }
}

Graph::~Graph() {
  if (pipe_) {
    for (cudaStream_t s : {pipe_->h2d, pipe_->h2d_b, pipe_->d2h})
      if (s) {
        cudaStreamSynchronize(s);
        cudaStreamDestroy(s);
      }
    for (int k = 0; k < 2; ++k) {
      if (pipe_->exec[k]) cudaGraphExecDestroy(pipe_->exec[k]);
      for (cudaEvent_t e : {pipe_->h2d_done[k], pipe_->h2d_b_done[k], pipe_->fwd_done[k], pipe_->d2h_done[k]})
        if (e) cudaEventDestroy(e);
    }
  }
  if (exec_) cudaGraphExecDestroy(exec_);
  if (stream_) {
    cudaStreamSynchronize(stream_);
    cudaStreamDestroy(stream_);
  }
}

void Graph::Build(const std::string& param_path, const std::string& bin_path) {
  pnnx::Graph g;
  g.Load(param_path, bin_path);

  std::map<std::string, const pnnx::Operator*> op_by_name;
  for (auto& op : g.ops) op_by_name[op.name] = &op;

  // graph input / output operands (source/graph.cpp:52-63)
  for (auto& op : g.ops) {
    if (op.type == "pnnx.Input") {
      if (!input_operand_.empty() || op.outputs.size() != 1) throw std::runtime_error("graph must have one input");
      input_operand_ = op.outputs[0];
    } else if (op.type == "pnnx.Output") {
      if (!output_operand_.empty() || op.inputs.size() != 1) throw std::runtime_error("graph must have one output");
      output_operand_ = op.inputs[0];
    }
  }
  if (input_operand_.empty() || output_operand_.empty()) throw std::runtime_error("graph input/output not found");

  // logical shapes with dim 0 := batch (source/graph.cpp:66-72)
  std::map<std::string, std::vector<uint32_t>> shapes;
  for (auto& kv : g.operands) {
    const auto& info = kv.second;
    if (info.type != "f32") throw std::runtime_error("operand " + kv.first + ": only f32 models are supported");
    std::vector<uint32_t> s;
    for (size_t i = 0; i < info.shape.size(); ++i) {
      if (i > 0 && info.shape[i] <= 0) throw std::runtime_error("operand " + kv.first + ": dynamic shape");
      s.push_back(i == 0 ? batch_ : static_cast<uint32_t>(info.shape[i]));
    }
    shapes[kv.first] = s;
  }

  // layers, with ReLU/sigmoid folded into the producer (source/layer/layer_conv2d.cu:129-141)
  for (auto& op : g.ops) {
    const std::string& t = op.type;
    if (t == "pnnx.Input" || t == "pnnx.Output" || is_act(t)) continue;
    std::shared_ptr<Layer> layer;
    if (t == "nn.Conv2d") {
      if (need(op, "groups").i != 1) throw std::runtime_error(op.name + ": only groups=1 is supported");
      const auto& dil = need(op, "dilation");
      if (pair0(dil) != 1 || pair1(dil) != 1) throw std::runtime_error(op.name + ": only dilation 1 is supported");
      auto pm = op.params.find("padding_mode");
      if (pm != op.params.end() && pm->second.s != "zeros") throw std::runtime_error(op.name + ": zero padding only");
      const auto& ks = need(op, "kernel_size");
      const auto& st = need(op, "stride");
      const auto& pd = need(op, "padding");
      if (pd.type == 4) throw std::runtime_error(op.name + ": string padding is not supported");
      const int cin = need(op, "in_channels").i;
      int s2d = 1;
      // stem rewrite: a strided conv on the graph input with few channels becomes
      // a stride-1 conv over the space-to-depth input (K = Cin*f^2*ceil(k/f)^2
      // instead of roundup(Cin,8)*k^2, contiguous 128-byte K rows)
      if (opt_.s2d_stem && op.inputs.at(0) == input_operand_ && g.operands.at(input_operand_).consumers.size() == 1 &&
          pair0(st) == pair1(st) && pair0(st) >= 2 && pair0(st) <= 8 && cin * pair0(st) * pair0(st) <= 64 &&
          shapes.at(op.outputs.at(0)).size() == 4) {
        s2d = pair0(st);
        const auto& os = shapes.at(op.outputs.at(0));
        stem_s2d_ = s2d;
        stem_pad_h_ = pair0(pd);
        stem_pad_w_ = pair1(pd);
        stem_shape_ = {os[0], static_cast<uint32_t>(cin * s2d * s2d), os[2] + (pair0(ks) + s2d - 1) / s2d - 1,
                       os[3] + (pair1(ks) + s2d - 1) / s2d - 1};
      }
      layer = std::make_shared<Conv2dLayer>(op, cin, need(op, "out_channels").i, pair0(ks), pair1(ks), pair0(st),
                                            pair1(st), pair0(pd), pair1(pd), stream_, s2d);
    } else if (t == "nn.ConvTranspose2d") {
      if (need(op, "groups").i != 1) throw std::runtime_error(op.name + ": only groups=1 is supported");
      const auto& dil = need(op, "dilation");
      if (pair0(dil) != 1 || pair1(dil) != 1) throw std::runtime_error(op.name + ": only dilation 1 is supported");
      const auto& ks = need(op, "kernel_size");
      const auto& st = need(op, "stride");
      const auto& pd = need(op, "padding");
      auto opad_it = op.params.find("output_padding");
      int oph = 0, opw = 0;
      if (opad_it != op.params.end()) {
        oph = pair0(opad_it->second);
        opw = pair1(opad_it->second);
      }
      layer = std::make_shared<TransposedConv2dLayer>(op, need(op, "in_channels").i, need(op, "out_channels").i,
                                                      pair0(ks), pair1(ks), pair0(st), pair1(st), pair0(pd),
                                                      pair1(pd), oph, opw, stream_);
    } else if (t == "nn.Linear") {
      int fc_c = 0, fc_h = 0, fc_w = 0;
      const auto& in_name = op.inputs.at(0);
      const auto& prod = g.operands.at(in_name).producer;
      if (!prod.empty() && op_by_name.at(prod)->type == "torch.flatten") {
        const auto& src = shapes.at(op_by_name.at(prod)->inputs.at(0));
        if (src.size() == 4 && (src[2] != 1 || src[3] != 1)) {
          fc_c = static_cast<int>(src[1]);
          fc_h = static_cast<int>(src[2]);
          fc_w = static_cast<int>(src[3]);
        }
      }
      layer = std::make_shared<LinearLayer>(op, need(op, "in_features").i, need(op, "out_features").i, fc_c, fc_h,
                                            fc_w, stream_);
    } else if (t == "nn.MaxPool2d") {
      auto cm = op.params.find("ceil_mode");
      if (cm != op.params.end() && cm->second.b) throw std::runtime_error(op.name + ": ceil_mode is not supported");
      auto ri = op.params.find("return_indices");
      if (ri != op.params.end() && ri->second.b)
        throw std::runtime_error(op.name + ": return_indices is not supported");
      const auto& ks = need(op, "kernel_size");
      const auto& st = need(op, "stride");
      const auto& pd = need(op, "padding");
      layer = std::make_shared<Maxpool2dLayer>(op, pair0(ks), pair1(ks), pair0(st), pair1(st), pair0(pd), pair1(pd));
    } else if (t == "nn.AdaptiveAvgPool2d") {
      const auto& os = need(op, "output_size");
      layer = std::make_shared<AdaptiveAvgpool2dLayer>(op, pair0(os), pair1(os));
    } else if (t == "pnnx.Expression") {
      layer = std::make_shared<ExpressionLayer>(op);
    } else if (t == "torch.flatten") {
      layer = std::make_shared<FlattenLayer>(op);
    } else if (t == "torch.cat") {
      layer = std::make_shared<CatLayer>(op);
    } else {
      throw std::runtime_error("unsupported layer type " + t);
    }
    // fold a sole ReLU / sigmoid consumer
    const auto& consumers = g.operands.at(op.outputs.at(0)).consumers;
    if (consumers.size() == 1 && is_act(op_by_name.at(consumers[0])->type) && t != "torch.flatten") {
      const auto* act = op_by_name.at(consumers[0]);
      layer->af_ = act->type == "nn.ReLU" ? RELU : SIGMOID;
      layer->outputs_name_ = {act->outputs.at(0)};
    }
    if (layers_.count(op.name)) throw std::runtime_error("duplicate layer name " + op.name);
    layers_[op.name] = layer;
    layer_order_.push_back(op.name);
  }
  // every activation op must have been folded
  for (auto& op : g.ops) {
    if (!is_act(op.type)) continue;
    bool folded = false;
    for (auto& kv : layers_)
      if (!kv.second->outputs_name_.empty() && kv.second->outputs_name_[0] == op.outputs.at(0)) folded = true;
    if (!folded) throw std::runtime_error(op.name + ": activation without a foldable producer is not supported");
  }

  // residual fusion: conv (sole consumer: add) -> add (-> act) becomes conv with residual
  auto consumers_of = [&](const std::string& operand) {
    std::vector<std::shared_ptr<Layer>> c;
    for (auto& kv : layers_)
      for (auto& in : kv.second->inputs_name_)
        if (in == operand) c.push_back(kv.second);
    return c;
  };
  auto producer_of = [&](const std::string& operand) -> std::shared_ptr<Layer> {
    for (auto& kv : layers_)
      for (auto& out : kv.second->outputs_name_)
        if (out == operand) return kv.second;
    return nullptr;
  };
  if (opt_.fuse_residual) {
    std::vector<std::string> fused;
    for (auto& name : layer_order_) {
      auto expr = std::dynamic_pointer_cast<ExpressionLayer>(layers_.at(name));
      if (!expr) continue;
      for (int side = 0; side < 2; ++side) {
        const std::string& mine = expr->inputs_name_[side];
        const std::string& other = expr->inputs_name_[1 - side];
        auto conv = std::dynamic_pointer_cast<Conv2dLayer>(producer_of(mine));
        if (!conv || conv->af_ != NONE || !conv->Residual().empty() || mine == other) continue;
        if (consumers_of(mine).size() != 1) continue;
        if (shapes.at(mine) != shapes.at(other)) continue;
        conv->SetResidual(other);
        conv->af_ = expr->af_;
        conv->outputs_name_ = expr->outputs_name_;
        fused.push_back(name);
        break;
      }
    }
    for (auto& n : fused) {
      layers_.erase(n);
      layer_order_.erase(std::find(layer_order_.begin(), layer_order_.end(), n));
    }
  }

  // pool fusion: conv (sole consumer: a 3x3/2 pad-1 max pool) -> pool becomes
  // one conv whose epilogue writes the pooled output (the ResNet stem; the
  // full-size conv output is never stored)
  if (opt_.fuse_pool) {
    std::vector<std::string> fused;
    for (auto& name : layer_order_) {
      auto pool = std::dynamic_pointer_cast<Maxpool2dLayer>(layers_.at(name));
      if (!pool) continue;
      const std::string& src = pool->inputs_name_.at(0);
      auto conv = std::dynamic_pointer_cast<Conv2dLayer>(producer_of(src));
      if (!conv || !conv->Residual().empty() || conv->HasPool() || consumers_of(src).size() != 1) continue;
      const std::string& cin = conv->inputs_name_.at(0);
      const auto& xs = (cin == input_operand_ && stem_s2d_ > 1) ? stem_shape_ : shapes.at(cin);
      const auto& ys = shapes.at(src);
      if (xs.size() != 4 || ys.size() != 4) continue;
      lotus_conv2d_desc d = conv->Desc();
      d.n = static_cast<int>(xs[0]);
      d.h = static_cast<int>(xs[2]);
      d.w = static_cast<int>(xs[3]);
      d.act = conv->af_;
      lotus_pool2d_desc pd = pool->Desc();
      pd.n = d.n;
      pd.c = static_cast<int>(ys[1]);
      pd.h = static_cast<int>(ys[2]);
      pd.w = static_cast<int>(ys[3]);
      if (lotus_conv2d_maxpool_supported(&d, &pd) != LOTUS_OK) continue;
      conv->SetPool(pd);
      conv->outputs_name_ = pool->outputs_name_;
      fused.push_back(name);
    }
    for (auto& n : fused) {
      layers_.erase(n);
      layer_order_.erase(std::find(layer_order_.begin(), layer_order_.end(), n));
    }
  }

  // operands that carry data after fusion
  std::set<std::string> live;
  for (auto& kv : layers_) {
    for (auto& n : kv.second->inputs_name_) live.insert(n);
    for (auto& n : kv.second->outputs_name_) live.insert(n);
  }
  live.insert(input_operand_);
  live.insert(output_operand_);

  // input conversion: NCHW fp32 -> NHWC fp16
  const std::string in_nhwc = input_operand_ + "@nhwc";
  for (auto& kv : layers_)
    for (auto& n : kv.second->inputs_name_)
      if (n == input_operand_) n = in_nhwc;
  {
    auto l = std::make_shared<InputConvertLayer>(input_operand_, in_nhwc);
    if (stem_s2d_ > 1) l->SetSpaceToDepth(stem_s2d_, stem_pad_h_, stem_pad_w_);
    layers_[l->Name()] = l;
    layer_order_.insert(layer_order_.begin(), l->Name());
  }
  shapes[in_nhwc] = stem_s2d_ > 1 ? stem_shape_ : shapes.at(input_operand_);

  // output: Linear and 1x1 adaptive pooling write fp32 rows directly, others convert
  auto out_prod = producer_of(output_operand_);
  if (!out_prod) throw std::runtime_error("graph output has no producer");
  const bool direct_f32 = std::dynamic_pointer_cast<LinearLayer>(out_prod) != nullptr ||
                          (std::dynamic_pointer_cast<AdaptiveAvgpool2dLayer>(out_prod) != nullptr &&
                           (shapes.at(output_operand_).size() == 2 ||
                            (shapes.at(output_operand_)[2] == 1 && shapes.at(output_operand_)[3] == 1)));
  if (!direct_f32) {
    const std::string out_nhwc = output_operand_ + "@nhwc";
    out_prod->outputs_name_ = {out_nhwc};
    shapes[out_nhwc] = shapes.at(output_operand_);
    auto l = std::make_shared<OutputConvertLayer>(out_nhwc, output_operand_);
    layers_[l->Name()] = l;
    layer_order_.push_back(l->Name());
  }

  // allocate operand tensors (flatten outputs alias their input)
  std::set<std::string> aliased;
  for (auto& kv : layers_)
    if (std::dynamic_pointer_cast<FlattenLayer>(kv.second)) aliased.insert(kv.second->outputs_name_[0]);
  std::set<std::string> needed;
  for (auto& kv : layers_) {
    for (auto& n : kv.second->inputs_name_) needed.insert(n);
    for (auto& n : kv.second->outputs_name_) needed.insert(n);
  }
  for (auto& n : needed) {
    auto opnd = std::make_shared<Operand>();
    opnd->name_ = n;
    auto pit = g.operands.find(n);
    if (pit != g.operands.end()) {
      opnd->producer_ = pit->second.producer;
      opnd->consumers_ = pit->second.consumers;
    }
    const auto& s = shapes.at(n);
    const bool f32 = (n == input_operand_) || (n == output_operand_);
    if (!aliased.count(n)) opnd->tensor_ = Tensor::Unallocated(s, f32 ? Format::kNCHW_F32 : Format::kNHWC_F16);
    operands_[n] = opnd;
  }

  TopoSortLayers();
  std::map<std::string, std::pair<std::string, uint32_t>> slice_of;  // operand -> (concat operand, first channel)
  if (opt_.fuse_concat) FuseConcats(&slice_of);
  PlanMemory(slice_of);
  // bind in order so flatten aliases exist before their consumers bind
  for (auto& l : topo_sorted_layers_) l->Bind(operands_);
  // one split-K workspace for the layer that wants the most
  size_t ws = 0;
  for (auto& l : topo_sorted_layers_) ws = std::max(ws, l->WorkspaceBytes());
  if (ws > 0) {
    void* p = nullptr;
    CudaCheck(cudaMalloc(&p, ws), "cudaMalloc(workspace)");
    workspace_ = std::shared_ptr<void>(p, [](void* q) { cudaFree(q); });
    for (auto& l : topo_sorted_layers_) l->SetWorkspace(p, ws);
  }
  CudaCheck(cudaStreamSynchronize(stream_), "graph build");
}

std::shared_ptr<Layer> Graph::ProducerOf(const std::string& operand) const {
  for (auto& l : topo_sorted_layers_)
    for (auto& o : l->outputs_name_)
      if (o == operand) return l;
  return nullptr;
}

void Graph::FuseConcats(std::map<std::string, std::pair<std::string, uint32_t>>* slice_of) {
  // torch.cat(a, b) along channels with both halves produced by a conv or a
  // transposed conv: the producers write straight into their channel slice of
  // the concat buffer (NHWC: a pixel-stride change), and the concat launches
  // nothing.  Other readers of a half must take a strided input: max pools
  // (the U-Net encoder output feeds both the next level's pool and the
  // decoder's concat).  The reference copies both halves into the concat
  // operand per sample (source/layer/concatenate.cpp:20-35).
  auto writes_slices = [](const std::shared_ptr<Layer>& l) {
    if (auto c = std::dynamic_pointer_cast<Conv2dLayer>(l)) return !c->HasPool();
    return std::dynamic_pointer_cast<TransposedConv2dLayer>(l) != nullptr;
  };
  for (auto& l : topo_sorted_layers_) {
    auto cat = std::dynamic_pointer_cast<CatLayer>(l);
    if (!cat) continue;
    const std::string a = cat->inputs_name_.at(0), b = cat->inputs_name_.at(1), y = cat->outputs_name_.at(0);
    if (a == b || a == input_operand_ || b == input_operand_ || y == output_operand_) continue;
    if (slice_of->count(a) || slice_of->count(b) || slice_of->count(y)) continue;
    const Tensor& ta = operands_.at(a)->tensor_;
    const Tensor& tb = operands_.at(b)->tensor_;
    const Tensor& ty = operands_.at(y)->tensor_;
    if (ta.Fmt() != Format::kNHWC_F16 || tb.Fmt() != Format::kNHWC_F16 || ty.Fmt() != Format::kNHWC_F16) continue;
    if (ta.DimSize() != 4 || tb.DimSize() != 4 || ty.DimSize() != 4 || ta.Dim(1) % 8 != 0) continue;
    if (!writes_slices(ProducerOf(a)) || !writes_slices(ProducerOf(b))) continue;
    bool other_readers_ok = true;
    for (auto& r : topo_sorted_layers_) {
      if (r == l) continue;
      for (auto& in : r->inputs_name_)
        if ((in == a || in == b) && !std::dynamic_pointer_cast<Maxpool2dLayer>(r)) other_readers_ok = false;
    }
    if (!other_readers_ok) continue;
    (*slice_of)[a] = {y, 0};
    (*slice_of)[b] = {y, ta.Dim(1)};
    cat->SetFused();
  }
}

void Graph::PlanMemory(const std::map<std::string, std::pair<std::string, uint32_t>>& slice_of) {
  // Storage roots: operands with storage of their own (channel slices live in
  // their concat buffer, flatten outputs alias their input).  A root is live
  // from the first layer that writes it (or a slice of it) to the last layer
  // that reads it (or an alias or slice of it), in the order the layers run.
  // With the plan on, a root takes the smallest free block of at least its
  // size whose last reader ran strictly before the root's first writer (the
  // layers run one after another on one stream, replayed from one CUDA
  // graph), else a new block.  The graph input and output keep their own
  // buffers (the caller copies into and out of them).  The reference
  // allocates every operand separately (source/graph.cpp:50-82).
  std::map<std::string, std::string> alias_of;
  for (auto& l : topo_sorted_layers_)
    if (std::dynamic_pointer_cast<FlattenLayer>(l)) alias_of[l->outputs_name_.at(0)] = l->inputs_name_.at(0);
  std::function<std::string(const std::string&)> root = [&](const std::string& n) -> std::string {
    auto s = slice_of.find(n);
    if (s != slice_of.end()) return root(s->second.first);
    auto a = alias_of.find(n);
    if (a != alias_of.end()) return root(a->second);
    return n;
  };
  std::map<std::string, int> first, last;
  for (size_t i = 0; i < topo_sorted_layers_.size(); ++i) {
    const int ii = static_cast<int>(i);
    for (auto& o : topo_sorted_layers_[i]->outputs_name_) {
      const std::string r = root(o);
      if (!first.count(r)) first[r] = ii;
      last[r] = std::max(last.count(r) ? last[r] : ii, ii);
    }
    for (auto& in : topo_sorted_layers_[i]->inputs_name_) {
      const std::string r = root(in);
      last[r] = std::max(last.count(r) ? last[r] : ii, ii);
    }
  }
  std::vector<std::string> roots;
  for (auto& kv : operands_)
    if (!slice_of.count(kv.first) && !alias_of.count(kv.first)) roots.push_back(kv.first);
  std::stable_sort(roots.begin(), roots.end(), [&](const std::string& x, const std::string& y) {
    const int fx = first.count(x) ? first.at(x) : -1, fy = first.count(y) ? first.at(y) : -1;
    return fx < fy;
  });
  struct Block {
    std::shared_ptr<void> mem;
    size_t bytes;
    int free_after;
  };
  std::vector<Block> blocks;
  auto alloc = [](size_t bytes) {
    void* p = nullptr;
    CudaCheck(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc(activations)");
    return std::shared_ptr<void>(p, [](void* q) { cudaFree(q); });
  };
  activation_bytes_ = 0;
  for (auto& r : roots) {
    Tensor& t = operands_.at(r)->tensor_;
    const size_t need = (t.Bytes() + 255) / 256 * 256;
    const bool dedicated = r == input_operand_ || r == output_operand_ || !first.count(r);
    if (!opt_.plan_memory || dedicated) {
      t.BindStorage(alloc(need), 0);
      activation_bytes_ += need;
      continue;
    }
    Block* best = nullptr;
    for (auto& b : blocks)
      if (b.free_after < first.at(r) && b.bytes >= need && (!best || b.bytes < best->bytes)) best = &b;
    if (!best) {
      blocks.push_back(Block{alloc(need), need, -1});
      activation_bytes_ += need;
      best = &blocks.back();
    }
    best->free_after = last.at(r);
    t.BindStorage(best->mem, 0);
  }
  // channel slices, parents first (a slice's parent is a root or a slice)
  std::function<void(const std::string&)> bind_slice = [&](const std::string& n) {
    const auto& sv = slice_of.at(n);
    if (slice_of.count(sv.first)) bind_slice(sv.first);
    Tensor& t = operands_.at(n)->tensor_;
    t = operands_.at(sv.first)->tensor_.ChannelSlice(sv.second, t.Dim(1));
  };
  for (auto& kv : slice_of) bind_slice(kv.first);
}

void Graph::TopoSortLayers() {
  // Kahn's algorithm over operand dependencies (source/graph.cpp:5-40);
  // ties keep the file order so the schedule is deterministic.
  std::map<std::string, std::string> producer;
  for (auto& kv : layers_)
    for (auto& o : kv.second->outputs_name_) producer[o] = kv.first;
  std::map<std::string, int> indeg;
  std::map<std::string, std::vector<std::string>> succ;
  for (auto& kv : layers_) {
    int d = 0;
    for (auto& in : kv.second->inputs_name_) {
      auto it = producer.find(in);
      if (it != producer.end()) {
        ++d;
        succ[it->second].push_back(kv.first);
      }
    }
    indeg[kv.first] = d;
  }
  std::map<std::string, size_t> rank;
  for (size_t i = 0; i < layer_order_.size(); ++i) rank[layer_order_[i]] = i;
  auto cmp = [&](const std::string& a, const std::string& b) { return rank.at(a) > rank.at(b); };
  std::priority_queue<std::string, std::vector<std::string>, decltype(cmp)> ready(cmp);
  for (auto& kv : indeg)
    if (kv.second == 0) ready.push(kv.first);
  topo_sorted_layers_.clear();
  while (!ready.empty()) {
    const std::string n = ready.top();
    ready.pop();
    topo_sorted_layers_.push_back(layers_.at(n));
    for (auto& s : succ[n])
      if (--indeg[s] == 0) ready.push(s);
  }
  if (topo_sorted_layers_.size() != layers_.size()) throw std::runtime_error("the graph is not acyclic");
}

void Graph::InitialiseInput(const std::vector<float>& input) { InputTensor().AssignData(input); }

std::shared_ptr<Operand> Graph::Output() { return operands_.at(output_operand_); }

void Graph::RunLayers(cudaStream_t s) {
  for (auto& l : topo_sorted_layers_) l->Forward(s);
}

void Graph::ForwardAsync(cudaStream_t stream) {
  cudaStream_t s = stream ? stream : stream_;
  CudaCheck(cudaSetDevice(device_), "cudaSetDevice");
  if (!opt_.cuda_graph || eager_runs_ == 0) {
    RunLayers(s);
    ++eager_runs_;
    return;
  }
  if (!exec_) {
    cudaGraph_t graph = nullptr;
    CudaCheck(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
      RunLayers(s);
    } catch (...) {
      cudaStreamEndCapture(s, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    CudaCheck(cudaStreamEndCapture(s, &graph), "end capture");
    cudaError_t e = cudaGraphInstantiate(&exec_, graph, 0);
    cudaGraphDestroy(graph);
    CudaCheck(e, "graph instantiate");
  }
  CudaCheck(cudaGraphLaunch(exec_, s), "graph launch");
}

void Graph::Forward() {
  ForwardAsync(stream_);
  Synchronize();
}

void Graph::Synchronize() {
  CudaCheck(cudaSetDevice(device_), "cudaSetDevice");
  if (pipe_) {
    CudaCheck(cudaStreamSynchronize(pipe_->h2d), "graph synchronize (input copies)");
    CudaCheck(cudaStreamSynchronize(pipe_->h2d_b), "graph synchronize (input copies)");
  }
  CudaCheck(cudaStreamSynchronize(stream_), "graph synchronize");
  if (pipe_) CudaCheck(cudaStreamSynchronize(pipe_->d2h), "graph synchronize (output copies)");
  // a kernel whose bounded wait ran out skipped its output tiles: report it
  // instead of handing back wrong results as a success
  const int dev_err = lotus_impl::read_device_error();
  if (dev_err != 0)
    throw std::runtime_error("a kernel's bounded wait expired (device error code " + std::to_string(dev_err) +
                             "); the outputs of this forward are invalid");
}

void Graph::SetupPipe() {
  auto p = std::make_unique<Pipe>();
  auto in_op = operands_.at(input_operand_);
  auto out_op = operands_.at(output_operand_);
  p->in[0] = in_op->tensor_;
  p->out[0] = out_op->tensor_;
  p->in[1] = Tensor(p->in[0].Shape(), p->in[0].Fmt());
  p->out[1] = Tensor(p->out[0].Shape(), p->out[0].Fmt());
  CudaCheck(cudaStreamCreateWithFlags(&p->h2d, cudaStreamNonBlocking), "cudaStreamCreate");
  CudaCheck(cudaStreamCreateWithFlags(&p->d2h, cudaStreamNonBlocking), "cudaStreamCreate");
  CudaCheck(cudaStreamCreateWithFlags(&p->h2d_b, cudaStreamNonBlocking), "cudaStreamCreate");
  for (int k = 0; k < 2; ++k)
    for (cudaEvent_t* e : {&p->h2d_done[k], &p->h2d_b_done[k], &p->fwd_done[k], &p->d2h_done[k]})
      CudaCheck(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "cudaEventCreate");
  // kernels set their launch attributes on their first (eager) launch, which
  // must not happen inside a capture
  if (eager_runs_ == 0) {
    RunLayers(stream_);
    ++eager_runs_;
  }
  // one captured forward per slot, with the input and output operands bound
  // to that slot's buffers
  for (int k = 0; k < 2; ++k) {
    in_op->tensor_ = p->in[k];
    out_op->tensor_ = p->out[k];
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
      try {
        RunLayers(stream_);
      } catch (...) {
        cudaStreamEndCapture(stream_, &graph);
        if (graph) cudaGraphDestroy(graph);
        in_op->tensor_ = p->in[0];
        out_op->tensor_ = p->out[0];
        throw;
      }
      e = cudaStreamEndCapture(stream_, &graph);
    }
    if (e == cudaSuccess) e = cudaGraphInstantiate(&p->exec[k], graph, 0);
    if (graph) cudaGraphDestroy(graph);
    in_op->tensor_ = p->in[0];
    out_op->tensor_ = p->out[0];
    CudaCheck(e, "pipeline graph capture");
  }
  pipe_ = std::move(p);
}

int Graph::Submit(const float* host_in, float* host_out) {
  CudaCheck(cudaSetDevice(device_), "cudaSetDevice");
  if (!pipe_) SetupPipe();
  Pipe& p = *pipe_;
  const int k = static_cast<int>(p.submitted & 1);
  const bool reuse = p.submitted >= 2;  // slot k was used by submission n-2
  // input copy, once the forward that last read this slot's input is done;
  // its two halves go on two streams so that two copy engines move them
  if (reuse) {
    CudaCheck(cudaStreamWaitEvent(p.h2d, p.fwd_done[k], 0), "wait");
    CudaCheck(cudaStreamWaitEvent(p.h2d_b, p.fwd_done[k], 0), "wait");
  }
  const size_t bytes = p.in[k].Bytes();
  const size_t half = (bytes / 2 + 4095) / 4096 * 4096;
  char* dst = static_cast<char*>(p.in[k].Data());
  const char* src = reinterpret_cast<const char*>(host_in);
  CudaCheck(cudaMemcpyAsync(dst, src, std::min(half, bytes), cudaMemcpyDefault, p.h2d), "input copy");
  if (bytes > half)
    CudaCheck(cudaMemcpyAsync(dst + half, src + half, bytes - half, cudaMemcpyDefault, p.h2d_b), "input copy");
  CudaCheck(cudaEventRecord(p.h2d_done[k], p.h2d), "record");
  CudaCheck(cudaEventRecord(p.h2d_b_done[k], p.h2d_b), "record");
  // forward, once its input landed and the output copy that last read this
  // slot's output is done
  CudaCheck(cudaStreamWaitEvent(stream_, p.h2d_done[k], 0), "wait");
  CudaCheck(cudaStreamWaitEvent(stream_, p.h2d_b_done[k], 0), "wait");
  if (reuse) CudaCheck(cudaStreamWaitEvent(stream_, p.d2h_done[k], 0), "wait");
  CudaCheck(cudaGraphLaunch(p.exec[k], stream_), "graph launch");
  CudaCheck(cudaEventRecord(p.fwd_done[k], stream_), "record");
  // output copy
  CudaCheck(cudaStreamWaitEvent(p.d2h, p.fwd_done[k], 0), "wait");
  CudaCheck(cudaMemcpyAsync(host_out, p.out[k].Data(), p.out[k].Bytes(), cudaMemcpyDefault, p.d2h), "output copy");
  CudaCheck(cudaEventRecord(p.d2h_done[k], p.d2h), "record");
  ++p.submitted;
  return k;
}

cudaStream_t Graph::CopyStream(int which) {
  CudaCheck(cudaSetDevice(device_), "cudaSetDevice");
  if (!pipe_) SetupPipe();
  return which == 0 ? pipe_->h2d : pipe_->d2h;
}

float* Graph::SlotOutput(int slot) {
  if (slot == 0 || !pipe_) return OutputTensor().DataF32();
  return pipe_->out[1].DataF32();
}

std::vector<float> Graph::ProfileLayers(int reps) {
  CudaCheck(cudaSetDevice(device_), "cudaSetDevice");
  const size_t n = topo_sorted_layers_.size();
  std::vector<cudaEvent_t> ev(n + 1);
  for (auto& e : ev) CudaCheck(cudaEventCreate(&e), "event");
  std::vector<double> acc(n, 0.0);
  for (int r = 0; r < reps; ++r) {
    CudaCheck(cudaEventRecord(ev[0], stream_), "record");
    for (size_t i = 0; i < n; ++i) {
      topo_sorted_layers_[i]->Forward(stream_);
      CudaCheck(cudaEventRecord(ev[i + 1], stream_), "record");
    }
    CudaCheck(cudaEventSynchronize(ev[n]), "sync");
    for (size_t i = 0; i < n; ++i) {
      float ms = 0.f;
      CudaCheck(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]), "elapsed");
      acc[i] += ms;
    }
  }
  for (auto& e : ev) cudaEventDestroy(e);
  std::vector<float> out(n);
  for (size_t i = 0; i < n; ++i) out[i] = static_cast<float>(acc[i] / std::max(reps, 1));
  return out;
}

int Graph::LaunchesPerForward() const {
  int n = 0;
  for (auto& l : topo_sorted_layers_) n += l->Launches();
  return n;
}

}  // namespace lotus
