// C ABI of the graph runtime (include/lotus_graph.h).
#include <cstring>
#include <exception>
#include <string>

#include "../../../include/lotus_graph.h"
#include "graph.hpp"

namespace lotus_impl {
int set_error(int code, const std::string& msg);  // abi.cu
}

struct lotus_graph {
  std::unique_ptr<lotus::Graph> g;
};

namespace {

int fill_shape(const lotus::Tensor& t, int64_t* dims, int* ndim) {
  if (!dims || !ndim) return lotus_impl::set_error(LOTUS_ERR_INVALID, "graph shape: null pointer");
  const auto& s = t.Shape();
  if (s.size() > 8) return lotus_impl::set_error(LOTUS_ERR_UNSUPPORTED, "graph shape: rank > 8");
  for (size_t i = 0; i < s.size(); ++i) dims[i] = s[i];
  *ndim = static_cast<int>(s.size());
  return lotus_impl::set_error(LOTUS_OK, "");
}

}  // namespace

extern "C" {

lotus_graph* lotus_graph_create(const char* param_path, const char* bin_path, int batch, int device, int flags) {
  if (!param_path || !bin_path || batch <= 0) {
    lotus_impl::set_error(LOTUS_ERR_INVALID, "graph_create: need param/bin paths and a positive batch");
    return nullptr;
  }
  try {
    lotus::Graph::Options o;
    o.device = device;
    o.cuda_graph = (flags & LOTUS_GRAPH_NO_CUDA_GRAPH) == 0;
    o.fuse_residual = (flags & LOTUS_GRAPH_NO_RESIDUAL_FUSION) == 0;
    o.s2d_stem = (flags & LOTUS_GRAPH_NO_S2D_STEM) == 0;
    o.fuse_pool = (flags & LOTUS_GRAPH_NO_POOL_FUSION) == 0;
    o.fuse_concat = (flags & LOTUS_GRAPH_NO_CONCAT_FUSION) == 0;
    o.plan_memory = (flags & LOTUS_GRAPH_NO_MEMORY_PLAN) == 0;
    std::unique_ptr<lotus::Graph> graph(new lotus::Graph(param_path, bin_path, static_cast<uint32_t>(batch), o));
    auto* h = new lotus_graph;
    h->g = std::move(graph);
    lotus_impl::set_error(LOTUS_OK, "");
    return h;
  } catch (const std::exception& e) {
    lotus_impl::set_error(LOTUS_ERR_INVALID, std::string("graph_create: ") + e.what());
    return nullptr;
  }
}

void lotus_graph_destroy(lotus_graph* g) { delete g; }

int lotus_graph_input_shape(const lotus_graph* g, int64_t* dims, int* ndim) {
  if (!g) return lotus_impl::set_error(LOTUS_ERR_INVALID, "null graph");
  return fill_shape(const_cast<lotus::Graph&>(*g->g).InputTensor(), dims, ndim);
}

int lotus_graph_output_shape(const lotus_graph* g, int64_t* dims, int* ndim) {
  if (!g) return lotus_impl::set_error(LOTUS_ERR_INVALID, "null graph");
  return fill_shape(const_cast<lotus::Graph&>(*g->g).OutputTensor(), dims, ndim);
}

float* lotus_graph_input_ptr(lotus_graph* g) { return g ? g->g->InputTensor().DataF32() : nullptr; }
const float* lotus_graph_output_ptr(lotus_graph* g) { return g ? g->g->OutputTensor().DataF32() : nullptr; }
cudaStream_t lotus_graph_stream(const lotus_graph* g) { return g ? g->g->Stream() : nullptr; }

int lotus_graph_set_input(lotus_graph* g, const float* host, size_t count, cudaStream_t stream) {
  if (!g || !host) return lotus_impl::set_error(LOTUS_ERR_INVALID, "graph_set_input: null pointer");
  auto& t = g->g->InputTensor();
  if (count != t.Size()) return lotus_impl::set_error(LOTUS_ERR_INVALID, "graph_set_input: wrong element count");
  const cudaError_t e =
      cudaMemcpyAsync(t.Data(), host, count * 4, cudaMemcpyDefault, stream ? stream : g->g->Stream());
  if (e != cudaSuccess) return lotus_impl::set_error(LOTUS_ERR_CUDA, cudaGetErrorString(e));
  return lotus_impl::set_error(LOTUS_OK, "");
}

int lotus_graph_get_output(lotus_graph* g, float* host, size_t count, cudaStream_t stream) {
  if (!g || !host) return lotus_impl::set_error(LOTUS_ERR_INVALID, "graph_get_output: null pointer");
  auto& t = g->g->OutputTensor();
  if (count != t.Size()) return lotus_impl::set_error(LOTUS_ERR_INVALID, "graph_get_output: wrong element count");
  const cudaError_t e =
      cudaMemcpyAsync(host, t.Data(), count * 4, cudaMemcpyDefault, stream ? stream : g->g->Stream());
  if (e != cudaSuccess) return lotus_impl::set_error(LOTUS_ERR_CUDA, cudaGetErrorString(e));
  return lotus_impl::set_error(LOTUS_OK, "");
}

int lotus_graph_forward(lotus_graph* g, cudaStream_t stream) {
  if (!g) return lotus_impl::set_error(LOTUS_ERR_INVALID, "null graph");
  try {
    g->g->ForwardAsync(stream);
  } catch (const std::exception& e) {
    return lotus_impl::set_error(LOTUS_ERR_CUDA, std::string("graph_forward: ") + e.what());
  }
  return lotus_impl::set_error(LOTUS_OK, "");
}

int lotus_graph_forward_sync(lotus_graph* g) {
  if (!g) return lotus_impl::set_error(LOTUS_ERR_INVALID, "null graph");
  try {
    g->g->Forward();
  } catch (const std::exception& e) {
    return lotus_impl::set_error(LOTUS_ERR_CUDA, std::string("graph_forward_sync: ") + e.what());
  }
  return lotus_impl::set_error(LOTUS_OK, "");
}

int lotus_graph_synchronize(lotus_graph* g) {
  if (!g) return lotus_impl::set_error(LOTUS_ERR_INVALID, "null graph");
  try {
    g->g->Synchronize();
  } catch (const std::exception& e) {
    return lotus_impl::set_error(LOTUS_ERR_CUDA, std::string("graph_synchronize: ") + e.what());
  }
  return lotus_impl::set_error(LOTUS_OK, "");
}

int lotus_graph_submit(lotus_graph* g, const float* host_in, float* host_out, int* slot) {
  if (!g || !host_in || !host_out) return lotus_impl::set_error(LOTUS_ERR_INVALID, "graph_submit: null pointer");
  try {
    const int k = g->g->Submit(host_in, host_out);
    if (slot) *slot = k;
  } catch (const std::exception& e) {
    return lotus_impl::set_error(LOTUS_ERR_CUDA, std::string("graph_submit: ") + e.what());
  }
  return lotus_impl::set_error(LOTUS_OK, "");
}

cudaStream_t lotus_graph_copy_stream(lotus_graph* g, int which) {
  if (!g || (which != 0 && which != 1)) return nullptr;
  try {
    return g->g->CopyStream(which);
  } catch (const std::exception& e) {
    lotus_impl::set_error(LOTUS_ERR_CUDA, std::string("graph_copy_stream: ") + e.what());
    return nullptr;
  }
}

float* lotus_graph_slot_output(lotus_graph* g, int slot) {
  if (!g || (slot != 0 && slot != 1)) return nullptr;
  return g->g->SlotOutput(slot);
}

int lotus_graph_layer_count(const lotus_graph* g) { return g ? static_cast<int>(g->g->Layers().size()) : -1; }

const char* lotus_graph_layer_name(const lotus_graph* g, int i) {
  if (!g || i < 0 || i >= static_cast<int>(g->g->Layers().size())) return nullptr;
  return g->g->Layers()[i]->Name().c_str();
}

const char* lotus_graph_layer_type(const lotus_graph* g, int i) {
  if (!g || i < 0 || i >= static_cast<int>(g->g->Layers().size())) return nullptr;
  return g->g->Layers()[i]->Type().c_str();
}

double lotus_graph_layer_flops(const lotus_graph* g, int i) {
  if (!g || i < 0 || i >= static_cast<int>(g->g->Layers().size())) return -1.0;
  return g->g->Layers()[i]->Flops();
}

double lotus_graph_layer_bytes(const lotus_graph* g, int i) {
  if (!g || i < 0 || i >= static_cast<int>(g->g->Layers().size())) return -1.0;
  return g->g->Layers()[i]->Bytes();
}

const void* lotus_graph_operand(const lotus_graph* g, const char* name, int* format, int64_t* dims, int* ndim) {
  if (!g || !name) return nullptr;
  auto o = g->g->FindOperand(name);
  if (!o || o->tensor_.Empty()) return nullptr;
  if (format) *format = o->tensor_.Fmt() == lotus::Format::kNHWC_F16 ? 1 : 0;
  if (dims && ndim) fill_shape(o->tensor_, dims, ndim);
  return o->tensor_.Data();
}

const void* lotus_graph_layer_weight(const lotus_graph* g, int i, size_t* bytes) {
  if (!g || i < 0 || i >= static_cast<int>(g->g->Layers().size())) return nullptr;
  return g->g->Layers()[i]->Weight(bytes);
}

int lotus_graph_launches_per_forward(const lotus_graph* g) { return g ? g->g->LaunchesPerForward() : -1; }

size_t lotus_graph_activation_bytes(const lotus_graph* g) { return g ? g->g->ActivationBytes() : 0; }

int lotus_graph_profile_layers(lotus_graph* g, int reps, float* ms) {
  if (!g || !ms || reps <= 0) return lotus_impl::set_error(LOTUS_ERR_INVALID, "graph_profile_layers: bad arguments");
  try {
    const auto v = g->g->ProfileLayers(reps);
    std::memcpy(ms, v.data(), v.size() * sizeof(float));
  } catch (const std::exception& e) {
    return lotus_impl::set_error(LOTUS_ERR_CUDA, std::string("graph_profile_layers: ") + e.what());
  }
  return lotus_impl::set_error(LOTUS_OK, "");
}

}  // extern "C"
