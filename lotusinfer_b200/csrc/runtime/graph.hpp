// lotus::Graph - loads a PNNX model and runs it on one GPU.
//
// Keeps the reference's public surface (include/graph.hpp:15-43:
// Graph(param, bin, batch), InitialiseInput, Forward, Output) and its build
// steps (source/graph.cpp:44-111: one operand per PNNX operand with dim 0 set
// to the batch, one layer per operator with ReLU/sigmoid folded into the
// producer, Kahn topological order).  Additions:
//   - residual fusion: `pnnx.Expression add` (+ReLU) whose operand is the
//     sole output of a Conv2d becomes that conv's residual epilogue;
//   - activations are NHWC fp16 between layers, converted once at the graph
//     input and output;
//   - Forward runs on one persistent stream with no per-layer sync, and is
//     captured into a CUDA graph after its first (eager) run.
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "layers.hpp"

namespace lotus {

class Graph {
 public:
  struct Options {
    int device = -1;             // -1: the current device
    bool cuda_graph = true;      // replay Forward from a CUDA graph after the first run
    bool fuse_residual = true;   // fold conv -> add (-> ReLU) into the conv epilogue
    bool s2d_stem = true;        // run a strided few-channel stem conv over the space-to-depth input
    bool fuse_pool = true;       // fold a 3x3/2 max pool into the conv that feeds it, where the fused kernel applies
    bool fuse_concat = true;     // producers of a torch.cat write their channel slice of it in place
    bool plan_memory = true;     // operands whose lifetimes do not overlap share device memory
  };

  Graph(const std::string& param_path, const std::string& bin_path, uint32_t batch_size);
  Graph(const std::string& param_path, const std::string& bin_path, uint32_t batch_size, const Options& opt);
  ~Graph();
  Graph(const Graph&) = delete;
  Graph& operator=(const Graph&) = delete;

  // Reference API: synchronous H2D of the NCHW fp32 input batch.
  void InitialiseInput(const std::vector<float>& input);
  std::shared_ptr<Operand> Output();
  // Reference API: runs every layer and waits for the result.
  void Forward();
  // Enqueues the forward pass on `stream` (nullptr = the graph's own stream).
  void ForwardAsync(cudaStream_t stream = nullptr);
  // Waits for the graph stream and the pipeline's copy streams; throws if a
  // kernel reported an expired bounded wait (its outputs are then invalid).
  void Synchronize();
  // Pipelined inference from host memory: host->device copy of `host_in` on a
  // copy stream, the forward on the graph stream once it landed, and the
  // device->host copy of the output into `host_out` on a second copy stream.
  // Two sets of device input/output buffers alternate, so the copies of one
  // batch overlap the forward of the previous one.  Returns the slot (0/1)
  // this batch used; does not wait.
  int Submit(const float* host_in, float* host_out);
  // Copy stream of the pipelined path: 0 host->device, 1 device->host.
  cudaStream_t CopyStream(int which);
  // Device output buffer of pipeline slot 0/1 (slot 0 is the graph's output).
  float* SlotOutput(int slot);

  Tensor& InputTensor() { return operands_.at(input_operand_)->tensor_; }
  Tensor& OutputTensor() { return operands_.at(output_operand_)->tensor_; }
  const std::vector<std::shared_ptr<Layer>>& Layers() const { return topo_sorted_layers_; }
  cudaStream_t Stream() const { return stream_; }
  int Device() const { return device_; }
  uint32_t Batch() const { return batch_; }
  // Mean device milliseconds of each layer over `reps` eager runs.
  std::vector<float> ProfileLayers(int reps);
  // Operand by name (nullptr if absent).
  std::shared_ptr<Operand> FindOperand(const std::string& name) const {
    auto it = operands_.find(name);
    return it == operands_.end() ? nullptr : it->second;
  }
  // Library kernel launches per Forward.
  int LaunchesPerForward() const;
  // Device bytes held by the operands (activations, graph input and output).
  size_t ActivationBytes() const { return activation_bytes_; }

 private:
  void Build(const std::string& param_path, const std::string& bin_path);
  void TopoSortLayers();
  std::shared_ptr<Layer> ProducerOf(const std::string& operand) const;
  void FuseConcats(std::map<std::string, std::pair<std::string, uint32_t>>* slice_of);
  void PlanMemory(const std::map<std::string, std::pair<std::string, uint32_t>>& slice_of);
  void RunLayers(cudaStream_t s);

  std::map<std::string, std::shared_ptr<Layer>> layers_;
  OperandMap operands_;
  std::vector<std::shared_ptr<Layer>> topo_sorted_layers_;
  std::vector<std::string> layer_order_;  // file order, for deterministic ties
  std::string input_operand_, output_operand_;
  uint32_t batch_;
  Options opt_;
  int device_ = 0;
  cudaStream_t stream_ = nullptr;
  cudaGraphExec_t exec_ = nullptr;
  int eager_runs_ = 0;
  // space-to-depth stem rewrite (factor 1 = none)
  int stem_s2d_ = 1, stem_pad_h_ = 0, stem_pad_w_ = 0;
  std::vector<uint32_t> stem_shape_;
  std::shared_ptr<void> workspace_;  // split-K scratch shared by the layers (one stream, one layer at a time)
  size_t activation_bytes_ = 0;

  // pipelined path (Submit): slot 1's buffers, one captured forward per slot,
  // the copy streams and the events that order them
  struct Pipe {
    Tensor in[2], out[2];
    cudaGraphExec_t exec[2] = {nullptr, nullptr};
    cudaStream_t h2d = nullptr, d2h = nullptr;
    cudaStream_t h2d_b = nullptr;  // second input-copy stream: each input copy is split over two copy engines
    cudaEvent_t h2d_done[2] = {}, h2d_b_done[2] = {}, fwd_done[2] = {}, d2h_done[2] = {};
    uint64_t submitted = 0;
  };
  void SetupPipe();
  std::unique_ptr<Pipe> pipe_;
};

}  // namespace lotus
