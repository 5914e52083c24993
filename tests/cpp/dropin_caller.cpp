// A C++ caller of liblotus_b200.so that binds the operators the way a
// maintainer would inside the reference's own layer classes: the layer keeps
// the reference's NCHW fp32 device tensors at its boundary (reference
// include/tensor.hpp:13-40, source/layer/layer_conv2d.cu:37-73) and converts
// to and from the library's NHWC fp16 activations around lotus_conv2d_fwd.
//
//   dropin_caller conv  <in.bin> <out.bin>   one Conv2dLayer forward
//   dropin_caller graph <param> <bin> <batch> <in.bin> <out.bin>
//                                            lotus_graph_* whole-model forward
//
// conv in.bin: int32 n, c, h, w, cout, k, stride, pad, act; then fp32 x
// [n,c,h,w], weight [cout,c,k,k], bias [cout].  out.bin: fp32 y [n,cout,oh,ow].
// graph in.bin: fp32 input [batch, ...]; out.bin: fp32 output.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "lotus_graph.h"
#include "lotus_ops.h"

#define CHECK_LOTUS(call)                                                                      \
  do {                                                                                         \
    if ((call) != LOTUS_OK) throw std::runtime_error(std::string(#call) + ": " + lotus_last_error_string()); \
  } while (0)
#define CHECK_CUDA(call)                                                                       \
  do {                                                                                         \
    cudaError_t e_ = (call);                                                                   \
    if (e_ != cudaSuccess) throw std::runtime_error(std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

// Device buffer owned like the reference Tensor's storage.
struct DeviceBuffer {
  void* p = nullptr;
  explicit DeviceBuffer(size_t bytes) { CHECK_CUDA(cudaMalloc(&p, bytes ? bytes : 16)); }
  ~DeviceBuffer() { cudaFree(p); }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
};

// The reference's Conv2dLayer with its per-sample Conv2d launches replaced by
// one lotus_conv2d_fwd per batch.  Input and output are NCHW fp32 device
// tensors, as everywhere in the reference.
class Conv2dLayer {
 public:
  Conv2dLayer(const std::vector<float>& weight_oihw, const std::vector<float>& bias, int c_in, int c_out, int k,
              int stride, int pad, int act, cudaStream_t stream)
      : stream_(stream) {
    d_ = lotus_conv2d_desc{1, c_in, k, k, c_out, k, k, stride, stride, pad, pad, act, LOTUS_OUT_NHWC_F16};
    DeviceBuffer w32(weight_oihw.size() * 4);
    CHECK_CUDA(cudaMemcpyAsync(w32.p, weight_oihw.data(), weight_oihw.size() * 4, cudaMemcpyHostToDevice, stream));
    packed_ = new DeviceBuffer(lotus_conv2d_packed_weight_bytes(&d_));
    CHECK_LOTUS(lotus_conv2d_prepack(static_cast<const float*>(w32.p), packed_->p, &d_, stream));
    bias_ = new DeviceBuffer(bias.size() * 4);
    CHECK_CUDA(cudaMemcpyAsync(bias_->p, bias.data(), bias.size() * 4, cudaMemcpyHostToDevice, stream));
    CHECK_CUDA(cudaStreamSynchronize(stream));  // w32 is freed on return
  }
  ~Conv2dLayer() {
    delete packed_;
    delete bias_;
    delete x16_;
    delete y16_;
  }

  // x: NCHW fp32 [n, c_in, h, w] -> y: NCHW fp32 [n, c_out, oh, ow]
  void Forward(const float* x, float* y, int n, int h, int w) {
    d_.n = n;
    d_.h = h;
    d_.w = w;
    int oh = 0, ow = 0;
    CHECK_LOTUS(lotus_conv2d_out_hw(&d_, &oh, &ow));
    const size_t x16_bytes = static_cast<size_t>(n) * h * w * lotus_channel_stride(d_.c_in) * 2;
    const size_t y16_bytes = static_cast<size_t>(n) * oh * ow * lotus_channel_stride(d_.c_out) * 2;
    if (!x16_ || x16_cap_ < x16_bytes) {
      delete x16_;
      x16_ = new DeviceBuffer(x16_bytes);
      x16_cap_ = x16_bytes;
    }
    if (!y16_ || y16_cap_ < y16_bytes) {
      delete y16_;
      y16_ = new DeviceBuffer(y16_bytes);
      y16_cap_ = y16_bytes;
    }
    CHECK_LOTUS(lotus_nchw_f32_to_nhwc_f16(x, x16_->p, n, d_.c_in, h, w, stream_));
    CHECK_LOTUS(lotus_conv2d_fwd(x16_->p, packed_->p, static_cast<const float*>(bias_->p), nullptr, y16_->p, &d_,
                                 stream_));
    CHECK_LOTUS(lotus_nhwc_f16_to_nchw_f32(y16_->p, y, n, d_.c_out, oh, ow, stream_));
  }

 private:
  lotus_conv2d_desc d_{};
  cudaStream_t stream_;
  DeviceBuffer* packed_ = nullptr;
  DeviceBuffer* bias_ = nullptr;
  DeviceBuffer* x16_ = nullptr;
  DeviceBuffer* y16_ = nullptr;
  size_t x16_cap_ = 0, y16_cap_ = 0;
};

static std::vector<char> read_file(const char* path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error(std::string("cannot open ") + path);
  return std::vector<char>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

static void write_file(const char* path, const void* data, size_t bytes) {
  std::ofstream f(path, std::ios::binary);
  f.write(static_cast<const char*>(data), static_cast<std::streamsize>(bytes));
  if (!f) throw std::runtime_error(std::string("cannot write ") + path);
}

static int run_conv(const char* in_path, const char* out_path) {
  const std::vector<char> raw = read_file(in_path);
  const int* hdr = reinterpret_cast<const int*>(raw.data());
  const int n = hdr[0], c = hdr[1], h = hdr[2], w = hdr[3], cout = hdr[4], k = hdr[5], s = hdr[6], p = hdr[7],
            act = hdr[8];
  const float* f = reinterpret_cast<const float*>(raw.data() + 9 * sizeof(int));
  const size_t nx = static_cast<size_t>(n) * c * h * w, nw = static_cast<size_t>(cout) * c * k * k;
  std::vector<float> x(f, f + nx), wt(f + nx, f + nx + nw), b(f + nx + nw, f + nx + nw + cout);
  cudaStream_t stream;
  CHECK_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  Conv2dLayer layer(wt, b, c, cout, k, s, p, act, stream);
  const int oh = (h + 2 * p - k) / s + 1, ow = (w + 2 * p - k) / s + 1;
  const size_t ny = static_cast<size_t>(n) * cout * oh * ow;
  DeviceBuffer xd(nx * 4), yd(ny * 4);
  CHECK_CUDA(cudaMemcpyAsync(xd.p, x.data(), nx * 4, cudaMemcpyHostToDevice, stream));
  layer.Forward(static_cast<const float*>(xd.p), static_cast<float*>(yd.p), n, h, w);
  std::vector<float> y(ny);
  CHECK_CUDA(cudaMemcpyAsync(y.data(), yd.p, ny * 4, cudaMemcpyDeviceToHost, stream));
  CHECK_CUDA(cudaStreamSynchronize(stream));
  if (lotus_device_error() != 0) throw std::runtime_error("device error word set");
  write_file(out_path, y.data(), ny * 4);
  CHECK_CUDA(cudaStreamDestroy(stream));
  return 0;
}

static int run_graph(const char* param, const char* bin, int batch, const char* in_path, const char* out_path) {
  lotus_graph* g = lotus_graph_create(param, bin, batch, 0, 0);
  if (!g) throw std::runtime_error(std::string("lotus_graph_create: ") + lotus_last_error_string());
  int64_t in_dims[8], out_dims[8];
  int in_nd = 0, out_nd = 0;
  CHECK_LOTUS(lotus_graph_input_shape(g, in_dims, &in_nd));
  CHECK_LOTUS(lotus_graph_output_shape(g, out_dims, &out_nd));
  size_t n_in = 1, n_out = 1;
  for (int i = 0; i < in_nd; ++i) n_in *= static_cast<size_t>(in_dims[i]);
  for (int i = 0; i < out_nd; ++i) n_out *= static_cast<size_t>(out_dims[i]);
  const std::vector<char> raw = read_file(in_path);
  if (raw.size() != n_in * 4) throw std::runtime_error("input file size does not match the graph input");
  std::vector<float> out(n_out);
  // the reference's InitialiseInput / Forward / Output sequence (source/graph.cpp:114-130)
  CHECK_LOTUS(lotus_graph_set_input(g, reinterpret_cast<const float*>(raw.data()), n_in, nullptr));
  CHECK_LOTUS(lotus_graph_forward_sync(g));
  CHECK_LOTUS(lotus_graph_get_output(g, out.data(), n_out, nullptr));
  CHECK_LOTUS(lotus_graph_synchronize(g));
  write_file(out_path, out.data(), n_out * 4);
  lotus_graph_destroy(g);
  return 0;
}

int main(int argc, char** argv) {
  try {
    const std::string mode = argc > 1 ? argv[1] : "";
    if (mode == "conv" && argc == 4) return run_conv(argv[2], argv[3]);
    if (mode == "graph" && argc == 7) return run_graph(argv[2], argv[3], std::atoi(argv[4]), argv[5], argv[6]);
    std::fprintf(stderr, "usage: %s conv <in> <out> | graph <param> <bin> <batch> <in> <out>\n", argv[0]);
    return 2;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "dropin_caller: %s\n", e.what());
    return 1;
  }
}
