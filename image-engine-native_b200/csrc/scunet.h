// SCUNet (denoising) on the CUDA backend.
//
// Replaces crates/scunet-native/src/gpu.rs (the Vulkan network) behind the
// model's public API (lib.rs): the U-Net of network.rs on the general
// tcgen05 implicit GEMM (1x1 convolutions, linear layers, the blocks' 3x3
// convolutions, 2x2 stride-2 halving and transposed doubling) with layer
// norm + shifted-window partition as one bandwidth kernel and the fused
// window attention (attention.cu). Residual adds, GELU/ReLU, the window
// reverse and the transposed-conv scatter are fused into GEMM epilogues.
#pragma once

#include <cuda_fp16.h>

#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "gemm.h"
#include "runtime.h"

namespace iec {

class Scunet {
 public:
  static constexpr int DIM = 64, BLOCKS = 4, STEPS = 7 * BLOCKS, MULTIPLE = 64, TILE = 896, MARGIN = 64;

  Scunet(const std::string& path, const Options& opt);
  ~Scunet();
  Device& device() { return dev_; }

  // network.rs:265-353 on device buffers: `src` one width x height x 3 image
  // (f32 or u8), `dst` its denoised copy (f32 or u8); `step` after each of
  // the 28 blocks (false cancels). The region [rx0, rx0 + rw) x [ry0, ry0 +
  // rh) of `src` is the network's input; the window [kx0, kx1) x [ky0, ky1)
  // of its output (region coordinates) goes to the same place of `dst`.
  bool run_region(const void* src, bool src_u8, void* dst, bool dst_u8, int src_w, int src_h, int rx0, int ry0,
                  int rw, int rh, int kx0, int ky0, int kx1, int ky1, const std::function<bool()>& step,
                  cudaStream_t s);
  // run_region over a whole f32 image on device buffers, replayed as a graph
  // while the buffers and size repeat (PassGraph).
  void run_whole_device(const float* src, float* dst, int width, int height, cudaStream_t s);
  // lib.rs:160-247: tiles of `tile` with `margin` context.
  void run_tiled_device(const void* src, bool src_u8, void* dst, bool dst_u8, size_t width, size_t height, size_t tile,
                        size_t margin, const std::function<bool(float)>& progress, cudaStream_t s);

  DeviceBuffer host_in, host_out;

  // Each transformer block runs fused (the default: LN1 folded into the qkv
  // product, the one-head window projection inside the attention kernel,
  // LayerNorm, fc1, GELU and fc2 in one kernel) or as LayerNorm launches and
  // GEMMs (for comparisons).
  void set_fused(bool on) {
    fused_mlp_ = on;
    alloc_gen_++;  // no captured pass of the other path replays
  }

  struct Block;
  struct Level;

 private:
  void ensure(int ph, int pw);

  Device dev_;
  PackedWeights head_, tail_;
  std::vector<std::unique_ptr<Level>> levels_;  // down 1..3, body, up 3..1
  int alloc_pixels_ = 0;
  // device working buffers (planar f16)
  DeviceBuffer img_, x_, y_, t_, tok_, qkv_, att_, ln2_, hid_, gat_, skip_[3], out_;
  std::vector<cudaEvent_t> step_events_;
  // Side stream of a block's convolution half, which runs beside its
  // attention half.
  cudaStream_t s_conv_ = nullptr;
  cudaEvent_t ev_in_ = nullptr, ev_conv_ = nullptr;
  PassGraph graph_;
  bool fused_mlp_ = true;
  uint64_t alloc_gen_ = 0;  // counts ensure()'s reallocations  // passes without progress reports
};

}  // namespace iec
