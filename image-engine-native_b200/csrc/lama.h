// Big LaMa (inpainting) on the CUDA backend.
//
// Replaces crates/lama-native/src/gpu.rs (the Vulkan network) behind the
// model's public API (lib.rs): the generator of network.rs on the general
// tcgen05 implicit GEMM (reflect-padded 7x7 and 3x3 convolutions, stride-2
// convolutions over space-to-depth phases, 1x1 spectral convolutions, the
// transposed convolutions as four phase products) and the planar Fourier
// transforms of fft.cu. Every map is written by its producing GEMM straight
// into the layout its consumer reads (reflect padding mirrored in the
// epilogue, space-to-depth phases for the stride-2 convolutions); ReLU,
// sigmoid, the spectral residual, the spectral accumulation and the blocks'
// residual adds are fused into GEMM epilogues.
#pragma once

#include <cuda_fp16.h>

#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "fft.h"
#include "gemm.h"
#include "runtime.h"

namespace iec {

class Lama {
 public:
  static constexpr int LOCAL = 128, GLOBAL = 384, CHANNELS = 512, SPECTRAL = 192, BLOCKS = 18, MIN_SIDE = 9,
                       STEPS = 1 + 3 + BLOCKS + 3 + 1, MULTIPLE = 8;

  Lama(const std::string& path, const Options& opt);
  ~Lama();
  Device& device() { return dev_; }

  // network.rs:405-488 (+ lib.rs:139-156 when `dst_u8`) on device buffers:
  // `image` width x height x 3 (f32 in 0..=1, or u8), `mask` width x height
  // (f32: 1 fills, or u8: non-zero fills). `dst` gets the prediction (f32
  // width x height x 3), or with `dst_u8` the 8-bit image (u8 `image`
  // required) with the masked pixels filled in. `step` after each of the 26
  // steps (false cancels: returns false).
  bool run(const void* image, bool image_u8, const void* mask, bool mask_u8, void* dst, bool dst_u8, int width,
           int height, const std::function<bool()>& step, cudaStream_t s);

  DeviceBuffer host_in, host_mask, host_out;  // staging of the host entry points

  // The fused Fourier unit (default) or rfft2, GEMM and irfft2 as separate
  // launches (for comparisons); the two give the same values.
  void set_fused(bool on) {
    fused_unit_ = on;
    alloc_gen_++;  // no captured pass of the other path replays
  }

  struct Ffc;

 private:
  void ensure(int hp, int wp);
  bool run_pass(const void* image, bool image_u8, const void* mask, bool mask_u8, void* dst, bool dst_u8, int width,
                int height, const std::function<bool()>& step, cudaStream_t s);
  void ffc(const Ffc& f, const __half* in, __half* out, __half* tmp, bool residual, cudaStream_t s);

  Device dev_;
  PackedWeights first_, down_[3], up_[3][4], last_;
  std::vector<std::unique_ptr<Ffc>> ffc_;  // block b: ffc_[2 b], ffc_[2 b + 1]
  int alloc_h_ = 0, alloc_w_ = 0;
  FourierPlan plan_;
  // device working buffers (planar f16)
  DeviceBuffer in0_, d0_, d1_, d2_, x_, mid_, tmp_, spectral_, spectrum_, filtered_, u0_, u1_, u2_, out_;
  std::vector<cudaEvent_t> step_events_;
  // Side streams of an FFC: its local convolution and its spectral chain run
  // beside the cross convolution (each alone fills a fraction of the GPU).
  cudaStream_t s_local_ = nullptr, s_spec_ = nullptr;
  cudaEvent_t ev_in_ = nullptr, ev_local_ = nullptr, ev_spec_ = nullptr;
  PassGraph graph_;
  bool fused_unit_ = true;
  uint64_t alloc_gen_ = 0;  // counts ensure()'s reallocations  // passes without progress reports
};

}  // namespace iec
