// Real-ESRGAN general-x4v3 (SRVGGNetCompact) on the CUDA backend.
//
// Replaces crates/realesrgan-native/src/gpu.rs (the Vulkan network) behind
// the model's public API (lib.rs): 34 3x3 convolutions on tcgen05 tensor
// cores, PReLU fused into each epilogue, and the pixel shuffle x4 plus the
// repeated input fused into the last one, which writes the final image
// (f32 or 8-bit) straight into the output, cropped to the tile it belongs to.
#pragma once

#include <cuda_fp16.h>

#include <array>
#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "runtime.h"

namespace iec {

class RealEsrgan {
 public:
  static constexpr int SCALE = 4, FEATURES = 64, STEPS = 34, GPU_TILE = 768, MARGIN = 34;

  RealEsrgan(const std::string& path, const Options& opt);
  ~RealEsrgan();

  Device& device() { return dev_; }

  // lib.rs:241-289 on device buffers: `src` is `count` images of
  // width x height x 3 (f32 or u8), `dst` their 4x outputs (f32 or u8).
  // Runs tile by tile; `progress` (may be empty) gets the share done after
  // each layer and returns false to cancel.
  // Only tiles first .. last - 1 of the grid (row-major) run when a range is
  // given; each writes just its own window of `dst`.
  void run_tiled_device(const void* src, bool src_u8, void* dst, bool dst_u8, size_t count, size_t width,
                        size_t height, size_t tile, size_t margin, const std::function<bool(float)>& progress,
                        cudaStream_t stream, size_t first = 0, size_t last = SIZE_MAX);

  // lib.rs:241-289's grid: the kept window {x0, y0, x1, y1} (input pixels)
  // of each tile first .. last - 1.
  static std::vector<std::array<size_t, 4>> tile_windows(size_t width, size_t height, size_t tile, size_t first,
                                                         size_t last);

  // Whole images (one region each), `count` at a time in chunks; no waits.
  void run_device(const float* src, float* dst, size_t count, size_t width, size_t height, cudaStream_t stream);

  // Host buffers (f32 or 8-bit images in and out), copies overlapped with
  // the kernels; returns when done.
  void run_batch_host(const void* src, bool src_u8, void* dst, bool dst_u8, size_t count, size_t width,
                      size_t height, cudaStream_t stream);

  // As run_device, but the feature maps live in a fixed scratch array that
  // the library holds on every device (no allocation at all); see
  // iec_realesrgan_run_device_noalloc in iec_cuda.h for the limit and rules.
  static constexpr size_t NOALLOC_MAX_PIXELS = 114688;
  void run_device_noalloc(const float* src, float* dst, size_t count, size_t width, size_t height,
                          cudaStream_t stream);

  size_t launches(size_t count, size_t width, size_t height) const;
  // Fused body on (default) or per-layer launches everywhere.
  void set_fused(bool on) { no_fuse_ = !on; }
  size_t chunk_for(size_t width, size_t height) const;

  // Measurement hooks: events around every launch (see iec_cuda.h).
  void set_timing(size_t capacity);
  size_t timing(int* kinds, float* ms, size_t n);

  // The host-API staging buffers.
  DeviceBuffer host_in, host_out;

 private:
  struct Layer {
    int cin = 0, cout = 0;  // cin as the kernel sees it (3 -> 16)
    int slope_unit = 0;     // all PReLU slopes in [0, 1]
    DeviceBuffer w, b, s;
  };
  struct Region {
    int rx0, ry0, rw, rh;     // region of the source image the network runs on
    int kx0, ky0, kx1, ky1;   // kept window, region coordinates
  };
  // One pass of the network over `count` regions at the same place of
  // `count` images; returns false when cancelled.
  bool run_network(const void* src, bool src_u8, void* dst, bool dst_u8, int count, int src_w, int src_h,
                   const Region& r, const std::function<bool()>& step, cudaStream_t stream);
  void ensure_maps(size_t count, int w, int h, cudaStream_t stream);
  // The 32 body layers as one persistent launch (conv3x3_body_sm100.cuh):
  // whether a pass of this size takes it, and the launch.
  bool body_fits(int count, int w, int h, int layers_per_launch) const;
  // Body layers first .. first + layers - 1 (0-based within the body).
  void launch_body(int count, int mw, int mh, const Region& r, int first, int layers, cudaStream_t stream);
  // Record a timing event before a launch of `kind` (-1: after the last).
  void mark(int kind, cudaStream_t stream);

  Device dev_;
  std::vector<Layer> layers_;
  DeviceBuffer prep_, map_a_, map_b_, rows_, items_;
  std::array<int, 4> items_key_ = {0, 0, 0, 0};  // pass shape (count, w, h, layers) of items_'s table
  // Images per layer sweep of the fused body: their two maps stay in L2.
  static constexpr int BODY_GROUP = 2;
  // Body layers per fused launch in passes with progress reports.
  static constexpr int BODY_STAGE = 8;
  bool body_pdl_ = true;   // the fused launch also takes programmatic dependent launch
  bool no_fuse_ = false;   // per-layer launches only (set_fused)
  size_t map_pixels_ = 0;
  int padded_ = 0;  // maps were zeroed for a region smaller than a TMA box
  std::vector<cudaEvent_t> layer_events_;
  DeviceBuffer batch_in_[2], batch_out_[2];
  cudaStream_t h2d_ = nullptr, d2h_ = nullptr;
  cudaEvent_t ev_h2d_[2] = {}, ev_done_[2] = {}, ev_d2h_[2] = {}, ev_start_ = nullptr;
  std::vector<cudaEvent_t> t_events_;
  std::vector<int> t_kinds_;
  size_t t_used_ = 0;
};

}  // namespace iec
