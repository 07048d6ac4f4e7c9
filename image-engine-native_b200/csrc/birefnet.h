// BiRefNet-lite (background removal) on the CUDA backend.
//
// Replaces crates/birefnet-native/src/gpu.rs (the Vulkan network) behind the
// model's public API (lib.rs): the Swin-T backbone of swin.rs (patch
// embedding, 7 x 7 shifted-window attention in 64-row window slots, MLPs,
// patch merges) on the general tcgen05 GEMM and the fused window attention,
// run on the image and on its half-size copy; and the decoder of decoder.rs
// (3x3 convolutions, deformable ASPPs as a bilinear-sample kernel feeding
// GEMMs, aligned-corner resizes, image patches, gates), ending in an f32
// head: the decoder's low-resolution logits resized and the full-resolution
// patch branch's composed 5x5 convolution added per pixel. Concatenations
// cost nothing: every map is planar, and each producer writes its channel
// planes straight into the consumer's input.
#pragma once

#include <cuda_fp16.h>

#include <memory>
#include <string>
#include <vector>

#include "gemm.h"
#include "runtime.h"

namespace iec {

class Birefnet {
 public:
  Birefnet(const std::string& path, const Options& opt);
  ~Birefnet();
  Device& device() { return dev_; }

  // lib.rs:116-172 on device buffers: `image` side x side x 3, 8-bit RGB
  // (`u8`) or already normalised f32; `logits` side x side f32.
  void run(const void* image, bool u8, int side, float* logits, cudaStream_t s);

  DeviceBuffer host_in, host_out;  // staging of the host entry points

  // Each backbone block's MLP runs fused where its width allows (the
  // default: norm2, fc1, GELU and fc2 in one kernel, mlp_sm100.cuh) or as a
  // LayerNorm launch and two GEMMs (for comparisons).
  void set_fused(bool on) {
    fused_mlp_ = on;
    alloc_gen_++;  // no captured pass of the other path replays
  }

  struct SwinBlock;
  struct Stage;
  struct DBlock;
  struct Patches;

 private:
  void ensure(int side);
  void run_pass(const void* image, bool u8, int side, float* logits, cudaStream_t s);
  // The backbone's working buffers (one set per concurrent pass).
  struct BackboneBuffers {
    DeviceBuffer patch_rows, x, tok, qkv, att, ln, hid, mrg;
  };
  void ensure_backbone(BackboneBuffers& b, int side);
  // swin.rs:162-215 on `img` (f32 NHWC, side x side); stage i's normalised
  // output goes to planes from plane0[i] of dst[i] (dst_plane[i] elements per
  // plane).
  void backbone(const float* img, int side, __half* const dst[4], const long long dst_plane[4], const int plane0[4],
                BackboneBuffers& bb, cudaStream_t s);
  // decoder.rs:343-406: `x` (cin channels, g x g) -> out planes from `plane0`
  // of `out` (cout channels).
  void block(const DBlock& b, const __half* x, long long x_plane, int cin, int g, __half* out, long long out_plane,
             int plane0, cudaStream_t s);

  Device dev_;
  PackedWeights embed_;
  DeviceBuffer embed_g_, embed_b_;
  std::vector<std::unique_ptr<Stage>> stages_;
  std::unique_ptr<DBlock> squeeze_;
  std::vector<std::unique_ptr<DBlock>> blocks_;
  PackedWeights laterals_[3];
  std::vector<std::unique_ptr<Patches>> patches_;
  DeviceBuffer head_w_, full_;  // head [96]; full-resolution branch tables
  float head_b_ = 0.0f;
  int alloc_side_ = 0;
  // working buffers
  DeviceBuffer img_, himg_;
  BackboneBuffers bb_[2];  // the full-size pass, the half-size pass
  DeviceBuffer lev_[3], hf_[4], x4_, in_[4], outb_[3], out1_, t_, t2_, offs_, samp_, cat_, g16_, sums_, low_, stack_,
      pmid_;
  DeviceBuffer offs_b_[3], samp_b_[3];  // ASPP branches 0-2, beside branch 3
  // Side streams: the half-size backbone pass, the image-patch branches of
  // the four levels, and the ASPP's small branches.
  cudaStream_t s_half_ = nullptr, s_patch_ = nullptr, s_aspp_ = nullptr;
  cudaEvent_t ev_prep_ = nullptr, ev_half_ = nullptr, ev_t_ = nullptr, ev_aspp_ = nullptr, ev_patch_[4] = {};
  PassGraph graph_;
  bool fused_mlp_ = true;
  uint64_t alloc_gen_ = 0;  // counts ensure()'s reallocations
};

}  // namespace iec
