// Test infrastructure: the model restatements of the CPU oracle.
#pragma once

#include "engine.h"

namespace ref {

// crates/realesrgan-native/src/network.rs + lib.rs (see realesrgan.cpp).
class RealEsrgan {
 public:
  static constexpr size_t SCALE = 4, FEATURES = 64, BODY = 32, STEPS = BODY + 2;
  explicit RealEsrgan(const std::string& path);
  static void check_size(size_t len, size_t width, size_t height);
  // network.rs:80-112: whole image, `step` after each layer (false = cancel).
  std::vector<float> run(const float* image, size_t width, size_t height,
                         const std::function<bool()>& step) const;
  // lib.rs:241-289 with identity load/store.
  std::vector<float> run_tiled(const float* image, size_t width, size_t height, size_t tile,
                               size_t margin, const std::function<bool(float)>& progress) const;

 private:
  struct Layer {
    Matrix conv;
    std::vector<float> slope;
  };
  std::vector<Layer> layers_;
};

// crates/scunet-native/src/network.rs + swin.rs + lib.rs (see scunet.cpp).
class Scunet {
 public:
  static constexpr size_t DIM = 64, BLOCKS = 4, STEPS = 7 * BLOCKS, MULTIPLE = 64, WINDOW = 8;
  static constexpr size_t TILE = 896, MARGIN = 64;
  explicit Scunet(const std::string& path);
  ~Scunet();
  // network.rs:265-353: whole image, `step` after each block (false = cancel).
  std::vector<float> run(const float* image, size_t width, size_t height,
                         const std::function<bool()>& step) const;
  // lib.rs:160-247 with identity load/store.
  std::vector<float> run_tiled(const float* image, size_t width, size_t height, size_t tile,
                               size_t margin, const std::function<bool(float)>& progress) const;
  struct Impl;

 private:
  Impl* impl_;
};

// crates/lama-native/src/network.rs + fourier.rs + lib.rs (see lama.cpp).
class Lama {
 public:
  static constexpr size_t MIN_SIDE = 9, STEPS = 26;
  explicit Lama(const std::string& path);
  ~Lama();
  // lib.rs:174-194 check_size.
  static void check_size(size_t image, size_t mask, size_t width, size_t height);
  // network.rs:405-488: the prediction for every pixel, `step` after each of
  // the 26 steps (false = cancel).
  std::vector<float> run(const float* image, const float* mask, size_t width, size_t height,
                         const std::function<bool()>& step) const;
  struct Impl;

 private:
  Impl* impl_;
};

// crates/birefnet-native/src/lib.rs + swin.rs + decoder.rs (see birefnet.cpp).
class Birefnet {
 public:
  explicit Birefnet(const std::string& path);
  ~Birefnet();
  // lib.rs:175-187 check_size.
  static void check_size(size_t len, size_t side);
  // lib.rs:134-172: the logit of every pixel of a normalised side x side image.
  std::vector<float> run_normalized(const float* image, size_t side) const;
  // lib.rs:116-133: an 8-bit image through the ImageNet normalisation table.
  static std::vector<float> normalize(const uint8_t* rgb, size_t pixels);
  struct Impl;

 private:
  Impl* impl_;
};

// decoder.rs:443-521: aligned-corner bilinear resize (ONNX Runtime's rule).
void resize(const float* src, size_t sh, size_t sw, size_t c, float* dst, size_t dh, size_t dw, size_t stride,
            bool add);

// fourier.rs: the ortho rfft2 of an h x w map of c channels (pixel p at
// x[p * stride]) into rows of h x (w / 2 + 1) pixels [re(c) | im(c)], and
// the ortho inverse added onto `out`.
void rfft2(const float* x, size_t stride, size_t h, size_t w, size_t c, std::vector<float>& out);
void irfft2_add(const std::vector<float>& spec, size_t h, size_t w, size_t c, float* out, size_t stride);

}  // namespace ref
