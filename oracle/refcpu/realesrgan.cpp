// Test infrastructure: CPU restatement of the reference's Real-ESRGAN
// (crates/realesrgan-native) on the engine restatement.
//   network.rs:22-29    constants: SCALE 4, 64 features, 32 body convs, 34 steps
//   network.rs:54-74    Network::load: body.{2i}.weight [9 cin, cout], bias, PReLU slopes
//   network.rs:80-112   Network::run: conv3 + PReLU per layer, two maps in turn
//   network.rs:118-140  shuffled: pixel shuffle x4 plus the input repeated
//   lib.rs:241-289      Model::tiled: equal grid tiles with a margin of context
//   lib.rs:302-316      check_size
#include <cmath>
#include <cstring>

#include "refcpu.h"

namespace ref {

RealEsrgan::RealEsrgan(const std::string& path) {
  WeightFile file = WeightFile::read(path, "REALESRG");
  for (size_t i = 0; i < STEPS; i++) {
    size_t cin = i == 0 ? 3 : FEATURES;
    bool last = i == STEPS - 1;
    size_t cout = last ? 3 * SCALE * SCALE : FEATURES;
    std::string name = "body." + std::to_string(2 * i);
    Weights w = file.take_weights(name + ".weight", {9 * cin, cout});
    std::vector<float> b = file.take(name + ".bias", {cout});
    Layer layer{Matrix(w, 9 * cin, cout, &b), {}};
    if (!last) layer.slope = file.take("body." + std::to_string(2 * i + 1) + ".weight", {FEATURES});
    layers_.push_back(std::move(layer));
  }
  file.finish();
}

void RealEsrgan::check_size(size_t len, size_t width, size_t height) {
  if (width == 0 || height == 0)
    throw Error(ERR_INPUT, "empty " + std::to_string(width) + " x " + std::to_string(height) + " image");
  if (width * height * 3 != len)
    throw Error(ERR_INPUT, std::to_string(len) + " values for a " + std::to_string(width) + " x " +
                               std::to_string(height) + " RGB image");
}

std::vector<float> RealEsrgan::run(const float* image, size_t width, size_t height,
                                   const std::function<bool()>& step) const {
  const size_t pixels = width * height;
  std::vector<float> a(pixels * FEATURES), b(pixels * FEATURES);
  size_t channels = 3;
  for (size_t i = 0; i < layers_.size(); i++) {
    const Layer& layer = layers_[i];
    const float* src = i == 0 ? image : a.data();
    Input in = Input::conv(src, height, width, channels, channels, 3);
    size_t n = layer.conv.n;
    const float* slope = layer.slope.empty() ? nullptr : layer.slope.data();
    conv3(in, layer.conv, b.data(), n, false, [slope, n](float* px) {
      if (!slope) return;
      for (size_t c = 0; c < n; c++) px[c] = px[c] < 0.0f ? px[c] * slope[c] : px[c];
    });
    std::swap(a, b);
    channels = n;
    if (step && !step()) throw Error(CANCELLED, "cancelled");
  }
  // network.rs:118-140.
  const size_t row = width * SCALE * 3;
  std::vector<float> out(height * SCALE * row);
#pragma omp parallel for schedule(static)
  for (long y = 0; y < (long)height; y++) {
    for (size_t x = 0; x < width; x++) {
      size_t p = (size_t)y * width + x;
      for (size_t i = 0; i < SCALE; i++)
        for (size_t j = 0; j < SCALE; j++) {
          size_t o = ((size_t)y * SCALE + i) * row + (x * SCALE + j) * 3;
          for (size_t c = 0; c < 3; c++)
            out[o + c] = a[p * 3 * SCALE * SCALE + c * SCALE * SCALE + i * SCALE + j] + image[p * 3 + c];
        }
    }
  }
  return out;
}

std::vector<float> RealEsrgan::run_tiled(const float* image, size_t width, size_t height, size_t tile,
                                         size_t margin, const std::function<bool(float)>& progress) const {
  check_size(width * height * 3, width, height);
  if (tile == 0) throw Error(ERR_INPUT, "tile size 0");
  const size_t ow = width * SCALE, oh = height * SCALE;
  std::vector<float> out(ow * oh * 3);
  const size_t cols = (width + tile - 1) / tile, rows = (height + tile - 1) / tile;
  const float steps = (float)(cols * rows * STEPS);
  size_t done = 0;
  std::vector<float> region;
  for (size_t j = 0; j < rows; j++) {
    size_t y0 = j * height / rows, y1 = (j + 1) * height / rows;
    for (size_t i = 0; i < cols; i++) {
      size_t x0 = i * width / cols, x1 = (i + 1) * width / cols;
      size_t rx0 = x0 > margin ? x0 - margin : 0, ry0 = y0 > margin ? y0 - margin : 0;
      size_t rx1 = margin > width - x1 ? width : x1 + margin;
      size_t ry1 = margin > height - y1 ? height : y1 + margin;
      size_t rw = rx1 - rx0;
      region.clear();
      for (size_t y = ry0; y < ry1; y++)
        region.insert(region.end(), image + (y * width + rx0) * 3, image + (y * width + rx0 + rw) * 3);
      std::vector<float> result = run(region.data(), rw, ry1 - ry0, [&]() {
        done++;
        return !progress || progress((float)done / steps);
      });
      size_t rws = rw * SCALE, cw = (x1 - x0) * SCALE;
      for (size_t y = y0 * SCALE; y < y1 * SCALE; y++) {
        size_t start = ((y - ry0 * SCALE) * rws + (x0 - rx0) * SCALE) * 3;
        std::memcpy(&out[(y * ow + x0 * SCALE) * 3], &result[start], cw * 3 * sizeof(float));
      }
    }
  }
  return out;
}

}  // namespace ref
