// CPU restatement of the reference's inference engine (crates/native-engine),
// used ONLY as test infrastructure: the parity oracle of the CUDA backend and
// the timed CPU baseline. Nothing in the product links it.
//
// It restates, in C++ of its own, the arithmetic of the reference's CPU f32
// path at its AVX2 tier, in the order the reference computes it:
//   half.rs:7-48,125        f32 <-> IEEE half, round to nearest even
//   weight_file.rs:40-145   the .weights container and its checks
//   gemm.rs:290-483,514-667 products and convolutions over "taps"; each output
//                           is bias (+ the old value when accumulating) then
//                           one fused multiply-add per tap and channel, in
//                           order (gemm/kernel.rs:112-270, the AVX2 kernel)
//   winograd.rs:53-773      3x3 stride-1 convolutions by F(4x4,3x3) or
//                           F(2x2,3x3), transforms without fused multiply-adds
//   math.rs                 GELU / sigmoid / layer norm / softmax
// Threads (OpenMP) split rows only: every value is computed by one thread in
// a fixed order, so results do not depend on the thread count.
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace ref {

enum Status { OK = 0, ERR_IO = 1, ERR_WEIGHTS = 2, ERR_INPUT = 3, CANCELLED = 4, ERR_GPU = 5 };

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

// half.rs:7-48 (f32_to_half) and half.rs:125 (half_to_f32).
uint16_t f32_to_half(float v);
float half_to_f32(uint16_t h);

// A tensor as a weights file stores it; `half` tells whether the file held
// IEEE halves (values are then those halves, widened exactly).
struct Weights {
  std::vector<size_t> shape;
  bool half = false;
  std::vector<float> values;
};

// weight_file.rs:28-145.
class WeightFile {
 public:
  static WeightFile read(const std::string& path, const char magic[8]);
  static WeightFile parse(const uint8_t* data, size_t len, const char magic[8]);
  Weights take_weights(const std::string& name, const std::vector<size_t>& shape);
  std::vector<float> take(const std::string& name, const std::vector<size_t>& shape) {
    return take_weights(name, shape).values;
  }
  void finish() const;

 private:
  std::map<std::string, Weights> tensors_;
};

// A layer's k x n weights, row-major, with its bias (zeros when it has none).
// gemm.rs:98-147.
struct Matrix {
  size_t k = 0, n = 0;
  bool half = false;
  std::vector<float> w;
  std::vector<float> bias;
  Matrix() = default;
  Matrix(const Weights& wt, size_t k, size_t n, const std::vector<float>* bias);
  Matrix(std::vector<float> w, size_t k, size_t n, const std::vector<float>* bias, bool half);
};

enum class Pad { Zero, Reflect };
enum class Act { None, Relu, Gelu };

// gemm.rs:274-304: where the rows of a product read their input.
struct Input {
  enum Kind { Rows, Image } kind = Rows;
  const float* data = nullptr;
  size_t stride = 0;
  // Image only:
  size_t height = 0, width = 0, channels = 0;
  enum TapKind { Conv, Offsets } taps = Conv;
  size_t size = 1, step = 1;
  Pad pad = Pad::Zero;
  size_t offsets[4][2] = {{0, 0}, {0, 0}, {0, 0}, {0, 0}};
  size_t count = 0;

  static Input rows(const float* data, size_t stride);
  static Input conv(const float* data, size_t height, size_t width, size_t channels, size_t stride,
                    size_t size, size_t step = 1, Pad pad = Pad::Zero);
  static Input phase(const float* data, size_t height, size_t width, size_t channels, size_t stride,
                     const size_t (*offs)[2], size_t count);
  void out_size(size_t* oh, size_t* ow) const;
  size_t tap_count() const;
  // Pointer to the `channels` values tap `t` of row `r` reads, or nullptr for zeros.
  const float* at(size_t r, size_t t) const;
};

// gemm.rs:408-441 reflect(): i mirrored into 0..n about the edge pixels.
inline size_t reflect(long i, size_t n) {
  long last = (long)n - 1;
  long a = i < 0 ? -i : i;
  long b = 2 * last - i;
  return (size_t)(a < b ? a : b);
}

// gemm.rs:514-667: out[r] = act(input[r] * w + bias), or with `accumulate`
// act(out[r] + bias + input[r] * w), for rows [r0, r1); row r of the result at
// out[(r - r0) * stride].
void multiply(const Input& input, size_t r0, size_t r1, const Matrix& w, float* out, size_t stride,
              Act act, bool accumulate);
// The same on the calling thread alone (for use inside a parallel region).
void multiply_serial(const Input& input, size_t r0, size_t r1, const Matrix& w, float* out, size_t stride,
                     Act act, bool accumulate);

// winograd.rs:612-672: the 3x3 stride-1 convolution of an image input with
// `w`, plus bias, stored to (or with `accumulate` added to) out pixels
// `stride` apart; `finish` then runs on each output pixel's n channels.
// `direct` forces the direct product (the oracle's noise-floor mode).
void conv3(const Input& input, const Matrix& w, float* out, size_t stride, bool accumulate,
           const std::function<void(float*)>& finish);

// Global switch: true makes conv3 use the direct product everywhere.
extern bool g_direct;
void set_threads(int n);
int threads();

// math.rs: exact GELU via an erf rational fit, sigmoid, layer norm, softmax.
float gelu_one(float x);
float sigmoid_one(float x);
float exp_neg(float x);

}  // namespace ref

namespace ref {

// math.rs:78-116: layer normalisation of one row in place (sums in eight
// interleaved lanes), epsilon 1e-5.
void layer_norm_row(float* x, size_t n, const float* gamma, const float* beta);
// math.rs:119-134: softmax of a row in place, given its largest value.
void softmax_from(float* x, size_t n, float max);
// attention.rs:25-209 at the AVX2 tier: head `head` (32 channels) of one
// window of `tokens` tokens; qkv rows of 3c (q | k | v); bias [tokens][tokens]
// (masks included); writes the head's 32 columns of `tokens` rows of `out`,
// `c` apart.
void attention(const float* qkv, size_t c, size_t head, const float* bias, size_t tokens, float* out);

}  // namespace ref
