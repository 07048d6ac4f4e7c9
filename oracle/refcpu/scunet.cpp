// Test infrastructure: CPU restatement of the reference's SCUNet
// (crates/scunet-native) on the engine restatement.
//   network.rs:27-35     DIM 64, 4 blocks per level, 28 steps, sides padded to 64
//   network.rs:113-153   Block: split 1x1, two 3x3 convolutions (ReLU, then
//                        accumulate) on the first half, transformer on the second
//   network.rs:162-215   run_level: each block's MLP, join (+= x) and the next
//                        block's split, per pixel
//   network.rs:234-353   Network::load / run: head, 3 levels down (2x2 stride-2
//                        halving), body, 3 levels up (skip add, 2x2 transposed
//                        doubling), head again (+=), tail, crop
//   network.rs:367-478   pad (edge repeat), add, halved, doubled
//   swin.rs:26-50        bias tables: position bias plus the shift masks of the
//                        4 window classes
//   swin.rs:124-254      attend (rolled 8x8 windows, LN, qkv, attention, proj,
//                        residual) and mlp (LN, fc1 GELU, fc2 residual)
//   lib.rs:160-247,302-316  the tiled runner and size checks
#include <cmath>
#include <cstring>

#include "refcpu.h"

namespace ref {

namespace {

constexpr size_t HEAD_DIM = 32, N_TOK = 64, SHIFT = 4;

Matrix linear(WeightFile& f, const std::string& name, size_t k, size_t n, bool bias) {
  Weights w = f.take_weights(name + ".weight", {k, n});
  std::vector<float> b;
  if (bias) b = f.take(name + ".bias", {n});
  return Matrix(w, k, n, bias ? &b : nullptr);
}

Matrix conv3_matrix(WeightFile& f, const std::string& name, size_t cin, size_t cout) {
  Weights w = f.take_weights(name + ".weight", {9 * cin, cout});
  return Matrix(w, 9 * cin, cout, nullptr);
}

// swin.rs:26-50.
std::vector<float> bias_tables(const std::vector<float>& position, bool shifted) {
  if (!shifted) return position;
  const size_t n = N_TOK;
  auto region = [](size_t v, bool last) -> size_t { return (last && v >= 8 - SHIFT) ? 1 : 0; };
  std::vector<float> t;
  t.reserve(4 * position.size());
  for (int cls = 0; cls < 4; cls++) {
    const bool last_col = cls & 1, last_row = cls & 2;
    auto id = [&](size_t i) { return region(i / 8, last_row) * 2 + region(i % 8, last_col); };
    for (size_t h = 0; h < position.size() / (n * n); h++)
      for (size_t i = 0; i < n; i++)
        for (size_t j = 0; j < n; j++) t.push_back(position[(h * n + i) * n + j] + (id(i) == id(j) ? 0.0f : -INFINITY));
  }
  return t;
}

struct Transformer {
  size_t c = 0;
  bool shifted = false;
  std::vector<float> g1, b1, g2, b2, bias;
  Matrix qkv, proj, fc1, fc2;

  Transformer(WeightFile& f, const std::string& name, size_t c_, bool shifted_) : c(c_), shifted(shifted_) {
    const size_t heads = c / HEAD_DIM;
    g1 = f.take(name + ".ln1.weight", {c});
    b1 = f.take(name + ".ln1.bias", {c});
    qkv = linear(f, name + ".msa.embedding_layer", c, 3 * c, true);
    bias = bias_tables(f.take(name + ".msa.position_bias", {heads, N_TOK, N_TOK}), shifted);
    proj = linear(f, name + ".msa.linear", c, c, true);
    g2 = f.take(name + ".ln2.weight", {c});
    b2 = f.take(name + ".ln2.bias", {c});
    fc1 = linear(f, name + ".mlp.0", c, 4 * c, true);
    fc2 = linear(f, name + ".mlp.2", 4 * c, c, true);
  }

  // swin.rs:124-220: attention with its residual on channels [0, c) of the
  // map whose pixel p starts at map[p * stride]; sides multiples of 8.
  void attend(float* map, size_t stride, size_t height, size_t width) const {
    const size_t rows_w = height / 8, cols_w = width / 8, heads = c / HEAD_DIM, n = N_TOK;
    const size_t shift = shifted ? SHIFT : 0;
    const long windows = (long)(rows_w * cols_w);
#pragma omp parallel
    {
      std::vector<float> tokens(n * c), q(n * 3 * c), out(n * c), proj_out(n * c);
      size_t source[N_TOK];
#pragma omp for schedule(dynamic, 1)
      for (long w = 0; w < windows; w++) {
        const size_t wy = (size_t)w / cols_w, wx = (size_t)w % cols_w;
        for (size_t i = 0; i < n; i++) {
          const size_t y = (wy * 8 + i / 8 + shift) % height, x = (wx * 8 + i % 8 + shift) % width;
          source[i] = y * width + x;
          std::memcpy(&tokens[i * c], map + source[i] * stride, c * sizeof(float));
          layer_norm_row(&tokens[i * c], c, g1.data(), b1.data());
        }
        multiply_serial(Input::rows(tokens.data(), c), 0, n, qkv, q.data(), 3 * c, Act::None, false);
        size_t cls = 0;
        if (shifted) cls = ((size_t)w % cols_w == cols_w - 1 ? 1 : 0) + 2 * ((size_t)w / cols_w == rows_w - 1 ? 1 : 0);
        for (size_t h = 0; h < heads; h++)
          attention(q.data(), c, h, &bias[(cls * heads + h) * n * n], n, out.data());
        multiply_serial(Input::rows(out.data(), c), 0, n, proj, proj_out.data(), c, Act::None, false);
        for (size_t i = 0; i < n; i++) {
          float* d = map + source[i] * stride;
          for (size_t k = 0; k < c; k++) d[k] += proj_out[i * c + k];
        }
      }
    }
  }

  // swin.rs:222-254: MLP with its residual on `rows` pixels at dst[r * stride].
  void mlp(float* dst, size_t stride, size_t rows, std::vector<float>& normed, std::vector<float>& hidden) const {
    normed.resize(rows * c);
    hidden.resize(rows * 4 * c);
    for (size_t r = 0; r < rows; r++) {
      std::memcpy(&normed[r * c], dst + r * stride, c * sizeof(float));
      layer_norm_row(&normed[r * c], c, g2.data(), b2.data());
    }
    multiply_serial(Input::rows(normed.data(), c), 0, rows, fc1, hidden.data(), 4 * c, Act::Gelu, false);
    multiply_serial(Input::rows(hidden.data(), 4 * c), 0, rows, fc2, dst, stride, Act::None, true);
  }
};

struct Block {
  size_t half;
  Matrix split, conv1, conv2, join;
  Transformer transformer;

  Block(WeightFile& f, const std::string& name, size_t c, bool shifted)
      : half(c / 2),
        split(linear(f, name + ".conv1_1", c, c, true)),
        conv1(conv3_matrix(f, name + ".conv_block.0", c / 2, c / 2)),
        conv2(conv3_matrix(f, name + ".conv_block.2", c / 2, c / 2)),
        join(linear(f, name + ".conv1_2", c, c, true)),
        transformer(f, name + ".trans_block", c / 2, shifted) {}

  // network.rs:136-153.
  void convolve(float* y, size_t height, size_t width, std::vector<float>& t) const {
    const size_t pixels = height * width;
    t.resize(pixels * half);
    conv3(Input::conv(y, height, width, half, 2 * half, 3), conv1, t.data(), half, false, [this](float* px) {
      for (size_t k = 0; k < half; k++) px[k] = px[k] > 0.0f ? px[k] : 0.0f;
    });
    conv3(Input::conv(t.data(), height, width, half, half, 3), conv2, y, 2 * half, true, nullptr);
  }
};

std::vector<Block> level(WeightFile& f, const std::string& name, size_t first, size_t c) {
  std::vector<Block> blocks;
  for (size_t b = 0; b < Scunet::BLOCKS; b++)
    blocks.emplace_back(f, name + "." + std::to_string(first + b), c, b % 2 == 1);
  return blocks;
}

// network.rs:162-215.
void run_level(const std::vector<Block>& blocks, std::vector<float>& x, size_t height, size_t width,
               const std::function<void()>& block_done) {
  const size_t half = blocks[0].half, c = 2 * half, pixels = height * width;
  std::vector<float> y(pixels * c), t;
  multiply(Input::rows(x.data(), c), 0, pixels, blocks[0].split, y.data(), c, Act::None, false);
  for (size_t b = 0; b < blocks.size(); b++) {
    const Block& block = blocks[b];
    block.convolve(y.data(), height, width, t);
    block.transformer.attend(y.data() + half, c, height, width);
    const Matrix* next = b + 1 < blocks.size() ? &blocks[b + 1].split : nullptr;
    const long chunks = (long)((pixels + 95) / 96);
#pragma omp parallel
    {
      std::vector<float> normed, hidden;
#pragma omp for schedule(dynamic, 4)
      for (long ch = 0; ch < chunks; ch++) {
        const size_t r0 = (size_t)ch * 96, r1 = std::min(pixels, r0 + 96), rows = r1 - r0;
        float* xr = x.data() + r0 * c;
        float* yr = y.data() + r0 * c;
        block.transformer.mlp(yr + half, c, rows, normed, hidden);
        multiply_serial(Input::rows(yr, c), 0, rows, block.join, xr, c, Act::None, true);
        if (next) multiply_serial(Input::rows(xr, c), 0, rows, *next, yr, c, Act::None, false);
      }
    }
    block_done();
  }
}

// network.rs:410-441: 2x2 stride-2 convolution, each output pixel reading its
// 2x2 input pixels in row-major order, channels within each.
std::vector<float> halved(const std::vector<float>& x, size_t height, size_t width, const Matrix& m) {
  const size_t c = m.k / 4, h = height / 2, w = width / 2;
  std::vector<float> rows(h * w * 4 * c), out(h * w * m.n);
#pragma omp parallel for schedule(static)
  for (long r = 0; r < (long)(h * w); r++) {
    const size_t y = 2 * ((size_t)r / w), xx = 2 * ((size_t)r % w);
    const size_t src[4] = {y * width + xx, y * width + xx + 1, (y + 1) * width + xx, (y + 1) * width + xx + 1};
    for (int q = 0; q < 4; q++) std::memcpy(&rows[((size_t)r * 4 + q) * c], &x[src[q] * c], c * sizeof(float));
  }
  multiply(Input::rows(rows.data(), 4 * c), 0, h * w, m, out.data(), m.n, Act::None, false);
  return out;
}

// network.rs:446-478: 2x2 stride-2 transposed convolution.
std::vector<float> doubled(const std::vector<float>& x, size_t height, size_t width, const Matrix& m) {
  const size_t cout = m.n / 4, w2 = 2 * width;
  std::vector<float> prod(height * width * m.n), out(4 * height * width * cout);
  multiply(Input::rows(x.data(), m.k), 0, height * width, m, prod.data(), m.n, Act::None, false);
#pragma omp parallel for schedule(static)
  for (long r = 0; r < (long)(height * width); r++) {
    const size_t y = (size_t)r / width, xx = (size_t)r % width;
    for (size_t q = 0; q < 4; q++) {
      const size_t pixel = (2 * y + q / 2) * w2 + 2 * xx + q % 2;
      std::memcpy(&out[pixel * cout], &prod[(size_t)r * m.n + q * cout], cout * sizeof(float));
    }
  }
  return out;
}

}  // namespace

struct Scunet::Impl {
  Matrix head, tail;
  std::vector<std::pair<std::vector<Block>, Matrix>> down;
  std::vector<Block> body;
  std::vector<std::pair<Matrix, std::vector<Block>>> up;
};

Scunet::Scunet(const std::string& path) : impl_(new Impl) {
  try {
    WeightFile f = WeightFile::read(path, std::string("SCUNET\0\0", 8).c_str());
    impl_->head = conv3_matrix(f, "m_head.0", 3, DIM);
    const size_t widths[3] = {DIM, 2 * DIM, 4 * DIM};
    for (int i = 0; i < 3; i++) {
      const std::string name = "m_down" + std::to_string(i + 1);
      auto blocks = level(f, name, 0, widths[i]);
      Matrix halve = linear(f, name + "." + std::to_string(BLOCKS), 4 * widths[i], 2 * widths[i], false);
      impl_->down.emplace_back(std::move(blocks), std::move(halve));
    }
    impl_->body = level(f, "m_body", 0, 8 * DIM);
    for (int i = 2; i >= 0; i--) {
      const std::string name = "m_up" + std::to_string(i + 1);
      Matrix dbl = linear(f, name + ".0", 2 * widths[i], 4 * widths[i], false);
      impl_->up.emplace_back(std::move(dbl), level(f, name, 1, widths[i]));
    }
    impl_->tail = conv3_matrix(f, "m_tail.0", DIM, 3);
    f.finish();
  } catch (...) {
    delete impl_;
    throw;
  }
}

Scunet::~Scunet() { delete impl_; }

std::vector<float> Scunet::run(const float* image, size_t width, size_t height,
                               const std::function<bool()>& step) const {
  const Impl& n = *impl_;
  auto done = [&]() {
    if (step && !step()) throw Error(CANCELLED, "cancelled");
  };
  // network.rs:358-379: pad to multiples of 64 by repeating the last row and column.
  const size_t ph = (height + MULTIPLE - 1) / MULTIPLE * MULTIPLE, pw = (width + MULTIPLE - 1) / MULTIPLE * MULTIPLE;
  std::vector<float> padded(ph * pw * 3);
  for (size_t y = 0; y < ph; y++) {
    const float* src = image + std::min(y, height - 1) * width * 3;
    std::memcpy(&padded[y * pw * 3], src, width * 3 * sizeof(float));
    for (size_t x = width; x < pw; x++)
      for (int k = 0; k < 3; k++) padded[(y * pw + x) * 3 + k] = src[(width - 1) * 3 + k];
  }
  size_t h = ph, w = pw;
  std::vector<float> x(h * w * DIM);
  auto head = [&](bool accumulate) {
    multiply(Input::conv(padded.data(), ph, pw, 3, 3, 3), 0, ph * pw, n.head, x.data(), DIM, Act::None, accumulate);
  };
  head(false);
  std::vector<std::vector<float>> skips;
  for (const auto& [blocks, halve] : n.down) {
    run_level(blocks, x, h, w, done);
    std::vector<float> next = halved(x, h, w, halve);
    x = next;
    skips.push_back(std::move(next));
    h /= 2;
    w /= 2;
  }
  run_level(n.body, x, h, w, done);
  for (const auto& [dbl, blocks] : n.up) {
    const std::vector<float>& skip = skips.back();
    for (size_t i = 0; i < x.size(); i++) x[i] += skip[i];
    skips.pop_back();
    x = doubled(x, h, w, dbl);
    h *= 2;
    w *= 2;
    run_level(blocks, x, h, w, done);
  }
  head(true);
  std::vector<float> out(h * w * 3);
  multiply(Input::conv(x.data(), h, w, DIM, DIM, 3), 0, h * w, n.tail, out.data(), 3, Act::None, false);
  std::vector<float> cropped(width * height * 3);
  for (size_t y = 0; y < height; y++)
    std::memcpy(&cropped[y * width * 3], &out[y * w * 3], width * 3 * sizeof(float));
  return cropped;
}

std::vector<float> Scunet::run_tiled(const float* image, size_t width, size_t height, size_t tile, size_t margin,
                                     const std::function<bool(float)>& progress) const {
  if (width == 0 || height == 0)
    throw Error(ERR_INPUT, "empty " + std::to_string(width) + " x " + std::to_string(height) + " image");
  if (tile == 0) throw Error(ERR_INPUT, "tile size 0");
  std::vector<float> out(width * height * 3);
  const size_t cols = (width + tile - 1) / tile, rows = (height + tile - 1) / tile;
  const float steps = (float)(cols * rows * STEPS);
  size_t done = 0;
  std::vector<float> region;
  for (size_t j = 0; j < rows; j++) {
    const size_t y0 = j * height / rows, y1 = (j + 1) * height / rows;
    for (size_t i = 0; i < cols; i++) {
      const size_t x0 = i * width / cols, x1 = (i + 1) * width / cols;
      const size_t rx0 = x0 > margin ? x0 - margin : 0, ry0 = y0 > margin ? y0 - margin : 0;
      const size_t rx1 = margin > width - x1 ? width : x1 + margin;
      const size_t ry1 = margin > height - y1 ? height : y1 + margin;
      const size_t rw = rx1 - rx0;
      region.clear();
      for (size_t y = ry0; y < ry1; y++)
        region.insert(region.end(), image + (y * width + rx0) * 3, image + (y * width + rx0 + rw) * 3);
      std::vector<float> result = run(region.data(), rw, ry1 - ry0, [&]() {
        done++;
        return !progress || progress((float)done / steps);
      });
      for (size_t y = y0; y < y1; y++)
        std::memcpy(&out[(y * width + x0) * 3], &result[((y - ry0) * rw + x0 - rx0) * 3], (x1 - x0) * 3 * sizeof(float));
    }
  }
  return out;
}

}  // namespace ref
