// Test infrastructure: CPU restatement of the reference's BiRefNet-lite
// (crates/birefnet-native) on the engine restatement.
//   lib.rs:36-37,134-172    ImageNet normalisation table, the half-size copy,
//                           the two backbone passes, the decoder
//   lib.rs:175-187          check_size (side a positive multiple of 64)
//   swin.rs:19-51           window 7, shift 3, mask -100, bias tables
//   swin.rs:115-215         Swin-T backbone: embed, stages, features, merges
//   swin.rs:219-346         window attention (tokens past the map are zero rows,
//                           not normalised) and the MLP
//   swin.rs:366-404         patch merging, order (0,0), (1,0), (0,1), (1,1)
//   decoder.rs:25-313       ASPP with deformable branches and the pooled bias,
//                           the torchvision-style bilinear sample
//   decoder.rs:343-406      a decoder block (conv_in, ASPP, conv_out, gate)
//   decoder.rs:443-521      aligned-corner bilinear resize (ONNX Runtime)
//   decoder.rs:549-601      image patches stacked as channels
//   decoder.rs:605-752      the full-resolution branch as a composed 5x5
//                           convolution with exact edges
//   decoder.rs:753-926      the decoder
#include <cmath>
#include <cstring>
#include <memory>

#include "refcpu.h"

namespace ref {

namespace {

constexpr size_t WINDOW = 7, SHIFT = 3, NTOK = 49, HEAD = 32, INTER = 64, BRANCH = 256;
constexpr float MASKED = -100.0f;
const size_t STAGES[4][2] = {{96, 2}, {192, 2}, {384, 6}, {768, 2}};
const size_t SIZES[4] = {1, 1, 3, 7};
const size_t LEVELS[4][2] = {{1728, 768}, {960, 384}, {480, 192}, {240, 96}};

struct Norm {
  std::vector<float> g, b;
  void apply(float* x) const { layer_norm_row(x, g.size(), g.data(), b.data()); }
};

Norm norm(WeightFile& f, const std::string& name, size_t c) {
  return Norm{f.take(name + ".weight", {c}), f.take(name + ".bias", {c})};
}

Matrix linear(WeightFile& f, const std::string& name, size_t k, size_t n, bool bias) {
  Weights w = f.take_weights(name + ".weight", {k, n});
  std::vector<float> b;
  if (bias) b = f.take(name + ".bias", {n});
  return Matrix(w, k, n, bias ? &b : nullptr);
}

// swin.rs:31-51.
std::vector<float> bias_tables(const std::vector<float>& position, bool shifted) {
  if (!shifted) return position;
  auto region = [](size_t v, bool last) { return (last && v >= WINDOW - SHIFT) ? 1 : 0; };
  std::vector<float> t;
  t.reserve(position.size() * 4);
  const size_t heads = position.size() / (NTOK * NTOK);
  for (int cls = 0; cls < 4; cls++) {
    const bool last_col = cls & 1, last_row = cls & 2;
    auto id = [&](size_t i) { return region(i / WINDOW, last_row) * 2 + region(i % WINDOW, last_col); };
    for (size_t h = 0; h < heads; h++)
      for (size_t i = 0; i < NTOK; i++)
        for (size_t j = 0; j < NTOK; j++)
          t.push_back(position[(h * NTOK + i) * NTOK + j] + (id(i) == id(j) ? 0.0f : MASKED));
  }
  return t;
}

struct SwinBlock {
  Norm n1, n2;
  Matrix qkv, proj, fc1, fc2;
  std::vector<float> bias;
  size_t heads = 0;

  // swin.rs:219-306.
  void attend(std::vector<float>& x, size_t grid, size_t c, size_t shift) const {
    const size_t padded = (grid + WINDOW - 1) / WINDOW * WINDOW, windows = padded / WINDOW;
    float* map = x.data();
#pragma omp parallel for schedule(dynamic, 1)
    for (long w = 0; w < (long)(windows * windows); w++) {
      std::vector<float> tokens(NTOK * c), qkv_rows(NTOK * 3 * c), heads_out(NTOK * c, 0.0f);
      size_t source[NTOK];
      const size_t wy = (size_t)w / windows, wx = (size_t)w % windows;
      for (size_t i = 0; i < NTOK; i++) {
        const size_t py = wy * WINDOW + i / WINDOW, px = wx * WINDOW + i % WINDOW;
        const size_t y = (py + shift) % padded, xx = (px + shift) % padded;
        float* row = &tokens[i * c];
        if (y < grid && xx < grid) {
          source[i] = y * grid + xx;
          std::memcpy(row, map + source[i] * c, c * sizeof(float));
          n1.apply(row);
        } else {
          source[i] = SIZE_MAX;
          std::fill(row, row + c, 0.0f);
        }
      }
      multiply_serial(Input::rows(tokens.data(), c), 0, NTOK, qkv, qkv_rows.data(), 3 * c, Act::None, false);
      size_t cls = 0;
      if (shift > 0) cls = ((size_t)w % windows == windows - 1 ? 1 : 0) + 2 * ((size_t)w / windows == windows - 1 ? 1 : 0);
      for (size_t h = 0; h < heads; h++)
        attention(qkv_rows.data(), c, h, &bias[(cls * heads + h) * NTOK * NTOK], NTOK, heads_out.data());
      multiply_serial(Input::rows(heads_out.data(), c), 0, NTOK, proj, tokens.data(), c, Act::None, false);
      for (size_t i = 0; i < NTOK; i++) {
        if (source[i] == SIZE_MAX) continue;
        float* dst = map + source[i] * c;
        for (size_t k = 0; k < c; k++) dst[k] += tokens[i * c + k];
      }
    }
  }

  // swin.rs:308-346.
  void mlp(std::vector<float>& x, size_t c) const {
    const size_t tokens = x.size() / c;
    std::vector<float> normed(x);
#pragma omp parallel for schedule(static)
    for (long r = 0; r < (long)tokens; r++) n2.apply(&normed[(size_t)r * c]);
    std::vector<float> hidden(tokens * 4 * c);
    multiply(Input::rows(normed.data(), c), 0, tokens, fc1, hidden.data(), 4 * c, Act::Gelu, false);
    multiply(Input::rows(hidden.data(), 4 * c), 0, tokens, fc2, x.data(), c, Act::None, true);
  }
};

struct Stage {
  size_t c = 0;
  std::vector<SwinBlock> blocks;
  Norm norm;
  bool merge = false;
  Norm merge_norm;
  Matrix reduction;
};

// swin.rs:366-404.
std::vector<float> merge(const std::vector<float>& x, size_t grid, size_t c, const Norm& n, const Matrix& red) {
  const size_t half = grid / 2, tokens = half * half;
  std::vector<float> buf(tokens * 4 * c), out(tokens * 2 * c);
  const size_t order[4][2] = {{0, 0}, {1, 0}, {0, 1}, {1, 1}};
#pragma omp parallel for schedule(static)
  for (long r = 0; r < (long)tokens; r++) {
    const size_t y = 2 * ((size_t)r / half), xx = 2 * ((size_t)r % half);
    float* row = &buf[(size_t)r * 4 * c];
    for (int q = 0; q < 4; q++)
      std::memcpy(row + q * c, &x[((y + order[q][0]) * grid + xx + order[q][1]) * c], c * sizeof(float));
    n.apply(row);
  }
  multiply(Input::rows(buf.data(), 4 * c), 0, tokens, red, out.data(), 2 * c, Act::None, false);
  return out;
}

struct Backbone {
  Matrix embed;
  Norm embed_norm;
  std::vector<Stage> stages;

  explicit Backbone(WeightFile& f) {
    embed = linear(f, "patch_embed", 48, 96, true);
    embed_norm = norm(f, "patch_embed.norm", 96);
    for (size_t s = 0; s < 4; s++) {
      Stage st;
      st.c = STAGES[s][0];
      const size_t c = st.c, heads = c / HEAD;
      for (size_t b = 0; b < STAGES[s][1]; b++) {
        const std::string p = "stage" + std::to_string(s) + ".block" + std::to_string(b);
        SwinBlock blk;
        blk.heads = heads;
        blk.n1 = norm(f, p + ".norm1", c);
        blk.qkv = linear(f, p + ".qkv", c, 3 * c, true);
        blk.bias = bias_tables(f.take(p + ".position_bias", {heads, NTOK, NTOK}), b % 2 == 1);
        blk.proj = linear(f, p + ".proj", c, c, true);
        blk.n2 = norm(f, p + ".norm2", c);
        blk.fc1 = linear(f, p + ".fc1", c, 4 * c, true);
        blk.fc2 = linear(f, p + ".fc2", 4 * c, c, true);
        st.blocks.push_back(std::move(blk));
      }
      if (s < 3) {
        st.merge = true;
        st.merge_norm = norm(f, "stage" + std::to_string(s) + ".merge.norm", 4 * c);
        st.reduction = linear(f, "stage" + std::to_string(s) + ".merge", 4 * c, 2 * c, false);
      }
      st.norm = norm(f, "stage" + std::to_string(s) + ".norm", c);
      stages.push_back(std::move(st));
    }
  }

  // swin.rs:162-215.
  std::vector<std::vector<float>> run(const float* image, size_t side) const {
    size_t grid = side / 4;
    const size_t tokens = grid * grid;
    std::vector<float> patches(tokens * 48), x(tokens * 96);
#pragma omp parallel for schedule(static)
    for (long r = 0; r < (long)tokens; r++) {
      const size_t ty = (size_t)r / grid, tx = (size_t)r % grid;
      for (size_t ky = 0; ky < 4; ky++)
        std::memcpy(&patches[(size_t)r * 48 + ky * 12], &image[((ty * 4 + ky) * side + tx * 4) * 3], 12 * sizeof(float));
    }
    multiply(Input::rows(patches.data(), 48), 0, tokens, embed, x.data(), 96, Act::None, false);
#pragma omp parallel for schedule(static)
    for (long r = 0; r < (long)tokens; r++) embed_norm.apply(&x[(size_t)r * 96]);
    std::vector<std::vector<float>> features;
    for (const Stage& st : stages) {
      for (size_t b = 0; b < st.blocks.size(); b++) {
        st.blocks[b].attend(x, grid, st.c, b % 2 == 1 ? SHIFT : 0);
        st.blocks[b].mlp(x, st.c);
      }
      std::vector<float> feat(x);
#pragma omp parallel for schedule(static)
      for (long r = 0; r < (long)(x.size() / st.c); r++) st.norm.apply(&feat[(size_t)r * st.c]);
      features.push_back(std::move(feat));
      if (st.merge) {
        x = merge(x, grid, st.c, st.merge_norm, st.reduction);
        grid /= 2;
      }
    }
    return features;
  }
};

// decoder.rs:443-487.
void axis(size_t out, size_t len_in, size_t len_out, size_t* i0, size_t* i1, float* w0, float* w1) {
  float pos = len_out == 1 ? 0.0f : (float)out * (float)(len_in - 1) / (float)(len_out - 1);
  pos = std::min(std::max(pos, 0.0f), (float)(len_in - 1));
  *i0 = (size_t)pos;
  *i1 = std::min(*i0 + 1, len_in - 1);
  if (*i0 == *i1) {
    *w0 = 0.5f;
    *w1 = 0.5f;
  } else {
    *w0 = std::fabs(pos - (float)*i0);
    *w1 = std::fabs(pos - (float)*i1);
  }
}

}  // namespace

// decoder.rs:443-521: aligned-corner bilinear resize of a sh x sw x c map into
// columns 0..c of the dh x dw rows of `dst`, `stride` apart (added with `add`).
void resize(const float* src, size_t sh, size_t sw, size_t c, float* dst, size_t dh, size_t dw, size_t stride,
            bool add) {
#pragma omp parallel for schedule(static)
  for (long y = 0; y < (long)dh; y++) {
    size_t y1, y2;
    float dy1, dy2;
    axis((size_t)y, sh, dh, &y1, &y2, &dy1, &dy2);
    for (size_t x = 0; x < dw; x++) {
      size_t x1, x2;
      float dx1, dx2;
      axis(x, sw, dw, &x1, &x2, &dx1, &dx2);
      const float* p11 = src + (y1 * sw + x1) * c;
      const float* p21 = src + (y1 * sw + x2) * c;
      const float* p12 = src + (y2 * sw + x1) * c;
      const float* p22 = src + (y2 * sw + x2) * c;
      float* d = dst + ((size_t)y * dw + x) * stride;
      for (size_t j = 0; j < c; j++) {
        const float v = dx2 * dy2 * p11[j] + dx1 * dy2 * p21[j] + dx2 * dy1 * p12[j] + dx1 * dy1 * p22[j];
        d[j] = add ? d[j] + v : v;
      }
    }
  }
}

namespace {

void place(const std::vector<float>& src, size_t c, float* dst, size_t stride, size_t offset) {
  const size_t pixels = src.size() / c;
#pragma omp parallel for schedule(static)
  for (long p = 0; p < (long)pixels; p++)
    std::memcpy(dst + (size_t)p * stride + offset, &src[(size_t)p * c], c * sizeof(float));
}

Matrix conv_matrix(WeightFile& f, const std::string& name, size_t cin, size_t cout) {
  return linear(f, name, 9 * cin, cout, true);
}

// decoder.rs:424-438: 3x3 "same" convolution (Winograd on the CPU).
void conv(const std::vector<float>& x, size_t h, size_t w, size_t cin, const Matrix& m, float* out, size_t stride,
          bool relu) {
  std::function<void(float*)> fin;
  const size_t n = m.n;
  if (relu)
    fin = [n](float* px) {
      for (size_t k = 0; k < n; k++) px[k] = px[k] > 0.0f ? px[k] : 0.0f;
    };
  conv3(Input::conv(x.data(), h, w, cin, cin, 3, 1, Pad::Zero), m, out, stride, false, fin);
}

// decoder.rs:265-313.
void sample(const float* t, size_t height, size_t width, size_t y, size_t x, size_t size, const float* offsets,
            float* out) {
  const size_t taps = size * size;
  const float half = (float)(size / 2);
  const float h = (float)height, w = (float)width;
  for (size_t tap = 0; tap < taps; tap++) {
    float* dst = out + tap * INTER;
    const float py = ((float)y - half + (float)(tap / size)) + offsets[2 * tap];
    const float px = ((float)x - half + (float)(tap % size)) + offsets[2 * tap + 1];
    const float m = 2.0f * offsets[2 * taps + tap];
    if (py <= -1.0f || py >= h || px <= -1.0f || px >= w) {
      std::fill(dst, dst + INTER, 0.0f);
      continue;
    }
    const float y0f = std::floor(py), x0f = std::floor(px);
    const float ly = py - y0f, lx = px - x0f, hy = 1.0f - ly, hx = 1.0f - lx;
    const long y0 = (long)y0f, x0 = (long)x0f;
    const long cy[4] = {y0, y0, y0 + 1, y0 + 1}, cx[4] = {x0, x0 + 1, x0, x0 + 1};
    const float cw[4] = {hy * hx, hy * lx, ly * hx, ly * lx};
    std::fill(dst, dst + INTER, 0.0f);
    for (int k = 0; k < 4; k++) {
      if (cy[k] < 0 || cx[k] < 0 || cy[k] >= (long)height || cx[k] >= (long)width) continue;
      const float* v = t + ((size_t)cy[k] * width + (size_t)cx[k]) * INTER;
      for (size_t j = 0; j < INTER; j++) dst[j] += cw[k] * v[j];
    }
    for (size_t j = 0; j < INTER; j++) dst[j] *= m;
  }
}

struct Aspp {
  struct Branch {
    size_t size;
    Matrix offsets, weight;
  };
  std::vector<Branch> branches;
  std::vector<float> pool_w, pool_b, conv1_pool, conv1_bias;
  Matrix conv1;

  Aspp(WeightFile& f, const std::string& p) {
    for (size_t i = 0; i < 4; i++) {
      const size_t taps = SIZES[i] * SIZES[i], k = taps * INTER;
      const std::string b = p + ".branch" + std::to_string(i);
      branches.push_back({SIZES[i], linear(f, b + ".offset", k, 3 * taps, true), linear(f, b, k, BRANCH, true)});
    }
    pool_w = f.take(p + ".pool.weight", {INTER, BRANCH});
    pool_b = f.take(p + ".pool.bias", {BRANCH});
    Weights w = f.take_weights(p + ".conv1.weight", {5 * BRANCH, INTER});
    conv1_bias = f.take(p + ".conv1.bias", {INTER});
    Weights rows;
    rows.shape = {4 * BRANCH, INTER};
    rows.half = w.half;
    rows.values.assign(w.values.begin(), w.values.begin() + 4 * BRANCH * INTER);
    conv1 = Matrix(rows, 4 * BRANCH, INTER, nullptr);
    conv1_pool.assign(w.values.begin() + 4 * BRANCH * INTER, w.values.end());
  }

  // decoder.rs:138-236.
  std::vector<float> run(const std::vector<float>& t, size_t height, size_t width) const {
    const size_t pixels = height * width;
    std::vector<double> mean(INTER, 0.0);
    for (size_t p = 0; p < pixels; p++)
      for (size_t c = 0; c < INTER; c++) mean[c] += (double)t[p * INTER + c];
    std::vector<float> pooled(pool_b);
    for (size_t c = 0; c < INTER; c++) {
      const float m = (float)(mean[c] / (double)pixels);
      for (size_t j = 0; j < BRANCH; j++) pooled[j] += m * pool_w[c * BRANCH + j];
    }
    std::vector<float> bias(conv1_bias);
    for (size_t j = 0; j < BRANCH; j++) {
      const float p = pooled[j] > 0.0f ? pooled[j] : 0.0f;
      for (size_t k = 0; k < INTER; k++) bias[k] += p * conv1_pool[j * INTER + k];
    }
    std::vector<float> out(pixels * INTER);
    const size_t chunk = 48;
#pragma omp parallel for schedule(dynamic, 1)
    for (long c0 = 0; c0 < (long)pixels; c0 += chunk) {
      const size_t r0 = (size_t)c0, rows = std::min(chunk, pixels - r0);
      std::vector<float> offsets(rows * 3 * 49), samples(rows * 49 * INTER), cat(rows * 4 * BRANCH);
      for (size_t i = 0; i < branches.size(); i++) {
        const Branch& br = branches[i];
        const size_t taps = br.size * br.size;
        multiply_serial(Input::conv(t.data(), height, width, INTER, INTER, br.size, 1, Pad::Zero), r0, r0 + rows,
                        br.offsets, offsets.data(), 3 * taps, Act::None, false);
        for (size_t r = 0; r < rows; r++) {
          float* o = &offsets[r * 3 * taps];
          for (size_t k = 2 * taps; k < 3 * taps; k++) o[k] = sigmoid_one(o[k]);
          const size_t p = r0 + r;
          sample(t.data(), height, width, p / width, p % width, br.size, o, &samples[r * taps * INTER]);
        }
        multiply_serial(Input::rows(samples.data(), taps * INTER), 0, rows, br.weight, &cat[i * BRANCH], 4 * BRANCH,
                        Act::Relu, false);
      }
      float* o = &out[r0 * INTER];
      multiply_serial(Input::rows(cat.data(), 4 * BRANCH), 0, rows, conv1, o, INTER, Act::None, false);
      for (size_t r = 0; r < rows; r++)
        for (size_t k = 0; k < INTER; k++) {
          const float v = o[r * INTER + k] + bias[k];
          o[r * INTER + k] = v > 0.0f ? v : 0.0f;
        }
    }
    return out;
  }
};

struct DBlock {
  Matrix conv_in, conv_out;
  Aspp aspp;
  bool gated = false;
  Matrix gdt;
  std::vector<float> gw;
  float gb = 0.0f;

  DBlock(WeightFile& f, const std::string& p, size_t cin, size_t cout, bool gate)
      : conv_in(conv_matrix(f, p + ".conv_in", cin, INTER)),
        conv_out(conv_matrix(f, p + ".conv_out", INTER, cout)),
        aspp(f, p + ".aspp") {
    if (gate) {
      gated = true;
      gdt = conv_matrix(f, p + ".gdt", cout, 16);
      gw = f.take(p + ".gdt_attn.weight", {16, 1});
      gb = f.take(p + ".gdt_attn.bias", {1})[0];
    }
  }

  // decoder.rs:343-406.
  std::vector<float> run(const std::vector<float>& x, size_t h, size_t w, size_t cin) const {
    const size_t pixels = h * w;
    std::vector<float> t(pixels * INTER);
    conv(x, h, w, cin, conv_in, t.data(), INTER, true);
    t = aspp.run(t, h, w);
    const size_t cout = conv_out.n;
    std::vector<float> out(pixels * cout);
    conv(t, h, w, INTER, conv_out, out.data(), cout, false);
    if (gated) {
      std::vector<float> g(pixels * 16);
      multiply(Input::conv(out.data(), h, w, cout, cout, 3, 1, Pad::Zero), 0, pixels, gdt, g.data(), 16, Act::Relu,
               false);
#pragma omp parallel for schedule(static)
      for (long p = 0; p < (long)pixels; p++) {
        float s = gb;
        for (size_t k = 0; k < 16; k++) s = s + g[(size_t)p * 16 + k] * gw[k];
        const float gate = sigmoid_one(s);
        for (size_t k = 0; k < cout; k++) out[(size_t)p * cout + k] *= gate;
      }
    }
    return out;
  }
};

struct Patches {
  Matrix conv1, conv_out;
  // decoder.rs:549-601.
  void run(const float* image, size_t side, size_t size, float* out, size_t stride) const {
    const size_t grid = side / size, channels = 3 * grid * grid;
    std::vector<float> stacked(size * size * channels);
#pragma omp parallel for schedule(static)
    for (long p = 0; p < (long)(size * size); p++) {
      const size_t y = (size_t)p / size, x = (size_t)p % size;
      float* row = &stacked[(size_t)p * channels];
      size_t k = 0;
      for (size_t c = 0; c < 3; c++)
        for (size_t gy = 0; gy < grid; gy++)
          for (size_t gx = 0; gx < grid; gx++) row[k++] = image[((gy * size + y) * side + gx * size + x) * 3 + c];
    }
    std::vector<float> mid(size * size * INTER);
    conv(stacked, size, size, channels, conv1, mid.data(), INTER, false);
    conv(mid, size, size, INTER, conv_out, out, stride, false);
  }
};

struct FullRes {
  std::vector<float> conv1, bias1, conv_out, composed;
  float bias_out = 0.0f, composed_bias = 0.0f;

  explicit FullRes(WeightFile& f) {
    conv1 = f.take("patches1.conv1.weight", {27, INTER});
    bias1 = f.take("patches1.conv1.bias", {INTER});
    conv_out = f.take("patches1.conv_out.weight", {9 * INTER, 1});
    bias_out = f.take("patches1.conv_out.bias", {1})[0];
    std::vector<double> comp(25 * 3, 0.0);
    double cb = bias_out;
    for (size_t d = 0; d < 9; d++)
      for (size_t k = 0; k < INTER; k++) {
        const double w2 = conv_out[d * INTER + k];
        cb += w2 * (double)bias1[k];
        for (size_t e = 0; e < 9; e++) {
          const size_t ey = d / 3 + e / 3, ex = d % 3 + e % 3;
          for (size_t c = 0; c < 3; c++) comp[(ey * 5 + ex) * 3 + c] += w2 * (double)conv1[(e * 3 + c) * INTER + k];
        }
      }
    for (double v : comp) composed.push_back((float)v);
    composed_bias = (float)cb;
  }

  float exact(const float* image, long side, long y, long x) const {
    auto inside = [&](long yy, long xx) { return yy >= 0 && xx >= 0 && yy < side && xx < side; };
    float s = bias_out;
    for (long d = 0; d < 9; d++) {
      const long qy = y + d / 3 - 1, qx = x + d % 3 - 1;
      if (!inside(qy, qx)) continue;
      std::vector<float> mid(bias1);
      for (long e = 0; e < 9; e++) {
        const long py = qy + e / 3 - 1, px = qx + e % 3 - 1;
        if (!inside(py, px)) continue;
        const float* p = image + ((size_t)py * side + (size_t)px) * 3;
        for (size_t c = 0; c < 3; c++)
          for (size_t k = 0; k < INTER; k++) mid[k] += p[c] * conv1[((size_t)e * 3 + c) * INTER + k];
      }
      float dot = 0.0f;
      for (size_t k = 0; k < INTER; k++) dot += mid[k] * conv_out[(size_t)d * INTER + k];
      s += dot;
    }
    return s;
  }

  // decoder.rs:637-752.
  void add(const float* image, size_t side, float* out) const {
    const size_t width = side + 4, plane = width * width;
    std::vector<float> planes(3 * plane, 0.0f);
    for (size_t y = 0; y < side; y++)
      for (size_t c = 0; c < 3; c++)
        for (size_t x = 0; x < side; x++) planes[(c * width + y + 2) * width + 2 + x] = image[(y * side + x) * 3 + c];
#pragma omp parallel for schedule(static)
    for (long y = 0; y < (long)side; y++) {
      float* row = out + (size_t)y * side;
      if (y == 0 || y + 1 == (long)side) {
        for (size_t x = 0; x < side; x++) row[x] += exact(image, (long)side, y, (long)x);
        continue;
      }
      row[0] += exact(image, (long)side, y, 0);
      row[side - 1] += exact(image, (long)side, y, (long)side - 1);
      for (size_t x = 1; x + 1 < side; x++) {
        float s = composed_bias;
        for (size_t e = 0; e < 25; e++) {
          const size_t at = ((size_t)y + e / 5) * width + 1 + e % 5 + (x - 1);
          s += composed[e * 3] * planes[at] + composed[e * 3 + 1] * planes[plane + at] +
               composed[e * 3 + 2] * planes[2 * plane + at];
        }
        row[x] += s;
      }
    }
  }
};

struct Decoder {
  std::unique_ptr<DBlock> squeeze;
  std::vector<std::unique_ptr<DBlock>> blocks;
  std::vector<Matrix> laterals;
  std::vector<Patches> patches;
  Matrix head;
  float head_bias = 0.0f;
  std::unique_ptr<FullRes> full;

  explicit Decoder(WeightFile& f) {
    squeeze = std::make_unique<DBlock>(f, "squeeze", 2880, 1536, false);
    for (size_t i = 0; i < 4; i++)
      blocks.push_back(std::make_unique<DBlock>(f, "block" + std::to_string(4 - i), LEVELS[i][0], LEVELS[i][1], i < 3));
    const size_t lat[3][2] = {{4, 768}, {3, 384}, {2, 192}};
    for (auto& l : lat) laterals.push_back(linear(f, "lateral" + std::to_string(l[0]), l[1], l[1], true));
    const size_t pt[4][3] = {{5, 3072, 192}, {4, 768, 192}, {3, 192, 96}, {2, 48, 48}};
    for (auto& q : pt) {
      const std::string p = "patches" + std::to_string(q[0]);
      patches.push_back(Patches{conv_matrix(f, p + ".conv1", q[1], INTER), conv_matrix(f, p + ".conv_out", INTER, q[2])});
    }
    Weights hw = f.take_weights("head.weight", {96, 1});
    head = Matrix(hw, 96, 1, nullptr);
    head_bias = f.take("head.bias", {1})[0];
    full = std::make_unique<FullRes>(f);
  }

  // decoder.rs:790-926.
  std::vector<float> run(const float* image, size_t side, std::vector<std::vector<float>> fullf,
                         std::vector<std::vector<float>> halff) const {
    struct Level {
      std::vector<float> x;
      size_t grid, c;
    };
    std::vector<Level> levels;
    for (size_t i = 0; i < 4; i++) {
      const size_t grid = side >> (i + 2), c = fullf[i].size() / (grid * grid);
      Level L{std::vector<float>(grid * grid * 2 * c), grid, 2 * c};
      place(fullf[i], c, L.x.data(), 2 * c, 0);
      resize(halff[i].data(), grid / 2, grid / 2, c, L.x.data() + c, grid, grid, 2 * c, false);
      levels.push_back(std::move(L));
    }
    const size_t g4 = side >> 5;
    std::vector<float> x4(g4 * g4 * 2880);
    size_t offset = 0;
    for (size_t i = 0; i < 3; i++) {
      resize(levels[i].x.data(), levels[i].grid, levels[i].grid, levels[i].c, x4.data() + offset, g4, g4, 2880, false);
      offset += levels[i].c;
    }
    place(levels[3].x, levels[3].c, x4.data(), 2880, offset);
    std::vector<float> previous = squeeze->run(x4, g4, g4, 2880);
    size_t previous_grid = g4;
    for (size_t i = 0; i < 4; i++) {
      const size_t level = 3 - i, cin = LEVELS[i][0], grid = side >> (level + 2);
      std::vector<float> input(grid * grid * cin);
      const size_t main_c = i == 0 ? 1536 : LEVELS[i - 1][1];
      if (i == 0) {
        place(previous, main_c, input.data(), cin, 0);
      } else {
        const Level& L = levels[level];
        multiply(Input::rows(L.x.data(), L.c), 0, grid * grid, laterals[i - 1], input.data(), cin, Act::None, false);
        resize(previous.data(), previous_grid, previous_grid, main_c, input.data(), grid, grid, cin, true);
      }
      patches[i].run(image, side, grid, input.data() + main_c, cin);
      previous = blocks[i]->run(input, grid, grid, cin);
      previous_grid = grid;
    }
    const size_t pixels = previous_grid * previous_grid;
    std::vector<float> low(pixels);
    multiply(Input::rows(previous.data(), 96), 0, pixels, head, low.data(), 1, Act::None, false);
    std::vector<float> logits(side * side, head_bias);
    resize(low.data(), previous_grid, previous_grid, 1, logits.data(), side, side, 1, true);
    full->add(image, side, logits.data());
    return logits;
  }
};

}  // namespace

struct Birefnet::Impl {
  std::unique_ptr<Backbone> backbone;
  std::unique_ptr<Decoder> decoder;
};

Birefnet::Birefnet(const std::string& path) : impl_(new Impl) {
  try {
    WeightFile f = WeightFile::read(path, "BIREFNET");
    impl_->backbone = std::make_unique<Backbone>(f);
    impl_->decoder = std::make_unique<Decoder>(f);
    f.finish();
  } catch (...) {
    delete impl_;
    throw;
  }
}

Birefnet::~Birefnet() { delete impl_; }

void Birefnet::check_size(size_t len, size_t side) {
  if (side == 0 || side % 64 != 0)
    throw Error(ERR_INPUT, "side " + std::to_string(side) + " is not a positive multiple of 64");
  if (side * side * 3 != len) throw Error(ERR_INPUT, "values do not make a side x side RGB image");
}

// lib.rs:134-172.
std::vector<float> Birefnet::run_normalized(const float* image, size_t side) const {
  const size_t hs = side / 2;
  std::vector<float> half(hs * hs * 3);
  resize(image, side, side, 3, half.data(), hs, hs, 3, false);
  auto full_features = impl_->backbone->run(image, side);
  auto half_features = impl_->backbone->run(half.data(), hs);
  return impl_->decoder->run(image, side, std::move(full_features), std::move(half_features));
}

// lib.rs:36-37,116-133: the 8-bit image normalised through the table.
std::vector<float> Birefnet::normalize(const uint8_t* rgb, size_t pixels) {
  const float mean[3] = {0.485f, 0.456f, 0.406f}, std_[3] = {0.229f, 0.224f, 0.225f};
  float table[256][3];
  for (int v = 0; v < 256; v++)
    for (int c = 0; c < 3; c++) table[v][c] = ((float)v / 255.0f - mean[c]) / std_[c];
  std::vector<float> out(pixels * 3);
  for (size_t p = 0; p < pixels; p++)
    for (int c = 0; c < 3; c++) out[p * 3 + c] = table[rgb[p * 3 + c]][c];
  return out;
}

}  // namespace ref
