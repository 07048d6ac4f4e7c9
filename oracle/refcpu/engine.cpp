// Test infrastructure: CPU restatement of crates/native-engine (see engine.h).
// Built with -ffp-contract=off so that only the explicit fmaf() calls fuse,
// as the reference's AVX2 tier fuses only inside its matrix kernel.
#include "engine.h"

#include <cmath>
#include <cstring>
#include <fstream>
#include <iterator>
#include <omp.h>

namespace ref {

bool g_direct = false;
static int g_threads = 0;

void set_threads(int n) {
  g_threads = n;
  if (n > 0) omp_set_num_threads(n);
}
int threads() { return g_threads > 0 ? g_threads : omp_get_max_threads(); }

// ---------------------------------------------------------------- half.rs:7-48
uint16_t f32_to_half(float v) {
  uint32_t x;
  std::memcpy(&x, &v, 4);
  uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
  uint32_t mant = x & 0x7fffff;
  if (((x >> 23) & 0xff) == 0xff) return sign | 0x7c00 | (mant == 0 ? 0 : 0x200);
  int e = (int)((x >> 23) & 0xff) - 112;
  auto round = [](uint32_t kept, uint32_t low, uint32_t shift) {
    uint32_t half = 1u << (shift - 1);
    return kept + ((low > half || (low == half && (kept & 1))) ? 1u : 0u);
  };
  if (e >= 31) return sign | 0x7c00;
  if (e <= 0) {
    if (e < -10) return sign;
    uint32_t sig = mant | 0x800000;
    uint32_t shift = (uint32_t)(14 - e);
    uint32_t low = sig & ((1u << shift) - 1);
    return sign | (uint16_t)round(sig >> shift, low, shift);
  }
  return sign | (uint16_t)round(((uint32_t)e << 10) | (mant >> 13), mant & 0x1fff, 13);
}

// half.rs:125-145
float half_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, bits;
  if (e == 0 && m == 0) {
    bits = sign;
  } else if (e == 0) {
    float mag = (float)m * 5.9604644775390625e-8f;  // 2^-24
    return sign ? -mag : mag;
  } else if (e == 0x1f) {
    bits = sign | 0x7f800000 | (m << 13);
  } else {
    bits = sign | ((e + 112) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// ------------------------------------------------------ weight_file.rs:40-145
WeightFile WeightFile::read(const std::string& path, const char magic[8]) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw Error(ERR_IO, path + ": cannot open");
  std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  return parse(bytes.data(), bytes.size(), magic);
}

WeightFile WeightFile::parse(const uint8_t* data, size_t len, const char magic[8]) {
  size_t at = 0;
  auto take = [&](size_t n) -> const uint8_t* {
    if (n > len - at) throw Error(ERR_WEIGHTS, "weights file is truncated");
    const uint8_t* p = data + at;
    at += n;
    return p;
  };
  auto u32 = [&]() { uint32_t v; std::memcpy(&v, take(4), 4); return v; };
  if (len < 8 || std::memcmp(take(8), magic, 8) != 0) {
    std::string kind(magic, 8);
    kind = kind.substr(0, kind.find('\0'));
    throw Error(ERR_WEIGHTS, "not a " + kind + " weights file");
  }
  uint32_t version = u32();
  if (version != 1)
    throw Error(ERR_WEIGHTS, "weights file version " + std::to_string(version) + ", expected 1");
  uint32_t count = u32();
  WeightFile wf;
  for (uint32_t i = 0; i < count; i++) {
    uint16_t name_len;
    std::memcpy(&name_len, take(2), 2);
    std::string name((const char*)take(name_len), name_len);
    const uint8_t* dr = take(2);
    uint8_t dtype = dr[0], rank = dr[1];
    size_t width;
    if (dtype == 0) width = 4;
    else if (dtype == 1) width = 2;
    else throw Error(ERR_WEIGHTS, name + ": unknown type " + std::to_string(dtype));
    Weights w;
    w.half = dtype == 1;
    size_t n = 1;
    for (int r = 0; r < rank; r++) {
      size_t d = u32();
      if (d != 0 && n > SIZE_MAX / d) throw Error(ERR_WEIGHTS, name + ": too large");
      n *= d;
      w.shape.push_back(d);
    }
    if (n > SIZE_MAX / width) throw Error(ERR_WEIGHTS, name + ": too large");
    const uint8_t* p = take(n * width);
    w.values.resize(n);
    if (width == 4) {
      std::memcpy(w.values.data(), p, n * 4);
    } else {
      for (size_t j = 0; j < n; j++) {
        uint16_t h;
        std::memcpy(&h, p + 2 * j, 2);
        w.values[j] = half_to_f32(h);
      }
    }
    if (!wf.tensors_.emplace(name, std::move(w)).second)
      throw Error(ERR_WEIGHTS, name + ": stored twice");
  }
  if (at != len) throw Error(ERR_WEIGHTS, "trailing bytes after the last tensor");
  return wf;
}

static std::string shape_str(const std::vector<size_t>& s) {
  std::string out = "[";
  for (size_t i = 0; i < s.size(); i++) out += (i ? ", " : "") + std::to_string(s[i]);
  return out + "]";
}

Weights WeightFile::take_weights(const std::string& name, const std::vector<size_t>& shape) {
  auto it = tensors_.find(name);
  if (it == tensors_.end()) throw Error(ERR_WEIGHTS, name + ": missing");
  if (it->second.shape != shape)
    throw Error(ERR_WEIGHTS, name + ": shape " + shape_str(it->second.shape) + ", expected " +
                                 shape_str(shape));
  Weights w = std::move(it->second);
  tensors_.erase(it);
  return w;
}

void WeightFile::finish() const {
  if (!tensors_.empty()) throw Error(ERR_WEIGHTS, tensors_.begin()->first + ": not used by this model");
}

// ------------------------------------------------------------ gemm.rs:98-147
Matrix::Matrix(const Weights& wt, size_t k_, size_t n_, const std::vector<float>* b)
    : Matrix(wt.values, k_, n_, b, wt.half) {}

Matrix::Matrix(std::vector<float> w_, size_t k_, size_t n_, const std::vector<float>* b, bool h)
    : k(k_), n(n_), half(h), w(std::move(w_)), bias(n_, 0.0f) {
  if (w.size() != k * n) throw Error(ERR_WEIGHTS, "weights are not " + std::to_string(k) + " x " + std::to_string(n));
  if (b) {
    if (b->size() != n) throw Error(ERR_WEIGHTS, "bias is not " + std::to_string(n) + " long");
    bias = *b;
  }
}

// ------------------------------------------------------------ gemm.rs:290-441
Input Input::rows(const float* d, size_t s) {
  Input in;
  in.kind = Rows;
  in.data = d;
  in.stride = s;
  return in;
}

Input Input::conv(const float* d, size_t h, size_t w, size_t c, size_t s, size_t size, size_t step, Pad pad) {
  Input in;
  in.kind = Image;
  in.data = d;
  in.height = h;
  in.width = w;
  in.channels = c;
  in.stride = s;
  in.taps = Conv;
  in.size = size;
  in.step = step;
  in.pad = pad;
  return in;
}

Input Input::phase(const float* d, size_t h, size_t w, size_t c, size_t s, const size_t (*offs)[2], size_t count) {
  Input in;
  in.kind = Image;
  in.data = d;
  in.height = h;
  in.width = w;
  in.channels = c;
  in.stride = s;
  in.taps = Offsets;
  in.count = count;
  for (size_t i = 0; i < count; i++) {
    in.offsets[i][0] = offs[i][0];
    in.offsets[i][1] = offs[i][1];
  }
  return in;
}

void Input::out_size(size_t* oh, size_t* ow) const {
  if (taps == Conv) {
    *oh = (height - 1) / step + 1;
    *ow = (width - 1) / step + 1;
  } else {
    *oh = height;
    *ow = width;
  }
}

size_t Input::tap_count() const {
  if (kind == Rows) return 1;
  return taps == Conv ? size * size : count;
}

const float* Input::at(size_t r, size_t t) const {
  if (kind == Rows) return data + r * stride;
  size_t oh, ow;
  out_size(&oh, &ow);
  size_t oy = r / ow, ox = r % ow;
  long y, x;
  if (taps == Conv) {
    long half = (long)(size / 2);
    y = (long)(oy * step + t / size) - half;
    x = (long)(ox * step + t % size) - half;
    bool inside = y >= 0 && y < (long)height && x >= 0 && x < (long)width;
    if (!inside) {
      if (pad == Pad::Zero) return nullptr;
      y = (long)reflect(y, height);
      x = (long)reflect(x, width);
    }
  } else {
    y = (long)(oy + offsets[t][0]);
    x = (long)(ox + offsets[t][1]);
    if (y >= (long)height || x >= (long)width) return nullptr;
  }
  return data + ((size_t)y * width + (size_t)x) * stride;
}

// ------------------------------------------------------------ gemm.rs:514-667
// The AVX2 kernel keeps, per output, acc = (accumulate ? old : 0) + bias and
// then one fused multiply-add per reduction element in tap-major, channel-
// minor order; blocks of the reduction store and reload the partial sum in
// f32, which changes nothing. ReLU applies at the last store, GELU after.
namespace {
void multiply_rows(const Input& input, size_t r0, size_t r1, long first, long last, const Matrix& w, float* out,
                   size_t stride, Act act, bool accumulate, std::vector<float>& acc, std::vector<const float*>& ptrs) {
  const size_t taps = input.tap_count();
  const size_t channels = input.kind == Input::Rows ? w.k : input.channels;
  const size_t n = w.n;
  const float* W = w.w.data();
  const float* B = w.bias.data();
  acc.resize(n);
  ptrs.resize(taps);
  for (long r = first; r < last; r++) {
    float* o = out + (size_t)(r - (long)r0) * stride;
    for (size_t j = 0; j < n; j++) acc[j] = (accumulate ? o[j] : 0.0f) + B[j];
    for (size_t t = 0; t < taps; t++) ptrs[t] = input.at((size_t)r, t);
    float* a_ = acc.data();
    for (size_t t = 0; t < taps; t++) {
      const float* p = ptrs[t];
      const float* wt = W + t * channels * n;
      for (size_t c = 0; c < channels; c++) {
        float a = p ? p[c] : 0.0f;
        const float* wr = wt + c * n;
        for (size_t j = 0; j < n; j++) a_[j] = std::fma(a, wr[j], a_[j]);
      }
    }
    if (act == Act::Relu)
      for (size_t j = 0; j < n; j++) o[j] = acc[j] > 0.0f ? acc[j] : 0.0f;
    else
      for (size_t j = 0; j < n; j++) o[j] = acc[j];
    if (act == Act::Gelu)
      for (size_t j = 0; j < n; j++) o[j] = gelu_one(o[j]);
  }
}

void check_multiply(const Input& input, const Matrix& w) {
  const size_t taps = input.tap_count();
  const size_t channels = input.kind == Input::Rows ? w.k : input.channels;
  if (taps * channels != w.k) throw Error(ERR_INPUT, "input does not match the weights");
}
}  // namespace

void multiply(const Input& input, size_t r0, size_t r1, const Matrix& w, float* out, size_t stride,
              Act act, bool accumulate) {
  if (r1 <= r0) return;
  check_multiply(input, w);
#pragma omp parallel
  {
    std::vector<float> acc;
    std::vector<const float*> ptrs;
#pragma omp for schedule(dynamic, 16)
    for (long r = (long)r0; r < (long)r1; r++)
      multiply_rows(input, r0, r1, r, r + 1, w, out, stride, act, accumulate, acc, ptrs);
  }
}

void multiply_serial(const Input& input, size_t r0, size_t r1, const Matrix& w, float* out, size_t stride,
                     Act act, bool accumulate) {
  if (r1 <= r0) return;
  check_multiply(input, w);
  std::vector<float> acc;
  std::vector<const float*> ptrs;
  multiply_rows(input, r0, r1, (long)r0, (long)r1, w, out, stride, act, accumulate, acc, ptrs);
}

// -------------------------------------------------------- winograd.rs:53-773
namespace {

constexpr size_t MIN_CHANNELS = 16;  // winograd.rs:53
constexpr size_t F4_CHANNELS = 576;  // winograd.rs:56

// F(2x2,3x3): winograd.rs:179-352.
struct F2 {
  static constexpr size_t BLOCK = 2, SIDE = 4, POINTS = 16;
  // G g G^T for one (cin, cout) pair: g holds the 3x3 taps row by row.
  static void weight(const float g[9], float v[16]) {
    float t[4][3];
    for (int x = 0; x < 3; x++) {
      float g0 = g[x], g1 = g[3 + x], g2 = g[6 + x];
      t[0][x] = g0;
      t[1][x] = 0.5f * (g0 + g1 + g2);
      t[2][x] = 0.5f * (g0 - g1 + g2);
      t[3][x] = g2;
    }
    for (int y = 0; y < 4; y++) {
      float t0 = t[y][0], t1 = t[y][1], t2 = t[y][2];
      v[4 * y] = t0;
      v[4 * y + 1] = 0.5f * (t0 + t1 + t2);
      v[4 * y + 2] = 0.5f * (t0 - t1 + t2);
      v[4 * y + 3] = t2;
    }
  }
  // B^T d B: d = 16 pixel pointers row by row, u = 16 runs of cin.
  static void input(const float* const* d, float* u, size_t cin) {
    for (size_t c = 0; c < cin; c++) {
      float q[4][4];
      for (int a = 0; a < 4; a++) {
        float v0 = d[4 * a][c], v1 = d[4 * a + 1][c], v2 = d[4 * a + 2][c], v3 = d[4 * a + 3][c];
        q[a][0] = v0 - v2;
        q[a][1] = v1 + v2;
        q[a][2] = v2 - v1;
        q[a][3] = v1 - v3;
      }
      for (int x = 0; x < 4; x++) {
        u[x * cin + c] = q[0][x] - q[2][x];
        u[(4 + x) * cin + c] = q[1][x] + q[2][x];
        u[(8 + x) * cin + c] = q[2][x] - q[1][x];
        u[(12 + x) * cin + c] = q[1][x] - q[3][x];
      }
    }
  }
  // A^T m A + bias: m = 16 runs of cout, y = 4 pixels row by row.
  static void output(const float* m, const float* bias, float* y, size_t cout) {
    for (size_t c = 0; c < cout; c++) {
      float s[4][2];
      for (int i = 0; i < 4; i++) {
        float v0 = m[(4 * i) * cout + c], v1 = m[(4 * i + 1) * cout + c];
        float v2 = m[(4 * i + 2) * cout + c], v3 = m[(4 * i + 3) * cout + c];
        s[i][0] = v0 + v1 + v2;
        s[i][1] = v1 - v2 - v3;
      }
      for (int x = 0; x < 2; x++) {
        y[x * cout + c] = s[0][x] + s[1][x] + s[2][x] + bias[c];
        y[(2 + x) * cout + c] = s[1][x] - s[2][x] - s[3][x] + bias[c];
      }
    }
  }
};

// F(4x4,3x3): winograd.rs:355-604.
struct F4 {
  static constexpr size_t BLOCK = 4, SIDE = 6, POINTS = 36;
  static void g_column(float a, float b, float c, float out[6]) {
    out[0] = a / 4.0f;
    out[1] = -(a + b + c) / 6.0f;
    out[2] = -(a - b + c) / 6.0f;
    out[3] = a / 24.0f + b / 12.0f + c / 6.0f;
    out[4] = a / 24.0f - b / 12.0f + c / 6.0f;
    out[5] = c;
  }
  static void weight(const float g[9], float v[36]) {
    float t[6][3];
    for (int x = 0; x < 3; x++) {
      float col[6];
      g_column(g[x], g[3 + x], g[6 + x], col);
      for (int r = 0; r < 6; r++) t[r][x] = col[r];
    }
    for (int y = 0; y < 6; y++) {
      float row[6];
      g_column(t[y][0], t[y][1], t[y][2], row);
      for (int x = 0; x < 6; x++) v[6 * y + x] = row[x];
    }
  }
  static inline void b_t(const float v[6], float o[6]) {
    float a = v[4] - 4.0f * v[2];
    float b = v[3] - 4.0f * v[1];
    float c = v[4] - v[2];
    float e = 2.0f * (v[3] - v[1]);
    o[0] = 4.0f * v[0] - 5.0f * v[2] + v[4];
    o[1] = a + b;
    o[2] = a - b;
    o[3] = c + e;
    o[4] = c - e;
    o[5] = 4.0f * v[1] - 5.0f * v[3] + v[5];
  }
  static inline void a_t(const float v[6], float bias, float o[4]) {
    float s = v[1] + v[2];
    float d = v[1] - v[2];
    float s2 = v[3] + v[4];
    float d2 = v[3] - v[4];
    o[0] = v[0] + s + s2 + bias;
    o[1] = d + 2.0f * d2 + bias;
    o[2] = s + 4.0f * s2 + bias;
    o[3] = d + 8.0f * d2 + v[5] + bias;
  }
  static void input(const float* const* d, float* u, size_t cin) {
    for (size_t c = 0; c < cin; c++) {
      float rows[6][6];
      for (int y = 0; y < 6; y++) {
        float v[6];
        for (int x = 0; x < 6; x++) v[x] = d[6 * y + x][c];
        b_t(v, rows[y]);
      }
      for (int x = 0; x < 6; x++) {
        float v[6], col[6];
        for (int y = 0; y < 6; y++) v[y] = rows[y][x];
        b_t(v, col);
        for (int y = 0; y < 6; y++) u[(6 * y + x) * cin + c] = col[y];
      }
    }
  }
  static void output(const float* m, const float* bias, float* y, size_t cout) {
    for (size_t c = 0; c < cout; c++) {
      float rows[6][4];
      for (int i = 0; i < 6; i++) {
        float v[6];
        for (int x = 0; x < 6; x++) v[x] = m[(6 * i + x) * cout + c];
        a_t(v, 0.0f, rows[i]);
      }
      for (int x = 0; x < 4; x++) {
        float v[6], col[4];
        for (int i = 0; i < 6; i++) v[i] = rows[i][x];
        a_t(v, bias[c], col);
        for (int i = 0; i < 4; i++) y[(4 * i + x) * cout + c] = col[i];
      }
    }
  }
};

template <class F>
void winograd(const Input& in, const Matrix& w, float* out, size_t stride, bool accumulate,
              const std::function<void(float*)>& finish) {
  const size_t cin = in.channels, cout = w.n, H = in.height, Wd = in.width;
  constexpr size_t P = F::POINTS, S = F::SIDE, BL = F::BLOCK;
  // winograd.rs:107-146: the transformed weights, [point][cin][cout]; from
  // half-float weights, rounded to half floats.
  std::vector<float> V(P * cin * cout);
#pragma omp parallel for schedule(static)
  for (long c = 0; c < (long)cin; c++) {
    float g[9], v[36];
    for (size_t o = 0; o < cout; o++) {
      for (int t = 0; t < 9; t++) g[t] = w.w[((size_t)t * cin + (size_t)c) * cout + o];
      F::weight(g, v);
      for (size_t p = 0; p < P; p++) {
        float x = v[p];
        if (w.half) x = half_to_f32(f32_to_half(x));
        V[(p * cin + (size_t)c) * cout + o] = x;
      }
    }
  }
  const size_t by_n = (H + BL - 1) / BL, bx_n = (Wd + BL - 1) / BL, blocks = by_n * bx_n;
  std::vector<float> zeros(cin, 0.0f);
#pragma omp parallel
  {
    std::vector<float> u(P * cin), m(P * cout), y(BL * BL * cout);
    const float* d[36];
#pragma omp for schedule(dynamic, 8)
    for (long b = 0; b < (long)blocks; b++) {
      size_t by = (size_t)b / bx_n, bx = (size_t)b % bx_n;
      for (size_t k = 0; k < P; k++) {
        long py = (long)(BL * by + k / S) - 1, px = (long)(BL * bx + k % S) - 1;
        auto near = [](long i, size_t n) { return i >= -1 && i <= (long)n; };
        auto inside = [](long i, size_t n) { return i >= 0 && i < (long)n; };
        if (in.pad == Pad::Reflect && near(py, H) && near(px, Wd)) {
          d[k] = in.data + (reflect(py, H) * Wd + reflect(px, Wd)) * in.stride;
        } else if (inside(py, H) && inside(px, Wd)) {
          d[k] = in.data + ((size_t)py * Wd + (size_t)px) * in.stride;
        } else {
          d[k] = zeros.data();
        }
      }
      F::input(d, u.data(), cin);
      // The 16 or 36 products, each a chain of fused multiply-adds from 0.
      for (size_t p = 0; p < P; p++) {
        float* mp = m.data() + p * cout;
        for (size_t o = 0; o < cout; o++) mp[o] = 0.0f;
        const float* up = u.data() + p * cin;
        const float* Vp = V.data() + p * cin * cout;
        for (size_t c = 0; c < cin; c++) {
          float a = up[c];
          const float* vr = Vp + c * cout;
          for (size_t o = 0; o < cout; o++) mp[o] = std::fma(a, vr[o], mp[o]);
        }
      }
      F::output(m.data(), w.bias.data(), y.data(), cout);
      for (size_t corner = 0; corner < BL * BL; corner++) {
        size_t py = BL * by + corner / BL, px = BL * bx + corner % BL;
        if (py >= H || px >= Wd) continue;
        float* pixel = out + (py * Wd + px) * stride;
        const float* vals = y.data() + corner * cout;
        if (accumulate)
          for (size_t o = 0; o < cout; o++) pixel[o] += vals[o];
        else
          std::memcpy(pixel, vals, cout * sizeof(float));
        if (finish) finish(pixel);
      }
    }
  }
}

}  // namespace

void conv3(const Input& in, const Matrix& w, float* out, size_t stride, bool accumulate,
           const std::function<void(float*)>& finish) {
  if (in.kind != Input::Image || in.taps != Input::Conv || in.size != 3 || in.step != 1)
    throw Error(ERR_INPUT, "Winograd's convolution needs a 3x3 stride-1 convolution");
  const size_t cin = in.channels, cout = w.n, pixels = in.height * in.width;
  if (w.k != 9 * cin || in.stride < cin || stride < cout)
    throw Error(ERR_INPUT, "convolution sizes do not match");
  if (g_direct || cin < MIN_CHANNELS) {
    multiply(in, 0, pixels, w, out, stride, Act::None, accumulate);
    if (finish) {
#pragma omp parallel for schedule(static)
      for (long p = 0; p < (long)pixels; p++) finish(out + (size_t)p * stride);
    }
    return;
  }
  if (cin + cout <= F4_CHANNELS)
    winograd<F4>(in, w, out, stride, accumulate, finish);
  else
    winograd<F2>(in, w, out, stride, accumulate, finish);
}

// ----------------------------------------------------------------- math.rs
// The reference evaluates exp by XNNPACK's p5 polynomial and erf by Eigen's
// rational fit (both within 5e-7 of the functions); this restatement calls
// libm's, a difference far below every parity tolerance.
float exp_neg(float x) { return std::exp(x); }
float sigmoid_one(float x) {
  float e = std::exp(-std::fabs(x));
  float s = e / (e + 1.0f);
  return x > 0.0f ? 1.0f - s : s;
}
float gelu_one(float x) { return 0.5f * x * (1.0f + std::erf(x * 0.70710678118654752f)); }

}  // namespace ref

namespace ref {

static float lane_sum(const float* v, size_t n) {
  float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t whole = n / 8 * 8;
  for (size_t i = 0; i < whole; i += 8)
    for (int l = 0; l < 8; l++) lanes[l] += v[i + l];
  float total = ((lanes[0] + lanes[4]) + (lanes[1] + lanes[5])) + ((lanes[2] + lanes[6]) + (lanes[3] + lanes[7]));
  for (size_t i = whole; i < n; i++) total += v[i];
  return total;
}

void layer_norm_row(float* x, size_t n, const float* gamma, const float* beta) {
  const float fn = (float)n;
  const float mean = lane_sum(x, n) / fn;
  float sq[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t whole = n / 8 * 8;
  for (size_t i = 0; i < whole; i += 8)
    for (int l = 0; l < 8; l++) {
      float d = x[i + l] - mean;
      sq[l] += d * d;
    }
  float var = lane_sum(sq, 8);
  for (size_t i = whole; i < n; i++) {
    float d = x[i] - mean;
    var += d * d;
  }
  const float inv = 1.0f / std::sqrt(var / fn + 1e-5f);
  for (size_t i = 0; i < n; i++) x[i] = (x[i] - mean) * inv * gamma[i] + beta[i];
}

void softmax_from(float* x, size_t n, float max) {
  for (size_t i = 0; i < n; i++) x[i] = exp_neg(x[i] - max);
  const float inv = 1.0f / lane_sum(x, n);
  for (size_t i = 0; i < n; i++) x[i] *= inv;
}

void attention(const float* qkv, size_t c, size_t head, const float* bias, size_t tokens, float* out) {
  constexpr size_t D = 32;
  const float scale = 1.0f / std::sqrt((float)D);
  const size_t q0 = head * D, k0 = c + head * D, v0 = 2 * c + head * D;
  std::vector<float> s(tokens);
  for (size_t i = 0; i < tokens; i++) {
    const float* q = qkv + i * 3 * c + q0;
    for (size_t j = 0; j < tokens; j++) s[j] = 0.0f;
    for (size_t d = 0; d < D; d++) {
      const float a = q[d] * scale;
      for (size_t j = 0; j < tokens; j++) s[j] = std::fma(a, qkv[j * 3 * c + k0 + d], s[j]);
    }
    float max = -INFINITY;
    for (size_t j = 0; j < tokens; j++) {
      s[j] += bias[i * tokens + j];
      max = s[j] > max ? s[j] : max;
    }
    softmax_from(s.data(), tokens, max);
    float acc[D];
    for (size_t d = 0; d < D; d++) acc[d] = 0.0f;
    for (size_t j = 0; j < tokens; j++) {
      const float* v = qkv + j * 3 * c + v0;
      for (size_t d = 0; d < D; d++) acc[d] = std::fma(s[j], v[d], acc[d]);
    }
    for (size_t d = 0; d < D; d++) out[i * c + head * D + d] = acc[d];
  }
}

}  // namespace ref
