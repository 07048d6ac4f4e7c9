// Test infrastructure: CPU restatement of the reference's Big LaMa
// (crates/lama-native) on the engine restatement.
//   network.rs:32-44    128 local + 384 global channels, 18 blocks, sides padded to 8, 26 steps
//   network.rs:151-248  Ffc::load / run: local conv3 (512 -> 128, ReLU), cross conv3
//                       (128 -> 384), spectral_in 1x1 (384 -> 192, ReLU), rfft2, fourier
//                       1x1 (384 -> 384, ReLU), irfft2 added onto the spectral input,
//                       spectral_out 1x1 (192 -> 384) accumulated, then ReLU
//   network.rs:271-333  Up: a 3x3 stride-2 transposed convolution as 4 phase products
//   network.rs:348-370  masked_rows: image * (1 - m), m; symmetric padding
//   network.rs:381-489  load / run: conv7 reflect, 3 conv3 stride-2 reflect, blocks,
//                       3 ups, conv7 reflect + sigmoid, crop
//   fourier.rs:16-436   rfftn / irfftn over the two spatial axes, "ortho": restated
//                       from their definition (the sums of the transforms), the
//                       inverse reading only the real part of the first column and,
//                       for an even width, of the last
//   lib.rs:139-194      compositing of the 8-bit run, check_size (sides >= 9)
#include <array>
#include <cmath>
#include <cstring>

#include "refcpu.h"

namespace ref {

namespace {
constexpr size_t LOCAL = 128, GLOBAL = 384, CHANNELS = 512, SPECTRAL = 192, BLOCKS = 18;

Matrix mat(WeightFile& f, const std::string& name, size_t k, size_t n, bool bias) {
  Weights w = f.take_weights(name + ".weight", {k, n});
  std::vector<float> b;
  if (bias) b = f.take(name + ".bias", {n});
  return Matrix(w, k, n, bias ? &b : nullptr);
}

}  // namespace

// The ortho 2-D real DFT of a h x w map of c channels (pixels `stride` apart
// from `x`): spectrum rows h x (w / 2 + 1), each pixel [re(c) | im(c)].
void rfft2(const float* x, size_t stride, size_t h, size_t w, size_t c, std::vector<float>& out) {
  const size_t half = w / 2 + 1;
  std::vector<double> cw(w), sw(w), ch(h), sh(h);
  for (size_t j = 0; j < w; j++) {
    cw[j] = std::cos(2 * M_PI * (double)j / (double)w);
    sw[j] = std::sin(2 * M_PI * (double)j / (double)w);
  }
  for (size_t j = 0; j < h; j++) {
    ch[j] = std::cos(2 * M_PI * (double)j / (double)h);
    sh[j] = std::sin(2 * M_PI * (double)j / (double)h);
  }
  // rows: R[y][k] = sum_x x[y][x] e^{-2 pi i k x / w}
  std::vector<double> rr(h * half * c), ri(h * half * c);
#pragma omp parallel for schedule(static)
  for (long y = 0; y < (long)h; y++)
    for (size_t k = 0; k < half; k++)
      for (size_t ch_ = 0; ch_ < c; ch_++) {
        double re = 0, im = 0;
        for (size_t xx = 0; xx < w; xx++) {
          const double v = x[((size_t)y * w + xx) * stride + ch_];
          const size_t j = (k * xx) % w;
          re += v * cw[j];
          im -= v * sw[j];
        }
        rr[((size_t)y * half + k) * c + ch_] = re;
        ri[((size_t)y * half + k) * c + ch_] = im;
      }
  const double scale = 1.0 / std::sqrt((double)(h * w));
  out.assign(h * half * 2 * c, 0.0f);
#pragma omp parallel for schedule(static)
  for (long ky = 0; ky < (long)h; ky++)
    for (size_t k = 0; k < half; k++)
      for (size_t ch_ = 0; ch_ < c; ch_++) {
        double re = 0, im = 0;
        for (size_t y = 0; y < h; y++) {
          const size_t j = ((size_t)ky * y) % h;
          const double a = rr[(y * half + k) * c + ch_], b = ri[(y * half + k) * c + ch_];
          // (a + i b) e^{-i t}
          re += a * ch[j] + b * sh[j];
          im += b * ch[j] - a * sh[j];
        }
        out[((size_t)ky * half + k) * 2 * c + ch_] = (float)(re * scale);
        out[((size_t)ky * half + k) * 2 * c + c + ch_] = (float)(im * scale);
      }
}

// The ortho inverse of rfft2, added onto `out` (pixels `stride` apart).
void irfft2_add(const std::vector<float>& spec, size_t h, size_t w, size_t c, float* out, size_t stride) {
  const size_t half = w / 2 + 1;
  std::vector<double> cw(w), sw(w), ch(h), sh(h);
  for (size_t j = 0; j < w; j++) {
    cw[j] = std::cos(2 * M_PI * (double)j / (double)w);
    sw[j] = std::sin(2 * M_PI * (double)j / (double)w);
  }
  for (size_t j = 0; j < h; j++) {
    ch[j] = std::cos(2 * M_PI * (double)j / (double)h);
    sh[j] = std::sin(2 * M_PI * (double)j / (double)h);
  }
  // columns: C[y][k] = sum_ky S[ky][k] e^{+2 pi i ky y / h}
  std::vector<double> cr(h * half * c), ci(h * half * c);
#pragma omp parallel for schedule(static)
  for (long y = 0; y < (long)h; y++)
    for (size_t k = 0; k < half; k++)
      for (size_t ch_ = 0; ch_ < c; ch_++) {
        double re = 0, im = 0;
        for (size_t ky = 0; ky < h; ky++) {
          const size_t j = (ky * (size_t)y) % h;
          const double a = spec[(ky * half + k) * 2 * c + ch_], b = spec[(ky * half + k) * 2 * c + c + ch_];
          re += a * ch[j] - b * sh[j];
          im += a * sh[j] + b * ch[j];
        }
        cr[((size_t)y * half + k) * c + ch_] = re;
        ci[((size_t)y * half + k) * c + ch_] = im;
      }
  // rows (Hermitian): x = C[0].re + (even w: C[w/2].re (-1)^x) + 2 sum_{0<k<w/2} Re(C[k] e^{+i})
  const double scale = 1.0 / std::sqrt((double)(h * w));
#pragma omp parallel for schedule(static)
  for (long y = 0; y < (long)h; y++)
    for (size_t xx = 0; xx < w; xx++)
      for (size_t ch_ = 0; ch_ < c; ch_++) {
        double v = cr[((size_t)y * half) * c + ch_];
        for (size_t k = 1; k < half; k++) {
          const double a = cr[((size_t)y * half + k) * c + ch_], b = ci[((size_t)y * half + k) * c + ch_];
          const size_t j = (k * xx) % w;
          if (2 * k == w)
            v += a * cw[j];  // the last column of an even width: real part only
          else
            v += 2.0 * (a * cw[j] - b * sw[j]);
        }
        out[((size_t)y * w + xx) * stride + ch_] += (float)(v * scale);
      }
}

namespace {

struct Ffc {
  Matrix local, cross, spectral_in, fourier, spectral_out;
  Ffc(WeightFile& f, const std::string& name)
      : local(mat(f, name + ".local", 9 * CHANNELS, LOCAL, true)),
        cross(mat(f, name + ".cross", 9 * LOCAL, GLOBAL, true)),
        spectral_in(mat(f, name + ".spectral_in", GLOBAL, SPECTRAL, true)),
        fourier(mat(f, name + ".fourier", 2 * SPECTRAL, 2 * SPECTRAL, true)),
        spectral_out(mat(f, name + ".spectral_out", SPECTRAL, GLOBAL, false)) {}

  // network.rs:174-248.
  void run(const std::vector<float>& x, std::vector<float>& out, size_t h, size_t w) const {
    const size_t pixels = h * w;
    conv3(Input::conv(x.data(), h, w, CHANNELS, CHANNELS, 3, 1, Pad::Reflect), local, out.data(), CHANNELS, false,
          [](float* px) {
            for (size_t k = 0; k < LOCAL; k++) px[k] = px[k] > 0.0f ? px[k] : 0.0f;
          });
    conv3(Input::conv(x.data(), h, w, LOCAL, CHANNELS, 3, 1, Pad::Reflect), cross, out.data() + LOCAL, CHANNELS,
          false, nullptr);
    std::vector<float> spectral(pixels * SPECTRAL);
    multiply(Input::rows(x.data() + LOCAL, CHANNELS), 0, pixels, spectral_in, spectral.data(), SPECTRAL, Act::Relu,
             false);
    std::vector<float> spectrum;
    rfft2(spectral.data(), SPECTRAL, h, w, SPECTRAL, spectrum);
    const size_t sp = h * (w / 2 + 1);
    std::vector<float> filtered(sp * 2 * SPECTRAL);
    multiply(Input::rows(spectrum.data(), 2 * SPECTRAL), 0, sp, fourier, filtered.data(), 2 * SPECTRAL, Act::Relu,
             false);
    irfft2_add(filtered, h, w, SPECTRAL, spectral.data(), SPECTRAL);
    multiply(Input::rows(spectral.data(), SPECTRAL), 0, pixels, spectral_out, out.data() + LOCAL, CHANNELS, Act::Relu,
             true);
  }
};

// network.rs:271: the offsets and taps of one output phase along an axis.
struct Up {
  std::vector<std::pair<Input, Matrix>> phases;  // Input data filled at run time
  std::vector<std::vector<std::array<size_t, 2>>> offsets;
  size_t cin, cout;
  Up(WeightFile& f, const std::string& name, size_t cin_, size_t cout_) : cin(cin_), cout(cout_) {
    const std::vector<size_t> taps[2] = {{0}, {0, 1}};  // offsets of phase 0 and 1 along an axis
    for (size_t p = 0; p < 4; p++) {
      std::vector<std::array<size_t, 2>> offs;
      for (size_t dy : taps[p / 2])
        for (size_t dx : taps[p % 2]) offs.push_back({dy, dx});
      Matrix m = mat(f, name + ".phase" + std::to_string(p), offs.size() * cin, cout, true);
      offsets.push_back(offs);
      phases.emplace_back(Input(), std::move(m));
    }
  }
  // network.rs:299-333: the doubled map through a ReLU.
  std::vector<float> run(const std::vector<float>& x, size_t h, size_t w) const {
    const size_t row = 2 * w * cout;
    std::vector<float> out(2 * h * row);
    for (size_t p = 0; p < 4; p++) {
      const size_t py = p / 2, px = p % 2;
      size_t offs[4][2];
      for (size_t t = 0; t < offsets[p].size(); t++) {
        offs[t][0] = offsets[p][t][0];
        offs[t][1] = offsets[p][t][1];
      }
      Input in = Input::phase(x.data(), h, w, cin, cin, offs, offsets[p].size());
#pragma omp parallel for schedule(static)
      for (long y = 0; y < (long)h; y++)
        multiply_serial(in, (size_t)y * w, ((size_t)y + 1) * w, phases[p].second,
                        out.data() + (2 * (size_t)y + py) * row + px * cout, 2 * cout, Act::Relu, false);
    }
    return out;
  }
};

}  // namespace

struct Lama::Impl {
  Matrix first, last;
  std::vector<Matrix> down;
  std::vector<std::pair<Ffc, Ffc>> blocks;
  std::vector<Up> up;
};

Lama::Lama(const std::string& path) : impl_(new Impl) {
  try {
    WeightFile f = WeightFile::read(path, std::string("LAMA\0\0\0\0", 8).c_str());
    impl_->first = mat(f, "first", 49 * 4, 64, true);
    const size_t dn[3][2] = {{64, 128}, {128, 256}, {256, CHANNELS}};
    for (int i = 0; i < 3; i++) impl_->down.push_back(mat(f, "down" + std::to_string(i), 9 * dn[i][0], dn[i][1], true));
    for (size_t b = 0; b < BLOCKS; b++)
      impl_->blocks.emplace_back(Ffc(f, "block" + std::to_string(b) + ".ffc0"), Ffc(f, "block" + std::to_string(b) + ".ffc1"));
    const size_t upc[3][2] = {{CHANNELS, 256}, {256, 128}, {128, 64}};
    for (int i = 0; i < 3; i++) impl_->up.emplace_back(f, "up" + std::to_string(i), upc[i][0], upc[i][1]);
    impl_->last = mat(f, "last", 49 * 64, 3, true);
    f.finish();
  } catch (...) {
    delete impl_;
    throw;
  }
}

Lama::~Lama() { delete impl_; }

void Lama::check_size(size_t image, size_t mask, size_t width, size_t height) {
  if (width < MIN_SIDE || height < MIN_SIDE)
    throw Error(ERR_INPUT, std::to_string(width) + " x " + std::to_string(height) + " image: sides of at least 9 pixels");
  if (width * height * 3 != image || width * height != mask)
    throw Error(ERR_INPUT, "image and mask sizes do not match");
}

std::vector<float> Lama::run(const float* image, const float* mask, size_t width, size_t height,
                             const std::function<bool()>& step) const {
  const Impl& n = *impl_;
  auto done = [&]() {
    if (step && !step()) throw Error(CANCELLED, "cancelled");
  };
  size_t h = (height + 7) / 8 * 8, w = (width + 7) / 8 * 8;
  // network.rs:348-370.
  std::vector<float> x(h * w * 4);
  for (size_t y = 0; y < h; y++) {
    const size_t sy = y < height ? y : 2 * height - 1 - y;
    for (size_t xx = 0; xx < w; xx++) {
      const size_t sx = xx < width ? xx : 2 * width - 1 - xx;
      const size_t p = sy * width + sx;
      const float m = mask[p];
      for (int c = 0; c < 3; c++) x[(y * w + xx) * 4 + c] = image[p * 3 + c] * (1.0f - m);
      x[(y * w + xx) * 4 + 3] = m;
    }
  }
  std::vector<float> a(h * w * 64);
  multiply(Input::conv(x.data(), h, w, 4, 4, 7, 1, Pad::Reflect), 0, h * w, n.first, a.data(), 64, Act::Relu, false);
  done();
  size_t channels = 64;
  for (const Matrix& m : n.down) {
    Input in = Input::conv(a.data(), h, w, channels, channels, 3, 2, Pad::Reflect);
    size_t nh, nw;
    in.out_size(&nh, &nw);
    std::vector<float> next(nh * nw * m.n);
    multiply(in, 0, nh * nw, m, next.data(), m.n, Act::Relu, false);
    a = std::move(next);
    h = nh;
    w = nw;
    channels = m.n;
    done();
  }
  std::vector<float> mid(h * w * CHANNELS), out(h * w * CHANNELS);
  for (const auto& [first, second] : n.blocks) {
    first.run(a, mid, h, w);
    second.run(mid, out, h, w);
    for (size_t i = 0; i < a.size(); i++) a[i] += out[i];
    done();
  }
  for (const Up& u : n.up) {
    a = u.run(a, h, w);
    h *= 2;
    w *= 2;
    done();
  }
  std::vector<float> rgb(h * w * 3);
  multiply(Input::conv(a.data(), h, w, 64, 64, 7, 1, Pad::Reflect), 0, h * w, n.last, rgb.data(), 3, Act::None, false);
  for (float& v : rgb) v = sigmoid_one(v);
  done();
  std::vector<float> cropped(width * height * 3);
  for (size_t y = 0; y < height; y++) std::memcpy(&cropped[y * width * 3], &rgb[y * w * 3], width * 3 * sizeof(float));
  return cropped;
}

}  // namespace ref
