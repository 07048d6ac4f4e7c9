// Test infrastructure: a C interface to the CPU oracle, for ctypes in tests/
// and for bench.py's timed CPU baseline. Not part of the product.
#include <cstring>
#include <memory>
#include <string>

#include "refcpu.h"

using namespace ref;

namespace {
thread_local std::string g_error;

template <class F>
int guard(F&& f) {
  try {
    f();
    return OK;
  } catch (const Error& e) {
    g_error = e.what();
    return e.code;
  } catch (const std::exception& e) {
    g_error = e.what();
    return ERR_INPUT;
  }
}
}  // namespace

extern "C" {

typedef int (*refcpu_progress_fn)(float fraction, void* user);

const char* refcpu_last_error(void) { return g_error.c_str(); }
void refcpu_set_threads(int n) { set_threads(n); }
int refcpu_threads(void) { return threads(); }
void refcpu_set_direct(int direct) { g_direct = direct != 0; }

uint16_t refcpu_f32_to_half(float v) { return f32_to_half(v); }
float refcpu_half_to_f32(uint16_t h) { return half_to_f32(h); }

// Parse a weights file held in memory; returns the status and, on success,
// the number of tensors named `probe` with `rank`/`dims` that match (0/1).
int refcpu_parse_weights(const uint8_t* data, size_t len, const char* magic) {
  return guard([&] { WeightFile::parse(data, len, magic); });
}

// gemm.rs multiply over an image input (`kind` 0 rows, 1 conv, 2 phase).
// `w` is k x n row-major; `bias` may be null; act 0 none, 1 relu, 2 gelu.
int refcpu_multiply(int kind, const float* data, size_t height, size_t width, size_t channels,
                    size_t in_stride, size_t size, size_t step, int reflect_pad, const size_t* offsets,
                    size_t count, size_t r0, size_t r1, const float* w, size_t k, size_t n,
                    const float* bias, int half, float* out, size_t stride, int act, int accumulate) {
  return guard([&] {
    std::vector<float> wv(w, w + k * n);
    std::vector<float> bv;
    if (bias) bv.assign(bias, bias + n);
    Matrix m(std::move(wv), k, n, bias ? &bv : nullptr, half != 0);
    Input in;
    if (kind == 0) {
      in = Input::rows(data, in_stride);
    } else if (kind == 1) {
      in = Input::conv(data, height, width, channels, in_stride, size, step,
                       reflect_pad ? Pad::Reflect : Pad::Zero);
    } else {
      size_t offs[4][2];
      for (size_t i = 0; i < count; i++) {
        offs[i][0] = offsets[2 * i];
        offs[i][1] = offsets[2 * i + 1];
      }
      in = Input::phase(data, height, width, channels, in_stride, offs, count);
    }
    multiply(in, r0, r1, m, out, stride, act == 1 ? Act::Relu : act == 2 ? Act::Gelu : Act::None,
             accumulate != 0);
  });
}

// winograd.rs conv3: 3x3 stride-1 convolution, `finish` doubling channel 0 when
// `double_first` (the reference test's finishing closure, winograd.rs:836-838).
int refcpu_conv3(const float* data, size_t height, size_t width, size_t channels, size_t in_stride,
                 int reflect_pad, const float* w, size_t n, const float* bias, int half, float* out,
                 size_t stride, int accumulate, int double_first) {
  return guard([&] {
    std::vector<float> wv(w, w + 9 * channels * n);
    std::vector<float> bv;
    if (bias) bv.assign(bias, bias + n);
    Matrix m(std::move(wv), 9 * channels, n, bias ? &bv : nullptr, half != 0);
    Input in = Input::conv(data, height, width, channels, in_stride, 3, 1,
                           reflect_pad ? Pad::Reflect : Pad::Zero);
    std::function<void(float*)> fin;
    if (double_first) fin = [](float* p) { p[0] *= 2.0f; };
    conv3(in, m, out, stride, accumulate != 0, fin);
  });
}

// ---------------------------------------------------------------- Real-ESRGAN
int refcpu_realesrgan_load(const char* path, void** out) {
  return guard([&] { *out = new RealEsrgan(path); });
}
void refcpu_realesrgan_free(void* h) { delete static_cast<RealEsrgan*>(h); }

// Model::run_float on the CPU engine: the whole image at once.
int refcpu_realesrgan_run_float(void* h, const float* image, size_t width, size_t height, float* out) {
  return guard([&] {
    auto* m = static_cast<RealEsrgan*>(h);
    RealEsrgan::check_size(width * height * 3, width, height);
    std::vector<float> r = m->run(image, width, height, nullptr);
    std::memcpy(out, r.data(), r.size() * sizeof(float));
  });
}

// Model::run_float_tiled.
int refcpu_realesrgan_run_tiled(void* h, const float* image, size_t width, size_t height, size_t tile,
                                size_t margin, float* out, refcpu_progress_fn cb, void* user) {
  return guard([&] {
    auto* m = static_cast<RealEsrgan*>(h);
    std::function<bool(float)> progress;
    if (cb) progress = [cb, user](float f) { return cb(f, user) == 0; };
    std::vector<float> r = m->run_tiled(image, width, height, tile, margin, progress);
    std::memcpy(out, r.data(), r.size() * sizeof(float));
  });
}

// ---------------------------------------------------------------------- SCUNet
int refcpu_scunet_load(const char* path, void** out) {
  return guard([&] { *out = new Scunet(path); });
}
void refcpu_scunet_free(void* h) { delete static_cast<Scunet*>(h); }

// Model::run_float on the CPU engine: the whole image (padded to 64).
int refcpu_scunet_run_float(void* h, const float* image, size_t width, size_t height, float* out) {
  return guard([&] {
    if (width == 0 || height == 0) throw Error(ERR_INPUT, "empty image");
    std::vector<float> r = static_cast<Scunet*>(h)->run(image, width, height, nullptr);
    std::memcpy(out, r.data(), r.size() * sizeof(float));
  });
}

int refcpu_scunet_run_tiled(void* h, const float* image, size_t width, size_t height, size_t tile, size_t margin,
                            float* out, refcpu_progress_fn cb, void* user) {
  return guard([&] {
    std::function<bool(float)> progress;
    if (cb) progress = [cb, user](float f) { return cb(f, user) == 0; };
    std::vector<float> r = static_cast<Scunet*>(h)->run_tiled(image, width, height, tile, margin, progress);
    std::memcpy(out, r.data(), r.size() * sizeof(float));
  });
}

// ------------------------------------------------------------------------ LaMa
int refcpu_lama_load(const char* path, void** out) {
  return guard([&] { *out = new Lama(path); });
}
void refcpu_lama_free(void* h) { delete static_cast<Lama*>(h); }

// Model::run_float: the prediction for every pixel (`out` width x height x 3).
int refcpu_lama_run_float(void* h, const float* image, const float* mask, size_t width, size_t height, float* out,
                          refcpu_progress_fn cb, void* user) {
  return guard([&] {
    Lama::check_size(width * height * 3, width * height, width, height);
    size_t done = 0;
    std::function<bool()> step;
    if (cb) step = [&] { return cb((float)++done / (float)Lama::STEPS, user) == 0; };
    std::vector<float> r = static_cast<Lama*>(h)->run(image, mask, width, height, step);
    std::memcpy(out, r.data(), r.size() * sizeof(float));
  });
}

// fourier.rs forward / inverse (the inverse adds onto `out`).
int refcpu_rfft2(const float* x, size_t h, size_t w, size_t c, float* out) {
  return guard([&] {
    std::vector<float> s;
    rfft2(x, c, h, w, c, s);
    std::memcpy(out, s.data(), s.size() * sizeof(float));
  });
}
int refcpu_irfft2_add(const float* spec, size_t h, size_t w, size_t c, float* out) {
  return guard([&] {
    std::vector<float> s(spec, spec + h * (w / 2 + 1) * 2 * c);
    irfft2_add(s, h, w, c, out, c);
  });
}

// -------------------------------------------------------------------- BiRefNet
int refcpu_birefnet_load(const char* path, void** out) {
  return guard([&] { *out = new Birefnet(path); });
}
void refcpu_birefnet_free(void* h) { delete static_cast<Birefnet*>(h); }

// Model::run_normalized: side x side logits.
int refcpu_birefnet_run_normalized(void* h, const float* image, size_t side, float* out) {
  return guard([&] {
    Birefnet::check_size(side * side * 3, side);
    std::vector<float> r = static_cast<Birefnet*>(h)->run_normalized(image, side);
    std::memcpy(out, r.data(), r.size() * sizeof(float));
  });
}

// Model::run: the 8-bit image normalised, then run_normalized.
int refcpu_birefnet_run(void* h, const uint8_t* rgb, size_t side, float* out) {
  return guard([&] {
    Birefnet::check_size(side * side * 3, side);
    std::vector<float> img = Birefnet::normalize(rgb, side * side);
    std::vector<float> r = static_cast<Birefnet*>(h)->run_normalized(img.data(), side);
    std::memcpy(out, r.data(), r.size() * sizeof(float));
  });
}

int refcpu_resize(const float* src, size_t sh, size_t sw, size_t c, float* dst, size_t dh, size_t dw, int add) {
  return guard([&] { resize(src, sh, sw, c, dst, dh, dw, c, add != 0); });
}

// The engine's window attention and layer norm, for the kernels' unit tests.
int refcpu_attention(const float* qkv, size_t c, size_t head, const float* bias, size_t tokens, float* out) {
  return guard([&] { attention(qkv, c, head, bias, tokens, out); });
}
void refcpu_gelu(float* x, size_t n) {
  for (size_t i = 0; i < n; i++) x[i] = gelu_one(x[i]);
}
void refcpu_sigmoid(float* x, size_t n) {
  for (size_t i = 0; i < n; i++) x[i] = sigmoid_one(x[i]);
}
int refcpu_layer_norm(float* x, size_t rows, size_t n, const float* gamma, const float* beta) {
  return guard([&] {
    for (size_t r = 0; r < rows; r++) layer_norm_row(x + r * n, n, gamma, beta);
  });
}

}  // extern "C"
