// The C ABI of include/iec_cuda.h: argument checks with the reference's
// messages, C++ exceptions turned into status codes, host <-> device copies
// of the host-buffer entry points.
#include <cuda_runtime.h>

#include <cstring>
#include <limits>
#include <functional>
#include <memory>
#include <string>

#include "../../include/iec_cuda.h"
#include "realesrgan.h"
#include "birefnet.h"
#include "lama.h"
#include "scunet.h"

using namespace iec;

namespace {

thread_local std::string g_error;

template <class F>
iec_status guard(F&& f) {
  try {
    f();
    g_error.clear();
    return IEC_OK;
  } catch (const Error& e) {
    g_error = e.what();
    return (iec_status)e.code;
  } catch (const std::bad_alloc&) {
    g_error = "out of host memory";
    return IEC_ERR_GPU;
  } catch (const std::exception& e) {
    g_error = e.what();
    return IEC_ERR_INPUT;
  }
}

Options to_options(const iec_options* o) {
  Options opt;
  if (o) {
    opt.device = o->device;
    opt.timeout_ms = o->timeout_ms;
    opt.batch_chunk = o->batch_chunk;
  }
  return opt;
}

// crates/realesrgan-native/src/lib.rs:302-316 (check_size): a nonempty image
// whose 16x larger output still has a size.
void check_realesrgan_size(size_t width, size_t height) {
  if (width == 0 || height == 0)
    throw Error(ERR_INPUT, "empty " + std::to_string(width) + " x " + std::to_string(height) + " image");
  const size_t max = std::numeric_limits<size_t>::max();
  if (width > max / height || width * height > max / (3 * 16) || width > (size_t)INT32_MAX / 4 ||
      height > (size_t)INT32_MAX / 4)
    throw Error(ERR_INPUT, "a " + std::to_string(width) + " x " + std::to_string(height) + " image is too large");
}

void need(const void* p, const char* what) {
  if (!p) throw Error(ERR_INPUT, std::string(what) + " is null");
}

}  // namespace

// Each handle carries a tag, so that a handle of one model passed where
// another's is expected fails with IEC_ERR_INPUT instead of being used.
struct iec_realesrgan {
  static constexpr uint32_t TAG = 0x52455347;  // "RESG"
  uint32_t tag = TAG;
  std::unique_ptr<RealEsrgan> model;
  ~iec_realesrgan() { tag = 0; }
};

namespace iec {

// The copies and kernels of a batched host entry point overlapped on three
// streams: the H2D copy of image i + 1 and the D2H copy of image i - 1 run
// while image i computes on the caller's stream; two device buffers of each
// kind alternate, so every image runs on one of two fixed buffer pairs.
struct BatchPipe {
  int device = -1;
  DeviceBuffer in[2], out[2];
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t ev_start = nullptr, ev_h2d[2] = {}, ev_done[2] = {}, ev_d2h[2] = {};

  struct Source {
    const void* ptr;
    size_t bytes;  // per image
  };
  using Compute = std::function<void(size_t, const uint8_t*, uint8_t*, cudaStream_t)>;

  ~BatchPipe() {
    if (device < 0) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    for (cudaEvent_t e : {ev_start, ev_h2d[0], ev_h2d[1], ev_done[0], ev_done[1], ev_d2h[0], ev_d2h[1]})
      if (e) cudaEventDestroy(e);
    for (cudaStream_t st : {h2d, d2h})
      if (st) cudaStreamDestroy(st);
    for (int b = 0; b < 2; b++) {
      in[b].release();
      out[b].release();
    }
    if (prev >= 0) cudaSetDevice(prev);
  }

  // `compute(i, d_in, d_out, s)` runs image i from d_in (the sources' bytes
  // one after another) into d_out (out_bytes) on s. Returns when every
  // output is in `dst` (image i at dst + i out_bytes).
  void run(Device& dev, size_t count, const std::vector<Source>& srcs, void* dst, size_t out_bytes, cudaStream_t s,
           const Compute& compute) {
    if (device < 0) {
      device = dev.ordinal();
      IEC_CUDA(cudaStreamCreateWithFlags(&h2d, cudaStreamNonBlocking));
      IEC_CUDA(cudaStreamCreateWithFlags(&d2h, cudaStreamNonBlocking));
      IEC_CUDA(cudaEventCreateWithFlags(&ev_start, cudaEventDisableTiming));
      for (int b = 0; b < 2; b++) {
        IEC_CUDA(cudaEventCreateWithFlags(&ev_h2d[b], cudaEventDisableTiming));
        IEC_CUDA(cudaEventCreateWithFlags(&ev_done[b], cudaEventDisableTiming));
        IEC_CUDA(cudaEventCreateWithFlags(&ev_d2h[b], cudaEventDisableTiming));
      }
    }
    size_t in_bytes = 0;
    for (const Source& src : srcs) in_bytes += src.bytes;
    for (int b = 0; b < 2; b++) {
      in[b].reserve(in_bytes);
      out[b].reserve(out_bytes);
    }
    IEC_CUDA(cudaEventRecord(ev_start, s));
    IEC_CUDA(cudaStreamWaitEvent(h2d, ev_start, 0));
    IEC_CUDA(cudaStreamWaitEvent(d2h, ev_start, 0));
    for (size_t i = 0; i < count; i++) {
      const int b = (int)(i & 1);
      if (i >= 2) IEC_CUDA(cudaStreamWaitEvent(h2d, ev_done[b], 0));  // image i - 2 has read in[b]
      size_t at = 0;
      for (const Source& src : srcs) {
        IEC_CUDA(cudaMemcpyAsync(in[b].as<uint8_t>() + at, static_cast<const uint8_t*>(src.ptr) + i * src.bytes,
                                 src.bytes, cudaMemcpyHostToDevice, h2d));
        at += src.bytes;
      }
      IEC_CUDA(cudaEventRecord(ev_h2d[b], h2d));
      IEC_CUDA(cudaStreamWaitEvent(s, ev_h2d[b], 0));
      if (i >= 2) IEC_CUDA(cudaStreamWaitEvent(s, ev_d2h[b], 0));  // image i - 2's output is copied out
      compute(i, in[b].as<uint8_t>(), out[b].as<uint8_t>(), s);
      IEC_CUDA(cudaEventRecord(ev_done[b], s));
      IEC_CUDA(cudaStreamWaitEvent(d2h, ev_done[b], 0));
      IEC_CUDA(cudaMemcpyAsync(static_cast<uint8_t*>(dst) + i * out_bytes, out[b].get(), out_bytes,
                               cudaMemcpyDeviceToHost, d2h));
      IEC_CUDA(cudaEventRecord(ev_d2h[b], d2h));
    }
    for (int b = 0; b < 2 && (size_t)b < count; b++) IEC_CUDA(cudaStreamWaitEvent(s, ev_d2h[b], 0));
    dev.sync(s);
  }
};

}  // namespace iec

struct iec_scunet {
  static constexpr uint32_t TAG = 0x53434e54;  // "SCNT"
  uint32_t tag = TAG;
  std::unique_ptr<Scunet> model;
  BatchPipe batch;
  ~iec_scunet() { tag = 0; }
};

struct iec_lama {
  static constexpr uint32_t TAG = 0x4c414d41;  // "LAMA"
  uint32_t tag = TAG;
  std::unique_ptr<Lama> model;
  BatchPipe batch;
  ~iec_lama() { tag = 0; }
};

struct iec_birefnet {
  static constexpr uint32_t TAG = 0x42524e54;  // "BRNT"
  uint32_t tag = TAG;
  std::unique_ptr<Birefnet> model;
  BatchPipe batch;
  ~iec_birefnet() { tag = 0; }
};

namespace {
template <class H>
bool valid(const H* h) {
  return h && h->tag == H::TAG && h->model;
}
template <class H>
void need_model(const H* h) {
  if (!h) throw Error(ERR_INPUT, "model is null");
  if (!valid(h)) throw Error(ERR_INPUT, "model is not a handle of this model type");
}
}  // namespace

extern "C" {

const char* iec_last_error(void) { return g_error.c_str(); }

int iec_device_count(void) { return device_count(); }

iec_status iec_realesrgan_load(const char* weights_path, const iec_options* options, iec_realesrgan** out) {
  return guard([&] {
    need(out, "out");
    *out = nullptr;
    need(weights_path, "weights_path");
    auto h = std::make_unique<iec_realesrgan>();
    h->model = std::make_unique<RealEsrgan>(weights_path, to_options(options));
    *out = h.release();
  });
}

void iec_realesrgan_free(iec_realesrgan* model) {
  if (valid(model)) delete model;
}

const char* iec_realesrgan_device_name(const iec_realesrgan* model) {
  return valid(model) ? model->model->device().name().c_str() : "";
}

static iec_status run_host(iec_realesrgan* model, const void* image, bool u8, size_t width, size_t height,
                           size_t tile, size_t margin, void* out, iec_progress_fn progress, void* user) {
  return guard([&] {
    need_model(model);
    need(image, "image");
    need(out, "out");
    check_realesrgan_size(width, height);
    RealEsrgan& m = *model->model;
    DeviceScope scope(m.device());
    const size_t elem = u8 ? 1 : 4;
    const size_t in_bytes = width * height * 3 * elem, out_bytes = in_bytes * 16;
    m.host_in.reserve(in_bytes);
    m.host_out.reserve(out_bytes);
    cudaStream_t s = m.device().stream();
    IEC_CUDA(cudaMemcpyAsync(m.host_in.get(), image, in_bytes, cudaMemcpyHostToDevice, s));
    std::function<bool(float)> cb;
    if (progress) cb = [progress, user](float f) { return progress(f, user) == 0; };
    m.run_tiled_device(m.host_in.get(), u8, m.host_out.get(), u8, 1, width, height, tile, margin, cb, s);
    IEC_CUDA(cudaMemcpyAsync(out, m.host_out.get(), out_bytes, cudaMemcpyDeviceToHost, s));
    m.device().sync(s);
  });
}

iec_status iec_realesrgan_run_float(iec_realesrgan* model, const float* image, size_t width, size_t height,
                                    float* out) {
  return run_host(model, image, false, width, height, RealEsrgan::GPU_TILE, RealEsrgan::MARGIN, out, nullptr,
                  nullptr);
}

iec_status iec_realesrgan_run_float_tiled(iec_realesrgan* model, const float* image, size_t width, size_t height,
                                          size_t tile, size_t margin, float* out, iec_progress_fn progress,
                                          void* user) {
  if (tile == 0) {
    g_error = "input: tile size 0";
    return IEC_ERR_INPUT;
  }
  return run_host(model, image, false, width, height, tile, margin, out, progress, user);
}

iec_status iec_realesrgan_run(iec_realesrgan* model, const uint8_t* rgb, size_t width, size_t height,
                              uint8_t* out, iec_progress_fn progress, void* user) {
  return run_host(model, rgb, true, width, height, RealEsrgan::GPU_TILE, RealEsrgan::MARGIN, out, progress, user);
}

iec_status iec_realesrgan_run_float_tiles(iec_realesrgan* model, const float* image, size_t width, size_t height,
                                          size_t tile, size_t margin, size_t first, size_t last, float* out) {
  return guard([&] {
    need_model(model);
    need(image, "image");
    need(out, "out");
    check_realesrgan_size(width, height);
    RealEsrgan& m = *model->model;
    DeviceScope scope(m.device());
    const auto windows = RealEsrgan::tile_windows(width, height, tile, first, last);
    const size_t in_bytes = width * height * 3 * 4;
    m.host_in.reserve(in_bytes);
    m.host_out.reserve(in_bytes * 16);
    cudaStream_t s = m.device().stream();
    IEC_CUDA(cudaMemcpyAsync(m.host_in.get(), image, in_bytes, cudaMemcpyHostToDevice, s));
    m.run_tiled_device(m.host_in.get(), false, m.host_out.get(), false, 1, width, height, tile, margin, nullptr, s,
                       first, last);
    // Only the tiles' own windows come back; the rest of `out` is untouched.
    const size_t pitch = width * 4 * 3 * sizeof(float);
    for (const auto& w : windows) {
      const size_t off = (w[1] * 4 * width * 4 + w[0] * 4) * 3;
      IEC_CUDA(cudaMemcpy2DAsync(out + off, pitch, m.host_out.as<float>() + off, pitch,
                                 (w[2] - w[0]) * 4 * 3 * sizeof(float), (w[3] - w[1]) * 4, cudaMemcpyDeviceToHost,
                                 s));
    }
    m.device().sync(s);
  });
}

iec_status iec_realesrgan_run_tiles_device(iec_realesrgan* model, const float* image, size_t width, size_t height,
                                           size_t tile, size_t margin, size_t first, size_t last, float* out,
                                           void* stream) {
  return guard([&] {
    need_model(model);
    need(image, "image");
    need(out, "out");
    check_realesrgan_size(width, height);
    if (reinterpret_cast<uintptr_t>(out) % 16 != 0) throw Error(ERR_INPUT, "out must be 16-byte aligned");
    RealEsrgan& m = *model->model;
    DeviceScope scope(m.device());
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.device().stream();
    m.run_tiled_device(image, false, out, false, 1, width, height, tile, margin, nullptr, s, first, last);
  });
}

iec_status iec_realesrgan_run_batch(iec_realesrgan* model, const float* images, size_t count, size_t width,
                                    size_t height, float* out, void* stream) {
  return guard([&] {
    need_model(model);
    need(images, "images");
    need(out, "out");
    if (count == 0) return;
    check_realesrgan_size(width, height);
    RealEsrgan& m = *model->model;
    DeviceScope scope(m.device());
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.device().stream();
    m.run_batch_host(images, false, out, false, count, width, height, s);
  });
}

iec_status iec_realesrgan_run_batch_u8(iec_realesrgan* model, const uint8_t* images, size_t count, size_t width,
                                       size_t height, uint8_t* out, void* stream) {
  return guard([&] {
    need_model(model);
    need(images, "images");
    need(out, "out");
    if (count == 0) return;
    check_realesrgan_size(width, height);
    RealEsrgan& m = *model->model;
    DeviceScope scope(m.device());
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.device().stream();
    m.run_batch_host(images, true, out, true, count, width, height, s);
  });
}

iec_status iec_realesrgan_run_device(iec_realesrgan* model, const float* images, size_t count, size_t width,
                                     size_t height, float* out, void* stream) {
  return guard([&] {
    need_model(model);
    need(images, "images");
    need(out, "out");
    if (count == 0) return;
    check_realesrgan_size(width, height);
    if (reinterpret_cast<uintptr_t>(out) % 16 != 0) throw Error(ERR_INPUT, "out must be 16-byte aligned");
    RealEsrgan& m = *model->model;
    DeviceScope scope(m.device());
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.device().stream();
    m.run_device(images, out, count, width, height, s);
  });
}

iec_status iec_realesrgan_run_device_noalloc(iec_realesrgan* model, const float* images, size_t count,
                                             size_t width, size_t height, float* out, void* stream) {
  return guard([&] {
    need_model(model);
    need(images, "images");
    need(out, "out");
    if (count == 0) return;
    check_realesrgan_size(width, height);
    if (reinterpret_cast<uintptr_t>(out) % 16 != 0) throw Error(ERR_INPUT, "out must be 16-byte aligned");
    RealEsrgan& m = *model->model;
    DeviceScope scope(m.device());
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.device().stream();
    m.run_device_noalloc(images, out, count, width, height, s);
  });
}

// ---------------------------------------------------------------------- SCUNet
iec_status iec_scunet_load(const char* weights_path, const iec_options* options, iec_scunet** out) {
  return guard([&] {
    need(out, "out");
    *out = nullptr;
    need(weights_path, "weights_path");
    auto h = std::make_unique<iec_scunet>();
    h->model = std::make_unique<Scunet>(weights_path, to_options(options));
    *out = h.release();
  });
}

void iec_scunet_free(iec_scunet* model) {
  if (valid(model)) delete model;
}

const char* iec_scunet_device_name(const iec_scunet* model) {
  return valid(model) ? model->model->device().name().c_str() : "";
}

// crates/scunet-native/src/lib.rs:256-267 (check_size).
static void check_scunet_size(size_t width, size_t height) {
  if (width == 0 || height == 0)
    throw Error(ERR_INPUT, "empty " + std::to_string(width) + " x " + std::to_string(height) + " image");
  if (width > (size_t)1 << 20 || height > (size_t)1 << 20 || width * height > ((size_t)1 << 31) / 64)
    throw Error(ERR_INPUT, "a " + std::to_string(width) + " x " + std::to_string(height) + " image is too large");
}

static iec_status scunet_host(iec_scunet* model, const void* image, bool u8, size_t width, size_t height, bool whole,
                              size_t tile, size_t margin, void* out, iec_progress_fn progress, void* user) {
  return guard([&] {
    need_model(model);
    need(image, "image");
    need(out, "out");
    check_scunet_size(width, height);
    Scunet& m = *model->model;
    DeviceScope scope(m.device());
    const size_t elem = u8 ? 1 : 4, bytes = width * height * 3 * elem;
    m.host_in.reserve(bytes);
    m.host_out.reserve(bytes);
    cudaStream_t s = m.device().stream();
    IEC_CUDA(cudaMemcpyAsync(m.host_in.get(), image, bytes, cudaMemcpyHostToDevice, s));
    std::function<bool(float)> cb;
    if (progress) cb = [progress, user](float f) { return progress(f, user) == 0; };
    if (whole) {
      m.run_region(m.host_in.get(), u8, m.host_out.get(), u8, (int)width, (int)height, 0, 0, (int)width, (int)height, 0,
                   0, (int)width, (int)height, nullptr, s);
    } else {
      m.run_tiled_device(m.host_in.get(), u8, m.host_out.get(), u8, width, height, tile, margin, cb, s);
    }
    IEC_CUDA(cudaMemcpyAsync(out, m.host_out.get(), bytes, cudaMemcpyDeviceToHost, s));
    m.device().sync(s);
  });
}

iec_status iec_scunet_run_float(iec_scunet* model, const float* image, size_t width, size_t height, float* out) {
  return scunet_host(model, image, false, width, height, true, 0, 0, out, nullptr, nullptr);
}

iec_status iec_scunet_run_float_tiled(iec_scunet* model, const float* image, size_t width, size_t height, size_t tile,
                                      size_t margin, float* out, iec_progress_fn progress, void* user) {
  if (tile == 0) {
    g_error = "input: tile size 0";
    return IEC_ERR_INPUT;
  }
  return scunet_host(model, image, false, width, height, false, tile, margin, out, progress, user);
}

iec_status iec_scunet_run_device(iec_scunet* model, const float* image, size_t width, size_t height, float* out,
                                 void* stream) {
  return guard([&] {
    need_model(model);
    need(image, "image");
    need(out, "out");
    check_scunet_size(width, height);
    Scunet& m = *model->model;
    DeviceScope scope(m.device());
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.device().stream();
    m.run_whole_device(image, out, (int)width, (int)height, s);
  });
}

iec_status iec_scunet_run_batch(iec_scunet* model, const float* images, size_t count, size_t width, size_t height,
                                float* out, void* stream) {
  return guard([&] {
    need_model(model);
    need(images, "images");
    need(out, "out");
    if (count == 0) return;
    check_scunet_size(width, height);
    Scunet& m = *model->model;
    DeviceScope scope(m.device());
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.device().stream();
    const size_t bytes = width * height * 3 * 4;
    model->batch.run(m.device(), count, {{images, bytes}}, out, bytes, s,
                     [&](size_t, const uint8_t* in, uint8_t* o, cudaStream_t st) {
                       m.run_whole_device(reinterpret_cast<const float*>(in), reinterpret_cast<float*>(o),
                                          (int)width, (int)height, st);
                     });
  });
}

iec_status iec_scunet_run(iec_scunet* model, const uint8_t* rgb, size_t width, size_t height, uint8_t* out,
                          iec_progress_fn progress, void* user) {
  return scunet_host(model, rgb, true, width, height, false, Scunet::TILE, Scunet::MARGIN, out, progress, user);
}

// ------------------------------------------------------------------------ LaMa
iec_status iec_lama_load(const char* weights_path, const iec_options* options, iec_lama** out) {
  return guard([&] {
    need(out, "out");
    *out = nullptr;
    need(weights_path, "weights_path");
    auto h = std::make_unique<iec_lama>();
    h->model = std::make_unique<Lama>(weights_path, to_options(options));
    *out = h.release();
  });
}

void iec_lama_free(iec_lama* model) {
  if (valid(model)) delete model;
}

const char* iec_lama_device_name(const iec_lama* model) { return valid(model) ? model->model->device().name().c_str() : ""; }

// crates/lama-native/src/lib.rs:180-194 (check_size), with a bound on the
// side the Fourier transforms take.
static void check_lama_size(size_t width, size_t height) {
  if (width < (size_t)Lama::MIN_SIDE || height < (size_t)Lama::MIN_SIDE)
    throw Error(ERR_INPUT, std::to_string(width) + " x " + std::to_string(height) +
                               " image: sides of at least " + std::to_string(Lama::MIN_SIDE) + " pixels");
  if (width > 12288 || height > 12288)
    throw Error(ERR_INPUT, "a " + std::to_string(width) + " x " + std::to_string(height) + " image is too large");
}

static iec_status lama_host(iec_lama* model, const void* image, const void* mask, bool u8, size_t width, size_t height,
                            void* out, iec_progress_fn progress, void* user) {
  return guard([&] {
    need_model(model);
    need(image, "image");
    need(mask, "mask");
    need(out, "out");
    check_lama_size(width, height);
    Lama& m = *model->model;
    DeviceScope scope(m.device());
    const size_t elem = u8 ? 1 : 4, bytes = width * height * 3 * elem, mbytes = width * height * elem;
    m.host_in.reserve(bytes);
    m.host_mask.reserve(mbytes);
    m.host_out.reserve(bytes);
    cudaStream_t s = m.device().stream();
    IEC_CUDA(cudaMemcpyAsync(m.host_in.get(), image, bytes, cudaMemcpyHostToDevice, s));
    IEC_CUDA(cudaMemcpyAsync(m.host_mask.get(), mask, mbytes, cudaMemcpyHostToDevice, s));
    size_t done = 0;
    std::function<bool()> step;
    if (progress)
      step = [&] { return progress((float)(++done) / (float)Lama::STEPS, user) == 0; };
    if (!m.run(m.host_in.get(), u8, m.host_mask.get(), u8, m.host_out.get(), u8, (int)width, (int)height, step, s))
      throw Error(CANCELLED, "cancelled");
    IEC_CUDA(cudaMemcpyAsync(out, m.host_out.get(), bytes, cudaMemcpyDeviceToHost, s));
    m.device().sync(s);
  });
}

iec_status iec_lama_run_float(iec_lama* model, const float* image, const float* mask, size_t width, size_t height,
                              float* out) {
  return lama_host(model, image, mask, false, width, height, out, nullptr, nullptr);
}

iec_status iec_lama_run(iec_lama* model, const uint8_t* rgb, const uint8_t* mask, size_t width, size_t height,
                        uint8_t* out, iec_progress_fn progress, void* user) {
  return lama_host(model, rgb, mask, true, width, height, out, progress, user);
}

iec_status iec_lama_run_device(iec_lama* model, const float* image, const float* mask, size_t width, size_t height,
                               float* out, void* stream) {
  return guard([&] {
    need_model(model);
    need(image, "image");
    need(mask, "mask");
    need(out, "out");
    check_lama_size(width, height);
    Lama& m = *model->model;
    DeviceScope scope(m.device());
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.device().stream();
    m.run(image, false, mask, false, out, false, (int)width, (int)height, nullptr, s);
  });
}

iec_status iec_scunet_set_fused(iec_scunet* model, int on) {
  return guard([&] {
    need_model(model);
    model->model->set_fused(on != 0);
  });
}

iec_status iec_birefnet_set_fused(iec_birefnet* model, int on) {
  return guard([&] {
    need_model(model);
    model->model->set_fused(on != 0);
  });
}

iec_status iec_lama_set_fused(iec_lama* model, int on) {
  return guard([&] {
    need_model(model);
    model->model->set_fused(on != 0);
  });
}

iec_status iec_lama_run_batch(iec_lama* model, const float* images, const float* masks, size_t count, size_t width,
                              size_t height, float* out, void* stream) {
  return guard([&] {
    need_model(model);
    need(images, "images");
    need(masks, "masks");
    need(out, "out");
    if (count == 0) return;
    check_lama_size(width, height);
    Lama& m = *model->model;
    DeviceScope scope(m.device());
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.device().stream();
    const size_t ib = width * height * 3 * 4, mb = width * height * 4;
    model->batch.run(m.device(), count, {{images, ib}, {masks, mb}}, out, ib, s,
                     [&](size_t, const uint8_t* in, uint8_t* o, cudaStream_t st) {
                       m.run(in, false, in + ib, false, o, false, (int)width, (int)height, nullptr, st);
                     });
  });
}

// -------------------------------------------------------------------- BiRefNet
iec_status iec_birefnet_load(const char* weights_path, const iec_options* options, iec_birefnet** out) {
  return guard([&] {
    need(out, "out");
    *out = nullptr;
    need(weights_path, "weights_path");
    auto h = std::make_unique<iec_birefnet>();
    h->model = std::make_unique<Birefnet>(weights_path, to_options(options));
    *out = h.release();
  });
}

void iec_birefnet_free(iec_birefnet* model) {
  if (valid(model)) delete model;
}

const char* iec_birefnet_device_name(const iec_birefnet* model) {
  return valid(model) ? model->model->device().name().c_str() : "";
}

// crates/birefnet-native/src/lib.rs:175-187 (check_size), with a bound on
// the side.
static void check_birefnet_size(size_t side) {
  if (side == 0 || side % 64 != 0)
    throw Error(ERR_INPUT, "side " + std::to_string(side) + " is not a positive multiple of 64");
  if (side > 8192) throw Error(ERR_INPUT, "side " + std::to_string(side) + " is too large");
}

static iec_status birefnet_host(iec_birefnet* model, const void* image, bool u8, size_t side, float* logits) {
  return guard([&] {
    need_model(model);
    need(image, "image");
    need(logits, "logits");
    check_birefnet_size(side);
    Birefnet& m = *model->model;
    DeviceScope scope(m.device());
    const size_t bytes = side * side * 3 * (u8 ? 1 : 4), obytes = side * side * 4;
    m.host_in.reserve(bytes);
    m.host_out.reserve(obytes);
    cudaStream_t s = m.device().stream();
    IEC_CUDA(cudaMemcpyAsync(m.host_in.get(), image, bytes, cudaMemcpyHostToDevice, s));
    m.run(m.host_in.get(), u8, (int)side, m.host_out.as<float>(), s);
    IEC_CUDA(cudaMemcpyAsync(logits, m.host_out.get(), obytes, cudaMemcpyDeviceToHost, s));
    m.device().sync(s);
  });
}

iec_status iec_birefnet_run(iec_birefnet* model, const uint8_t* rgb, size_t side, float* logits) {
  return birefnet_host(model, rgb, true, side, logits);
}

iec_status iec_birefnet_run_normalized(iec_birefnet* model, const float* image, size_t side, float* logits) {
  return birefnet_host(model, image, false, side, logits);
}

iec_status iec_birefnet_run_device(iec_birefnet* model, const void* image, int image_u8, size_t side, float* logits,
                                   void* stream) {
  return guard([&] {
    need_model(model);
    need(image, "image");
    need(logits, "logits");
    check_birefnet_size(side);
    Birefnet& m = *model->model;
    DeviceScope scope(m.device());
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.device().stream();
    m.run(image, image_u8 != 0, (int)side, logits, s);
  });
}

iec_status iec_birefnet_run_batch(iec_birefnet* model, const uint8_t* images, size_t count, size_t side,
                                  float* logits, void* stream) {
  return guard([&] {
    need_model(model);
    need(images, "images");
    need(logits, "logits");
    if (count == 0) return;
    check_birefnet_size(side);
    Birefnet& m = *model->model;
    DeviceScope scope(m.device());
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.device().stream();
    model->batch.run(m.device(), count, {{images, side * side * 3}}, logits, side * side * 4, s,
                     [&](size_t, const uint8_t* in, uint8_t* o, cudaStream_t st) {
                       m.run(in, true, (int)side, reinterpret_cast<float*>(o), st);
                     });
  });
}

namespace {
// The device of a model handle of any kind (by its type tag), or null.
Device* handle_device(void* handle) {
  if (!handle) return nullptr;
  const uint32_t tag = *static_cast<const uint32_t*>(handle);
  if (tag == iec_scunet::TAG) return &static_cast<iec_scunet*>(handle)->model->device();
  if (tag == iec_lama::TAG) return &static_cast<iec_lama*>(handle)->model->device();
  if (tag == iec_birefnet::TAG) return &static_cast<iec_birefnet*>(handle)->model->device();
  if (tag == iec_realesrgan::TAG) return &static_cast<iec_realesrgan*>(handle)->model->device();
  return nullptr;
}
}  // namespace

iec_status iec_set_launch_timing(void* model, int on) {
  return guard([&] {
    Device* d = handle_device(model);
    if (!d) throw Error(ERR_INPUT, "not a model handle");
    d->set_timing(on != 0);
  });
}

size_t iec_launch_timing(void* model, iec_launch_record* records, size_t n) {
  size_t written = 0;
  iec_status st = guard([&] {
    Device* d = handle_device(model);
    if (!d) throw Error(ERR_INPUT, "not a model handle");
    need(records, "records");
    DeviceScope scope(*d);
    const auto& t = d->timed();
    for (size_t i = 0; i < t.size() && written < n; i++, written++) {
      iec_launch_record& r = records[written];
      std::memset(r.name, 0, sizeof r.name);
      std::strncpy(r.name, t[i].name.c_str(), sizeof r.name - 1);
      r.flop = t[i].flop;
      r.bytes = t[i].bytes;
      r.ms = d->timed_ms(i);
    }
  });
  return st == IEC_OK ? written : 0;
}

size_t iec_realesrgan_launches(const iec_realesrgan* model, size_t count, size_t width, size_t height) {
  return valid(model) ? model->model->launches(count, width, height) : 0;
}

iec_status iec_realesrgan_set_timing(iec_realesrgan* model, size_t capacity) {
  return guard([&] {
    need_model(model);
    DeviceScope scope(model->model->device());
    model->model->set_timing(capacity);
  });
}

iec_status iec_realesrgan_set_fused(iec_realesrgan* model, int on) {
  return guard([&] {
    need_model(model);
    model->model->set_fused(on != 0);
  });
}

size_t iec_realesrgan_timing(iec_realesrgan* model, int* kinds, float* ms, size_t n) {
  size_t written = 0;
  iec_status st = guard([&] {
    need_model(model);
    need(kinds, "kinds");
    need(ms, "ms");
    DeviceScope scope(model->model->device());
    written = model->model->timing(kinds, ms, n);
  });
  return st == IEC_OK ? written : 0;
}

}  // extern "C"
