// Big LaMa on the CUDA backend (see lama.h).
//
// Network (crates/lama-native/src/network.rs:32-489): the masked image and
// mask padded to a multiple of 8 by mirroring (symmetric), conv7 4 -> 64,
// three conv3 stride 2 to 512 channels at an eighth of the size, 18 residual
// blocks of two fast Fourier convolutions, three stride-2 transposed
// convolutions back to 64 channels, conv7 64 -> 3 and a sigmoid, cropped.
// All convolutions but the transposed ones pad by reflection.
//
// Stored layouts (planar f16, [channels / 8][pixels][8]):
//   in0   the first convolution's input with its 7 horizontal taps folded into
//         32 channels (kx * 4 + c), reflect-padded by 3 rows: the 7x7
//         convolution becomes 7 taps of K = 32
//   d0-d2 each stride-2 convolution's input: reflect-padded by 1 and split
//         into its four space-to-depth phases, so the convolution reads 9
//         taps of stride 1 (tap (ky, kx) = phase (ky % 2, kx % 2), offset
//         (ky / 2, kx / 2))
//   x, mid, tmp  the eighth-scale maps, reflect-padded by 1 (the FFCs' 3x3
//         convolutions read them directly)
//   spectral (rows y w + x), spectrum / filtered (rows ky half + k, real
//         planes then imaginary)
//   u0, u1 the first two doublings, unpadded (the phase taps read zeros past
//         the edge from TMA's fill); u2 reflect-padded by 3 for the last conv7
#include "lama.h"

#include <algorithm>
#include <cmath>
#include <cstring>

#include "igemm_sm100.cuh"

namespace iec {

struct Lama::Ffc {
  PackedWeights local, cross, spectral_in, fourier, spectral_out;
  FourierWeights fourier_unit;  // the same Fourier matrix for the fused unit
};

namespace {

int blocks_for(long long n, int sms) {
  return (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, (long long)sms * 16));
}

__device__ __forceinline__ int reflect_index(int i, int n) {
  const int a = i < 0 ? -i : i, b = 2 * (n - 1) - i;
  return a < b ? a : b;
}

// network.rs:348-370 masked_rows + the first convolution's reflect padding:
// padded row r (logical row r - 3 of the hp x wp map), column x, channel
// kx * 4 + c = the masked input at (reflect(r - 3), reflect(x + kx - 3)),
// the hp x wp map mirroring the image past its bottom and right edges.
__global__ void lama_prep(const void* __restrict__ image, int image_u8, const void* __restrict__ mask, int mask_u8,
                          int width, int height, int hp, int wp, __half* __restrict__ dst, long long plane) {
  griddep_wait();
  griddep_launch_dependents();
  const long long total = (long long)(hp + 6) * wp;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / wp), x = (int)(i % wp);
    int sy = reflect_index(r - 3, hp);
    sy = sy < height ? sy : 2 * height - 1 - sy;
    float v[32];
#pragma unroll
    for (int kx = 0; kx < 7; kx++) {
      int sx = reflect_index(x + kx - 3, wp);
      sx = sx < width ? sx : 2 * width - 1 - sx;
      const long long p = (long long)sy * width + sx;
      const float m = mask_u8 ? (static_cast<const uint8_t*>(mask)[p] != 0 ? 1.0f : 0.0f)
                              : static_cast<const float*>(mask)[p];
#pragma unroll
      for (int c = 0; c < 3; c++) {
        const float px = image_u8 ? (float)static_cast<const uint8_t*>(image)[p * 3 + c] / 255.0f
                                  : static_cast<const float*>(image)[p * 3 + c];
        v[kx * 4 + c] = px * (1.0f - m);
      }
      v[kx * 4 + 3] = m;
    }
#pragma unroll
    for (int j = 28; j < 32; j++) v[j] = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; q++) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; e++) {
        __half2 h2 = __floats2half2_rn(v[8 * q + 2 * e], v[8 * q + 2 * e + 1]);
        w[e] = *reinterpret_cast<uint32_t*>(&h2);
      }
      *reinterpret_cast<uint4*>(dst + q * plane + i * 8) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// Zero the one-pixel border of a map reflect-padded by 1 (h x w inside), so
// that the transposed convolution's phase taps read zeros past the edge.
__global__ void lama_zero_border(__half* __restrict__ x, long long plane, int planes, int h, int w) {
  griddep_wait();
  griddep_launch_dependents();
  const int ring = 2 * (w + 2) + 2 * h;
  const long long total = (long long)ring * planes;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int q = (int)(i / ring), k = (int)(i % ring);
    int r, c;
    if (k < w + 2) {
      r = 0;
      c = k;
    } else if (k < 2 * (w + 2)) {
      r = h + 1;
      c = k - (w + 2);
    } else {
      const int j = k - 2 * (w + 2);
      r = 1 + j / 2;
      c = (j & 1) ? w + 1 : 0;
    }
    *reinterpret_cast<uint4*>(x + q * plane + ((long long)r * (w + 2) + c) * 8) = make_uint4(0u, 0u, 0u, 0u);
  }
}

// The prediction (plane 0 of the last convolution, rows y wp + x) cropped to
// the image: f32, or lib.rs:146-153's 8-bit composite.
__global__ void lama_output(const __half* __restrict__ pred, int wp, int width, int height, void* __restrict__ dst,
                            int dst_u8, const uint8_t* __restrict__ rgb, const void* __restrict__ mask,
                            int mask_u8) {
  griddep_wait();
  griddep_launch_dependents();
  const long long total = (long long)width * height;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int y = (int)(i / width), x = (int)(i % width);
    const __half* p = pred + ((long long)y * wp + x) * 8;
    if (!dst_u8) {
      float* o = static_cast<float*>(dst) + i * 3;
      for (int c = 0; c < 3; c++) o[c] = __half2float(p[c]);
      continue;
    }
    const bool hole = mask_u8 ? static_cast<const uint8_t*>(mask)[i] != 0 : static_cast<const float*>(mask)[i] != 0.0f;
    uint8_t* o = static_cast<uint8_t*>(dst) + i * 3;
    for (int c = 0; c < 3; c++) {
      if (hole) {
        const float v = fminf(fmaxf(__half2float(p[c]), 0.0f), 1.0f);
        o[c] = (uint8_t)roundf(v * 255.0f);
      } else {
        o[c] = rgb[i * 3 + c];
      }
    }
  }
}

void matrix(WeightFile& f, PackedWeights& pw, const std::string& name, int taps, int k, int n, bool bias) {
  HostTensor w = f.take_tensor(name + ".weight", {(size_t)taps * k, (size_t)n});
  std::vector<float> b;
  if (bias) b = f.take(name + ".bias", {(size_t)n});
  pack_weights(pw, w.values, taps, k, n, bias ? b.data() : nullptr);
}

std::vector<Tap> conv_taps(int size) {
  std::vector<Tap> t;
  for (int ky = 0; ky < size; ky++)
    for (int kx = 0; kx < size; kx++) t.push_back({ky, kx, 0});
  return t;
}

// network.rs:271: offsets of output phase 0 (input m) and 1 (m, m + 1).
std::vector<int> phase_offsets(int phase) { return phase == 0 ? std::vector<int>{0} : std::vector<int>{0, 1}; }

}  // namespace

Lama::Lama(const std::string& path, const Options& opt) : dev_(opt) {
  WeightFile f = WeightFile::read(path, std::string("LAMA\0\0\0\0", 8).c_str());
  DeviceScope scope(dev_);
  {
    // first [(ky, kx, c), 64] -> 7 taps (ky) of 32 channels (kx * 4 + c).
    HostTensor w = f.take_tensor("first.weight", {49 * 4, 64});
    std::vector<float> b = f.take("first.bias", {64});
    std::vector<float> folded((size_t)7 * 32 * 64, 0.0f);
    for (int ky = 0; ky < 7; ky++)
      for (int j = 0; j < 28; j++)
        for (int o = 0; o < 64; o++)
          folded[((size_t)ky * 32 + j) * 64 + o] = w.values[((size_t)(ky * 7 + j / 4) * 4 + j % 4) * 64 + o];
    pack_weights(first_, folded, 7, 32, 64, b.data());
  }
  const int dn[3][2] = {{64, 128}, {128, 256}, {256, CHANNELS}};
  for (int i = 0; i < 3; i++) matrix(f, down_[i], "down" + std::to_string(i), 9, dn[i][0], dn[i][1], true);
  for (int b = 0; b < BLOCKS; b++)
    for (int k = 0; k < 2; k++) {
      auto F = std::make_unique<Ffc>();
      const std::string name = "block" + std::to_string(b) + ".ffc" + std::to_string(k);
      matrix(f, F->local, name + ".local", 9, CHANNELS, LOCAL, true);
      matrix(f, F->cross, name + ".cross", 9, LOCAL, GLOBAL, true);
      matrix(f, F->spectral_in, name + ".spectral_in", 1, GLOBAL, SPECTRAL, true);
      {
        HostTensor w = f.take_tensor(name + ".fourier.weight", {2 * SPECTRAL, 2 * SPECTRAL});
        std::vector<float> b = f.take(name + ".fourier.bias", {2 * SPECTRAL});
        pack_weights(F->fourier, w.values, 1, 2 * SPECTRAL, 2 * SPECTRAL, b.data());
        pack_fourier_weights(F->fourier_unit, w.values, b);
      }
      matrix(f, F->spectral_out, name + ".spectral_out", 1, SPECTRAL, GLOBAL, false);
      ffc_.push_back(std::move(F));
    }
  const int upc[3][2] = {{CHANNELS, 256}, {256, 128}, {128, 64}};
  for (int i = 0; i < 3; i++)
    for (int p = 0; p < 4; p++) {
      const int count = (int)(phase_offsets(p / 2).size() * phase_offsets(p % 2).size());
      matrix(f, up_[i][p], "up" + std::to_string(i) + ".phase" + std::to_string(p), count, upc[i][0], upc[i][1],
             true);
    }
  matrix(f, last_, "last", 49, 64, 3, true);
  f.finish();
  step_events_.resize(STEPS);
  for (auto& e : step_events_) IEC_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  IEC_CUDA(cudaStreamCreateWithFlags(&s_local_, cudaStreamNonBlocking));
  IEC_CUDA(cudaStreamCreateWithFlags(&s_spec_, cudaStreamNonBlocking));
  for (cudaEvent_t* e : {&ev_in_, &ev_local_, &ev_spec_}) IEC_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
  IEC_CUDA(cudaDeviceSynchronize());
}

Lama::~Lama() {
  if (dev_.poisoned()) {
    graph_.leak();
    for (DeviceBuffer* b : {&in0_, &d0_, &d1_, &d2_, &x_, &mid_, &tmp_, &spectral_, &spectrum_, &filtered_, &u0_,
                            &u1_, &u2_, &out_, &host_in, &host_mask, &host_out, &plan_.twiddles, &plan_.scratch})
      b->leak();
    return;
  }
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(dev_.ordinal());
  for (auto& e : step_events_) cudaEventDestroy(e);
  for (cudaEvent_t e : {ev_in_, ev_local_, ev_spec_})
    if (e) cudaEventDestroy(e);
  for (cudaStream_t st : {s_local_, s_spec_})
    if (st) cudaStreamDestroy(st);
  if (prev >= 0) cudaSetDevice(prev);
}

void Lama::ensure(int hp, int wp) {
  if (hp == alloc_h_ && wp == alloc_w_) return;
  alloc_gen_++;  // buffers may move: captured passes must not replay
  const int h8 = hp / 8, w8 = wp / 8, half = w8 / 2 + 1;
  auto bytes = [](long long planes, long long elems) { return (size_t)(planes * elems * 2); };
  in0_.reserve(bytes(4, (long long)(hp + 6) * wp * 8));
  d0_.reserve(bytes(8, MapGeom{hp, wp, 1, 2}.plane_elems()));
  d1_.reserve(bytes(16, MapGeom{hp / 2, wp / 2, 1, 2}.plane_elems()));
  d2_.reserve(bytes(32, MapGeom{hp / 4, wp / 4, 1, 2}.plane_elems()));
  const long long e8 = MapGeom{h8, w8, 1, 1}.plane_elems();
  x_.reserve(bytes(64, e8));
  mid_.reserve(bytes(64, e8));
  tmp_.reserve(bytes(64, e8));
  spectral_.reserve(bytes(SPECTRAL / 8, (long long)gemm_rows_alloc(h8 * w8) * 8));
  spectrum_.reserve(bytes(2 * SPECTRAL / 8, (long long)gemm_rows_alloc(h8 * half) * 8));
  filtered_.reserve(bytes(2 * SPECTRAL / 8, (long long)gemm_rows_alloc(h8 * half) * 8));
  u0_.reserve(bytes(32, (long long)(2 * h8) * (2 * w8) * 8));
  u1_.reserve(bytes(16, (long long)(4 * h8) * (4 * w8) * 8));
  u2_.reserve(bytes(8, MapGeom{hp, wp, 3, 1}.plane_elems()));
  out_.reserve(bytes(1, (long long)gemm_rows_alloc(hp * wp) * 8));
  fourier_plan(plan_, h8, w8, SPECTRAL);
  alloc_h_ = hp;
  alloc_w_ = wp;
}

// network.rs:174-248. `out` = ffc(`in`); with `residual`, `out` (the block's
// input) gets ffc(`in`) added instead, its global part staged in `tmp`.
// Three independent chains run on three streams: the local convolution
// (writes the local planes of `out`), the spectral chain (spectral_in,
// rfft2, the Fourier 1x1, irfft2: its own buffers) and the cross
// convolution (the global planes of `out` or `tmp`); spectral_out joins the
// last two, and `s` waits for all before the next layer.
void Lama::ffc(const Ffc& F, const __half* in, __half* out, __half* tmp, bool residual, cudaStream_t s) {
  const int h8 = alloc_h_ / 8, w8 = alloc_w_ / 8, half = w8 / 2 + 1;
  const MapGeom g{h8, w8, 1, 1};
  static const std::vector<Tap> taps3 = conv_taps(3);
  IEC_CUDA(cudaEventRecord(ev_in_, s));
  IEC_CUDA(cudaStreamWaitEvent(s_local_, ev_in_, 0));
  IEC_CUDA(cudaStreamWaitEvent(s_spec_, ev_in_, 0));
  // local = relu(conv3(all 512 channels)) [+ out]
  GemmOutSpec o = map_out(g, out, 0);
  if (residual) o.resid = out;
  gemm_taps(dev_, F.local, g.source(in), taps3, h8, w8, ACT_RELU, o, s_local_);
  IEC_CUDA(cudaEventRecord(ev_local_, s_local_));
  // the spectral chain
  const long long spec_plane = (long long)gemm_rows_alloc(h8 * w8) * 8;
  const long long freq_plane = (long long)gemm_rows_alloc(h8 * half) * 8;
  __half* spectral = spectral_.as<__half>();
  {
    GemmOutSpec so;
    so.mode = OUT_STORE;
    so.out = spectral;
    so.plane_elems = spec_plane;
    gemm_taps(dev_, F.spectral_in, g.source(in, LOCAL / 8), {{1, 1, 0}}, h8, w8, ACT_RELU, so, s_spec_);
  }
  if (fused_unit_ && fourier_unit_fits(plan_)) {
    // rfft2, the Fourier 1x1 (ReLU) and irfft2 added on the spectral map,
    // the spectrum kept on chip (fft.h)
    fourier_unit_planar(plan_, F.fourier_unit, spectral, spec_plane, dev_.dev_err(), s_spec_);
  } else {
    rfft2_planar(plan_, spectral, spec_plane, spectrum_.as<__half>(), freq_plane, s_spec_);
    GemmOutSpec fo;
    fo.mode = OUT_STORE;
    fo.out = filtered_.as<__half>();
    fo.plane_elems = freq_plane;
    gemm_rows(dev_, F.fourier, spectrum_.as<__half>(), freq_plane, h8 * half, ACT_RELU, fo, s_spec_);
    irfft2_add_planar(plan_, filtered_.as<__half>(), freq_plane, spectral, spec_plane, s_spec_);
  }
  IEC_CUDA(cudaEventRecord(ev_spec_, s_spec_));
  // global = cross(local part) + spectral_out(spectral + irfft2(...)), then ReLU
  __half* global = residual ? tmp : out;
  gemm_taps(dev_, F.cross, g.source(in), taps3, h8, w8, ACT_NONE, map_out(g, global, LOCAL / 8), s);
  IEC_CUDA(cudaStreamWaitEvent(s, ev_spec_, 0));
  GemmOutSpec go = map_out(g, out, LOCAL / 8);
  go.acc_src = global;
  if (residual) go.resid = out;
  gemm_rows(dev_, F.spectral_out, spectral, spec_plane, h8 * w8, ACT_RELU, go, s);
  IEC_CUDA(cudaStreamWaitEvent(s, ev_local_, 0));
}

bool Lama::run(const void* image, bool image_u8, const void* mask, bool mask_u8, void* dst, bool dst_u8, int width,
               int height, const std::function<bool()>& step, cudaStream_t s) {
  // Progress reports wait on the GPU between steps: those passes run as plain
  // launches; the others replay as a graph (PassGraph).
  if (step) return run_pass(image, image_u8, mask, mask_u8, dst, dst_u8, width, height, step, s);
  graph_.run({(long long)(uintptr_t)image, image_u8, (long long)(uintptr_t)mask, mask_u8, (long long)(uintptr_t)dst,
              dst_u8, width, height, (long long)alloc_gen_, (long long)dev_.scratch_generation()},
             s, [&](cudaStream_t st) { run_pass(image, image_u8, mask, mask_u8, dst, dst_u8, width, height, {}, st); });
  return true;
}

bool Lama::run_pass(const void* image, bool image_u8, const void* mask, bool mask_u8, void* dst, bool dst_u8, int width,
               int height, const std::function<bool()>& step, cudaStream_t s) {
  SerialStreams serial(dev_.timing(), {&s_local_, &s_spec_}, s);
  if (width < MIN_SIDE || height < MIN_SIDE)
    throw Error(ERR_INPUT, std::to_string(width) + " x " + std::to_string(height) + " image: sides of at least " +
                               std::to_string(MIN_SIDE) + " pixels");
  if (dst_u8 && !image_u8) throw Error(ERR_INPUT, "the 8-bit composite needs the 8-bit image");
  const int hp = (height + MULTIPLE - 1) / MULTIPLE * MULTIPLE, wp = (width + MULTIPLE - 1) / MULTIPLE * MULTIPLE;
  ensure(hp, wp);
  const int sms = dev_.sms();

  int done = 0;
  bool cancelled = false;
  auto step_done = [&]() {
    if (!step || cancelled) return;
    IEC_CUDA(cudaEventRecord(step_events_[done], s));
    if (done >= 1) {
      dev_.wait_event(step_events_[done - 1]);
      if (!step()) cancelled = true;
    }
    done++;
  };

  // first: conv7 over the folded input, into down0's phases.
  {
    const long long plane = (long long)(hp + 6) * wp * 8;
    launch_pdl(lama_prep, blocks_for((long long)(hp + 6) * wp, sms), 256, 0, s, image, image_u8 ? 1 : 0, mask,
                                                                         mask_u8 ? 1 : 0, width, height, hp, wp,
                                                                         in0_.as<__half>(), plane);
    IEC_CUDA(cudaGetLastError());
    std::vector<Tap> taps;
    for (int ky = 0; ky < 7; ky++) taps.push_back({ky, 0, 0});
    const TapSource src{in0_.as<__half>(), plane, wp, hp + 6, 1};
    gemm_taps(dev_, first_, src, taps, hp, wp, ACT_RELU, map_out(MapGeom{hp, wp, 1, 2}, d0_.as<__half>()), s);
  }
  step_done();
  // down: conv3 stride 2 (reflect) over the phases of the padded map.
  {
    std::vector<Tap> taps;
    for (int ky = 0; ky < 3; ky++)
      for (int kx = 0; kx < 3; kx++) taps.push_back({ky / 2, kx / 2, (ky % 2) * 2 + kx % 2});
    DeviceBuffer* ins[3] = {&d0_, &d1_, &d2_};
    int h = hp, w = wp;
    for (int i = 0; i < 3; i++) {
      const MapGeom gin{h, w, 1, 2};
      const MapGeom gout = i < 2 ? MapGeom{h / 2, w / 2, 1, 2} : MapGeom{h / 2, w / 2, 1, 1};
      __half* dst_map = i < 2 ? ins[i + 1]->as<__half>() : x_.as<__half>();
      gemm_taps(dev_, down_[i], gin.source(ins[i]->as<__half>()), taps, h / 2, w / 2, ACT_RELU,
                map_out(gout, dst_map), s);
      h /= 2;
      w /= 2;
      step_done();
    }
  }
  // blocks: x += ffc1(ffc0(x)).
  for (int b = 0; b < BLOCKS && !cancelled; b++) {
    ffc(*ffc_[2 * b], x_.as<__half>(), mid_.as<__half>(), nullptr, false, s);
    ffc(*ffc_[2 * b + 1], mid_.as<__half>(), x_.as<__half>(), tmp_.as<__half>(), true, s);
    step_done();
  }
  if (cancelled) {
    dev_.sync(s);
    return false;
  }
  // up: three transposed convolutions, each as its four output phases.
  {
    const int h8 = hp / 8, w8 = wp / 8;
    const MapGeom g8{h8, w8, 1, 1};
    launch_pdl(lama_zero_border, blocks_for((long long)(2 * (w8 + 2) + 2 * h8) * 64, sms), 256, 0, s, 
        x_.as<__half>(), g8.plane_elems(), 64, h8, w8);
    IEC_CUDA(cudaGetLastError());
    int h = h8, w = w8;
    for (int i = 0; i < 3; i++) {
      TapSource src;
      int base = 0;  // offset of pixel (0, 0) in the source's padding
      if (i == 0) {
        src = g8.source(x_.as<__half>());
        base = 1;
      } else {
        src = MapGeom{h, w, 0, 1}.source((i == 1 ? u0_ : u1_).as<__half>());
      }
      const MapGeom gout = i < 2 ? MapGeom{2 * h, 2 * w, 0, 1} : MapGeom{2 * h, 2 * w, 3, 1};
      __half* dst_map = (i == 0 ? u0_ : i == 1 ? u1_ : u2_).as<__half>();
      for (int p = 0; p < 4; p++) {
        std::vector<Tap> taps;
        for (int dy : phase_offsets(p / 2))
          for (int dx : phase_offsets(p % 2)) taps.push_back({base + dy, base + dx, 0});
        GemmOutSpec o = map_out(gout, dst_map);
        o.ostep = 2;
        o.phase_y = p / 2;
        o.phase_x = p % 2;
        gemm_taps(dev_, up_[i][p], src, taps, h, w, ACT_RELU, o, s);
      }
      h *= 2;
      w *= 2;
      step_done();
    }
  }
  if (cancelled) {
    dev_.sync(s);
    return false;
  }
  // last: conv7 (reflect) + sigmoid, cropped.
  {
    static const std::vector<Tap> taps7 = conv_taps(7);
    GemmOutSpec o;
    o.mode = OUT_STORE;
    o.out = out_.as<__half>();
    o.plane_elems = (long long)gemm_rows_alloc(hp * wp) * 8;
    gemm_taps(dev_, last_, MapGeom{hp, wp, 3, 1}.source(u2_.as<__half>()), taps7, hp, wp, ACT_SIGMOID, o, s);
    launch_pdl(lama_output, blocks_for((long long)width * height, sms), 256, 0, s, 
        out_.as<__half>(), wp, width, height, dst, dst_u8 ? 1 : 0, static_cast<const uint8_t*>(image), mask,
        mask_u8 ? 1 : 0);
    IEC_CUDA(cudaGetLastError());
  }
  step_done();
  if (step && !cancelled) {
    dev_.wait_event(step_events_[done - 1]);
    if (!step()) cancelled = true;
  }
  if (cancelled) {
    dev_.sync(s);
    return false;
  }
  return true;
}

}  // namespace iec
