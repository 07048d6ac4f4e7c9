// Real-ESRGAN general-x4v3 on the CUDA backend (see realesrgan.h).
//
// Network (crates/realesrgan-native/src/network.rs:22-140): conv3x3 3 -> 64
// + PReLU, 32 x [conv3x3 64 -> 64 + PReLU], conv3x3 64 -> 48, pixel shuffle
// x4, plus the input repeated. Tiling (lib.rs:241-289): equal grid tiles,
// each run with `margin` pixels of context, only its own output kept.
#include "realesrgan.h"

#include <algorithm>
#include <cstring>
#include <mutex>

#include "conv3x3_body_sm100.cuh"
#include "conv3x3_sm100.cuh"

namespace iec {

// The network's input, a region of the source image (f32 or 8-bit, whose
// value v means v / 255 as lib.rs:293-295 to_float), as the first layer's
// f16 channel-group planes: group 0 holds R, G, B and five zeros, group 1
// zeros (the first convolution runs with 16 input channels).
__global__ void realesrgan_prep(const void* __restrict__ src, int src_u8, int src_w, int src_h, int rx0, int ry0,
                                int rw, int rh, int mw, int mh, int count, __half* __restrict__ dst,
                                int* __restrict__ rows, int nrows) {
  griddep_wait();
  griddep_launch_dependents();
  // The fused body's row counters start at zero (it runs two launches on).
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nrows; i += gridDim.x * blockDim.x) rows[i] = 0;
  const size_t total = (size_t)count * rw * rh;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t per = (size_t)rw * rh;
    const int img = (int)(i / per);
    const int rem = (int)(i - (size_t)img * per);
    const int y = rem / rw, x = rem - y * rw;
    const size_t spix = ((size_t)img * src_h + ry0 + y) * src_w + rx0 + x;
    float c[3];
    if (src_u8) {
      const uint8_t* s = static_cast<const uint8_t*>(src) + spix * 3;
      for (int k = 0; k < 3; k++) c[k] = (float)s[k] / 255.0f;
    } else {
      const float* s = static_cast<const float*>(src) + spix * 3;
      for (int k = 0; k < 3; k++) c[k] = s[k];
    }
    __half2 rg = __floats2half2_rn(c[0], c[1]);
    __half2 b0 = __floats2half2_rn(c[2], 0.0f);
    const size_t plane = (size_t)mw * mh;
    uint4* g0 = reinterpret_cast<uint4*>(dst + ((size_t)img * 2 * plane + (size_t)y * mw + x) * 8);
    *g0 = make_uint4(*reinterpret_cast<uint32_t*>(&rg), *reinterpret_cast<uint32_t*>(&b0), 0u, 0u);
    *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(g0) + plane * 8) = make_uint4(0u, 0u, 0u, 0u);
  }
}

namespace {

template <int CIN, int COUT, int MODE>
void launch_conv(Device& dev, const void* in_maps, int count, int mw, int mh, ConvParams p, cudaStream_t s) {
  using L = ConvSmem<CIN, COUT>;
  constexpr int KCH = CIN / 8;
  // The maps as 4-D tensors: a plane row of mw pixels x 8 channels (one
  // contiguous run), rows, channel groups, images. A box is one tile's halo:
  // 16 pixels of 10 rows of every channel group.
  CUtensorMap map;
  const uint64_t dims[4] = {(uint64_t)mw * 8, (uint64_t)mh, (uint64_t)KCH, (uint64_t)count};
  const uint64_t plane = (uint64_t)mw * mh * 16;
  const uint64_t strides[3] = {(uint64_t)mw * 16, plane, plane * KCH};
  const uint32_t box[4] = {CONV_HALO_W * 8, CONV_HALO_H, (uint32_t)KCH, 1};
  encode_tensor_map(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, in_maps, dims, strides, box);
  auto kernel = conv3x3_sm100<CIN, COUT, MODE>;
  // Every variant takes the whole opt-in shared memory: one CTA per SM (so
  // the TMEM columns never run short) and room past every operand it reads.
  static int smem_bytes[64] = {};
  int& bytes = smem_bytes[dev.ordinal() & 63];
  if (bytes == 0) {
    int optin = 0;
    IEC_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev.ordinal()));
    if (optin < L::DYN_BYTES) throw Error(ERR_GPU, "not enough shared memory per block");
    IEC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
    bytes = optin;
  }
  const int grid = std::min(p.tiles, dev.sms());
  launch_pdl(kernel, grid, CONV_THREADS, (size_t)bytes, s, map, p);
}

}  // namespace

RealEsrgan::RealEsrgan(const std::string& path, const Options& opt) : dev_(opt) {
  WeightFile file = WeightFile::read(path, "REALESRG");
  DeviceScope scope(dev_);
  // network.rs:54-74: body.{2i}.weight [9 cin, cout], body.{2i}.bias, and
  // the PReLU slopes body.{2i+1}.weight of every layer but the last.
  for (int i = 0; i < STEPS; i++) {
    const int cin = i == 0 ? 3 : FEATURES;
    const bool last = i == STEPS - 1;
    const int cout = last ? 3 * SCALE * SCALE : FEATURES;
    const std::string name = "body." + std::to_string(2 * i);
    HostTensor w = file.take_tensor(name + ".weight", {(size_t)(9 * cin), (size_t)cout});
    std::vector<float> b = file.take(name + ".bias", {(size_t)cout});
    std::vector<float> slope;
    if (!last) slope = file.take("body." + std::to_string(2 * i + 1) + ".weight", {(size_t)FEATURES});
    Layer layer;
    layer.cin = i == 0 ? 16 : FEATURES;
    layer.cout = cout;
    // The K-major core-matrix image of B: [ky][cin / 8][kx][cout][8] halves
    // (a tap row's three taps side by side as the MMA's N = 3 cout).
    const int kch = layer.cin / 8;
    std::vector<uint16_t> packed((size_t)9 * kch * cout * 8, 0);
    for (int ky = 0; ky < 3; ky++)
      for (int kx = 0; kx < 3; kx++)
        for (int c = 0; c < cin; c++)
          for (int o = 0; o < cout; o++)
            packed[((((size_t)ky * kch + c / 8) * 3 + kx) * cout + o) * 8 + c % 8] =
                f32_to_half(w.values[((size_t)(ky * 3 + kx) * cin + c) * cout + o]);
    layer.w.reserve(packed.size() * 2);
    IEC_CUDA(cudaMemcpy(layer.w.get(), packed.data(), packed.size() * 2, cudaMemcpyHostToDevice));
    layer.b.reserve(cout * 4);
    IEC_CUDA(cudaMemcpy(layer.b.get(), b.data(), cout * 4, cudaMemcpyHostToDevice));
    // Slopes in [0, 1] (0.25 at initialisation) let the epilogue take
    // max(v, s v), which equals v < 0 ? s v : v for them.
    layer.slope_unit = 1;
    for (float v : slope) layer.slope_unit &= (v >= 0.0f && v <= 1.0f) ? 1 : 0;
    if (!last) {
      layer.s.reserve(FEATURES * 4);
      IEC_CUDA(cudaMemcpy(layer.s.get(), slope.data(), FEATURES * 4, cudaMemcpyHostToDevice));
    }
    layers_.push_back(std::move(layer));
  }
  file.finish();
  layer_events_.resize(STEPS);
  for (auto& e : layer_events_) IEC_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  IEC_CUDA(cudaStreamCreateWithFlags(&h2d_, cudaStreamNonBlocking));
  IEC_CUDA(cudaStreamCreateWithFlags(&d2h_, cudaStreamNonBlocking));
  for (int i = 0; i < 2; i++) {
    IEC_CUDA(cudaEventCreateWithFlags(&ev_h2d_[i], cudaEventDisableTiming));
    IEC_CUDA(cudaEventCreateWithFlags(&ev_done_[i], cudaEventDisableTiming));
    IEC_CUDA(cudaEventCreateWithFlags(&ev_d2h_[i], cudaEventDisableTiming));
  }
  IEC_CUDA(cudaEventCreateWithFlags(&ev_start_, cudaEventDisableTiming));
  IEC_CUDA(cudaDeviceSynchronize());
}

RealEsrgan::~RealEsrgan() {
  if (dev_.poisoned()) {
    // A device that failed a wait may still be running this model's work:
    // its memory is leaked rather than freed under it.
    for (auto& L : layers_) {
      L.w.leak();
      L.b.leak();
      L.s.leak();
    }
    for (DeviceBuffer* b : {&prep_, &map_a_, &map_b_, &rows_, &items_, &host_in, &host_out, &batch_in_[0], &batch_in_[1],
                            &batch_out_[0], &batch_out_[1]})
      b->leak();
    return;
  }
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(dev_.ordinal());
  for (auto& e : layer_events_) cudaEventDestroy(e);
  for (auto& e : t_events_) cudaEventDestroy(e);
  for (int i = 0; i < 2; i++) {
    cudaEventDestroy(ev_h2d_[i]);
    cudaEventDestroy(ev_done_[i]);
    cudaEventDestroy(ev_d2h_[i]);
  }
  if (ev_start_) cudaEventDestroy(ev_start_);
  if (h2d_) cudaStreamDestroy(h2d_);
  if (d2h_) cudaStreamDestroy(d2h_);
  if (prev >= 0) cudaSetDevice(prev);
}

void RealEsrgan::ensure_maps(size_t count, int w, int h, cudaStream_t stream) {
  // A region narrower or shorter than the TMA box is kept in zero-filled
  // maps of the box's size, so the box never outgrows the tensor.
  const int mw = std::max(w, CONV_HALO_W), mh = std::max(h, CONV_HALO_H);
  const size_t pixels = count * (size_t)mw * mh;
  prep_.reserve(pixels * 2 * 16);
  map_a_.reserve(pixels * 8 * 16);
  map_b_.reserve(pixels * 8 * 16);
  if (mw != w || mh != h) {
    IEC_CUDA(cudaMemsetAsync(prep_.get(), 0, pixels * 2 * 16, stream));
    IEC_CUDA(cudaMemsetAsync(map_a_.get(), 0, pixels * 8 * 16, stream));
    IEC_CUDA(cudaMemsetAsync(map_b_.get(), 0, pixels * 8 * 16, stream));
  }
}

void RealEsrgan::set_timing(size_t capacity) {
  for (auto& e : t_events_) cudaEventDestroy(e);
  t_events_.clear();
  t_kinds_.clear();
  t_used_ = 0;
  for (size_t i = 0; i < capacity; i++) {
    cudaEvent_t e;
    IEC_CUDA(cudaEventCreate(&e));
    t_events_.push_back(e);
  }
  t_kinds_.resize(capacity);
}

void RealEsrgan::mark(int kind, cudaStream_t s) {
  if (t_used_ >= t_events_.size()) return;
  IEC_CUDA(cudaEventRecord(t_events_[t_used_], s));
  t_kinds_[t_used_++] = kind;
}

size_t RealEsrgan::timing(int* kinds, float* ms, size_t n) {
  size_t w = 0;
  for (size_t i = 0; i + 1 < t_used_ && w < n; i++) {
    if (t_kinds_[i] < 0) continue;
    dev_.wait_event(t_events_[i + 1]);
    float t = 0;
    IEC_CUDA(cudaEventElapsedTime(&t, t_events_[i], t_events_[i + 1]));
    kinds[w] = t_kinds_[i];
    ms[w] = t;
    w++;
  }
  t_used_ = 0;
  return w;
}

bool RealEsrgan::body_fits(int count, int w, int h, int layers_per_launch) const {
  const long long tiles_img = (long long)((w + CONV_TILE_W - 1) / CONV_TILE_W) * ((h + CONV_TILE_H - 1) / CONV_TILE_H);
  const long long group = std::min(count, BODY_GROUP);
  const long long layers = layers_per_launch;
  const long long items = layers * count * tiles_img, group_items = layers * group * tiles_img;
  const long long group_tiles = group * tiles_img, tiles_x = (w + CONV_TILE_W - 1) / CONV_TILE_W;
  // FastDiv's exactness (numerator x divisor < 2^40) for every division of
  // an item index (body_item), and a fused launch that never runs short of
  // work.
  const long long lim = 1LL << 40;
  const long long tiles_y = (h + CONV_TILE_H - 1) / CONV_TILE_H;
  return !no_fuse_ && items < (1LL << 24) && items * group_items < lim && group_items * group_tiles < lim &&
         group_tiles * tiles_img < lim && tiles_img * tiles_x < lim && items >= 4LL * dev_.sms() &&
         count <= 256 && tiles_y <= 1024 && tiles_x <= 512;  // body_pack's fields
}

void RealEsrgan::launch_body(int count, int mw, int mh, const Region& r, int first, int layers, cudaStream_t s) {
  BodyParams bp{};
  bp.H = r.rh;
  bp.W = r.rw;
  bp.MH = mh;
  bp.MW = mw;
  bp.tiles_x = (r.rw + CONV_TILE_W - 1) / CONV_TILE_W;
  bp.tiles_y = (r.rh + CONV_TILE_H - 1) / CONV_TILE_H;
  bp.tiles_img = bp.tiles_x * bp.tiles_y;
  bp.count = count;
  bp.layers = layers;
  bp.group = std::min(count, BODY_GROUP);
  const int groups = (count + bp.group - 1) / bp.group;
  const int last_images = count - (groups - 1) * bp.group;
  bp.items = bp.layers * count * bp.tiles_img;
  bp.group_items = bp.layers * bp.group * bp.tiles_img;
  bp.last_group = groups - 1;
  bp.div_tiles_x = FastDiv((uint32_t)bp.tiles_x);
  bp.div_tiles_img = FastDiv((uint32_t)bp.tiles_img);
  bp.div_group_items = FastDiv((uint32_t)bp.group_items);
  bp.div_group_tiles = FastDiv((uint32_t)(bp.group * bp.tiles_img));
  bp.div_last_tiles = FastDiv((uint32_t)(last_images * bp.tiles_img));
  static_assert(STEPS - 2 <= BODY_MAX_LAYERS, "body layers");
  if (first < 0 || layers < 1 || first + layers > STEPS - 2) throw Error(ERR_INPUT, "body layer range");
  for (int l = 0; l < bp.layers; l++) {
    const Layer& L = layers_[first + l + 1];
    bp.weights[l] = L.w.as<uint16_t>();
    bp.bias[l] = L.b.as<float>();
    bp.slope[l] = L.s.as<float>();
    if (L.slope_unit) bp.slope_unit |= 1u << l;
  }
  // Body layer f reads map A when f is even (the first layer wrote A).
  bp.maps[0] = (first % 2 == 0 ? map_a_ : map_b_).as<__half>();
  bp.maps[1] = (first % 2 == 0 ? map_b_ : map_a_).as<__half>();
  bp.rows = rows_.as<int>() + (size_t)first * count * bp.tiles_y;
  // The item table (body_item of every index, packed), built once per shape.
  const std::array<int, 4> key = {count, r.rw, r.rh, layers};
  if (key != items_key_) {
    std::vector<uint32_t> words((size_t)bp.items);
    for (int k = 0; k < bp.items; k++) {
      const int grp = std::min(k / bp.group_items, bp.last_group);
      const int rem = k - grp * bp.group_items;
      const int per_layer = (grp == bp.last_group ? last_images : bp.group) * bp.tiles_img;
      const int l = rem / per_layer, t = rem - l * per_layer;
      const int gi = t / bp.tiles_img, tt = t - gi * bp.tiles_img;
      words[(size_t)k] = body_pack(l, grp * bp.group + gi, tt / bp.tiles_x, tt % bp.tiles_x);
    }
    items_.reserve(words.size() * 4);
    IEC_CUDA(cudaMemcpyAsync(items_.get(), words.data(), words.size() * 4, cudaMemcpyHostToDevice, s));
    IEC_CUDA(cudaStreamSynchronize(s));
    items_key_ = key;
  }
  bp.item_words = items_.as<uint32_t>();
  bp.dev_err = dev_.dev_err();
  CUtensorMap maps[2];
  for (int m = 0; m < 2; m++) {
    const uint64_t dims[4] = {(uint64_t)mw * 8, (uint64_t)mh, 8, (uint64_t)count};
    const uint64_t plane = (uint64_t)mw * mh * 16;
    const uint64_t strides[3] = {(uint64_t)mw * 16, plane, plane * 8};
    const uint32_t box[4] = {CONV_HALO_W * 8, CONV_HALO_H, 8, 1};
    encode_tensor_map(&maps[m], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, bp.maps[m], dims, strides, box);
  }
  auto kernel = conv3x3_body_sm100;
  static int smem_bytes[64] = {};
  int& bytes = smem_bytes[dev_.ordinal() & 63];
  if (bytes == 0) {
    int optin = 0;
    IEC_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev_.ordinal()));
    if (optin < BodySmem::DYN_BYTES) throw Error(ERR_GPU, "not enough shared memory per block");
    IEC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
    bytes = optin;
  }
  // Every CTA resident at once (the dataflow waits need it): a cooperative
  // launch, one CTA per SM.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::min(bp.items, dev_.sms()));
  cfg.blockDim = dim3(BODY_THREADS);
  cfg.dynamicSmemBytes = (size_t)bytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = body_pdl_ ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, maps[0], maps[1], bp);
  if (e != cudaSuccess && body_pdl_) {
    // A driver that refuses the two attributes together gets the
    // cooperative launch alone.
    (void)cudaGetLastError();
    body_pdl_ = false;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kernel, maps[0], maps[1], bp);
  }
  IEC_CUDA(e);
}

bool RealEsrgan::run_network(const void* src, bool src_u8, void* dst, bool dst_u8, int count, int src_w, int src_h,
                             const Region& r, const std::function<bool()>& step, cudaStream_t s) {
  ensure_maps(count, r.rw, r.rh, s);
  const int mw = std::max(r.rw, CONV_HALO_W), mh = std::max(r.rh, CONV_HALO_H);
  // The 32 body layers run as one fused launch, or with progress reports as
  // fused launches of BODY_STAGE layers (their reports follow each launch).
  const int stage = step ? BODY_STAGE : STEPS - 2;
  const bool fused = body_fits(count, r.rw, r.rh, stage);
  const int body_rows = (STEPS - 2) * count * ((r.rh + CONV_TILE_H - 1) / CONV_TILE_H);
  if (fused) rows_.reserve((size_t)body_rows * sizeof(int));
  mark(0, s);
  {
    const size_t total = (size_t)count * r.rw * r.rh;
    const int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)dev_.sms() * 16);
    launch_pdl(realesrgan_prep, blocks, 256, 0, s, src, (int)src_u8, src_w, src_h, r.rx0, r.ry0, r.rw, r.rh, mw, mh,
               count, prep_.as<__half>(), fused ? rows_.as<int>() : (int*)nullptr, fused ? body_rows : 0);
    IEC_CUDA(cudaGetLastError());
  }
  ConvParams p{};
  p.H = r.rh;
  p.W = r.rw;
  p.MW = mw;
  p.MH = mh;
  p.tiles_x = (r.rw + CONV_TILE_W - 1) / CONV_TILE_W;
  p.tiles_y = (r.rh + CONV_TILE_H - 1) / CONV_TILE_H;
  p.tiles = p.tiles_x * p.tiles_y * count;
  if ((size_t)p.tiles_x * p.tiles_y * count >= (1u << 24) || p.tiles_x >= (1 << 16) || p.tiles_y >= (1 << 16))
    throw Error(ERR_INPUT, "too many tiles for one pass");
  p.div_tiles_x = FastDiv((uint32_t)p.tiles_x);
  p.div_tiles_y = FastDiv((uint32_t)p.tiles_y);
  p.dev_err = dev_.dev_err();
  const void* in = prep_.get();
  // Launch units (first layer, layer count): the first layer, the body (fused
  // launches, or one launch per layer), the last layer.
  std::vector<std::array<int, 2>> units;
  units.push_back({0, 1});
  for (int f = 1; f < STEPS - 1; f += fused ? stage : 1) units.push_back({f, fused ? std::min(stage, STEPS - 1 - f) : 1});
  units.push_back({STEPS - 1, 1});
  bool cancelled = false;
  for (size_t u = 0; u < units.size(); u++) {
    const int i = units[u][0], n = units[u][1];
    // the unit's output map: the one its last layer writes
    __half* out = ((i + n - 1) % 2 == 0 ? map_a_ : map_b_).as<__half>();
    if (fused && i >= 1 && i < STEPS - 1) {
      mark(4, s);
      launch_body(count, mw, mh, r, i - 1, n, s);
    } else {
      const Layer& L = layers_[i];
      p.weights = L.w.as<uint16_t>();
      p.bias = L.b.as<float>();
      p.slope = L.s.get() ? L.s.as<float>() : nullptr;
      p.slope_unit = L.slope_unit;
      p.out = out;
      mark(i == 0 ? 1 : i < STEPS - 1 ? 2 : 3, s);
      if (i == 0) {
        launch_conv<16, 64, CONV_PRELU>(dev_, in, count, mw, mh, p, s);
      } else if (i < STEPS - 1) {
        launch_conv<64, 64, CONV_PRELU>(dev_, in, count, mw, mh, p, s);
      } else {
        ShuffleOut& so = p.shuffle;
        so.src = src;
        so.dst = dst;
        so.src_w = src_w;
        so.src_h = src_h;
        so.rx0 = r.rx0;
        so.ry0 = r.ry0;
        so.kx0 = r.kx0;
        so.ky0 = r.ky0;
        so.kx1 = r.kx1;
        so.ky1 = r.ky1;
        so.src_u8 = src_u8;
        so.dst_u8 = dst_u8;
        launch_conv<64, 48, CONV_SHUFFLE>(dev_, in, count, mw, mh, p, s);
        mark(-1, s);
      }
    }
    in = out;
    if (step) {
      // Two slots, as the reference's Steps (native-vulkan lib.rs:521-572):
      // unit u is queued before unit u - 1 is waited for and its layers
      // reported, so the progress reports cost the GPU no idle time.
      IEC_CUDA(cudaEventRecord(layer_events_[u], s));
      if (u >= 1) {
        dev_.wait_event(layer_events_[u - 1]);
        for (int k = 0; k < units[u - 1][1] && !cancelled; k++) cancelled = !step();
        if (cancelled) break;
      }
    }
  }
  if (step && !cancelled) {
    dev_.wait_event(layer_events_[units.size() - 1]);
    if (!step()) cancelled = true;
  }
  if (cancelled) dev_.sync(s);  // nothing may still use the buffers
  return !cancelled;
}

std::vector<std::array<size_t, 4>> RealEsrgan::tile_windows(size_t width, size_t height, size_t tile, size_t first,
                                                            size_t last) {
  if (tile == 0) throw Error(ERR_INPUT, "tile size 0");
  const size_t cols = (width + tile - 1) / tile, rows = (height + tile - 1) / tile;
  std::vector<std::array<size_t, 4>> out;
  for (size_t t = first; t < std::min(last, cols * rows); t++) {
    const size_t j = t / cols, i = t % cols;
    out.push_back({i * width / cols, j * height / rows, (i + 1) * width / cols, (j + 1) * height / rows});
  }
  return out;
}

void RealEsrgan::run_tiled_device(const void* src, bool src_u8, void* dst, bool dst_u8, size_t count, size_t width,
                                  size_t height, size_t tile, size_t margin,
                                  const std::function<bool(float)>& progress, cudaStream_t s, size_t first,
                                  size_t last) {
  const std::vector<std::array<size_t, 4>> windows = tile_windows(width, height, tile, first, last);
  const float steps = (float)(windows.size() * STEPS);
  size_t done = 0;
  std::function<bool()> step;
  if (progress) step = [&] { return progress((float)(++done) / steps); };
  for (const auto& wnd : windows) {
    const size_t x0 = wnd[0], y0 = wnd[1], x1 = wnd[2], y1 = wnd[3];
    const size_t rx0 = x0 > margin ? x0 - margin : 0, ry0 = y0 > margin ? y0 - margin : 0;
    const size_t rx1 = margin > width - x1 ? width : x1 + margin;
    const size_t ry1 = margin > height - y1 ? height : y1 + margin;
    Region r;
    r.rx0 = (int)rx0;
    r.ry0 = (int)ry0;
    r.rw = (int)(rx1 - rx0);
    r.rh = (int)(ry1 - ry0);
    r.kx0 = (int)(x0 - rx0);
    r.ky0 = (int)(y0 - ry0);
    r.kx1 = (int)(x1 - rx0);
    r.ky1 = (int)(y1 - ry0);
    if (!run_network(src, src_u8, dst, dst_u8, (int)count, (int)width, (int)height, r, step, s))
      throw Error(CANCELLED, "cancelled");
  }
}

size_t RealEsrgan::chunk_for(size_t width, size_t height) const {
  if (dev_.batch_chunk() > 0) return (size_t)dev_.batch_chunk();
  // About a million pixels per pass: the two 64-channel maps (256 MB) stay
  // near the 126 MB L2 while each layer still fills the GPU many times over.
  const size_t px = std::max<size_t>(1, width * height);
  return std::max<size_t>(1, ((size_t)1 << 20) / px);
}

size_t RealEsrgan::launches(size_t count, size_t width, size_t height) const {
  const size_t chunk = chunk_for(width, height);
  size_t n = 0;
  for (size_t c0 = 0; c0 < count; c0 += chunk) {
    const int m = (int)std::min(chunk, count - c0);
    n += body_fits(m, (int)width, (int)height, STEPS - 2) ? 4 : STEPS + 1;
  }
  return n;
}

void RealEsrgan::run_device(const float* src, float* dst, size_t count, size_t width, size_t height,
                            cudaStream_t s) {
  const size_t chunk = chunk_for(width, height);
  Region r{0, 0, (int)width, (int)height, 0, 0, (int)width, (int)height};
  for (size_t c0 = 0; c0 < count; c0 += chunk) {
    const size_t n = std::min(chunk, count - c0);
    run_network(src + c0 * width * height * 3, false, dst + c0 * width * height * 3 * SCALE * SCALE, false, (int)n,
                (int)width, (int)height, r, nullptr, s);
  }
}

void RealEsrgan::run_batch_host(const void* src, bool src_u8, void* dst, bool dst_u8, size_t count, size_t width,
                                size_t height, cudaStream_t s) {
  // Three streams: H2D of chunk c + 1 and D2H of chunk c - 1 run while chunk
  // c computes; two device buffers of each kind alternate. 8-bit images move
  // a quarter of the bytes of f32 ones over the host link.
  const size_t chunk = chunk_for(width, height);
  const size_t in_elem = src_u8 ? 1 : 4, out_elem = dst_u8 ? 1 : 4;
  const size_t img_vals = width * height * 3, out_vals = img_vals * SCALE * SCALE;
  for (int b = 0; b < 2; b++) {
    batch_in_[b].reserve(chunk * img_vals * in_elem);
    batch_out_[b].reserve(chunk * out_vals * out_elem);
  }
  Region r{0, 0, (int)width, (int)height, 0, 0, (int)width, (int)height};
  IEC_CUDA(cudaEventRecord(ev_start_, s));
  IEC_CUDA(cudaStreamWaitEvent(h2d_, ev_start_, 0));
  IEC_CUDA(cudaStreamWaitEvent(d2h_, ev_start_, 0));
  const uint8_t* in_bytes = static_cast<const uint8_t*>(src);
  uint8_t* out_bytes = static_cast<uint8_t*>(dst);
  size_t k = 0;
  for (size_t c0 = 0; c0 < count; c0 += chunk, k++) {
    const int b = (int)(k & 1);
    const size_t n = std::min(chunk, count - c0);
    const size_t ib = n * img_vals * in_elem, ob = n * out_vals * out_elem;
    if (k >= 2) IEC_CUDA(cudaStreamWaitEvent(h2d_, ev_done_[b], 0));  // chunk k - 2 has read batch_in_[b]
    IEC_CUDA(cudaMemcpyAsync(batch_in_[b].get(), in_bytes + c0 * img_vals * in_elem, ib, cudaMemcpyHostToDevice, h2d_));
    IEC_CUDA(cudaEventRecord(ev_h2d_[b], h2d_));
    IEC_CUDA(cudaStreamWaitEvent(s, ev_h2d_[b], 0));
    if (k >= 2) IEC_CUDA(cudaStreamWaitEvent(s, ev_d2h_[b], 0));  // chunk k - 2's output is copied out
    run_network(batch_in_[b].get(), src_u8, batch_out_[b].get(), dst_u8, (int)n, (int)width, (int)height, r, nullptr,
                s);
    IEC_CUDA(cudaEventRecord(ev_done_[b], s));
    IEC_CUDA(cudaStreamWaitEvent(d2h_, ev_done_[b], 0));
    IEC_CUDA(cudaMemcpyAsync(out_bytes + c0 * out_vals * out_elem, batch_out_[b].get(), ob, cudaMemcpyDeviceToHost,
                             d2h_));
    IEC_CUDA(cudaEventRecord(ev_d2h_[b], d2h_));
  }
  // The caller's stream completes only once every output is in host memory.
  for (int b = 0; b < 2 && (size_t)b < k; b++) IEC_CUDA(cudaStreamWaitEvent(s, ev_d2h_[b], 0));
  dev_.sync(s);
}

}  // namespace iec

// ------------------------------------------------------- allocation-free path
namespace iec {

namespace {

// The feature maps of iec_realesrgan_run_device_noalloc: the first layer's
// two channel groups and the two 64-channel maps, 18 x 16 bytes per pixel,
// for at most NOALLOC_MAX_PIXELS pixels (31.5 MiB). The array is part of the
// library's device code, so every GPU that loads the library holds it until
// the process exits, and every call on a device shares it.
constexpr size_t NOALLOC_PREP_BYTES = RealEsrgan::NOALLOC_MAX_PIXELS * 2 * 16;
constexpr size_t NOALLOC_MAP_BYTES = RealEsrgan::NOALLOC_MAX_PIXELS * 8 * 16;
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_PREP_BYTES + 2 * NOALLOC_MAP_BYTES];

// The array's device address on each device. In host code the name
// g_noalloc_scratch is only a host-side stand-in, so the address is looked
// up once per device, with that device current, and passed to the kernels.
std::mutex g_noalloc_mutex;
uint8_t* g_noalloc_ptr[64] = {};

uint8_t* noalloc_scratch(int device) {
  if (device < 0 || device >= 64) throw Error(ERR_GPU, "device ordinal out of range for the fixed scratch");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      throw Error(ERR_GPU, std::string("cudaGetSymbolAddress of the fixed scratch: ") + cudaGetErrorString(e));
    g_noalloc_ptr[device] = static_cast<uint8_t*>(p);
  }
  return g_noalloc_ptr[device];
}

}  // namespace

void RealEsrgan::run_device_noalloc(const float* src, float* dst, size_t count, size_t width, size_t height,
                                    cudaStream_t s) {
  const int w = (int)width, h = (int)height;
  const int mw = std::max(w, CONV_HALO_W), mh = std::max(h, CONV_HALO_H);
  // Every input check comes before any work is queued. The scratch holds
  // count x mw x mh pixels; each factor is compared against the limit
  // divided by the others, so no product can wrap around.
  const size_t per_image = (size_t)mw * (size_t)mh;
  const bool fits = count >= 1 && per_image <= NOALLOC_MAX_PIXELS && count <= NOALLOC_MAX_PIXELS / per_image;
  if (!fits)
    throw Error(ERR_INPUT, std::to_string(count) + " images of " + std::to_string(width) + " x " +
                               std::to_string(height) + " need " + std::to_string(count) + " x " +
                               std::to_string(per_image) + " pixels of scratch; the allocation-free entry point holds " +
                               std::to_string(NOALLOC_MAX_PIXELS));
  const size_t pixels = count * per_image;
  ConvParams p{};
  p.H = h;
  p.W = w;
  p.MW = mw;
  p.MH = mh;
  p.tiles_x = (w + CONV_TILE_W - 1) / CONV_TILE_W;
  p.tiles_y = (h + CONV_TILE_H - 1) / CONV_TILE_H;
  if ((size_t)p.tiles_x * p.tiles_y * count >= (1u << 24) || p.tiles_x >= (1 << 16) || p.tiles_y >= (1 << 16))
    throw Error(ERR_INPUT, "too many tiles for one pass");
  p.tiles = p.tiles_x * p.tiles_y * (int)count;
  uint8_t* base = noalloc_scratch(dev_.ordinal());
  __half* prep = reinterpret_cast<__half*>(base);
  __half* maps[2] = {reinterpret_cast<__half*>(base + NOALLOC_PREP_BYTES),
                     reinterpret_cast<__half*>(base + NOALLOC_PREP_BYTES + NOALLOC_MAP_BYTES)};
  // The array keeps the previous call's values; the margin of maps kept
  // larger than the image (too small for a TMA box) must read as zeros.
  if (mw != w || mh != h) {
    IEC_CUDA(cudaMemsetAsync(prep, 0, pixels * 2 * 16, s));
    IEC_CUDA(cudaMemsetAsync(maps[0], 0, pixels * 8 * 16, s));
    IEC_CUDA(cudaMemsetAsync(maps[1], 0, pixels * 8 * 16, s));
  }
  {
    const size_t total = count * (size_t)w * h;
    const int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)dev_.sms() * 16);
    launch_pdl(realesrgan_prep, blocks, 256, 0, s, src, 0, w, h, 0, 0, w, h, mw, mh, (int)count, prep, (int*)nullptr, 0);
    IEC_CUDA(cudaGetLastError());
  }
  p.div_tiles_x = FastDiv((uint32_t)p.tiles_x);
  p.div_tiles_y = FastDiv((uint32_t)p.tiles_y);
  p.dev_err = dev_.dev_err();
  const void* in = prep;
  for (int i = 0; i < STEPS; i++) {
    const Layer& L = layers_[i];
    p.weights = L.w.as<uint16_t>();
    p.bias = L.b.as<float>();
    p.slope = L.s.get() ? L.s.as<float>() : nullptr;
    p.slope_unit = L.slope_unit;
    p.out = maps[i % 2];
    if (i == 0) {
      launch_conv<16, 64, CONV_PRELU>(dev_, in, (int)count, mw, mh, p, s);
    } else if (i < STEPS - 1) {
      launch_conv<64, 64, CONV_PRELU>(dev_, in, (int)count, mw, mh, p, s);
    } else {
      ShuffleOut& so = p.shuffle;
      so.src = src;
      so.dst = dst;
      so.src_w = w;
      so.src_h = h;
      so.rx0 = so.ry0 = 0;
      so.kx0 = so.ky0 = 0;
      so.kx1 = w;
      so.ky1 = h;
      so.src_u8 = 0;
      so.dst_u8 = 0;
      launch_conv<64, 48, CONV_SHUFFLE>(dev_, in, (int)count, mw, mh, p, s);
    }
    in = p.out;
  }
}

}  // namespace iec
