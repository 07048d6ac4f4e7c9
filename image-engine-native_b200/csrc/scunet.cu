// SCUNet on the CUDA backend (see scunet.h).
//
// Network (crates/scunet-native/src/network.rs:27-478, swin.rs:18-254):
// pad to a multiple of 64 by edge repeat, head conv3 3 -> 64, three levels
// down (4 Swin-Conv blocks, then 2x2 stride-2 halving into a skip), body
// (512 channels), three levels up (skip add, 2x2 transposed doubling, 4
// blocks), head conv again added onto x, tail conv3 64 -> 3, crop.
#include "scunet.h"

#include <algorithm>
#include <cmath>
#include <cstring>

#include "igemm_sm100.cuh"

namespace iec {

struct Scunet::Block {
  int c = 0, h = 0;
  bool shifted = false;
  PackedWeights split, conv1, conv2, join, qkv, proj, fc1, fc2;
  WindowBlockWeights wblock;  // LN1, qkv, attention and projection in one kernel, where the width fits
  JoinSplitWeights joinsplit;  // this block's join and the next one's split in one kernel, where the width fits
  MlpWeights mlp;  // LN2, fc1, GELU and fc2 fused (mlp_sm100.cuh), where the width fits
  LnRowsWeights lnqkv;  // LN1 + window partition + qkv (lnrows_sm100.cuh), where the width fits
  DeviceBuffer ln1g, ln1b, ln2g, ln2b, bias;  // LN params f32; attention bias tables f32
};

struct Scunet::Level {
  int c = 0;
  std::vector<Block> blocks;
  PackedWeights resample;  // down: halving [4c, 2c]; up: doubling [2c, 4c]
  bool down = false, up = false;
};

namespace {

constexpr int N_TOK = 64, SHIFT = 4;

long long rows_alloc(long long rows) { return std::max<long long>(rows, 128); }

void upload(DeviceBuffer& b, const std::vector<float>& v) {
  b.reserve(v.size() * 4);
  IEC_CUDA(cudaMemcpy(b.get(), v.data(), v.size() * 4, cudaMemcpyHostToDevice));
}

// A 1x1 layer's host values, kept where another kernel packs them again.
struct Linear {
  std::vector<float> w, b;
};

void linear(WeightFile& f, PackedWeights& pw, const std::string& name, int k, int n, bool bias,
            Linear* keep = nullptr) {
  HostTensor w = f.take_tensor(name + ".weight", {(size_t)k, (size_t)n});
  std::vector<float> b;
  if (bias) b = f.take(name + ".bias", {(size_t)n});
  pack_weights(pw, w.values, 1, k, n, bias ? b.data() : nullptr);
  if (keep) {
    keep->w = std::move(w.values);
    keep->b = std::move(b);
  }
}

void conv3(WeightFile& f, PackedWeights& pw, const std::string& name, int cin, int cout, int cin_pad) {
  HostTensor w = f.take_tensor(name + ".weight", {(size_t)(9 * cin), (size_t)cout});
  std::vector<float> wv((size_t)9 * cin_pad * cout, 0.0f);
  for (int tap = 0; tap < 9; tap++)
    for (int c = 0; c < cin; c++)
      for (int o = 0; o < cout; o++)
        wv[((size_t)tap * cin_pad + c) * cout + o] = w.values[((size_t)tap * cin + c) * cout + o];
  pack_weights(pw, wv, 9, cin_pad, cout, nullptr);
}

// swin.rs:26-50: the position bias, and for a shifted block its sums with the
// masks of the four window classes (last column 1, last row 2).
std::vector<float> bias_tables(const std::vector<float>& position, bool shifted) {
  if (!shifted) return position;
  auto region = [](int v, bool last) { return (last && v >= 8 - SHIFT) ? 1 : 0; };
  std::vector<float> t;
  t.reserve(position.size() * 4);
  const size_t heads = position.size() / (N_TOK * N_TOK);
  for (int cls = 0; cls < 4; cls++) {
    const bool last_col = cls & 1, last_row = cls & 2;
    auto id = [&](int i) { return region(i / 8, last_row) * 2 + region(i % 8, last_col); };
    for (size_t hd = 0; hd < heads; hd++)
      for (int i = 0; i < N_TOK; i++)
        for (int j = 0; j < N_TOK; j++)
          t.push_back(position[(hd * N_TOK + i) * N_TOK + j] + (id(i) == id(j) ? 0.0f : -INFINITY));
  }
  return t;
}

// The network's input: the region of the source image, padded to (ph, pw)
// by repeating its last row and column (network.rs:358-379), as two f16
// planes (R, G, B and zeros; zeros) for the 16-channel head convolution.
__global__ void scunet_prep(const void* __restrict__ src, int src_u8, int src_w, int rx0, int ry0, int rw, int rh,
                            int ph, int pw, __half* __restrict__ dst, long long plane) {
  griddep_wait();
  griddep_launch_dependents();
  const long long total = (long long)ph * pw;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int y = (int)(i / pw), x = (int)(i % pw);
    const long long sp = ((long long)(ry0 + min(y, rh - 1))) * src_w + rx0 + min(x, rw - 1);
    float c[3];
    for (int k = 0; k < 3; k++)
      c[k] = src_u8 ? (float)static_cast<const uint8_t*>(src)[sp * 3 + k] / 255.0f
                    : static_cast<const float*>(src)[sp * 3 + k];
    __half2 rg = __floats2half2_rn(c[0], c[1]), b0 = __floats2half2_rn(c[2], 0.0f);
    *reinterpret_cast<uint4*>(dst + i * 8) =
        make_uint4(*reinterpret_cast<uint32_t*>(&rg), *reinterpret_cast<uint32_t*>(&b0), 0u, 0u);
    *reinterpret_cast<uint4*>(dst + plane + i * 8) = make_uint4(0u, 0u, 0u, 0u);
  }
}

// network.rs:410-441: rows of the 2x2 stride-2 convolution, each the four
// input pixels (y, x), (y, x + 1), (y + 1, x), (y + 1, x + 1) in turn.
__global__ void scunet_halve_gather(const __half* __restrict__ x, long long x_plane, int groups, int h, int w,
                                    __half* __restrict__ out, long long out_plane) {
  griddep_wait();
  griddep_launch_dependents();
  const int oh = h / 2, ow = w / 2;
  const long long total = (long long)oh * ow * 4 * groups;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i % ((long long)oh * ow);
    const int rest = (int)(i / ((long long)oh * ow));  // q * groups + g
    const int q = rest / groups, g = rest % groups;
    const int y = 2 * (int)(r / ow) + (q >> 1), xx = 2 * (int)(r % ow) + (q & 1);
    *reinterpret_cast<uint4*>(out + (long long)rest * out_plane + r * 8) =
        *reinterpret_cast<const uint4*>(x + (long long)g * x_plane + ((long long)y * w + xx) * 8);
  }
}

// x += s over `planes` planes of `rows` rows (network.rs:382-393).
__global__ void scunet_add(__half* __restrict__ x, const __half* __restrict__ s, long long plane, int planes,
                           long long rows) {
  griddep_wait();
  griddep_launch_dependents();
  const long long total = (long long)planes * rows;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long at = (i / rows) * plane + (i % rows) * 8;
    uint4 a = *reinterpret_cast<uint4*>(x + at);
    const uint4 b = *reinterpret_cast<const uint4*>(s + at);
    __half2* ha = reinterpret_cast<__half2*>(&a);
    const __half2* hb = reinterpret_cast<const __half2*>(&b);
    for (int e = 0; e < 4; e++) {
      const float2 fa = __half22float2(ha[e]), fb = __half22float2(hb[e]);
      ha[e] = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);
    }
    *reinterpret_cast<uint4*>(x + at) = a;
  }
}

// The tail's three channels (plane 0) of the kept window, to the output
// image (f32 or 8-bit, lib.rs:264-270 to_byte).
__global__ void scunet_store(const __half* __restrict__ y, int pw, int kx0, int ky0, int kx1, int ky1, int rx0,
                             int ry0, void* __restrict__ dst, int dst_u8, int dst_w) {
  griddep_wait();
  griddep_launch_dependents();
  const int kw = kx1 - kx0;
  const long long total = (long long)kw * (ky1 - ky0);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int yy = ky0 + (int)(i / kw), xx = kx0 + (int)(i % kw);
    const __half* px = y + ((long long)yy * pw + xx) * 8;
    const long long o = ((long long)(ry0 + yy) * dst_w + rx0 + xx) * 3;
    for (int k = 0; k < 3; k++) {
      const float v = __half2float(px[k]);
      if (dst_u8)
        static_cast<uint8_t*>(dst)[o + k] = (uint8_t)roundf(fminf(fmaxf(v, 0.0f), 1.0f) * 255.0f);
      else
        static_cast<float*>(dst)[o + k] = v;
    }
  }
}

int blocks_for(long long n, int sms) { return (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, (long long)sms * 16)); }

}  // namespace

Scunet::Scunet(const std::string& path, const Options& opt) : dev_(opt) {
  WeightFile f = WeightFile::read(path, std::string("SCUNET\0\0", 8).c_str());
  DeviceScope scope(dev_);
  conv3(f, head_, "m_head.0", 3, DIM, 16);
  auto load_block = [&](Block& b, const std::string& name, int c, bool shifted, Linear* split, Linear* join) {
    b.c = c;
    b.h = c / 2;
    b.shifted = shifted;
    const int h = b.h;
    linear(f, b.split, name + ".conv1_1", c, c, true, split);
    conv3(f, b.conv1, name + ".conv_block.0", h, h, h);
    conv3(f, b.conv2, name + ".conv_block.2", h, h, h);
    const std::string t = name + ".trans_block";
    std::vector<float> wq_keep, bq_keep, g1_keep, be1_keep;  // LN1 and qkv again for the fused window block
    {
      // LN1 and the qkv layer: the separate launches' weights, and the same
      // values for the kernel that folds LN1 and the window partition into
      // the product's staged rows
      const std::vector<float> g1 = f.take(t + ".ln1.weight", {(size_t)h}), be1 = f.take(t + ".ln1.bias", {(size_t)h});
      HostTensor wq = f.take_tensor(t + ".msa.embedding_layer.weight", {(size_t)h, (size_t)(3 * h)});
      const std::vector<float> bq = f.take(t + ".msa.embedding_layer.bias", {(size_t)(3 * h)});
      upload(b.ln1g, g1);
      upload(b.ln1b, be1);
      pack_weights(b.qkv, wq.values, 1, h, 3 * h, bq.data());
      if (lnrows_fits(h, 3 * h)) pack_lnrows(b.lnqkv, h, 3 * h, wq.values, bq, g1, be1);
      wq_keep = std::move(wq.values);
      bq_keep = bq;
      g1_keep = g1;
      be1_keep = be1;
    }
    upload(b.bias, attention_bias_layout(bias_tables(f.take(t + ".msa.position_bias", {(size_t)(h / 32), 64, 64}), shifted)));
    {
      HostTensor w = f.take_tensor(t + ".msa.linear.weight", {(size_t)h, (size_t)h});
      const std::vector<float> pb = f.take(t + ".msa.linear.bias", {(size_t)h});
      pack_weights(b.proj, w.values, 1, h, h, pb.data());
      if (window_block_fits(h)) pack_window_block(b.wblock, h, wq_keep, bq_keep, w.values, pb, g1_keep, be1_keep);
    }
    {
      // LN2 and the MLP: the separate launches' weights, and the same values
      // packed for the fused MLP kernel.
      const std::vector<float> g2 = f.take(t + ".ln2.weight", {(size_t)h}), be2 = f.take(t + ".ln2.bias", {(size_t)h});
      HostTensor w1 = f.take_tensor(t + ".mlp.0.weight", {(size_t)h, (size_t)(4 * h)});
      const std::vector<float> bb1 = f.take(t + ".mlp.0.bias", {(size_t)(4 * h)});
      HostTensor w2 = f.take_tensor(t + ".mlp.2.weight", {(size_t)(4 * h), (size_t)h});
      const std::vector<float> bb2 = f.take(t + ".mlp.2.bias", {(size_t)h});
      upload(b.ln2g, g2);
      upload(b.ln2b, be2);
      pack_weights(b.fc1, w1.values, 1, h, 4 * h, bb1.data());
      pack_weights(b.fc2, w2.values, 1, 4 * h, h, bb2.data());
      if (mlp_fits(h)) pack_mlp(b.mlp, h, w1.values, bb1, w2.values, bb2, g2, be2);
      if (b.wblock.c == 32) pack_window_block_mlp(b.wblock, w1.values, bb1, w2.values, bb2, g2, be2);
    }
    linear(f, b.join, name + ".conv1_2", c, c, true, join);
  };
  auto load_level = [&](Level& L, const std::string& name, int first, int c) {
    L.c = c;
    L.blocks.resize(BLOCKS);
    std::vector<Linear> splits(BLOCKS), joins(BLOCKS);
    for (int b = 0; b < BLOCKS; b++)
      load_block(L.blocks[b], name + "." + std::to_string(first + b), c, b % 2 == 1, &splits[b], &joins[b]);
    // a block's join with the next block's split, for the fused boundary
    if (joinsplit_fits(c))
      for (int b = 0; b + 1 < BLOCKS; b++)
        pack_joinsplit(L.blocks[b].joinsplit, c, joins[b].w, joins[b].b, splits[b + 1].w, splits[b + 1].b);
  };
  const int widths[3] = {DIM, 2 * DIM, 4 * DIM};
  for (int i = 0; i < 3; i++) {
    auto L = std::make_unique<Level>();
    const std::string name = "m_down" + std::to_string(i + 1);
    load_level(*L, name, 0, widths[i]);
    L->down = true;
    linear(f, L->resample, name + "." + std::to_string(BLOCKS), 4 * widths[i], 2 * widths[i], false);
    levels_.push_back(std::move(L));
  }
  {
    auto L = std::make_unique<Level>();
    load_level(*L, "m_body", 0, 8 * DIM);
    levels_.push_back(std::move(L));
  }
  for (int i = 2; i >= 0; i--) {
    auto L = std::make_unique<Level>();
    const std::string name = "m_up" + std::to_string(i + 1);
    L->up = true;
    linear(f, L->resample, name + ".0", 2 * widths[i], 4 * widths[i], false);
    load_level(*L, name, 1, widths[i]);
    levels_.push_back(std::move(L));
  }
  conv3(f, tail_, "m_tail.0", DIM, 3, DIM);
  f.finish();
  step_events_.resize(STEPS);
  for (auto& e : step_events_) IEC_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  IEC_CUDA(cudaStreamCreateWithFlags(&s_conv_, cudaStreamNonBlocking));
  IEC_CUDA(cudaEventCreateWithFlags(&ev_in_, cudaEventDisableTiming));
  IEC_CUDA(cudaEventCreateWithFlags(&ev_conv_, cudaEventDisableTiming));
  IEC_CUDA(cudaDeviceSynchronize());
}

Scunet::~Scunet() {
  if (dev_.poisoned()) {
    graph_.leak();
    for (DeviceBuffer* b : {&img_, &x_, &y_, &t_, &tok_, &qkv_, &att_, &ln2_, &hid_, &gat_, &skip_[0], &skip_[1],
                            &skip_[2], &out_, &host_in, &host_out})
      b->leak();
    return;  // the weights stay with the leaked device too
  }
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(dev_.ordinal());
  for (auto& e : step_events_) cudaEventDestroy(e);
  for (cudaEvent_t e : {ev_in_, ev_conv_})
    if (e) cudaEventDestroy(e);
  if (s_conv_) cudaStreamDestroy(s_conv_);
  if (prev >= 0) cudaSetDevice(prev);
}

void Scunet::ensure(int ph, int pw) {
  const long long P = (long long)ph * pw;
  if (P <= alloc_pixels_) return;
  alloc_gen_++;  // buffers may move: captured passes must not replay
  // Per level (c channels, Pl pixels): the largest need of each buffer, in
  // planes x max(rows, 128) x 8 halves.
  auto bytes = [](long long planes, long long rows) { return (size_t)(planes * rows_alloc(rows) * 8 * 2); };
  size_t bx = 0, by = 0, bt = 0, bq = 0, bh = 0, bg = 0, bs[3] = {0, 0, 0};
  for (int l = 0; l < 4; l++) {
    const long long c = (long long)DIM << l, Pl = P >> (2 * l), h = c / 2;
    bx = std::max(bx, bytes(c / 8, Pl));
    by = std::max(by, bytes(c / 8, Pl));
    bt = std::max(bt, bytes(h / 8, Pl));
    bq = std::max(bq, bytes(3 * h / 8, Pl));
    bh = std::max(bh, bytes(4 * h / 8, Pl));
    if (l < 3) {
      bg = std::max(bg, bytes(4 * c / 8, Pl / 4));
      bs[l] = bytes(2 * c / 8, Pl / 4);
    }
  }
  img_.reserve(bytes(2, P));
  x_.reserve(bx);
  y_.reserve(by);
  t_.reserve(bt);
  tok_.reserve(bt);
  att_.reserve(bt);
  ln2_.reserve(bt);
  qkv_.reserve(bq);
  hid_.reserve(bh);
  gat_.reserve(bg);
  for (int i = 0; i < 3; i++) skip_[i].reserve(bs[i]);
  out_.reserve(bytes(1, P));
  alloc_pixels_ = (int)P;
}

bool Scunet::run_region(const void* src, bool src_u8, void* dst, bool dst_u8, int src_w, int src_h, int rx0,
                        int ry0, int rw, int rh, int kx0, int ky0, int kx1, int ky1,
                        const std::function<bool()>& step, cudaStream_t s) {
  (void)src_h;
  SerialStreams serial(dev_.timing(), {&s_conv_}, s);
  const int ph = (rh + MULTIPLE - 1) / MULTIPLE * MULTIPLE, pw = (rw + MULTIPLE - 1) / MULTIPLE * MULTIPLE;
  ensure(ph, pw);
  const int sms = dev_.sms();
  const long long P = (long long)ph * pw;
  __half* img = img_.as<__half>();
  const long long img_plane = rows_alloc(P) * 8;
  launch_pdl(scunet_prep, blocks_for(P, sms), 256, 0, s, src, src_u8, src_w, rx0, ry0, rw, rh, ph, pw, img, img_plane);
  IEC_CUDA(cudaGetLastError());

  int done = 0;
  bool cancelled = false;
  auto block_done = [&]() {
    if (!step) return;
    IEC_CUDA(cudaEventRecord(step_events_[done], s));
    if (done >= 1) {
      dev_.wait_event(step_events_[done - 1]);
      if (!step()) cancelled = true;
    }
    done++;
  };

  int H = ph, W = pw;
  __half* x = x_.as<__half>();
  auto plane = [](long long rows) { return rows_alloc(rows) * 8; };
  // x = head(image)
  {
    GemmOutSpec o;
    o.mode = OUT_STORE;
    o.out = x;
    o.plane_elems = plane(P);
    gemm_conv3(dev_, head_, img, img_plane, H, W, ACT_NONE, o, s);
  }

  auto run_level = [&](Level& L) {
    const int c = L.c, h = c / 2, Pl = H * W;
    const long long pl = plane(Pl);
    __half* y = y_.as<__half>();
    __half *t = t_.as<__half>(), *tok = tok_.as<__half>(), *qkv = qkv_.as<__half>(), *att = att_.as<__half>();
    __half *ln2 = ln2_.as<__half>(), *hid = hid_.as<__half>();
    GemmOutSpec o;
    o.plane_elems = pl;
    // y = split_0(x)
    o.mode = OUT_STORE;
    o.out = y;
    o.plane0 = 0;
    gemm_rows(dev_, L.blocks[0].split, x, pl, Pl, ACT_NONE, o, s);
    for (int b = 0; b < BLOCKS && !cancelled; b++) {
      Block& B = L.blocks[b];
      const int shift = B.shifted ? SHIFT : 0;
      // Convolution half (network.rs:136-153): t = relu(conv(y[:h])); y[:h] += conv(t),
      // on the side stream: it touches only y's first h channels and t, the
      // attention half below only y's last h channels and its own buffers.
      IEC_CUDA(cudaEventRecord(ev_in_, s));
      IEC_CUDA(cudaStreamWaitEvent(s_conv_, ev_in_, 0));
      {
        GemmOutSpec c;
        c.plane_elems = pl;
        c.mode = OUT_STORE;
        c.out = t;
        gemm_conv3(dev_, B.conv1, y, pl, H, W, ACT_RELU, c, s_conv_);
        c.mode = OUT_ACCUM;
        c.out = y;
        gemm_conv3(dev_, B.conv2, t, pl, H, W, ACT_NONE, c, s_conv_);
      }
      IEC_CUDA(cudaEventRecord(ev_conv_, s_conv_));
      // Attention (swin.rs:124-220) on y[h:]: LN1 + window partition, qkv,
      // attention, projection added back at the tokens' pixels.
      const WindowMap wm{8, H, W, H, W, shift};
      if (fused_mlp_ && B.wblock.c == h) {
        // LN1, qkv, attention, projection and the residual add in one kernel
        window_block(dev_, B.wblock, B.bias.as<float>(), B.shifted, H / 8, W / 8, y, pl, h / 8, wm, s);
      } else {
        if (fused_mlp_ && B.lnqkv.c == h) {
          lnrows_planar(dev_, B.lnqkv, y + (long long)(h / 8) * pl, pl, Pl, wm, qkv, pl, s);
        } else {
          layer_norm_planar(y, pl, h / 8, Pl, h, B.ln1g.as<float>(), B.ln1b.as<float>(), tok, pl, &wm, s);
          o.mode = OUT_STORE;
          o.out = qkv;
          o.plane0 = 0;
          gemm_rows(dev_, B.qkv, tok, pl, Pl, ACT_NONE, o, s);
        }
        window_attention(qkv, pl, h, Pl / 64, B.bias.as<float>(), B.shifted, H / 8, W / 8, att, pl, dev_.dev_err(), s);
        o.mode = OUT_WINDOW_ACCUM;
        o.out = y;
        o.plane0 = h / 8;
        o.map_h = H;
        o.map_w = W;
        o.shift = shift;
        gemm_rows(dev_, B.proj, att, pl, Pl, ACT_NONE, o, s);
      }
      // MLP (swin.rs:222-254): y[h:] += fc2(gelu(fc1(LN2(y[h:])))).
      if (fused_mlp_ && B.wblock.c == h && B.wblock.mlp) {
        // folded into the window block above
      } else if (fused_mlp_ && B.mlp.c == h && mlp_preferred(h)) {
        mlp_planar(dev_, B.mlp, y + (long long)(h / 8) * pl, pl, Pl, s);
      } else {
        layer_norm_planar(y, pl, h / 8, Pl, h, B.ln2g.as<float>(), B.ln2b.as<float>(), ln2, pl, nullptr, s);
        o.mode = OUT_STORE;
        o.out = hid;
        o.plane0 = 0;
        gemm_rows(dev_, B.fc1, ln2, pl, Pl, ACT_GELU, o, s);
        o.mode = OUT_ACCUM;
        o.out = y;
        o.plane0 = h / 8;
        gemm_rows(dev_, B.fc2, hid, pl, Pl, ACT_NONE, o, s);
      }
      // x += join(y); y = next split(x) (network.rs:190-212).
      IEC_CUDA(cudaStreamWaitEvent(s, ev_conv_, 0));
      if (fused_mlp_ && b + 1 < BLOCKS && B.joinsplit.c == c) {
        joinsplit_planar(dev_, B.joinsplit, x, y, pl, Pl, s);
      } else {
        o.mode = OUT_ACCUM;
        o.out = x;
        o.plane0 = 0;
        gemm_rows(dev_, B.join, y, pl, Pl, ACT_NONE, o, s);
        if (b + 1 < BLOCKS) {
          o.mode = OUT_STORE;
          o.out = y;
          gemm_rows(dev_, L.blocks[b + 1].split, x, pl, Pl, ACT_NONE, o, s);
        }
      }
      block_done();
    }
  };

  int level_index = 0;
  for (auto& Lp : levels_) {
    if (cancelled) break;
    Level& L = *Lp;
    if (L.up) {
      // x += skip; x = doubled(x) (network.rs:333-339, 446-478).
      const int si = 2 - (level_index - 4);  // up levels 3, 2, 1 use skips 2, 1, 0
      const int cin = 2 * L.c;
      const long long pin = plane((long long)H * W);
      launch_pdl(scunet_add, blocks_for((long long)(cin / 8) * H * W, sms), 256, 0, s, x, skip_[si].as<__half>(), pin,
                                                                               cin / 8, (long long)H * W);
      IEC_CUDA(cudaGetLastError());
      // The doubled map goes to y's buffer first, then becomes x.
      GemmOutSpec o;
      o.mode = OUT_DOUBLE;
      o.out = y_.as<__half>();
      o.plane_elems = plane((long long)4 * H * W);
      o.dbl_w = W;
      o.dbl_cout = L.c;
      gemm_rows(dev_, L.resample, x, pin, H * W, ACT_NONE, o, s);
      H *= 2;
      W *= 2;
      IEC_CUDA(cudaMemcpyAsync(x, y_.get(), (size_t)(L.c / 8) * plane((long long)H * W) * 2, cudaMemcpyDeviceToDevice, s));
    }
    run_level(L);
    if (L.down && !cancelled) {
      // halved(x) -> skip and the next level's x (network.rs:310-318).
      const int c = L.c;
      const long long pin = plane((long long)H * W), pout = plane((long long)H * W / 4);
      launch_pdl(scunet_halve_gather, blocks_for((long long)H * W / 4 * 4 * (c / 8), sms), 256, 0, s, 
          x, pin, c / 8, H, W, gat_.as<__half>(), pout);
      IEC_CUDA(cudaGetLastError());
      GemmOutSpec o;
      o.mode = OUT_STORE;
      o.out = skip_[level_index].as<__half>();
      o.plane_elems = pout;
      gemm_rows(dev_, L.resample, gat_.as<__half>(), pout, H * W / 4, ACT_NONE, o, s);
      H /= 2;
      W /= 2;
      IEC_CUDA(cudaMemcpyAsync(x, skip_[level_index].get(), (size_t)(2 * c / 8) * pout * 2, cudaMemcpyDeviceToDevice, s));
    }
    level_index++;
  }
  if (step && !cancelled) {
    dev_.wait_event(step_events_[done - 1]);
    if (!step()) cancelled = true;
  }
  if (cancelled) {
    dev_.sync(s);
    return false;
  }
  // x += head(image); out = tail(x); crop (network.rs:340-352).
  GemmOutSpec o;
  o.mode = OUT_ACCUM;
  o.out = x;
  o.plane_elems = plane(P);
  gemm_conv3(dev_, head_, img, img_plane, H, W, ACT_NONE, o, s);
  o.mode = OUT_STORE;
  o.out = out_.as<__half>();
  gemm_conv3(dev_, tail_, x, plane(P), H, W, ACT_NONE, o, s);
  launch_pdl(scunet_store, blocks_for((long long)(kx1 - kx0) * (ky1 - ky0), sms), 256, 0, s, 
      out_.as<__half>(), pw, kx0, ky0, kx1, ky1, rx0, ry0, dst, dst_u8 ? 1 : 0, src_w);
  IEC_CUDA(cudaGetLastError());
  return true;
}

void Scunet::run_whole_device(const float* src, float* dst, int width, int height, cudaStream_t s) {
  graph_.run({(long long)(uintptr_t)src, (long long)(uintptr_t)dst, width, height, -1, (long long)alloc_gen_,
              (long long)dev_.scratch_generation()},
             s, [&](cudaStream_t st) {
               run_region(src, false, dst, false, width, height, 0, 0, width, height, 0, 0, width, height, nullptr,
                          st);
             });
}

void Scunet::run_tiled_device(const void* src, bool src_u8, void* dst, bool dst_u8, size_t width, size_t height,
                              size_t tile, size_t margin, const std::function<bool(float)>& progress,
                              cudaStream_t s) {
  if (tile == 0) throw Error(ERR_INPUT, "tile size 0");
  const size_t cols = (width + tile - 1) / tile, rows = (height + tile - 1) / tile;
  const float steps = (float)(cols * rows * STEPS);
  size_t done = 0;
  std::function<bool()> step;
  if (progress) step = [&] { return progress((float)(++done) / steps); };
  auto pass = [&](cudaStream_t st) {
    for (size_t j = 0; j < rows; j++) {
      const size_t y0 = j * height / rows, y1 = (j + 1) * height / rows;
      for (size_t i = 0; i < cols; i++) {
        const size_t x0 = i * width / cols, x1 = (i + 1) * width / cols;
        const size_t rx0 = x0 > margin ? x0 - margin : 0, ry0 = y0 > margin ? y0 - margin : 0;
        const size_t rx1 = margin > width - x1 ? width : x1 + margin;
        const size_t ry1 = margin > height - y1 ? height : y1 + margin;
        if (!run_region(src, src_u8, dst, dst_u8, (int)width, (int)height, (int)rx0, (int)ry0, (int)(rx1 - rx0),
                        (int)(ry1 - ry0), (int)(x0 - rx0), (int)(y0 - ry0), (int)(x1 - rx0), (int)(y1 - ry0), step,
                        st))
          throw Error(CANCELLED, "cancelled");
      }
    }
  };
  // Progress reports wait on the GPU between blocks: those passes run as
  // plain launches; the others replay as a graph (PassGraph).
  if (progress) return pass(s);
  graph_.run({(long long)(uintptr_t)src, src_u8, (long long)(uintptr_t)dst, dst_u8, (long long)width,
              (long long)height, (long long)tile, (long long)margin, (long long)alloc_gen_,
              (long long)dev_.scratch_generation()},
             s, pass);
}

}  // namespace iec
