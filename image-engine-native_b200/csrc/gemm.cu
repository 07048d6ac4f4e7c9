// Host side of the general implicit GEMM and the bandwidth kernels around it
// (see gemm.h).
#include "gemm.h"

#include <algorithm>

#include "igemm_sm100.cuh"
#include "joinsplit_sm100.cuh"
#include "mlp_sm100.cuh"
#include "lnrows_sm100.cuh"

namespace iec {

namespace {

int choose_bn(int n) {
  // Up to 256 columns: one tile, the narrowest that covers them (its
  // padding columns are zero weights); above: the widest tile that divides.
  const int up[] = {32, 64, 96, 128, 192, 256};
  if (n <= 256)
    for (int bn : up)
      if (bn >= n) return bn;
  const int cands[] = {256, 192, 128, 96, 64, 32};
  for (int bn : cands)
    if (n % bn == 0) return bn;
  return 128;  // n padded to a multiple of 128 with zero columns
}

int choose_kb(int k) {
  if (k % 64 == 0) return 64;
  if (k % 32 == 0) return 32;
  if (k % 16 == 0) return 16;
  throw Error(ERR_INPUT, "GEMM reduction of " + std::to_string(k) + " channels: not a multiple of 16");
}

template <int BN, int KB, int AMODE>
void launch(Device& dev, const CUtensorMap& map, const GemmParams& p, cudaStream_t s) {
  auto kernel = igemm_sm100<BN, KB, AMODE>;
  static int smem_bytes[64] = {};
  int& bytes = smem_bytes[dev.ordinal() & 63];
  if (bytes == 0) {
    int optin = 0;
    IEC_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev.ordinal()));
    if (optin < GemmSmem<BN, KB>::DYN_BYTES) throw Error(ERR_GPU, "not enough shared memory per block");
    IEC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
    bytes = optin;  // one CTA per SM: its TMEM columns are always free
  }
  const int grid = std::min(p.tiles, dev.sms());
  // Programmatic dependent launch (the kernel waits for its predecessor's
  // completion before touching global memory; see igemm_sm100).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = (size_t)bytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  IEC_CUDA(cudaLaunchKernelEx(&cfg, kernel, map, p));
  IEC_CUDA(cudaGetLastError());
}

template <int AMODE>
void dispatch(Device& dev, int bn, int kb, const CUtensorMap& map, const GemmParams& p, cudaStream_t s) {
#define IEC_GEMM_CASE(BN_, KB_) \
  if (bn == BN_ && kb == KB_) return launch<BN_, KB_, AMODE>(dev, map, p, s);
#define IEC_GEMM_BN(KB_)  \
  IEC_GEMM_CASE(32, KB_)  \
  IEC_GEMM_CASE(64, KB_)  \
  IEC_GEMM_CASE(96, KB_)  \
  IEC_GEMM_CASE(128, KB_) \
  IEC_GEMM_CASE(192, KB_) \
  IEC_GEMM_CASE(256, KB_)
  IEC_GEMM_BN(64)
  IEC_GEMM_BN(32)
  IEC_GEMM_BN(16)
#undef IEC_GEMM_BN
#undef IEC_GEMM_CASE
  throw Error(ERR_GPU, "no GEMM kernel for this tile shape");
}

// Launch the GEMM of `p` (tiles set, split-K not yet): launches whose tiles
// fill less than half the GPU and that have at least 32 K steps run their K
// steps in slices of at least 16 steps on more CTAs (one wave), and a reduce
// kernel adds the slices in order and applies the epilogue.
template <int AMODE>
void run_gemm(Device& dev, const PackedWeights& pw, const CUtensorMap& map, GemmParams& p, cudaStream_t s) {
  p.tiles_mn = p.tiles;
  p.ksplit = 1;
  p.kslice = p.ksteps;
  p.ws = nullptr;
  p.ws_n = p.tiles_n * pw.bn;
  const bool splittable =
      AMODE != A_HALO && (p.out_mode == OUT_STORE || p.out_mode == OUT_ACCUM || p.out_mode == OUT_MAP);
  if (splittable && p.tiles_mn * 2 <= dev.sms() && p.ksteps >= 32) {
    const int want = std::min(dev.sms() / p.tiles_mn, p.ksteps / 16);  // one wave of tiles
    if (want >= 2) {
      p.kslice = (p.ksteps + want - 1) / want;
      p.ksplit = (p.ksteps + p.kslice - 1) / p.kslice;
    }
  }
  if (p.ksplit > 1) {
    p.ws = static_cast<float*>(dev.scratch((size_t)p.ksplit * p.M * p.ws_n * sizeof(float), s));
    p.tiles = p.tiles_mn * p.ksplit;
  }
  // Algorithmic work of the product: 2 M N K FLOPs (K over all taps); bytes:
  // the input read once (M x K), the weights, the output and the old values
  // the epilogue reads (accumulate, acc_src, resid).
  const double M = p.M, N = p.N, K1 = p.K, KT = pw.ktot;
  const int sources = (p.out_mode == OUT_ACCUM || p.out_mode == OUT_WINDOW_ACCUM ? 1 : 0) +
                      (p.acc_src ? 1 : 0) + (p.resid ? 1 : 0);
  const double gbytes = M * K1 * 2 + KT * N * 2 + M * N * 2 * (1 + sources);
  char name[96];
  snprintf(name, sizeof name, "igemm_sm100<%d,%d,%d> %dx%dx%d", pw.bn, pw.kb, AMODE, p.M, p.N, pw.ktot);
  timed_launch(name, 2.0 * M * N * KT, gbytes, s, [&] { dispatch<AMODE>(dev, pw.bn, pw.kb, map, p, s); });
  if (p.ksplit > 1) {
    const long long total = (long long)p.M * ((p.N + 7) / 8);
    const int grid = (int)std::max<long long>(1, std::min<long long>((total + 255) / 256, (long long)dev.sms() * 16));
    // programmatic dependent of the GEMM: it waits for the partial sums
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const double rbytes = (double)p.ksplit * p.M * p.ws_n * 4 + M * N * 2 * (1 + sources);
    timed_launch("gemm_splitk_reduce", 0.0, rbytes, s, [&] {
      IEC_CUDA(cudaLaunchKernelEx(&cfg, gemm_splitk_reduce, p));
      IEC_CUDA(cudaGetLastError());
    });
  }
}

void fill_out(GemmParams& p, const GemmOutSpec& o) {
  p.out_mode = o.mode;
  p.out = o.out;
  p.out_plane_elems = o.plane_elems;
  p.out_plane0 = o.plane0;
  p.map_h = o.map_h;
  p.map_w = o.map_w;
  p.shift = o.shift;
  p.win_ws = o.win_ws ? o.win_ws : 8;
  p.pad_h = o.pad_h ? o.pad_h : o.map_h;
  p.pad_w = o.pad_w ? o.pad_w : o.map_w;
  if (o.mode == OUT_WINDOW_ACCUM && (p.win_ws < 1 || p.win_ws > 8 || p.pad_h % p.win_ws || p.pad_w % p.win_ws ||
                                     p.pad_h < o.map_h || p.pad_w < o.map_w))
    throw Error(ERR_INPUT, "window partition geometry is inconsistent");
  p.dbl_w = o.dbl_w;
  p.dbl_cout = o.dbl_cout;
  p.phase_y = o.phase_y;
  p.phase_x = o.phase_x;
  p.ostep = o.ostep;
  p.dst_h = o.dst_h;
  p.dst_w = o.dst_w;
  p.dst_pad = o.dst_pad;
  p.dst_split = o.dst_split;
  p.dst_pw = o.dst_pw;
  p.dst_ph = o.dst_ph;
  p.acc_src = o.acc_src;
  p.resid = o.resid;
  if (o.mode == OUT_MAP) {
    const MapGeom g{o.dst_h, o.dst_w, o.dst_pad, o.dst_split};
    if (o.ostep < 1 || o.ostep > 2 || o.phase_y < 0 || o.phase_y >= o.ostep || o.phase_x < 0 ||
        o.phase_x >= o.ostep || o.dst_pad < 0 || o.dst_pad >= o.dst_h || o.dst_pad >= o.dst_w ||
        (o.dst_split != 1 && o.dst_split != 2) || o.dst_pw != g.pw() || o.dst_ph != g.ph() ||
        o.plane_elems < g.plane_elems() || o.dst_w % o.ostep != 0 || o.dst_h % o.ostep != 0)
      throw Error(ERR_INPUT, "GEMM output map geometry is inconsistent");
  }
}

}  // namespace

GemmOutSpec map_out(const MapGeom& g, __half* out, int plane0) {
  GemmOutSpec o;
  o.mode = OUT_MAP;
  o.out = out;
  o.plane_elems = g.plane_elems();
  o.plane0 = plane0;
  o.dst_h = g.h;
  o.dst_w = g.w;
  o.dst_pad = g.pad;
  o.dst_split = g.split;
  o.dst_pw = g.pw();
  o.dst_ph = g.ph();
  return o;
}

void pack_weights(PackedWeights& pw, const std::vector<float>& w, int taps, int k, int n, const float* bias) {
  pw.n = n;
  pw.k = k;
  pw.taps = taps;
  pw.ktot = taps * k;
  pw.bn = choose_bn(n);
  pw.kb = choose_kb(k);
  const int n_pad = (n + pw.bn - 1) / pw.bn * pw.bn;
  pw.n_tiles = n_pad / pw.bn;
  pw.ksteps = pw.ktot / pw.kb;
  if ((size_t)pw.ktot * n != w.size()) throw Error(ERR_WEIGHTS, "weight matrix size does not match");
  // [n tile][k step][kb / 8 groups][bn][8]
  std::vector<uint16_t> packed((size_t)n_pad * pw.ktot, 0);
  const int kg = pw.kb / 8;
  for (int nt = 0; nt < pw.n_tiles; nt++)
    for (int ks = 0; ks < pw.ksteps; ks++)
      for (int g = 0; g < kg; g++)
        for (int j = 0; j < pw.bn; j++)
          for (int e = 0; e < 8; e++) {
            const int kk = ks * pw.kb + g * 8 + e, nn = nt * pw.bn + j;
            const size_t at = ((((size_t)nt * pw.ksteps + ks) * kg + g) * pw.bn + j) * 8 + e;
            packed[at] = nn < n ? f32_to_half(w[(size_t)kk * n + nn]) : 0;
          }
  pw.w.reserve(packed.size() * 2);
  IEC_CUDA(cudaMemcpy(pw.w.get(), packed.data(), packed.size() * 2, cudaMemcpyHostToDevice));
  // The row-tap packing of an s x s grid (taps in row-major order).
  int side = 0;
  for (int c = 3; c <= 7; c += 2)
    if (c * c == taps) side = c;
  if (side && side * pw.bn <= 256 && k % pw.kb == 0) {
    const int chunks = k / pw.kb, np = side * pw.bn;
    std::vector<uint16_t> rt((size_t)pw.n_tiles * side * chunks * kg * np * 8, 0);
    for (int nt = 0; nt < pw.n_tiles; nt++)
      for (int ky = 0; ky < side; ky++)
        for (int kb = 0; kb < chunks; kb++)
          for (int g = 0; g < kg; g++)
            for (int dx = 0; dx < side; dx++)
              for (int j = 0; j < pw.bn; j++) {
                const int nn = nt * pw.bn + j;
                if (nn >= n) continue;
                const size_t at = (((((size_t)nt * side + ky) * chunks + kb) * kg + g) * np + dx * pw.bn + j) * 8;
                const size_t kk = (size_t)(ky * side + dx) * k + kb * pw.kb + g * 8;
                for (int e = 0; e < 8; e++) rt[at + e] = f32_to_half(w[(kk + e) * n + nn]);
              }
    pw.rt.reserve(rt.size() * 2);
    IEC_CUDA(cudaMemcpy(pw.rt.get(), rt.data(), rt.size() * 2, cudaMemcpyHostToDevice));
    pw.rt_kw = side;
  }
  pw.has_bias = bias != nullptr;
  if (bias) {
    pw.bias.reserve((size_t)n * 4);
    IEC_CUDA(cudaMemcpy(pw.bias.get(), bias, (size_t)n * 4, cudaMemcpyHostToDevice));
  }
}

void gemm_rows(Device& dev, const PackedWeights& pw, const __half* a, long long a_plane_elems, int m, int act,
               const GemmOutSpec& out, cudaStream_t s) {
  if (pw.taps != 1) throw Error(ERR_INPUT, "gemm_rows needs a 1x1 weight matrix");
  if (m <= 0) throw Error(ERR_INPUT, "GEMM without rows");
  const int rows = gemm_rows_alloc(m);
  if (a_plane_elems < (long long)rows * 8) throw Error(ERR_INPUT, "GEMM input planes too short");
  if (out.mode == OUT_MAP && (m % (out.dst_w / out.ostep) != 0 || m / (out.dst_w / out.ostep) != out.dst_h / out.ostep))
    throw Error(ERR_INPUT, "GEMM rows do not match the output map");
  const int kg = pw.kb / 8;
  CUtensorMap map;
  // Planes hold at least 128 rows, so the 128-row box never outgrows them.
  const uint64_t dims[3] = {128, (uint64_t)rows / 16, (uint64_t)pw.k / 8};
  const uint64_t strides[2] = {256, (uint64_t)a_plane_elems * 2};
  const uint32_t box[3] = {128, 8, (uint32_t)kg};
  encode_tensor_map(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, a, dims, strides, box);
  GemmParams p{};
  p.M = m;
  p.N = pw.n;
  p.K = pw.k;
  p.tiles_m = ((m + 127) / 128 + gemm_msub(pw.bn) - 1) / gemm_msub(pw.bn);
  p.tiles_n = pw.n_tiles;
  p.tiles = p.tiles_m * p.tiles_n;
  p.div_tiles_n = FastDiv((uint32_t)p.tiles_n);
  p.ksteps = pw.ksteps;
  p.b = pw.w.as<uint16_t>();
  p.bias = pw.has_bias ? pw.bias.as<float>() : nullptr;
  p.act = act;
  fill_out(p, out);
  if (out.mode == OUT_MAP) {
    p.W = out.dst_w / out.ostep;
    p.H = out.dst_h / out.ostep;
  }
  p.dev_err = dev.dev_err();
  if (p.tiles >= (1 << 24)) throw Error(ERR_INPUT, "GEMM too large for one launch");
  run_gemm<A_ROWS>(dev, pw, map, p, s);
}

bool mlp_fits(int c) {
  return c == 32 || c == 64 || c == 96 || c == 128 || c == 192 || c == 256 || c == 384;
}

// Wider MLPs run as LayerNorm and two GEMM launches: with their few row
// tiles and many hidden chunks the fused kernel's per-chunk hand-offs cost
// more than the launches it saves (measured: 256 channels over 6144 rows
// took 74 us fused against about 42 as three launches).
bool mlp_preferred(int c) { return mlp_fits(c) && c <= 192; }

void pack_mlp(MlpWeights& mw, int c, const std::vector<float>& w1, const std::vector<float>& b1,
              const std::vector<float>& w2, const std::vector<float>& b2, const std::vector<float>& gamma,
              const std::vector<float>& beta) {
  if (!mlp_fits(c)) throw Error(ERR_INPUT, "fused MLP of " + std::to_string(c) + " channels");
  const size_t hid = (size_t)4 * c;
  if (w1.size() != c * hid || w2.size() != c * hid || b1.size() != hid || b2.size() != (size_t)c ||
      gamma.size() != (size_t)c || beta.size() != (size_t)c)
    throw Error(ERR_WEIGHTS, "MLP weights of the wrong size");
  const int nh = mlp_nh(c), chunks = (int)hid / nh;
  // per chunk j: W1 columns j nh .. as [c / 8][nh][8], then W2 rows j nh ..
  // as [nh / 8][c][8] (the core-matrix images of fc1's and fc2's B operands)
  std::vector<uint16_t> w((size_t)chunks * 2 * c * nh);
  size_t at = 0;
  for (int j = 0; j < chunks; j++) {
    for (int g = 0; g < c / 8; g++)
      for (int n = 0; n < nh; n++)
        for (int e = 0; e < 8; e++) w[at++] = f32_to_half(w1[(size_t)(8 * g + e) * hid + (size_t)j * nh + n]);
    for (int g = 0; g < nh / 8; g++)
      for (int n = 0; n < c; n++)
        for (int e = 0; e < 8; e++) w[at++] = f32_to_half(w2[((size_t)j * nh + 8 * g + e) * c + n]);
  }
  std::vector<float> par;
  par.insert(par.end(), gamma.begin(), gamma.end());
  par.insert(par.end(), beta.begin(), beta.end());
  par.insert(par.end(), b1.begin(), b1.end());
  par.insert(par.end(), b2.begin(), b2.end());
  mw.c = c;
  mw.w.reserve(w.size() * 2);
  mw.params.reserve(par.size() * 4);
  IEC_CUDA(cudaMemcpy(mw.w.get(), w.data(), w.size() * 2, cudaMemcpyHostToDevice));
  IEC_CUDA(cudaMemcpy(mw.params.get(), par.data(), par.size() * 4, cudaMemcpyHostToDevice));
}

namespace {

template <int C>
void launch_mlp(Device& dev, const CUtensorMap& map, const MlpParams& p, cudaStream_t s) {
  using L = MlpSmem<C>;
  static bool prepared[64] = {};
  if (!prepared[dev.ordinal() & 63]) {
    IEC_CUDA(cudaFuncSetAttribute(mlp_sm100<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    prepared[dev.ordinal() & 63] = true;
  }
  launch_pdl(mlp_sm100<C>, std::min(p.tiles, dev.sms() * L::CTAS), L::THREADS, (size_t)L::TOTAL, s, map, p);
  IEC_CUDA(cudaGetLastError());
}

}  // namespace

void mlp_planar(Device& dev, const MlpWeights& mw, __half* x, long long plane_elems, int rows, cudaStream_t s) {
  const int c = mw.c;
  if (!mlp_fits(c) || rows <= 0) throw Error(ERR_INPUT, "fused MLP shape");
  const int alloc = gemm_rows_alloc(rows);
  if (plane_elems < (long long)alloc * 8) throw Error(ERR_INPUT, "MLP planes too short");
  // the A_ROWS box of gemm_rows with every channel group in one box
  CUtensorMap map;
  const uint64_t dims[3] = {128, (uint64_t)alloc / 16, (uint64_t)c / 8};
  const uint64_t strides[2] = {256, (uint64_t)plane_elems * 2};
  const uint32_t box[3] = {128, 8, (uint32_t)c / 8};
  encode_tensor_map(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, x, dims, strides, box);
  MlpParams p{};
  p.M = rows;
  p.tiles = (rows + 127) / 128;
  p.x = x;
  p.plane_elems = plane_elems;
  p.w = mw.w.as<uint8_t>();
  p.params = mw.params.as<float>();
  p.dev_err = dev.dev_err();
  const double hid = 4.0 * c;
  char name[64];
  snprintf(name, sizeof name, "mlp_sm100<%d> %dx%d", c, rows, c);
  // FLOPs of fc1 and fc2; bytes: the rows read and written, the weights
  timed_launch(name, 4.0 * rows * c * hid, (double)rows * c * 4 + 4.0 * c * hid, s, [&] {
    switch (c) {
      case 32: return launch_mlp<32>(dev, map, p, s);
      case 64: return launch_mlp<64>(dev, map, p, s);
      case 96: return launch_mlp<96>(dev, map, p, s);
      case 128: return launch_mlp<128>(dev, map, p, s);
      case 192: return launch_mlp<192>(dev, map, p, s);
      case 256: return launch_mlp<256>(dev, map, p, s);
      default: return launch_mlp<384>(dev, map, p, s);
    }
  });
}

bool joinsplit_fits(int c) { return c == 64 || c == 128 || c == 256; }

void pack_joinsplit(JoinSplitWeights& jw, int c, const std::vector<float>& wj, const std::vector<float>& bj,
                    const std::vector<float>& ws, const std::vector<float>& bs) {
  if (!joinsplit_fits(c)) throw Error(ERR_INPUT, "fused join and split of " + std::to_string(c) + " channels");
  const size_t cc = (size_t)c * c;
  if (wj.size() != cc || ws.size() != cc || bj.size() != (size_t)c || bs.size() != (size_t)c)
    throw Error(ERR_WEIGHTS, "join and split weights of the wrong size");
  // each matrix as [c / 8][c][8]: the core-matrix image of a B operand of K c
  std::vector<uint16_t> w(2 * cc);
  size_t at = 0;
  for (const std::vector<float>* m : {&wj, &ws})
    for (int g = 0; g < c / 8; g++)
      for (int n = 0; n < c; n++)
        for (int e = 0; e < 8; e++) w[at++] = f32_to_half((*m)[(size_t)(8 * g + e) * c + n]);
  std::vector<float> b(bj);
  b.insert(b.end(), bs.begin(), bs.end());
  jw.c = c;
  jw.w.reserve(w.size() * 2);
  jw.bias.reserve(b.size() * 4);
  IEC_CUDA(cudaMemcpy(jw.w.get(), w.data(), w.size() * 2, cudaMemcpyHostToDevice));
  IEC_CUDA(cudaMemcpy(jw.bias.get(), b.data(), b.size() * 4, cudaMemcpyHostToDevice));
}

namespace {

template <int C>
void launch_joinsplit(Device& dev, const CUtensorMap& ymap, const CUtensorMap& xmap, const JoinSplitParams& p,
                      cudaStream_t s) {
  using L = JoinSplitSmem<C>;
  static bool prepared[64] = {};
  if (!prepared[dev.ordinal() & 63]) {
    IEC_CUDA(cudaFuncSetAttribute(joinsplit_sm100<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    prepared[dev.ordinal() & 63] = true;
  }
  launch_pdl(joinsplit_sm100<C>, std::min(p.tiles, dev.sms() * L::CTAS), L::THREADS, (size_t)L::TOTAL, s, ymap,
             xmap, p);
  IEC_CUDA(cudaGetLastError());
}

}  // namespace

void joinsplit_planar(Device& dev, const JoinSplitWeights& jw, __half* x, __half* y, long long plane_elems, int rows,
                      cudaStream_t s) {
  const int c = jw.c;
  if (!joinsplit_fits(c) || rows <= 0) throw Error(ERR_INPUT, "fused join and split shape");
  const int alloc = gemm_rows_alloc(rows);
  if (plane_elems < (long long)alloc * 8) throw Error(ERR_INPUT, "join and split planes too short");
  // the A_ROWS box of gemm_rows with every channel group in one box, for
  // both maps
  CUtensorMap ymap, xmap;
  const uint64_t dims[3] = {128, (uint64_t)alloc / 16, (uint64_t)c / 8};
  const uint64_t strides[2] = {256, (uint64_t)plane_elems * 2};
  const uint32_t box[3] = {128, 8, (uint32_t)c / 8};
  encode_tensor_map(&ymap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, y, dims, strides, box);
  encode_tensor_map(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, x, dims, strides, box);
  JoinSplitParams p{};
  p.M = rows;
  p.tiles = (rows + 127) / 128;
  p.x = x;
  p.y = y;
  p.plane_elems = plane_elems;
  p.w = jw.w.as<uint8_t>();
  p.bias = jw.bias.as<float>();
  p.dev_err = dev.dev_err();
  char name[64];
  snprintf(name, sizeof name, "joinsplit_sm100<%d> %dx%d", c, rows, c);
  // FLOPs of both products; bytes: y and x read and written, the weights
  timed_launch(name, 4.0 * rows * c * c, (double)rows * c * 8 + 4.0 * c * c, s, [&] {
    if (c == 64) return launch_joinsplit<64>(dev, ymap, xmap, p, s);
    if (c == 128) return launch_joinsplit<128>(dev, ymap, xmap, p, s);
    return launch_joinsplit<256>(dev, ymap, xmap, p, s);
  });
}

bool lnrows_fits(int c, int n) {
  return (c == 32 && n == 96) || (c == 64 && n == 192) || (c == 96 && n == 288) || (c == 128 && n == 384);
}

void pack_lnrows(LnRowsWeights& lw, int c, int n, const std::vector<float>& w, const std::vector<float>& bias,
                 const std::vector<float>& gamma, const std::vector<float>& beta) {
  if (!lnrows_fits(c, n)) throw Error(ERR_INPUT, "folded LayerNorm product of this shape");
  if (w.size() != (size_t)c * n || bias.size() != (size_t)n || gamma.size() != (size_t)c || beta.size() != (size_t)c)
    throw Error(ERR_WEIGHTS, "folded LayerNorm product weights of the wrong size");
  std::vector<uint16_t> img((size_t)c * n);
  size_t at = 0;
  for (int g = 0; g < c / 8; g++)
    for (int j = 0; j < n; j++)
      for (int e = 0; e < 8; e++) img[at++] = f32_to_half(w[(size_t)(8 * g + e) * n + j]);
  std::vector<float> par;
  par.insert(par.end(), gamma.begin(), gamma.end());
  par.insert(par.end(), beta.begin(), beta.end());
  par.insert(par.end(), bias.begin(), bias.end());
  lw.c = c;
  lw.n = n;
  lw.w.reserve(img.size() * 2);
  lw.params.reserve(par.size() * 4);
  IEC_CUDA(cudaMemcpy(lw.w.get(), img.data(), img.size() * 2, cudaMemcpyHostToDevice));
  IEC_CUDA(cudaMemcpy(lw.params.get(), par.data(), par.size() * 4, cudaMemcpyHostToDevice));
}

namespace {

template <int C, int N>
void launch_lnrows(Device& dev, const LnRowsParams& p, cudaStream_t s) {
  using L = LnRowsSmem<C, N>;
  static bool prepared[64] = {};
  if (!prepared[dev.ordinal() & 63]) {
    IEC_CUDA(cudaFuncSetAttribute(lnrows_sm100<C, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    prepared[dev.ordinal() & 63] = true;
  }
  launch_pdl(lnrows_sm100<C, N>, std::min(p.tiles, dev.sms()), L::THREADS, (size_t)L::TOTAL, s, p);
  IEC_CUDA(cudaGetLastError());
}

}  // namespace

void lnrows_planar(Device& dev, const LnRowsWeights& lw, const __half* src, long long src_plane, int rows,
                   const WindowMap& wm, __half* out, long long out_plane, cudaStream_t s) {
  if (!lnrows_fits(lw.c, lw.n) || rows <= 0) throw Error(ERR_INPUT, "folded LayerNorm product shape");
  if (wm.ws < 1 || wm.ws > 8 || wm.pad_h % wm.ws || wm.pad_w % wm.ws || wm.pad_h < wm.map_h || wm.pad_w < wm.map_w)
    throw Error(ERR_INPUT, "window partition geometry is inconsistent");
  if (out_plane < (long long)rows * 8) throw Error(ERR_INPUT, "output planes too short");
  LnRowsParams p{};
  p.rows = rows;
  p.tiles = (rows + 127) / 128;
  p.src = src;
  p.src_plane = src_plane;
  p.wm = wm;
  p.w = lw.w.as<uint8_t>();
  p.params = lw.params.as<float>();
  p.out = out;
  p.out_plane = out_plane;
  p.dev_err = dev.dev_err();
  char name[64];
  snprintf(name, sizeof name, "lnrows_sm100<%d,%d> %dx%dx%d", lw.c, lw.n, rows, lw.n, lw.c);
  // FLOPs of the product; bytes: the rows gathered once, the output, the weights
  timed_launch(name, 2.0 * rows * lw.n * lw.c, (double)rows * (lw.c + lw.n) * 2 + 2.0 * lw.c * lw.n, s, [&] {
    if (lw.c == 32) return launch_lnrows<32, 96>(dev, p, s);
    if (lw.c == 64) return launch_lnrows<64, 192>(dev, p, s);
    if (lw.c == 96) return launch_lnrows<96, 288>(dev, p, s);
    return launch_lnrows<128, 384>(dev, p, s);
  });
}

void gemm_conv3(Device& dev, const PackedWeights& pw, const __half* map_ptr, long long map_plane_elems, int h, int w,
                int act, const GemmOutSpec& out, cudaStream_t s) {
  std::vector<Tap> taps;
  for (int t = 0; t < 9; t++) taps.push_back({t / 3 - 1, t % 3 - 1, 0});
  TapSource src{map_ptr, map_plane_elems, w, h, 1};
  gemm_taps(dev, pw, src, taps, h, w, act, out, s);
}

namespace {

// The taps as a kh x kw grid from (dy0, dx0), row-major, over phase 0; or false.
bool tap_grid(const std::vector<Tap>& taps, int& kh, int& kw, int& dy0, int& dx0) {
  if (taps.empty()) return false;
  dy0 = taps[0].dy;
  dx0 = taps[0].dx;
  kw = 0;
  while (kw < (int)taps.size() && taps[kw].dy == dy0) kw++;
  kh = (int)taps.size() / kw;
  if (kh * kw != (int)taps.size()) return false;
  for (int t = 0; t < (int)taps.size(); t++)
    if (taps[t].dy != dy0 + t / kw || taps[t].dx != dx0 + t % kw || taps[t].phase != 0) return false;
  return true;
}

}  // namespace

void gemm_taps(Device& dev, const PackedWeights& pw, const TapSource& src, const std::vector<Tap>& taps, int h, int w,
               int act, const GemmOutSpec& out, cudaStream_t s, int halo) {
  if (pw.taps != (int)taps.size() || taps.size() > (size_t)GEMM_MAX_TAPS)
    throw Error(ERR_INPUT, "tap table does not match the weights");
  if (w < 1 || h < 1) throw Error(ERR_INPUT, "empty convolution output");
  if (out.mode == OUT_MAP && (out.dst_w != w * out.ostep || out.dst_h != h * out.ostep))
    throw Error(ERR_INPUT, "convolution output does not match the output map");
  // Halo tiles (A_HALO): a full kh x kw grid of taps over a single-phase
  // source at least 32 pixels wide, with the row-tap packing; tiles of
  // 4 msub rows x (33 - kw) outputs, each channel chunk's halo box loaded
  // once and read by one MMA of N = kw bn per kernel row. Taken when the
  // tiles fill at least half the GPU (fewer tiles keep the tap boxes and
  // split-K) and two halo boxes and two weight stages fit the ring; `halo`
  // 0 never, 1 whenever it fits.
  int kh = 0, kw = 0, dy0 = 0, dx0 = 0;
  if (halo != 0 && pw.rt_kw > 0 && src.phases == 1 && src.w >= 32 && out.mode != OUT_WINDOW_ACCUM &&
      tap_grid(taps, kh, kw, dy0, dx0) && kw == pw.rt_kw && kh == pw.rt_kw &&
      ((kw == 3 && pw.bn <= 64) || ((kw == 5 || kw == 7) && pw.bn <= 32))) {
    const int np = kw * pw.bn, msub = halo_msub(pw.bn, kw);
    const int th = 4 * msub, tv = 33 - kw, kg = pw.kb / 8;
    const int tiles_w = (w + tv - 1) / tv, tiles_h = (h + th - 1) / th;
    const int halo_rows = th + kh - 1;
    // Shared memory (200 KB): the weights resident when one n tile's fit
    // beside two halo buffers, else a ring of up to 2 kh weight stages; the
    // rest a ring of up to 8 halo buffers.
    constexpr int RING = 200 * 1024;
    const int stride = (kg * halo_rows * 32 * 16 + 1023) / 1024 * 1024;
    const int b_stage = kg * np * 16, chunks = pw.k / pw.kb;
    const int b_all = kh * chunks * b_stage;
    const bool resident = pw.n_tiles == 1 && b_all + 2 * stride <= RING;
    const int b_stages = resident ? 1 : std::min({8, 2 * kh, (RING - 2 * stride) / b_stage});
    const int b_bytes = resident ? b_all : b_stages * b_stage;
    const int bufs = std::min(8, (RING - b_bytes) / stride);
    const long long tiles = (long long)tiles_w * tiles_h * pw.n_tiles;
    if (src.h >= halo_rows && (resident || b_stages >= 2) && bufs >= 2 && (halo == 1 || tiles * 2 >= dev.sms()) &&
        tiles < (1 << 24)) {
      CUtensorMap map;
      const uint64_t dims[5] = {(uint64_t)src.w * 8, (uint64_t)src.h, 1, (uint64_t)pw.k / 8, 1};
      const uint64_t strides[4] = {(uint64_t)src.w * 16, (uint64_t)src.w * src.h * 16, (uint64_t)src.plane_elems * 2,
                                   (uint64_t)src.plane_elems * 2 * (pw.k / 8)};
      const uint32_t box[5] = {32 * 8, (uint32_t)halo_rows, 1, (uint32_t)kg, 1};
      encode_tensor_map(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, src.ptr, dims, strides, box);
      GemmParams p{};
      p.taps = (int)taps.size();
      p.phase_y = out.phase_y;
      p.phase_x = out.phase_x;
      p.M = h * w;
      p.N = pw.n;
      p.K = pw.k;
      p.H = h;
      p.W = w;
      p.TW = 32;
      p.tiles_w = tiles_w;
      p.tiles_m = tiles_w * tiles_h;
      p.tiles_n = pw.n_tiles;
      p.tiles = (int)tiles;
      p.div_tiles_n = FastDiv((uint32_t)p.tiles_n);
      p.div_tiles_w = FastDiv((uint32_t)p.tiles_w);
      p.ksteps = pw.ksteps;
      p.b = pw.rt.as<uint16_t>();
      p.bias = pw.has_bias ? pw.bias.as<float>() : nullptr;
      p.act = act;
      fill_out(p, out);
      p.dev_err = dev.dev_err();
      p.halo_kh = kh;
      p.halo_kw = kw;
      p.halo_dy0 = dy0;
      p.halo_dx0 = dx0;
      p.halo_rows = halo_rows;
      p.halo_tv = tv;
      p.halo_stride = stride;
      p.halo_msub = msub;
      p.halo_np = np;
      p.b_stage = b_stage;
      p.halo_bufs = bufs;
      p.b_resident = resident ? 1 : 0;
      p.b_off = bufs * stride;
      p.b_stages = b_stages;
      run_gemm<A_HALO>(dev, pw, map, p, s);
      return;
    }
  }
  // Tiles of 8 rows x 16 (or, for narrow outputs, 8) columns; boxes that
  // reach past the source read TMA's zero fill.
  const int tw = w > 8 ? 16 : 8;
  const int kg = pw.kb / 8;
  CUtensorMap map;
  const uint64_t phase_bytes = (uint64_t)src.w * src.h * 16;
  const uint64_t dims[5] = {(uint64_t)src.w * 8, (uint64_t)src.h, (uint64_t)src.phases, (uint64_t)pw.k / 8, 1};
  const uint64_t strides[4] = {(uint64_t)src.w * 16, phase_bytes, (uint64_t)src.plane_elems * 2,
                               (uint64_t)src.plane_elems * 2 * (pw.k / 8)};
  const uint32_t box[5] = {(uint32_t)tw * 8, 8, 1, (uint32_t)kg, 1};
  encode_tensor_map(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, src.ptr, dims, strides, box);
  GemmParams p{};
  p.taps = (int)taps.size();
  for (size_t t = 0; t < taps.size(); t++) {
    p.dy[t] = (signed char)taps[t].dy;
    p.dx[t] = (signed char)taps[t].dx;
    p.phase[t] = (signed char)taps[t].phase;
  }
  p.phase_y = out.phase_y;
  p.phase_x = out.phase_x;
  p.M = h * w;
  p.N = pw.n;
  p.K = pw.k;
  p.H = h;
  p.W = w;
  p.TW = tw;
  p.tiles_w = (w + tw - 1) / tw;
  // groups of gemm_msub consecutive 8 x tw blocks, row-major
  p.tiles_m = (p.tiles_w * ((h + 7) / 8) + gemm_msub(pw.bn) - 1) / gemm_msub(pw.bn);
  p.tiles_n = pw.n_tiles;
  p.tiles = p.tiles_m * p.tiles_n;
  p.div_tiles_n = FastDiv((uint32_t)p.tiles_n);
  p.div_tiles_w = FastDiv((uint32_t)p.tiles_w);
  p.ksteps = pw.ksteps;
  p.b = pw.w.as<uint16_t>();
  p.bias = pw.has_bias ? pw.bias.as<float>() : nullptr;
  p.act = act;
  fill_out(p, out);
  p.dev_err = dev.dev_err();
  if (p.tiles >= (1 << 24) || p.tiles_w >= (1 << 16)) throw Error(ERR_INPUT, "GEMM too large for one launch");
  run_gemm<A_TAPS>(dev, pw, map, p, s);
}

// ---------------------------------------------------------- bandwidth kernels
__global__ void rows_to_planar_kernel(const float* __restrict__ src, int rows, int c, __half* __restrict__ dst,
                                      long long plane) {
  griddep_wait();
  griddep_launch_dependents();
  const int groups = c / 8;
  const long long total = (long long)rows * groups;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int g = (int)(i % groups);
    const long long r = i / groups;
    const float4* s4 = reinterpret_cast<const float4*>(src + r * c + g * 8);
    const float4 a = s4[0], b = s4[1];
    __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
    __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
    *reinterpret_cast<uint4*>(dst + g * plane + r * 8) =
        make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                   *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
  }
}

__global__ void planar_to_rows_kernel(const __half* __restrict__ src, long long plane, int rows, int c,
                                      float* __restrict__ dst) {
  griddep_wait();
  griddep_launch_dependents();
  const long long total = (long long)rows * c;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int ch = (int)(i % c);
    const long long r = i / c;
    dst[i] = __half2float(src[(ch / 8) * plane + r * 8 + ch % 8]);
  }
}

static int grid_for(long long n, int block, int sms) {
  return (int)std::max<long long>(1, std::min<long long>((n + block - 1) / block, (long long)sms * 32));
}

void rows_to_planar(const float* src, int rows, int c, __half* dst, long long dst_plane_elems, cudaStream_t s) {
  if (c % 8 != 0) throw Error(ERR_INPUT, "channels must be a multiple of 8");
  launch_pdl(rows_to_planar_kernel, grid_for((long long)rows * c / 8, 256, 148), 256, 0, s, src, rows, c, dst, dst_plane_elems);
  IEC_CUDA(cudaGetLastError());
}

void planar_to_rows(const __half* src, long long src_plane_elems, int rows, int c, float* dst, cudaStream_t s) {
  launch_pdl(planar_to_rows_kernel, grid_for((long long)rows * c, 256, 148), 256, 0, s, src, src_plane_elems, rows, c, dst);
  IEC_CUDA(cudaGetLastError());
}

// S threads per output row (token or pixel), each holding up to G of the
// row's channel groups in registers: one read of the row, the mean and the
// variance by shuffles within the S threads (two passes, as math.rs:78-116
// computes them), then the normalised groups. mode 0: row r is pixel r;
// mode 1: window order (zero rows where WindowMap says so); mode 2: patch
// merge, row r of the (grid / 2)^2 map gathering its 2 x 2 pixels in the
// order (0,0), (1,0), (0,1), (1,1) (birefnet swin.rs:366-404). The scales
// and shifts (weights, which no kernel writes) are staged in shared memory
// before the wait for the previous kernel, so their fetch overlaps its tail
// instead of following the two reductions.
template <int S, int G>
__global__ void __launch_bounds__(256) layer_norm_rows(const __half* __restrict__ src, long long src_plane, int plane0,
                                                       int rows, int c, const float* __restrict__ gamma,
                                                       const float* __restrict__ beta, __half* __restrict__ dst,
                                                       long long dst_plane, int mode, WindowMap wm, int grid) {
  extern __shared__ float4 ln_params[];  // [c / 4] scales, then [c / 4] shifts
  for (int i = threadIdx.x; i < c / 4; i += blockDim.x) {
    ln_params[i] = __ldg(reinterpret_cast<const float4*>(gamma) + i);
    ln_params[c / 4 + i] = __ldg(reinterpret_cast<const float4*>(beta) + i);
  }
  __syncthreads();
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x % S, sub = threadIdx.x / S;
  const int r = blockIdx.x * (256 / S) + sub;
  const bool valid = r < rows;
  const int groups = c / 8;
  bool zero = false;
  long long pix = r;
  int src_groups = groups;
  if (valid && mode == 1) {
    const int win = r >> 6, i = r & 63, ws = wm.ws, cols = wm.pad_w / ws;
    const int wy = win / cols, wx = win - wy * cols;
    const int y = (wy * ws + i / ws + wm.shift) % wm.pad_h, x = (wx * ws + i % ws + wm.shift) % wm.pad_w;
    if (i >= ws * ws || y >= wm.map_h || x >= wm.map_w)
      zero = true;
    else
      pix = (long long)y * wm.map_w + x;
  }
  if (mode == 2) src_groups = groups / 4;
  float v[G][8];
  float sum = 0.0f;
#pragma unroll
  for (int k = 0; k < G; k++) {
    const int g = lane + k * S;
#pragma unroll
    for (int e = 0; e < 8; e++) v[k][e] = 0.0f;
    if (!valid || zero || g >= groups) continue;
    const __half* at;
    if (mode == 2) {
      const int q = g / src_groups, gs = g - q * src_groups, half = grid / 2;
      const long long p2 = (long long)(2 * (r / half) + (q & 1)) * grid + 2 * (r % half) + (q >> 1);
      at = src + (long long)gs * src_plane + p2 * 8;
    } else {
      at = src + (long long)(plane0 + g) * src_plane + pix * 8;
    }
    const uint4 u = *reinterpret_cast<const uint4*>(at);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float2 f = __half22float2(h[e]);
      v[k][2 * e] = f.x;
      v[k][2 * e + 1] = f.y;
      sum += f.x + f.y;
    }
  }
#pragma unroll
  for (int o = S / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o, S);
  const float mean = sum / (float)c;
  float var = 0.0f;
#pragma unroll
  for (int k = 0; k < G; k++) {
    if (lane + k * S >= groups) continue;
#pragma unroll
    for (int e = 0; e < 8; e++) var += (v[k][e] - mean) * (v[k][e] - mean);
  }
#pragma unroll
  for (int o = S / 2; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o, S);
  if (!valid) return;
  const float inv = 1.0f / sqrtf(var / (float)c + 1e-5f);
#pragma unroll
  for (int k = 0; k < G; k++) {
    const int g = lane + k * S;
    if (g >= groups) continue;
    // the group's 8 scales and 8 shifts: four 16-byte shared-memory loads
    float gm[8], bt[8];
    if (!zero) {
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const float4 gq = ln_params[g * 2 + h], bq = ln_params[c / 4 + g * 2 + h];
        gm[4 * h] = gq.x;
        gm[4 * h + 1] = gq.y;
        gm[4 * h + 2] = gq.z;
        gm[4 * h + 3] = gq.w;
        bt[4 * h] = bq.x;
        bt[4 * h + 1] = bq.y;
        bt[4 * h + 2] = bq.z;
        bt[4 * h + 3] = bq.w;
      }
    }
    uint32_t packed[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      float a = 0.0f, b = 0.0f;
      if (!zero) {
        a = (v[k][2 * e] - mean) * inv * gm[2 * e] + bt[2 * e];
        b = (v[k][2 * e + 1] - mean) * inv * gm[2 * e + 1] + bt[2 * e + 1];
      }
      __half2 o = __floats2half2_rn(a, b);
      packed[e] = *reinterpret_cast<uint32_t*>(&o);
    }
    *reinterpret_cast<uint4*>(dst + g * dst_plane + (long long)r * 8) =
        make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
}

static void launch_ln(const __half* src, long long src_plane, int plane0, int rows, int c, const float* gamma,
                      const float* beta, __half* dst, long long dst_plane, int mode, const WindowMap& wm, int grid,
                      cudaStream_t s) {
  const int groups = c / 8;
  if (c % 8 != 0 || groups < 1) throw Error(ERR_INPUT, "layer norm over a channel count not a multiple of 8");
  if (((uintptr_t)gamma | (uintptr_t)beta) % 16 != 0) throw Error(ERR_INPUT, "layer norm parameters not 16-byte aligned");
  const size_t smem = (size_t)2 * c * sizeof(float);  // at most 24 KB (3072 channels)
  // bytes: every output row's c values read and written once (f16)
  timed_launch("layer_norm_rows", 0.0, (double)rows * c * 4, s, [&] {
  if (groups <= 8) {
    launch_pdl(layer_norm_rows<2, 4>, (rows + 127) / 128, 256, smem, s, src, src_plane, plane0, rows, c, gamma, beta, dst,
                                                             dst_plane, mode, wm, grid);
  } else if (groups <= 16) {
    launch_pdl(layer_norm_rows<4, 4>, (rows + 63) / 64, 256, smem, s, src, src_plane, plane0, rows, c, gamma, beta, dst,
                                                           dst_plane, mode, wm, grid);
  } else if (groups <= 48) {
    launch_pdl(layer_norm_rows<8, 6>, (rows + 31) / 32, 256, smem, s, src, src_plane, plane0, rows, c, gamma, beta, dst,
                                                           dst_plane, mode, wm, grid);
  } else if (groups <= 384) {
    launch_pdl(layer_norm_rows<32, 12>, (rows + 7) / 8, 256, smem, s, src, src_plane, plane0, rows, c, gamma, beta, dst,
                                                           dst_plane, mode, wm, grid);
  } else {
    throw Error(ERR_INPUT, "layer norm over more than 3072 channels");
  }
  IEC_CUDA(cudaGetLastError());
  });
}

void layer_norm_planar(const __half* src, long long src_plane_elems, int plane0, int rows, int c, const float* gamma,
                       const float* beta, __half* dst, long long dst_plane_elems, const WindowMap* window,
                       cudaStream_t s) {
  WindowMap wm;
  if (window) {
    wm = *window;
    if (wm.ws < 1 || wm.ws > 8 || wm.pad_h % wm.ws || wm.pad_w % wm.ws || wm.pad_h < wm.map_h || wm.pad_w < wm.map_w)
      throw Error(ERR_INPUT, "window partition geometry is inconsistent");
  }
  launch_ln(src, src_plane_elems, plane0, rows, c, gamma, beta, dst, dst_plane_elems, window ? 1 : 0, wm, 0, s);
}

void merge_layer_norm_planar(const __half* src, long long src_plane_elems, int grid, int c, const float* gamma,
                             const float* beta, __half* dst, long long dst_plane_elems, cudaStream_t s) {
  if (grid % 2 != 0) throw Error(ERR_INPUT, "patch merge of an odd grid");
  const int rows = (grid / 2) * (grid / 2);
  launch_ln(src, src_plane_elems, 0, rows, 4 * c, gamma, beta, dst, dst_plane_elems, 2, WindowMap{}, grid, s);
}

}  // namespace iec
