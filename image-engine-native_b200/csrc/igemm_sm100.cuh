// General implicit GEMM on sm_100a tensor cores: every 1x1 convolution,
// linear layer, 2x2 stride-2 (transposed) convolution and wide 3x3
// convolution of the networks. f16 inputs, f32 accumulators in TMEM.
//
// Semantics: crates/native-engine/src/gemm.rs:514-667 (multiply): out[r] =
// act(input[r] * w + bias), or accumulated onto out[r], over Input::Rows or a
// centred 3x3 stride-1 zero-padded convolution (Taps::Conv), with the GELU of
// math.rs:63-75 (exact, through erf) or ReLU applied after the sum.
//
// Layout. Every activation is f16 "channel-group planar": [channels / 8]
// [rows][8] with rows = pixels (or tokens) row-major, so the 8 channels of
// one row form one 16-byte K-unit of a tensor-core core matrix, and a plane
// is one contiguous run. A-tiles come in by TMA in the no-swizzle K-major
// core-matrix layout [k-group][128 rows][8] that tcgen05 reads directly:
//   A_ROWS   128 consecutive rows: a 3-D box {16 rows x 8 channels, 8 blocks of
//            16 rows, KB/8 groups} (256-byte inner runs).
//   A_TAPS   a tile of 8 output rows x TW pixels (TW = 16, or 8 for 8-wide
//            outputs): per tap t a 5-D box of the source map, phase
//            phase[t], shifted by (dy[t], dx[t]) from the tile (zero fill
//            outside the map), K = taps x cin. A 3x3 zero-padded convolution
//            is 9 taps of offsets -1..1 over the map itself; a reflect-padded
//            one reads a map padded beforehand with offsets 0..k-1; a stride-2
//            one reads the four space-to-depth phases of the (padded) map;
//            one output phase of a stride-2 transposed convolution reads
//            offsets 0..1 (gemm.rs:274-286 Taps, lama network.rs:271-333).
// B-tiles (weights) are pre-arranged on the host per (N tile, K step) as the
// core-matrix image [KB/8][BN][8] and brought in by one cp.async.bulk.
//
// Persistent CTAs walk (M tile, N tile) pairs; 320 threads: warp 0 issues
// the TMA / bulk loads into a ring of stages, warp 1 the MMAs (M 128, N BN,
// K 16) into one of two TMEM accumulators, warps 2..9 (two per TMEM lane
// quarter, half the columns each) run the epilogue while the next tile's
// MMAs proceed:
//   OUT_STORE        act(acc + bias) -> f16 planes (at a channel offset)
//   OUT_ACCUM        out += act(acc + bias)                (residual adds)
//   OUT_WINDOW_ACCUM out[pixel(token)] += acc + bias, the token's pixel from
//                    the (shifted) window partition: scunet swin.rs:174-178,
//                    212-219 (8 x 8), birefnet swin.rs:219-306 (7 x 7 windows
//                    of a map padded to a multiple of 7, in 64-row slots)
//   OUT_DOUBLE       2x2 stride-2 transposed convolution: column q cout + o of
//                    input pixel (y, x) -> output pixel (2y + q / 2, 2x + q % 2),
//                    channel o (crates/scunet-native/src/network.rs:446-478)
//   OUT_PHASE        one output phase (py, px) of a stride-2 transposed
//                    convolution: row (y, x) -> output pixel (2y + py, 2x + px)
//   OUT_MAP          row (y, x) -> pixel (ostep y + phase_y, ostep x + phase_x)
//                    of a map stored reflect-padded by dst_pad (every pixel
//                    also written where the padding mirrors it: gemm.rs:408-441
//                    reflect) and, with dst_split 2, as the four space-to-depth
//                    phases a stride-2 convolution reads; the value is
//                    act(acc + bias [+ acc_src]) [+ resid], the two optional
//                    sources read at the pixel in the same geometry
// When accumulating, the activation applies after the add, as multiply does.
// All waits are bounded as in conv3x3_sm100.cuh.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "sm100.cuh"

namespace iec {

enum GemmA { A_ROWS = 0, A_TAPS = 1, A_HALO = 2 };
enum GemmOut { OUT_STORE = 0, OUT_ACCUM = 1, OUT_WINDOW_ACCUM = 2, OUT_DOUBLE = 3, OUT_PHASE = 4, OUT_MAP = 5 };
enum GemmAct { ACT_NONE = 0, ACT_RELU = 1, ACT_GELU = 2, ACT_SIGMOID = 3 };

constexpr int GEMM_EPI_WARPS = 16;
constexpr int GEMM_THREADS = 64 + 32 * GEMM_EPI_WARPS;
constexpr int GEMM_MAX_TAPS = 49;

struct GemmParams {
  int M;                    // output rows (A_ROWS) or output pixels H * W (A_TAPS)
  int N, K;                 // output columns; reduction per tap (channels)
  int H, W, TW;             // A_TAPS: output size, tile width (16, or 8 for 8-wide outputs)
  int tiles_m, tiles_n, tiles, tiles_w;
  FastDiv div_tiles_n, div_tiles_w;
  int ksteps;               // K steps of KB channels (A_TAPS: taps x K / KB)
  int taps;
  signed char dy[GEMM_MAX_TAPS], dx[GEMM_MAX_TAPS], phase[GEMM_MAX_TAPS];
  int phase_y, phase_x;     // OUT_PHASE
  const uint16_t* b;        // [n tile][k step][KB / 8][BN][8] f16
  const float* bias;        // [N] or null
  int act;
  int out_mode;
  __half* out;              // planar f16: plane p at out + p * out_plane_elems
  long long out_plane_elems;  // elements per plane (rows * 8)
  int out_plane0;           // plane of output column 0
  int map_h, map_w, shift;  // OUT_WINDOW_ACCUM: the map the tokens came from,
  int win_ws, pad_h, pad_w; // its window side and the padded size the windows tile
  int dbl_w, dbl_cout;      // OUT_DOUBLE: input width, output channels
  // OUT_MAP: logical map size, reflect padding, phase split (1 or 2), pitch
  // and rows of one stored phase image, output step (1, or 2 for one phase
  // of a transposed convolution); A_ROWS reads the pixel (m / W, m % W).
  int dst_h, dst_w, dst_pad, dst_split, dst_pw, dst_ph, ostep;
  const __half* acc_src;    // added before the activation, or null
  const __half* resid;      // added after the activation, or null
  // Split-K: the K steps of each output tile in `ksplit` slices of `kslice`,
  // one tile per (slice, M tile, N tile); each writes its f32 partial sums
  // to ws[slice][row][ws_n], summed by gemm_splitk_reduce.
  int ksplit, kslice, tiles_mn, ws_n;
  float* ws;
  // A_HALO: a kh x kw grid of taps from (dy0, dx0); tiles of 4 halo_msub
  // rows x halo_tv (33 - kw) outputs; each channel chunk's halo box
  // (halo_rows x 32 pixels) in a ring of halo_bufs buffers halo_stride
  // bytes apart. The weights are packed per kernel row (ky) and chunk with
  // the kw taps of the row side by side in N (halo_np = kw BN columns,
  // b_stage bytes per block) from byte b_off: resident (b_resident, all
  // blocks loaded once) or through a ring of b_stages stages. One MMA per
  // kernel row gives each position's products with all kw taps, and the
  // epilogue adds the products of tap dx found dx positions to the right.
  int halo_kh, halo_kw, halo_dy0, halo_dx0, halo_rows, halo_tv, halo_stride, b_off, b_stages;
  int halo_msub, halo_np, b_stage, halo_bufs, b_resident;
  int* dev_err;
};

// OUT_MAP: the stored rows (or columns) that hold logical row `y` of a map of
// `n` rows reflect-padded by `pad` (pad < n): its own, and where the padding
// mirrors it, reflect(i) = min(|i|, 2 (n - 1) - i).
__device__ __forceinline__ int map_mirrors(int y, int n, int pad, int* r) {
  int k = 0;
  r[k++] = y + pad;
  if (y >= 1 && y <= pad) r[k++] = pad - y;
  if (y >= n - 1 - pad && y <= n - 2) r[k++] = pad + 2 * (n - 1) - y;
  return k;
}

__device__ __forceinline__ long long map_offset(const GemmParams& p, int r, int c) {
  if (p.dst_split == 2)
    return ((long long)(((r & 1) * 2 + (c & 1)) * p.dst_ph + (r >> 1))) * p.dst_pw + (c >> 1);
  return (long long)r * p.dst_pw + c;
}

// M blocks of 128 rows per tile: narrow tiles (N <= 64) take several, so that
// each tile's pipeline hand-offs and weight loads serve more rows and all
// four epilogue column parts have work.
__host__ __device__ constexpr int gemm_msub(int bn) { return bn <= 32 ? 4 : bn <= 64 ? 2 : 1; }

template <int BN, int KB>
struct GemmSmem {
  static constexpr int MSUB = gemm_msub(BN);
  static constexpr int A_ONE = (KB / 8) * 128 * 16;  // one M block
  static constexpr int A_BYTES = MSUB * A_ONE;
  static constexpr int B_BYTES = (KB / 8) * BN * 16;
  static constexpr int STAGE = ((A_BYTES + B_BYTES) + 1023) / 1024 * 1024;
  static constexpr int RING = 200 * 1024;  // the stages (or, for A_HALO, two halo boxes and a weight ring)
  static constexpr int NSTAGE = RING / STAGE > 8 ? 8 : RING / STAGE;
  static constexpr int NSLOT = 8;  // full / empty barrier pairs (A_HALO's weight ring may use all)
  static constexpr int BAR_OFF = RING;
  static constexpr int NBARS = 2 * NSLOT + 4 + 2 * NSLOT;  // + A_HALO's halo ring
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  // The bias, staged once per CTA for the epilogue (when N fits).
  static constexpr int BIAS_FLOATS = 4096;
  static constexpr int BIAS_OFF = (MISC_OFF + 16 + 15) / 16 * 16;
  static constexpr int TOTAL = BIAS_OFF + BIAS_FLOATS * 4;
  static constexpr int DYN_BYTES = TOTAL + 1024;
  static constexpr int ACC_COLS = MSUB * (BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256);
  static constexpr int TMEM_COLS = 2 * ACC_COLS < 32 ? 32 : 2 * ACC_COLS;
};

// w[e] += the 8 halves of `old`.
__device__ __forceinline__ void add_half8(float* w, const uint4 old) {
  const __half2* oh = reinterpret_cast<const __half2*>(&old);
#pragma unroll
  for (int e = 0; e < 4; e++) {
    const float2 f = __half22float2(oh[e]);
    w[2 * e] += f.x;
    w[2 * e + 1] += f.y;
  }
}

__device__ __forceinline__ uint4 pack_half8(const float* w) {
  uint32_t packed[4];
#pragma unroll
  for (int e = 0; e < 4; e++) {
    __half2 h2 = __floats2half2_rn(w[2 * e], w[2 * e + 1]);
    packed[e] = *reinterpret_cast<uint32_t*>(&h2);
  }
  return make_uint4(packed[0], packed[1], packed[2], packed[3]);
}

// Sigmoid stays out of line (and GELU compact): inlined into every element of
// the unrolled epilogue they made its loop body too large for the
// instruction cache, and the common ReLU / identity path would pay for them.
// GELU(v) = v Phi(v) = max(v, 0) - |v| (1 - erf(|v| / sqrt 2)) / 2, with erf
// by Abramowitz & Stegun 7.1.28: 1 - erf(a) = P(a)^-16 for a >= 0, P(a) = 1 +
// a1 a + ... + a6 a^6 (|error| <= 3e-7 in exact arithmetic). So
//   GELU(v) = max(v, 0) - |v| / (2 P(a)^16),  a = |v| / sqrt 2:
// one MUFU reciprocal per value (7.1.26 needs a reciprocal and an
// exponential; the fused MLP's hidden layer, 16,384 GELUs per 128-row tile,
// is bound by this arithmetic), and for negative v no cancellation between
// 1 and erf. Past a of about 13 the 16th power overflows to +inf, whose
// approximate reciprocal is +0 (PTX rcp.approx), which is the limit: GELU(v)
// = max(v, 0). Compact enough to stay inline in the epilogue (an IEEE
// division here cost more than the rest of the activation).
__device__ __forceinline__ float gelu_rcp(float q) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(q));
  return r;
}
__device__ __forceinline__ float gemm_gelu(float v) {
  const float av = fabsf(v), a = av * 0.70710678118654752f;
  float q = fmaf(fmaf(fmaf(fmaf(fmaf(fmaf(4.30638e-5f, a, 2.765672e-4f), a, 1.520143e-4f), a, 9.2705272e-3f), a,
                          4.22820123e-2f),
                     a, 7.05230784e-2f),
                a, 1.0f);
  q *= q;
  q *= q;
  q *= q;
  q *= q;
  return fmaf(-0.5f * av, gelu_rcp(q), fmaxf(v, 0.0f));
}

// The same GELU for two values, its multiplies and fused multiply-adds on
// packed f32 pairs (each lane the scalar operation, so the results equal two
// gemm_gelu calls), half the FP32 instructions; the reciprocal stays per value.
__device__ __forceinline__ float2 gemm_gelu2(float2 v) {
  auto both = [](float c) { return make_float2(c, c); };
  const float2 av = make_float2(fabsf(v.x), fabsf(v.y));
  const float2 a = fmul2(av, both(0.70710678118654752f));
  float2 q = ffma2(both(4.30638e-5f), a, both(2.765672e-4f));
  q = ffma2(q, a, both(1.520143e-4f));
  q = ffma2(q, a, both(9.2705272e-3f));
  q = ffma2(q, a, both(4.22820123e-2f));
  q = ffma2(q, a, both(7.05230784e-2f));
  q = ffma2(q, a, both(1.0f));
  q = fmul2(q, q);
  q = fmul2(q, q);
  q = fmul2(q, q);
  q = fmul2(q, q);
  return ffma2(fmul2(both(-0.5f), av), make_float2(gelu_rcp(q.x), gelu_rcp(q.y)),
               make_float2(fmaxf(v.x, 0.0f), fmaxf(v.y, 0.0f)));
}

static __device__ __noinline__ float gemm_sigmoid(float v) {
  // math.rs:33-39: from exp(-|x|), so that neither tail cancels.
  const float e = expf(-fabsf(v)), s = __fdividef(e, e + 1.0f);
  return v > 0.0f ? 1.0f - s : s;
}

// The activation of 16 values, one branch for all of them.
__device__ __forceinline__ void act16(float* v, int act) {
  if (act == ACT_RELU) {
#pragma unroll
    for (int e = 0; e < 16; e++) v[e] = v[e] > 0.0f ? v[e] : 0.0f;
  } else if (act == ACT_GELU) {
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
      const float2 g = gemm_gelu2(make_float2(v[e], v[e + 1]));
      v[e] = g.x;
      v[e + 1] = g.y;
    }
  } else if (act == ACT_SIGMOID) {
#pragma unroll
    for (int e = 0; e < 16; e++) v[e] = gemm_sigmoid(v[e]);
  }
}

__device__ __forceinline__ float gemm_act(float v, int act) {
  if (act == ACT_RELU) return v > 0.0f ? v : 0.0f;
  if (act == ACT_GELU) return gemm_gelu(v);
  if (act == ACT_SIGMOID) return gemm_sigmoid(v);
  return v;
}

// 16 accumulator columns from output column c0 (a multiple of 16) for the
// warp's 32 rows. A_HALO: the sum over the kernel row's kw taps of the
// products of tap dx held by the position dx to the right (lane + dx), which
// is this row's output; lanes past the last output read their own values.
template <int BN, int AMODE>
__device__ __forceinline__ void acc_ld16(const GemmParams& p, uint32_t taddr, int c0, uint32_t* r) {
  if constexpr (AMODE == A_HALO) {
    const int sb = c0 / BN, c = c0 - sb * BN;
    const uint32_t base = taddr + (uint32_t)(sb * p.halo_np + c);
    // the loads of two taps in flight together, one wait per pair
    uint32_t t1[16], t2[16];
    tmem_ld16(base, r);
    tmem_ld16(base + (uint32_t)BN, t1);
    tmem_ld16(base + (uint32_t)(2 * BN), t2);
    tmem_wait_ld();
#pragma unroll
    for (int e = 0; e < 16; e++)
      r[e] = __float_as_uint(__uint_as_float(r[e]) + __shfl_down_sync(0xffffffffu, __uint_as_float(t1[e]), 1) +
                             __shfl_down_sync(0xffffffffu, __uint_as_float(t2[e]), 2));
#pragma unroll 1
    for (int dx = 3; dx < p.halo_kw; dx += 2) {
      tmem_ld16(base + (uint32_t)(dx * BN), t1);
      tmem_ld16(base + (uint32_t)((dx + 1) * BN), t2);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 16; e++)
        r[e] = __float_as_uint(__uint_as_float(r[e]) + __shfl_down_sync(0xffffffffu, __uint_as_float(t1[e]), dx) +
                               __shfl_down_sync(0xffffffffu, __uint_as_float(t2[e]), dx + 1));
    }
  } else {
    tmem_ld16(taddr + (uint32_t)c0, r);
    tmem_wait_ld();
  }
}

// The OUT_MAP epilogue of one thread's row over accumulator columns
// [c_begin, c_end) of its tile (output column = that - cb + the N tile's):
// in batches of 32 columns (two TMEM loads), the old values of the batch's
// four 8-column groups are loaded together ahead of the accumulators, so
// that their latencies overlap.
template <int BN, int AMODE>
__device__ __forceinline__ void map_epilogue(const GemmParams& p, const float* bias, uint32_t taddr, int c_begin,
                                             int c_end, int cb, int nt, int m, const int* ry, const int* rx, int nry,
                                             int nrx) {
  const bool live = m >= 0;
  const long long pix = live ? map_offset(p, ry[0], rx[0]) * 8 : 0;
#pragma unroll 1
  for (int c0 = c_begin; c0 < c_end; c0 += 32) {
    const bool two = c0 + 16 < c_end;  // uniform across the warp
    uint4 oa[4], orr[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int n = nt * BN + (c0 - cb) + 8 * q;
      oa[q] = make_uint4(0u, 0u, 0u, 0u);
      orr[q] = oa[q];
      if (live && (q < 2 || two) && n < p.N) {
        const long long at = (long long)(p.out_plane0 + n / 8) * p.out_plane_elems + pix;
        if (p.acc_src) oa[q] = *reinterpret_cast<const uint4*>(p.acc_src + at);
        if (p.resid) orr[q] = *reinterpret_cast<const uint4*>(p.resid + at);
      }
    }
    uint32_t r[32];
    if constexpr (AMODE == A_HALO) {
      acc_ld16<BN, AMODE>(p, taddr, c0, r);  // 16 columns per part: `two` is false
    } else {
      tmem_ld16(taddr + (uint32_t)c0, r);
      if (two) tmem_ld16(taddr + (uint32_t)c0 + 16, r + 16);
      tmem_wait_ld();
    }
    if (!live) continue;
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int n = nt * BN + (c0 - cb) + 8 * q;
      if ((q >= 2 && !two) || n >= p.N) continue;
      float w[8];
#pragma unroll
      for (int e = 0; e < 8; e++) {
        float x = __uint_as_float(r[8 * q + e]);
        if (bias) x += bias[n + e < p.N ? n + e : 0];
        w[e] = x;
      }
      if (p.acc_src) add_half8(w, oa[q]);
#pragma unroll
      for (int e = 0; e < 8; e++) w[e] = gemm_act(w[e], p.act);
      if (p.resid) add_half8(w, orr[q]);
      const uint4 val = pack_half8(w);
      __half* plane = p.out + (long long)(p.out_plane0 + n / 8) * p.out_plane_elems;
      for (int iy = 0; iy < nry; iy++)
        for (int ix = 0; ix < nrx; ix++)
          *reinterpret_cast<uint4*>(plane + map_offset(p, ry[iy], rx[ix]) * 8) = val;
    }
  }
}

// M blocks per A_HALO tile for kernel width kw: as many as two accumulators
// of kw BN columns each leave room for in 512 TMEM columns (at most MSUB).
__host__ __device__ constexpr int halo_msub(int bn, int kw) {
  return gemm_msub(bn) < 256 / (kw * bn) ? gemm_msub(bn) : 256 / (kw * bn);
}

// The A_HALO MMA issuer for kernels of KW x KW taps. Kernel row ky of M
// block sb reads the halo box from row 4 sb + ky: its 128 MMA rows are the
// 4 x 32 positions of box rows 4 sb + ky .. 4 sb + ky + 3, its N = KW BN
// columns the row's KW taps; the accumulator of M block sb starts at column
// sb KW BN. Every MMA of a channel chunk is unrolled, with its descriptors
// a stage's base plus constant offsets: a loop or branch between MMAs costs
// the single issuing thread about as much as an MMA. RES: the weights are
// resident (all loaded once on full[0]), else they stream through the ring.
template <int BN, int KB, int KW, bool RES>
__device__ __forceinline__ void halo_mma_issuer(const GemmParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                                                uint64_t* acc_full, uint64_t* acc_empty, uint64_t* halo_full,
                                                uint64_t* halo_empty, uint32_t tmem_base, volatile int* abort_flag) {
  constexpr int NP = KW * BN, MS = halo_msub(BN, KW), ROWS = 4 * MS + KW - 1;
  constexpr uint32_t LBO_A = ROWS * 32 * 16, LBO_B = NP * 16;
  constexpr uint32_t IDESC = idesc_f16_f32(128, NP);
  const int chunks = p.K / KB, stages = p.b_stages, nh = p.halo_bufs;
  int hb = 0, s = 0, i = 0, last_acc = -1;
  uint32_t hph = 0, phase = 0, last_parity = 0;
  bool ok = true;
  if (RES) {
    ok = mbar_wait(&full[0], 0, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL);
    tc_fence_after();
  }
  const uint32_t bres = smem_u32(smem + p.b_off);
  for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, i++) {
    const int a = i & 1;
    const uint32_t acc_phase = (uint32_t)(i >> 1) & 1;
    if (!mbar_wait(&acc_empty[a], acc_phase ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_EMPTY)) break;
    tc_fence_after();
    const uint32_t d = tmem_base + (uint32_t)(a * 256);
    for (int kb = 0; kb < chunks && ok; kb++) {
      if (!mbar_wait(&halo_full[hb], hph, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t a0 = smem_desc(smem_u32(smem + hb * p.halo_stride), LBO_A, 128);
      const uint32_t more = kb != 0 ? 1u : 0u;
#pragma unroll
      for (int ky = 0; ky < KW; ky++) {
        uint64_t b0;
        if (RES) {
          b0 = smem_desc(bres + (uint32_t)((ky * chunks + kb) * p.b_stage), LBO_B, 128);
        } else {
          if (!mbar_wait(&full[s], phase, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          b0 = smem_desc(smem_u32(smem + p.b_off + s * p.b_stage), LBO_B, 128);
        }
#pragma unroll
        for (int j = 0; j < KB / 16; j++)
#pragma unroll
          for (int sb = 0; sb < MS; sb++)
            umma_f16(d + (uint32_t)(sb * NP), a0 + (uint64_t)((2 * j * LBO_A + (4 * sb + ky) * 512) >> 4),
                     b0 + (uint64_t)((2 * j * LBO_B) >> 4), IDESC, (ky != 0 || j != 0) ? 1u : more);
        if (!RES) {
          umma_commit(&empty[s]);
          const bool wrap = s + 1 == stages;
          s = wrap ? 0 : s + 1;
          phase ^= wrap ? 1u : 0u;
        }
      }
      if (!ok) break;
      umma_commit(&halo_empty[hb]);
      const bool hwrap = hb + 1 == nh;
      hb = hwrap ? 0 : hb + 1;
      hph ^= hwrap ? 1u : 0u;
    }
    if (!ok) break;
    umma_commit(&acc_full[a]);
    last_acc = a;
    last_parity = acc_phase;
  }
  if (last_acc >= 0) mbar_wait(&acc_full[last_acc], last_parity, abort_flag, p.dev_err, 0);
}

template <int BN, int KB, int AMODE>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    igemm_sm100(const __grid_constant__ CUtensorMap a_map, const GemmParams p) {
  static_assert(BN % 16 == 0 && BN <= 256 && (KB == 16 || KB == 32 || KB == 64), "tile shape");
  using L = GemmSmem<BN, KB>;
  constexpr int KG = KB / 8;  // channel groups per K step
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + L::NSLOT;
  uint64_t* acc_full = bars + 2 * L::NSLOT;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* halo_full = acc_empty + 2;  // A_HALO: the ring of halo buffers
  uint64_t* halo_empty = halo_full + L::NSLOT;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // A tile: rows of the box, and the A-side bytes one TMA load delivers.
  const int a_rows = AMODE == A_ROWS ? 128 : 8 * p.TW;
  const uint32_t a_bytes = AMODE == A_HALO ? (uint32_t)(KG * p.halo_rows * 32 * 16) : (uint32_t)(KG * a_rows * 16);
  // TMEM: two accumulators; A_HALO's hold up to 256 columns each.
  constexpr int ACC = AMODE == A_HALO ? 256 : L::ACC_COLS;
  constexpr int TMEM_COLS = AMODE == A_HALO ? 512 : L::TMEM_COLS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::NSLOT; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], GEMM_EPI_WARPS);
    }
    for (int h = 0; h < L::NSLOT; h++) {
      mbar_init(&halo_full[h], 1);
      mbar_init(&halo_empty[h], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: let the next kernel's CTAs start their
  // own set-up as SMs free up. The producer and the epilogue wait for the
  // previous kernel's results (and for its reads of what this one
  // overwrites) before they touch activations; the weights and the bias,
  // which no kernel writes, are fetched before that wait, so the ring's
  // first weight stages fill while the previous kernel drains. The MMA
  // issuer touches no global memory. Without the launch attribute the
  // waits are no-ops.
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      prefetch_tensor_map(&a_map);
      if constexpr (AMODE == A_HALO) {
        // Per tile and channel chunk one halo box through the ring of
        // halo_bufs buffers. The weights of each kernel row and chunk (block
        // (nt kh + ky) chunks + chunk) either stream through the weight ring
        // after their chunk's box, or, with b_resident, are all loaded once
        // up front on full[0] and stay.
        const int chunks = p.K / KB, nh = p.halo_bufs;
        int hb = 0, s = 0, n_halo = 0, n_b = 0;
        uint32_t hph = 0, phase = 0;
        bool ok = true;
        if (p.b_resident) {
          const uint32_t total = (uint32_t)(p.halo_kh * chunks * p.b_stage);
          mbar_arrive_expect_tx(&full[0], total);
          for (int blk = 0; blk < p.halo_kh * chunks; blk++)
            bulk_load(smem + p.b_off + blk * p.b_stage, reinterpret_cast<const uint8_t*>(p.b) + (size_t)blk * p.b_stage,
                      (uint32_t)p.b_stage, &full[0]);
        }
        griddep_wait();
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
          const int mt = (int)p.div_tiles_n.div((uint32_t)tile), nt = tile - mt * p.tiles_n;
          const int ty = (int)p.div_tiles_w.div((uint32_t)mt), tx = mt - ty * p.tiles_w;
          const int x0 = tx * p.halo_tv, y0 = ty * 4 * p.halo_msub;
          const uint8_t* bsrc = reinterpret_cast<const uint8_t*>(p.b) + (size_t)nt * p.halo_kh * chunks * p.b_stage;
          for (int kb = 0; kb < chunks && ok; kb++) {
            if (!mbar_wait(&halo_empty[hb], hph ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_EMPTY)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&halo_full[hb], a_bytes);
            tma_load_5d(smem + hb * p.halo_stride, &a_map, &halo_full[hb], (x0 + p.halo_dx0) * 8, y0 + p.halo_dy0, 0,
                        kb * KG, 0);
            n_halo++;
            if (++hb == nh) {
              hb = 0;
              hph ^= 1;
            }
            if (p.b_resident) continue;
            for (int ky = 0; ky < p.halo_kh; ky++) {
              if (!mbar_wait(&empty[s], phase ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_EMPTY)) {
                ok = false;
                break;
              }
              uint8_t* st = smem + p.b_off + s * p.b_stage;
              mbar_arrive_expect_tx(&full[s], (uint32_t)p.b_stage);
              bulk_load(st, bsrc + (size_t)(ky * chunks + kb) * p.b_stage, (uint32_t)p.b_stage, &full[s]);
              n_b++;
              if (++s == p.b_stages) {
                s = 0;
                phase ^= 1;
              }
            }
          }
        }
        // the copies in flight land before the CTA may leave
        for (int c = n_halo - nh; c < n_halo; c++)
          if (c >= 0) mbar_wait(&halo_full[c % nh], (uint32_t)(c / nh) & 1, abort_flag, p.dev_err, 0);
        if (p.b_resident) mbar_wait(&full[0], 0, abort_flag, p.dev_err, 0);
        for (int c = n_b - p.b_stages; c < n_b; c++)
          if (c >= 0) mbar_wait(&full[c % p.b_stages], (uint32_t)(c / p.b_stages) & 1, abort_flag, p.dev_err, 0);
      } else {
      int s = 0;
      uint32_t phase = 0;
      int issued[L::NSTAGE];
      for (int i = 0; i < L::NSTAGE; i++) issued[i] = -1;
      bool ok = true;
      // The first NSTAGE stages (fresh, so free) get their weights and their
      // whole transaction count now; their A boxes follow after the wait.
      int pre = 0;
      for (int tile = blockIdx.x; tile < p.tiles && pre < L::NSTAGE; tile += gridDim.x) {
        const int split = p.ksplit > 1 ? tile / p.tiles_mn : 0, tmn = tile - split * p.tiles_mn;
        const int nt = tmn - (int)p.div_tiles_n.div((uint32_t)tmn) * p.tiles_n;
        const int ks0 = split * p.kslice, ks1 = min(ks0 + p.kslice, p.ksteps);
        const uint8_t* bsrc = reinterpret_cast<const uint8_t*>(p.b) + (size_t)nt * p.ksteps * L::B_BYTES;
        for (int ks = ks0; ks < ks1 && pre < L::NSTAGE; ks++, pre++) {
          mbar_arrive_expect_tx(&full[pre], (uint32_t)L::MSUB * a_bytes + (uint32_t)L::B_BYTES);
          bulk_load(smem + pre * L::STAGE + L::A_BYTES, bsrc + (size_t)ks * L::B_BYTES, L::B_BYTES, &full[pre]);
        }
      }
      griddep_wait();
      int n_issue = 0;
      for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
        const int split = p.ksplit > 1 ? tile / p.tiles_mn : 0, tmn = tile - split * p.tiles_mn;
        const int mt = (int)p.div_tiles_n.div((uint32_t)tmn), nt = tmn - mt * p.tiles_n;
        const int ks0 = split * p.kslice, ks1 = min(ks0 + p.kslice, p.ksteps);
        const uint8_t* bsrc = reinterpret_cast<const uint8_t*>(p.b) + (size_t)nt * p.ksteps * L::B_BYTES;
        for (int ks = ks0; ks < ks1; ks++, n_issue++) {
          const bool early = n_issue < pre;  // weights already in flight
          if (!early && !mbar_wait(&empty[s], phase ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_EMPTY)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * L::STAGE;
          if (!early) mbar_arrive_expect_tx(&full[s], (uint32_t)L::MSUB * a_bytes + (uint32_t)L::B_BYTES);
#pragma unroll
          for (int sb = 0; sb < L::MSUB; sb++) {
            const int blk = mt * L::MSUB + sb;
            uint8_t* sa = st + sb * L::A_ONE;
            if (AMODE == A_ROWS) {
              tma_load_3d(sa, &a_map, &full[s], 0, blk * 8, ks * KG);
            } else {
              const int by = (int)p.div_tiles_w.div((uint32_t)blk);
              const int bx0 = (blk - by * p.tiles_w) * p.TW, by0 = by * 8;
              const int per_tap = p.K / KB;
              const int tap = ks / per_tap, kb = ks - tap * per_tap;
              tma_load_5d(sa, &a_map, &full[s], (bx0 + p.dx[tap]) * 8, by0 + p.dy[tap], p.phase[tap], kb * KG, 0);
            }
          }
          if (!early) bulk_load(st + L::A_BYTES, bsrc + (size_t)ks * L::B_BYTES, L::B_BYTES, &full[s]);
          issued[s] = (int)phase;
          if (++s == L::NSTAGE) {
            s = 0;
            phase ^= 1;
          }
        }
      }
      for (int i = 0; i < L::NSTAGE; i++)
        if (issued[i] >= 0) mbar_wait(&full[i], (uint32_t)issued[i], abort_flag, p.dev_err, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = idesc_f16_f32(128, BN);
      if constexpr (AMODE == A_HALO) {
        // (the launch checks kw: 3 for bn <= 64, 5 and 7 for bn 32)
#define IEC_HALO_ISSUE(KW_)                                                                                        \
  do {                                                                                                             \
    if (p.b_resident)                                                                                              \
      halo_mma_issuer<BN, KB, KW_, true>(p, smem, full, empty, acc_full, acc_empty, halo_full, halo_empty, tmem_base, \
                                         abort_flag);                                                              \
    else                                                                                                           \
      halo_mma_issuer<BN, KB, KW_, false>(p, smem, full, empty, acc_full, acc_empty, halo_full, halo_empty,          \
                                          tmem_base, abort_flag);                                                  \
  } while (0)
        if constexpr (BN <= 64) {
          if (p.halo_kw == 3) IEC_HALO_ISSUE(3);
        }
        if constexpr (BN <= 32) {
          if (p.halo_kw == 5) IEC_HALO_ISSUE(5);
          if (p.halo_kw == 7) IEC_HALO_ISSUE(7);
        }
#undef IEC_HALO_ISSUE
      } else {
      const uint32_t lbo_a = (uint32_t)(a_rows * 16);
      int s = 0, i = 0, last_acc = -1;
      uint32_t phase = 0, last_parity = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, i++) {
        const int a = i & 1;
        const uint32_t acc_phase = (uint32_t)(i >> 1) & 1;
        if (!mbar_wait(&acc_empty[a], acc_phase ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_EMPTY)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(a * L::ACC_COLS);
        const int split = p.ksplit > 1 ? tile / p.tiles_mn : 0;  // no division without split-K
        const int ks0 = split * p.kslice, ks1 = min(ks0 + p.kslice, p.ksteps);
        for (int ks = ks0; ks < ks1; ks++) {
          if (!mbar_wait(&full[s], phase, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t abase = smem_u32(smem + s * L::STAGE), bbase = abase + (uint32_t)L::A_BYTES;
#pragma unroll
          for (int sb = 0; sb < L::MSUB; sb++)
#pragma unroll
            for (int j = 0; j < KB / 16; j++) {
              const uint64_t adesc = smem_desc(abase + (uint32_t)(sb * L::A_ONE + 2 * j * lbo_a), lbo_a, 128);
              const uint64_t bdesc = smem_desc(bbase + (uint32_t)(2 * j * BN * 16), BN * 16, 128);
              umma_f16(d + (uint32_t)(sb * BN), adesc, bdesc, idesc, (ks != ks0) || (j != 0));
            }
          umma_commit(&empty[s]);
          const bool wrap = s + 1 == L::NSTAGE;
          s = wrap ? 0 : s + 1;
          phase ^= wrap ? 1u : 0u;
        }
        if (!ok) break;
        umma_commit(&acc_full[a]);
        last_acc = a;
        last_parity = acc_phase;
      }
      if (last_acc >= 0) mbar_wait(&acc_full[last_acc], last_parity, abort_flag, p.dev_err, 0);
      }
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    const int part = (warp - 2) >> 2;  // which quarter of the columns
    const int row = quarter * 32 + lane;
    // columns per part (a multiple of 16); with several M blocks a part's
    // columns lie in one block's accumulator
    // (A_HALO: 16 columns per part, of halo_msub M blocks)
    const int HALF = AMODE == A_HALO ? 16 : (L::MSUB * BN + 63) / 64 * 16;
    const int ACC_USED = AMODE == A_HALO ? p.halo_msub * BN : L::MSUB * BN;
    const int sb = (part * HALF) / BN;  // this part's M block within the tile
    const int cb = sb * BN;             // its first accumulator column
    // Stage the bias in shared memory: the epilogue then reads it at shared
    // memory latency instead of a round trip to L2 per column chunk.
    float* sbias = reinterpret_cast<float*>(smem + L::BIAS_OFF);
    const int n_pad = p.tiles_n * BN;
    const bool bias_staged = p.bias && n_pad <= L::BIAS_FLOATS;
    if (bias_staged)
      for (int j = (int)threadIdx.x - 64; j < n_pad; j += 32 * GEMM_EPI_WARPS) sbias[j] = j < p.N ? p.bias[j] : 0.0f;
    asm volatile("bar.sync 1, %0;" ::"n"(32 * GEMM_EPI_WARPS) : "memory");
    const float* bias = bias_staged ? sbias : p.bias;
    griddep_wait();
    int i = 0;
    for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, i++) {
      const int a = i & 1;
      const uint32_t acc_phase = (uint32_t)(i >> 1) & 1;
      const int split = p.ksplit > 1 ? tile / p.tiles_mn : 0, tmn = tile - split * p.tiles_mn;
      const int mt = (int)p.div_tiles_n.div((uint32_t)tmn), nt = tmn - mt * p.tiles_n;
      // This thread's output row, and for A_TAPS its pixel.
      int m = -1, oy = 0, ox = 0;
      const int blk = mt * L::MSUB + sb;
      if (AMODE == A_ROWS) {
        m = blk * 128 + row;
        if (m >= p.M) m = -1;
      } else if (AMODE == A_HALO) {
        // M block sb: tile rows 4 sb .. 4 sb + 3 (one per lane quarter),
        // positions 0 .. 31 (one per lane), of which halo_tv are outputs
        const int ty = (int)p.div_tiles_w.div((uint32_t)mt), tx = mt - ty * p.tiles_w;
        oy = ty * 4 * p.halo_msub + 4 * sb + quarter;
        ox = tx * p.halo_tv + lane;
        if (lane < p.halo_tv && oy < p.H && ox < p.W) m = oy * p.W + ox;
      } else {
        const int ty = (int)p.div_tiles_w.div((uint32_t)blk);
        const int x0 = (blk - ty * p.tiles_w) * p.TW, y0 = ty * 8;
        oy = y0 + row / p.TW;
        ox = x0 + row % p.TW;
        if (row < a_rows && oy < p.H && ox < p.W) m = oy * p.W + ox;
      }
      // OUT_MAP: the stored pixels that hold this row's output.
      int ry[3], rx[3], nry = 0, nrx = 0;
      if (p.out_mode == OUT_MAP && m >= 0) {
        if (AMODE == A_ROWS) {
          oy = m / p.W;
          ox = m - oy * p.W;
        }
        nry = map_mirrors(oy * p.ostep + p.phase_y, p.dst_h, p.dst_pad, ry);
        nrx = map_mirrors(ox * p.ostep + p.phase_x, p.dst_w, p.dst_pad, rx);
      }
      // Destination pixel of the row for the scattering epilogues.
      long long dest = m;
      if (m >= 0 && p.out_mode == OUT_WINDOW_ACCUM) {
        // Window slots of 64 rows: rows past ws * ws tokens, and tokens of
        // the padding past the map's edge, are dropped.
        const int win = m >> 6, t = m & 63, ws = p.win_ws, cols = p.pad_w / ws;
        const int wy = win / cols, wx = win - wy * cols;
        const int py = (wy * ws + t / ws + p.shift) % p.pad_h, px = (wx * ws + t % ws + p.shift) % p.pad_w;
        if (t >= ws * ws || py >= p.map_h || px >= p.map_w)
          m = -1;
        else
          dest = (long long)py * p.map_w + px;
      }
      // The accumulating epilogues read the old values of their rows: fetch
      // them towards L1 before waiting for the accumulator, so that their
      // latency overlaps the tile's MMAs instead of following each TMEM load
      // (a hint: nothing is held in registers; the rows are this launch's own).
      if (p.ksplit == 1 && (p.out_mode == OUT_ACCUM || p.out_mode == OUT_WINDOW_ACCUM) && m >= 0) {
#pragma unroll 1
        for (int c = part * HALF; c < part * HALF + HALF && c < ACC_USED; c += 8) {
          const int n = nt * BN + (c - cb);
          if (n >= p.N) break;
          prefetch_l1(p.out + (long long)(p.out_plane0 + n / 8) * p.out_plane_elems + dest * 8);
        }
      }
      if (!mbar_wait(&acc_full[a], acc_phase, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_FULL)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * ACC);
      if (p.ksplit > 1) {
        // the slice's raw partial sums, f32
#pragma unroll 1
        for (int c0 = part * HALF; c0 < part * HALF + HALF && c0 < ACC_USED; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(taddr + (uint32_t)c0, r);
          tmem_wait_ld();
          if (m < 0) continue;
          float4* w = reinterpret_cast<float4*>(p.ws + ((size_t)split * p.M + m) * p.ws_n + nt * BN + (c0 - cb));
#pragma unroll
          for (int q = 0; q < 4; q++)
            w[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                               __uint_as_float(r[4 * q + 3]));
        }
      } else if (p.out_mode == OUT_MAP)
        map_epilogue<BN, AMODE>(p, bias, taddr, part * HALF, min(part * HALF + HALF, ACC_USED), cb, nt, m, ry, rx, nry, nrx);
#pragma unroll 1
      for (int c0 = part * HALF; p.ksplit == 1 && p.out_mode != OUT_MAP && c0 < part * HALF + HALF && c0 < ACC_USED;
           c0 += 16) {
        uint32_t r[16];
        acc_ld16<BN, AMODE>(p, taddr, c0, r);
        const int n0 = nt * BN + (c0 - cb);
        if (m < 0 || n0 >= p.N) continue;
        float v[16];
        if (bias_staged) {
          const float4* b4 = reinterpret_cast<const float4*>(sbias + n0);
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const float4 b = b4[q];
            v[4 * q] = __uint_as_float(r[4 * q]) + b.x;
            v[4 * q + 1] = __uint_as_float(r[4 * q + 1]) + b.y;
            v[4 * q + 2] = __uint_as_float(r[4 * q + 2]) + b.z;
            v[4 * q + 3] = __uint_as_float(r[4 * q + 3]) + b.w;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; e++) {
            float x = __uint_as_float(r[e]);
            if (bias) x += bias[n0 + e < p.N ? n0 + e : 0];
            v[e] = x;
          }
        }
        if (p.out_mode == OUT_STORE) {
          // the common case without per-group branches
          act16(v, p.act);
          __half* dst = p.out + (long long)(p.out_plane0 + n0 / 8) * p.out_plane_elems + dest * 8;
          *reinterpret_cast<uint4*>(dst) = pack_half8(v);
          if (n0 + 8 < p.N) *reinterpret_cast<uint4*>(dst + p.out_plane_elems) = pack_half8(v + 8);
          continue;
        }
#pragma unroll
        for (int g = 0; g < 2; g++) {
          const int n = n0 + 8 * g;
          if (n >= p.N) break;
          __half* dst;
          if (p.out_mode == OUT_DOUBLE) {
            const int q = n / p.dbl_cout, o = n - q * p.dbl_cout;
            const int iy = m / p.dbl_w, ix = m - iy * p.dbl_w;
            const long long op = (long long)(2 * iy + (q >> 1)) * (2 * p.dbl_w) + 2 * ix + (q & 1);
            dst = p.out + (long long)(p.out_plane0 + o / 8) * p.out_plane_elems + op * 8;
          } else if (p.out_mode == OUT_PHASE) {
            const int iy = m / p.W, ix = m - iy * p.W;
            const long long op = (long long)(2 * iy + p.phase_y) * (2 * p.W) + 2 * ix + p.phase_x;
            dst = p.out + (long long)(p.out_plane0 + n / 8) * p.out_plane_elems + op * 8;
          } else {
            dst = p.out + (long long)(p.out_plane0 + n / 8) * p.out_plane_elems + dest * 8;
          }
          float w8[8];
#pragma unroll
          for (int e = 0; e < 8; e++) w8[e] = v[8 * g + e];
          if (p.out_mode == OUT_ACCUM || p.out_mode == OUT_WINDOW_ACCUM) {
            const uint4 old = *reinterpret_cast<const uint4*>(dst);
            const __half2* oh = reinterpret_cast<const __half2*>(&old);
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const float2 f = __half22float2(oh[e]);
              w8[2 * e] += f.x;
              w8[2 * e + 1] += f.y;
            }
          }
#pragma unroll
          for (int e = 0; e < 8; e++) w8[e] = gemm_act(w8[e], p.act);
          uint32_t packed[4];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            __half2 h2 = __floats2half2_rn(w8[2 * e], w8[2 * e + 1]);
            packed[e] = *reinterpret_cast<uint32_t*>(&h2);
          }
          *reinterpret_cast<uint4*>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// Split-K: out = the slices' partial sums added in slice order, then the
// tile epilogue's bias, activation and store (OUT_STORE, OUT_ACCUM, OUT_MAP).
// One thread per (row, 8-column group).
static __global__ void __launch_bounds__(256) gemm_splitk_reduce(const GemmParams p) {
  griddep_wait();  // launched as a programmatic dependent of the GEMM
  const int groups = (p.N + 7) / 8;
  const long long total = (long long)p.M * groups;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / groups), g = (int)(i - (long long)m * groups), n0 = 8 * g;
    float w[8];
#pragma unroll
    for (int e = 0; e < 8; e++) w[e] = 0.0f;
    for (int sp = 0; sp < p.ksplit; sp++) {
      const float4* src = reinterpret_cast<const float4*>(p.ws + ((size_t)sp * p.M + m) * p.ws_n + n0);
      const float4 a = src[0], b = src[1];
      w[0] += a.x;
      w[1] += a.y;
      w[2] += a.z;
      w[3] += a.w;
      w[4] += b.x;
      w[5] += b.y;
      w[6] += b.z;
      w[7] += b.w;
    }
    if (p.bias)
#pragma unroll
      for (int e = 0; e < 8; e++) w[e] += p.bias[n0 + e < p.N ? n0 + e : 0];
    __half* plane = p.out + (long long)(p.out_plane0 + g) * p.out_plane_elems;
    if (p.out_mode == OUT_MAP) {
      const int oy = m / p.W, ox = m - oy * p.W;
      int ry[3], rx[3];
      const int nry = map_mirrors(oy * p.ostep + p.phase_y, p.dst_h, p.dst_pad, ry);
      const int nrx = map_mirrors(ox * p.ostep + p.phase_x, p.dst_w, p.dst_pad, rx);
      const long long at = (long long)(p.out_plane0 + g) * p.out_plane_elems + map_offset(p, ry[0], rx[0]) * 8;
      if (p.acc_src) add_half8(w, *reinterpret_cast<const uint4*>(p.acc_src + at));
#pragma unroll
      for (int e = 0; e < 8; e++) w[e] = gemm_act(w[e], p.act);
      if (p.resid) add_half8(w, *reinterpret_cast<const uint4*>(p.resid + at));
      const uint4 val = pack_half8(w);
      for (int iy = 0; iy < nry; iy++)
        for (int ix = 0; ix < nrx; ix++) *reinterpret_cast<uint4*>(plane + map_offset(p, ry[iy], rx[ix]) * 8) = val;
      continue;
    }
    __half* dst = plane + (long long)m * 8;
    if (p.out_mode == OUT_ACCUM) add_half8(w, *reinterpret_cast<const uint4*>(dst));
#pragma unroll
    for (int e = 0; e < 8; e++) w[e] = gemm_act(w[e], p.act);
    *reinterpret_cast<uint4*>(dst) = pack_half8(w);
  }
}

}  // namespace iec
