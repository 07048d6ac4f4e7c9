// Implicit-GEMM 3x3 convolution (stride 1, zero padding) on sm_100a tensor
// cores: f16 inputs, f32 accumulators in TMEM, fused epilogues.
//
// Semantics: crates/native-engine/src/gemm.rs:514-667 (multiply over
// Taps::Conv { size: 3, step: 1, pad: Zero }) with the epilogue of
// crates/realesrgan-native/src/network.rs:31-41,80-112 (bias, PReLU) or
// network.rs:118-140 (pixel shuffle x4 plus the input repeated).
//
// Layout. Feature maps are f16 and "channel-group planar": [image][cin / 8]
// [height][width][8], so a row of one plane is contiguous. One tile is 4 rows
// x 30 columns of output pixels. Its MMA rows (M = 128) are the 4 x 32
// positions x0 - 1 .. x0 + 30 of those rows (one row per TMEM lane quarter,
// so per epilogue warp), and its MMA columns are the three horizontal taps
// side by side (N = 3 * cout): row (r, c), column kx * cout + o accumulates
// Q_kx(r, c)[o] = sum over ky and channels of in(r + ky - 1, c - 1) *
// w[ky][kx][.][o]. Output pixel (r, c) (c = 1..30) is then Q_0(r, c - 1) +
// Q_1(r, c) + Q_2(r, c + 1): its neighbours' partial sums sit in the
// adjacent TMEM lanes, one warp shuffle away. Three MMAs of N = 192 fetch as
// many shared-memory operand bytes as three of N = 64 but do three times the
// math, which is what bounds this convolution (its narrow N otherwise leaves
// the tensor core waiting on operand fetches). 30 of every 32 positions are
// outputs (an 8 x 16 block of positions kept 14 of 16: the MMAs and the
// epilogue did 7 % more work per output pixel).
//
// A single 4-D TMA box (inner row 32 pixels x 8 channels = 512 bytes) brings
// the tile's 6 x 32 pixel halo of every channel group into shared memory as
// [group][6][32][8]: the no-swizzle K-major core-matrix layout tcgen05
// reads, 8 consecutive positions of a row per core matrix (SBO 128 bytes),
// the next channel group 3072 bytes on (LBO). Tap row ky is a start offset
// of ky * 512 bytes into the same halo; out-of-image pixels are TMA's zero
// fill.
//
// The weights of the layer, pre-arranged on the host as [ky][cin / 8]
// [kx][cout][8] (the K-major core-matrix image of B), stay in shared memory
// for the whole persistent kernel (72 KB for 64 -> 64).
//
// Roles (576 threads): warp 0 one thread issues TMA loads into a ring of
// NSTAGE halo stages; warp 1 one thread issues 3 * cin / 16 UMMAs
// (M 128, N 3 cout, K 16) per tile into one of two TMEM accumulators; warps
// 2..17 (four per TMEM lane quarter, each with a quarter of the channels, or
// one output row of the pixel shuffle) drain an accumulator while the next
// tile's MMAs run, combine the taps, apply the epilogue and store. Per tile
// the epilogue issues several times the MMA warp's instructions and waits on
// TMEM loads and shuffles, so it gets four warps per SM sub-partition to
// hide those latencies.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "sm100.cuh"

namespace iec {

constexpr int CONV_TILE_H = 4;                    // output rows of a tile
constexpr int CONV_TILE_W = 30;                   // output columns of a tile
constexpr int CONV_HALO_H = CONV_TILE_H + 2;      // 6
constexpr int CONV_HALO_W = CONV_TILE_W + 2;      // 32: also the partial-sum positions of a row (one warp)
constexpr int CONV_CHUNK_BYTES = CONV_HALO_H * CONV_HALO_W * 16;  // 3072: one channel group
constexpr int CONV_NSTAGE = 6;
constexpr int CONV_EPI_WARPS = 16;                // four per TMEM lane quarter
constexpr int CONV_THREADS = 64 + 32 * CONV_EPI_WARPS;
constexpr int CONV_ACC_COLS = 256;                // TMEM columns between the two accumulators
constexpr int CONV_TMEM_COLS = 2 * CONV_ACC_COLS;

enum ConvMode { CONV_PRELU = 0, CONV_SHUFFLE = 1 };

// Where the pixel-shuffle epilogue adds the input and stores the result: the
// network ran on a region of a larger source image (a tile with its margin),
// and only the window [kx0, kx1) x [ky0, ky1) of the region is kept.
struct ShuffleOut {
  const void* src;  // network input images: f32 or u8, [image][src_h][src_w][3]
  void* dst;        // output: f32 or u8, [image][4 src_h][4 src_w][3]
  int src_w, src_h;
  int rx0, ry0;     // region origin in the source image
  int kx0, ky0, kx1, ky1;
  int src_u8, dst_u8;
};

struct ConvParams {
  int H, W;                    // valid size of the maps (the region)
  int MH, MW;                  // allocated size of the maps (>= H, W; the excess stays zero)
  int tiles_x, tiles_y, tiles;  // tile grid over all images (tiles < 2^24, sides < 2^16)
  FastDiv div_tiles_x, div_tiles_y;
  int slope_unit;              // every PReLU slope is in [0, 1]: max(v, s v) is PReLU
  const uint16_t* weights;     // [3 ky][cin / 8][3 kx][cout][8] f16
  const float* bias;           // [cout]
  const float* slope;          // [cout] PReLU slopes, or null
  __half* out;                 // CONV_PRELU: [image][cout / 8][MH][MW][8]
  ShuffleOut shuffle;          // CONV_SHUFFLE
  int* dev_err;
};

template <int CIN, int COUT>
struct ConvSmem {
  static constexpr int KCH = CIN / 8;
  static constexpr int W_BYTES = 9 * KCH * COUT * 16;
  static constexpr int W_ALLOC = (W_BYTES + 1023) / 1024 * 1024;
  static constexpr int STAGE_BYTES = (KCH * CONV_CHUNK_BYTES + 1023) / 1024 * 1024;
  static constexpr int A_OFF = W_ALLOC;
  static constexpr int BAR_OFF = A_OFF + CONV_NSTAGE * STAGE_BYTES;
  // full[NSTAGE], empty[NSTAGE], acc_full[2], acc_empty[2], weights
  static constexpr int NBARS = 2 * CONV_NSTAGE + 5;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;      // tmem slot, abort flag
  static constexpr int BIAS_OFF = (MISC_OFF + 16 + 15) / 16 * 16;
  static constexpr int TOTAL = BIAS_OFF + 2 * COUT * 4;
  static constexpr int DYN_BYTES = TOTAL + 1024;             // room to align the base
};

template <int CIN, int COUT, int MODE>
__global__ void __launch_bounds__(CONV_THREADS, 1)
    conv3x3_sm100(const __grid_constant__ CUtensorMap in_map, const ConvParams p) {
  static_assert(CIN % 16 == 0 && COUT % 16 == 0 && COUT <= 64, "tile shape");
  using L = ConvSmem<CIN, COUT>;
  constexpr int KCH = L::KCH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* w_smem = smem;
  uint8_t* a_smem = smem + L::A_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + CONV_NSTAGE;
  uint64_t* acc_full = bars + 2 * CONV_NSTAGE;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* wbar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);
  float* s_bias = reinterpret_cast<float*>(smem + L::BIAS_OFF);
  float* s_slope = s_bias + COUT;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Programmatic dependent launch: the next layer's CTAs may take each SM as
  // this grid's CTA there exits, and run their prologue (barriers, TMEM,
  // weights) while the other SMs finish. One CTA fills an SM's shared memory,
  // so they never share one.
  griddep_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < CONV_NSTAGE; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], CONV_EPI_WARPS);
    }
    mbar_init(wbar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, CONV_TMEM_COLS);
    tmem_relinquish();
  }
  for (int c = threadIdx.x; c < COUT; c += CONV_THREADS) {
    s_bias[c] = p.bias[c];
    s_slope[c] = p.slope ? p.slope[c] : 1.0f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      prefetch_tensor_map(&in_map);
      mbar_arrive_expect_tx(wbar, L::W_BYTES);
      for (int off = 0; off < L::W_BYTES; off += 32768) {
        int bytes = L::W_BYTES - off < 32768 ? L::W_BYTES - off : 32768;
        bulk_load(w_smem + off, reinterpret_cast<const uint8_t*>(p.weights) + off, bytes, wbar);
      }
      // The previous layer wrote this layer's input and reads its output
      // buffer: nothing of either is touched before it has completed (the
      // epilogue's stores follow these loads).
      griddep_wait();
      int s = 0;
      uint32_t phase = 0;
      int issued[CONV_NSTAGE];  // parity of the last load into each stage, -1 none
      for (int i = 0; i < CONV_NSTAGE; i++) issued[i] = -1;
      for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x) {
        if (!mbar_wait(&empty[s], phase ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_EMPTY)) break;
        const int row_id = (int)p.div_tiles_x.div((uint32_t)tile);  // image * tiles_y + ty
        const int tx = tile - row_id * p.tiles_x;
        const int img = (int)p.div_tiles_y.div((uint32_t)row_id), ty = row_id - img * p.tiles_y;
        mbar_arrive_expect_tx(&full[s], KCH * CONV_CHUNK_BYTES);
        // x in elements of a plane row: (x0 - 1) * 8 halves, 16-byte aligned.
        tma_load_4d(a_smem + s * L::STAGE_BYTES, &in_map, &full[s], (tx * CONV_TILE_W - 1) * 8,
                    ty * CONV_TILE_H - 1, 0, img);
        issued[s] = (int)phase;
        if (++s == CONV_NSTAGE) {
          s = 0;
          phase ^= 1;
        }
      }
      // No copy may still be writing shared memory when the CTA exits.
      for (int i = 0; i < CONV_NSTAGE; i++)
        if (issued[i] >= 0) mbar_wait(&full[i], (uint32_t)issued[i], abort_flag, p.dev_err, 0);
      mbar_wait(wbar, 0, abort_flag, p.dev_err, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr int N = 3 * COUT;
      constexpr uint32_t idesc = idesc_f16_f32(128, N);
      const uint32_t abase0 = smem_u32(a_smem), wbase = smem_u32(w_smem);
      int last_acc = -1;
      uint32_t last_parity = 0;
      if (mbar_wait(wbar, 0, abort_flag, p.dev_err, DEV_ERR_WAIT_WEIGHTS)) {
        int s = 0, i = 0;
        uint32_t phase = 0;
        for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, i++) {
          const int a = i & 1;
          const uint32_t acc_phase = (uint32_t)(i >> 1) & 1;
          if (!mbar_wait(&acc_empty[a], acc_phase ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_EMPTY)) break;
          if (!mbar_wait(&full[s], phase, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL)) break;
          tc_fence_after();
          const uint32_t d = tmem_base + (uint32_t)(a * CONV_ACC_COLS);
          const uint32_t abase = abase0 + (uint32_t)(s * L::STAGE_BYTES);
#pragma unroll
          for (int ky = 0; ky < 3; ky++) {
#pragma unroll
            for (int ks = 0; ks < KCH / 2; ks++) {
              // A: positions (r, c) of the tile read halo pixel (r + ky, c);
              // B: the three kx taps' weights of row ky, N = 3 cout.
              const uint64_t adesc = smem_desc(abase + (uint32_t)(2 * ks * CONV_CHUNK_BYTES + ky * CONV_HALO_W * 16),
                                               CONV_CHUNK_BYTES, 128);
              const uint64_t bdesc = smem_desc(wbase + (uint32_t)((ky * KCH + 2 * ks) * N * 16), N * 16, 128);
              umma_f16(d, adesc, bdesc, idesc, (ky | ks) != 0);
            }
          }
          umma_commit(&empty[s]);
          umma_commit(&acc_full[a]);
          last_acc = a;
          last_parity = acc_phase;
          if (++s == CONV_NSTAGE) {
            s = 0;
            phase ^= 1;
          }
        }
      }
      // The accumulators must be written before TMEM is released.
      if (last_acc >= 0) mbar_wait(&acc_full[last_acc], last_parity, abort_flag, p.dev_err, 0);
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int quarter = warp & 3;            // TMEM lanes 32 q .. 32 q + 31
    const int part = (warp - 2) >> 2;        // which quarter of the channels (0..3)
    const int row = quarter * 32 + lane;     // M row = partial-sum position (r, c) of the tile
    const int pr = row / CONV_HALO_W, pc = row % CONV_HALO_W;
    // This warp's channels' bias and PReLU slope, kept in registers.
    constexpr int NB = MODE == CONV_PRELU ? COUT / 4 : 12;
    float r_bias[NB], r_slope[NB];
#pragma unroll
    for (int e = 0; e < NB; e++) {
      const int k = MODE == CONV_PRELU ? part * NB + e : 16 * (e / 4) + 4 * part + (e % 4);
      r_bias[e] = s_bias[k];
      r_slope[e] = s_slope[k];
    }
    const bool slope_unit = p.slope_unit != 0;
    int i = 0;
    for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, i++) {
      const int a = i & 1;
      const uint32_t acc_phase = (uint32_t)(i >> 1) & 1;
      if (!mbar_wait(&acc_full[a], acc_phase, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_FULL)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * CONV_ACC_COLS);
      // out(r, c) = Q_0(r, c - 1) + Q_1(r, c) + Q_2(r, c + 1): the left and
      // right partial sums come from the neighbouring lanes (a warp holds
      // one whole row of 32 positions).
      constexpr int NV = MODE == CONV_PRELU ? COUT / 4 : 12;
      float v[NV];
      if constexpr (MODE == CONV_PRELU) {
        // channels 16 part .. 16 part + 15
        static_assert(COUT == 64, "four parts of 16 channels");
        uint32_t q0[16], q1[16], q2[16];
        const uint32_t col = (uint32_t)(part * 16);
        tmem_ld16(taddr + col, q0);
        tmem_ld16(taddr + (uint32_t)COUT + col, q1);
        tmem_ld16(taddr + (uint32_t)(2 * COUT) + col, q2);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float2 left = make_float2(__shfl_up_sync(0xffffffffu, __uint_as_float(q0[e]), 1),
                                          __shfl_up_sync(0xffffffffu, __uint_as_float(q0[e + 1]), 1));
          const float2 right = make_float2(__shfl_down_sync(0xffffffffu, __uint_as_float(q2[e]), 1),
                                           __shfl_down_sync(0xffffffffu, __uint_as_float(q2[e + 1]), 1));
          const float2 sum =
              fadd2(fadd2(left, make_float2(__uint_as_float(q1[e]), __uint_as_float(q1[e + 1]))), right);
          v[e] = sum.x;
          v[e + 1] = sum.y;
        }
      } else {
        // output row i = part of the pixel shuffle needs channels
        // 16 c + 4 part .. + 3 of each colour c
        static_assert(COUT == 48, "three colours of 16 channels");
        uint32_t q0[12], q1[12], q2[12];
#pragma unroll
        for (int c = 0; c < 3; c++) {
          const uint32_t col = (uint32_t)(16 * c + 4 * part);
          tmem_ld4(taddr + col, q0 + 4 * c);
          tmem_ld4(taddr + (uint32_t)COUT + col, q1 + 4 * c);
          tmem_ld4(taddr + (uint32_t)(2 * COUT) + col, q2 + 4 * c);
        }
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 12; e++) {
          const float left = __shfl_up_sync(0xffffffffu, __uint_as_float(q0[e]), 1);
          const float right = __shfl_down_sync(0xffffffffu, __uint_as_float(q2[e]), 1);
          v[e] = (left + __uint_as_float(q1[e])) + right;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);

      const int row_id = (int)p.div_tiles_x.div((uint32_t)tile);
      const int tx = tile - row_id * p.tiles_x;
      const int img = (int)p.div_tiles_y.div((uint32_t)row_id), ty = row_id - img * p.tiles_y;
      const int y = ty * CONV_TILE_H + pr, x = tx * CONV_TILE_W + pc - 1;
      if (pc < 1 || pc > CONV_TILE_W || y >= p.H || x >= p.W) continue;

      if constexpr (MODE == CONV_PRELU) {
        const size_t plane = (size_t)p.MH * p.MW;
        __half* base = p.out + ((size_t)img * (COUT / 8) * plane + (size_t)y * p.MW + x) * 8;
#pragma unroll
        for (int g = 0; g < NV / 8; g++) {
          const int c0 = part * NV + g * 8;  // first channel of the group
          uint32_t packed[4];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const int k = g * 8 + 2 * e;
            const float2 w = fadd2(make_float2(v[k], v[k + 1]), make_float2(r_bias[k], r_bias[k + 1]));
            float v0, v1;
            if (slope_unit) {
              const float2 sw = fmul2(w, make_float2(r_slope[k], r_slope[k + 1]));
              v0 = fmaxf(w.x, sw.x);
              v1 = fmaxf(w.y, sw.y);
            } else {
              v0 = w.x < 0.0f ? w.x * r_slope[k] : w.x;
              v1 = w.y < 0.0f ? w.y * r_slope[k + 1] : w.y;
            }
            __half2 h = __floats2half2_rn(v0, v1);
            packed[e] = *reinterpret_cast<uint32_t*>(&h);
          }
          *reinterpret_cast<uint4*>(base + (size_t)(c0 / 8) * plane * 8) =
              make_uint4(packed[0], packed[1], packed[2], packed[3]);
        }
      } else {
        // Pixel shuffle x4 plus the input repeated (network.rs:118-140):
        // output pixel (4y + i, 4x + j) channel c = last[16c + 4i + j] + in[c].
        const ShuffleOut& so = p.shuffle;
        if (x < so.kx0 || x >= so.kx1 || y < so.ky0 || y >= so.ky1) continue;
        const int gy = so.ry0 + y, gx = so.rx0 + x;
        const size_t spix = ((size_t)img * so.src_h + gy) * so.src_w + gx;
        float in[3];
#pragma unroll
        for (int c = 0; c < 3; c++)
          in[c] = so.src_u8 ? (float)reinterpret_cast<const uint8_t*>(so.src)[spix * 3 + c] / 255.0f
                            : reinterpret_cast<const float*>(so.src)[spix * 3 + c];
        const size_t ow = (size_t)so.src_w * 4;
        {
          const int ii = part;
          float o[12];
#pragma unroll
          for (int j = 0; j < 4; j++)
#pragma unroll
            for (int c = 0; c < 3; c++) o[j * 3 + c] = (v[4 * c + j] + r_bias[4 * c + j]) + in[c];
          const size_t opix = ((size_t)img * so.src_h * 4 + (size_t)gy * 4 + ii) * ow + (size_t)gx * 4;
          if (so.dst_u8) {
            uint8_t* d = reinterpret_cast<uint8_t*>(so.dst) + opix * 3;
#pragma unroll
            for (int e = 0; e < 12; e++) d[e] = (uint8_t)roundf(fminf(fmaxf(o[e], 0.0f), 1.0f) * 255.0f);
          } else {
            float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(so.dst) + opix * 3);
            d[0] = make_float4(o[0], o[1], o[2], o[3]);
            d[1] = make_float4(o[4], o[5], o[6], o[7]);
            d[2] = make_float4(o[8], o[9], o[10], o[11]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, CONV_TMEM_COLS);
  }
}

}  // namespace iec
