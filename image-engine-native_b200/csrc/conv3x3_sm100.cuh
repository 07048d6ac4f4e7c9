// Implicit-GEMM 3x3 convolution (stride 1, zero padding) on sm_100a tensor
// cores: f16 inputs, f32 accumulators in TMEM, fused epilogues.
//
// Semantics: crates/native-engine/src/gemm.rs:514-667 (multiply over
// Taps::Conv { size: 3, step: 1, pad: Zero }) with the epilogue of
// crates/realesrgan-native/src/network.rs:31-41,80-112 (bias, PReLU) or
// network.rs:118-140 (pixel shuffle x4 plus the input repeated).
//
// Layout. Feature maps are f16 and "channel-group planar": [image][cin / 8]
// [height][width][8]. One tile is 16 rows x 8 columns of output pixels (the
// M = 128 rows of one UMMA). A single 5-D TMA box brings the tile's 18 x 10
// pixel halo of every channel group into shared memory as [group][18][10][8],
// which is exactly the no-swizzle K-major core-matrix layout tcgen05 reads:
// 8 consecutive pixels of a halo row are one 8 x 16-byte core matrix, the
// next tile row is 160 bytes on (SBO), the next channel group 2880 bytes on
// (LBO). Each of the 9 taps is therefore just a start-address offset of
// (ky * 10 + kx) * 16 bytes into the same halo: no im2col, one TMA load per
// tile, out-of-image pixels zero-filled by TMA itself.
//
// The weights of the layer, pre-arranged on the host as [tap][cin / 8][cout]
// [8] (the K-major core-matrix image of B), stay in shared memory for the
// whole persistent kernel (72 KB for 64 -> 64).
//
// Roles (192 threads): warp 0 one thread issues TMA loads into a ring of
// NSTAGE halo stages; warp 1 one thread issues 9 * cin / 16 UMMAs
// (M 128, N cout, K 16) per tile into one of two TMEM accumulators; warps
// 2..5 (one per TMEM lane quarter) drain an accumulator while the next
// tile's MMAs run, apply the epilogue and store.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "sm100.cuh"

namespace iec {

constexpr int CONV_TILE_H = 16;
constexpr int CONV_TILE_W = 8;
constexpr int CONV_HALO_H = CONV_TILE_H + 2;
constexpr int CONV_HALO_W = CONV_TILE_W + 2;
constexpr int CONV_CHUNK_BYTES = CONV_HALO_H * CONV_HALO_W * 16;  // 2880
constexpr int CONV_NSTAGE = 4;
constexpr int CONV_THREADS = 192;
constexpr int CONV_TMEM_COLS = 128;  // two accumulators of up to 64 columns

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
  int tiles_x, tiles_y, tiles;  // tile grid over all images
  const uint16_t* weights;     // [9][cin / 8][cout][8] f16
  const float* bias;           // [cout]
  const float* slope;          // [cout] PReLU slopes, or null
  __half* out;                 // CONV_PRELU: [image][cout / 8][H][W][8]
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

  if (threadIdx.x == 0) {
    for (int s = 0; s < CONV_NSTAGE; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
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
  const int tiles_per_img = p.tiles_x * p.tiles_y;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      prefetch_tensor_map(&in_map);
      mbar_arrive_expect_tx(wbar, L::W_BYTES);
      for (int off = 0; off < L::W_BYTES; off += 32768) {
        int bytes = L::W_BYTES - off < 32768 ? L::W_BYTES - off : 32768;
        bulk_load(w_smem + off, reinterpret_cast<const uint8_t*>(p.weights) + off, bytes, wbar);
      }
      int s = 0;
      uint32_t phase = 0;
      int issued[CONV_NSTAGE];  // parity of the last load into each stage, -1 none
      for (int i = 0; i < CONV_NSTAGE; i++) issued[i] = -1;
      for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x) {
        if (!mbar_wait(&empty[s], phase ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_EMPTY)) break;
        const int img = tile / tiles_per_img;
        const int rem = tile - img * tiles_per_img;
        const int ty = rem / p.tiles_x, tx = rem - ty * p.tiles_x;
        mbar_arrive_expect_tx(&full[s], KCH * CONV_CHUNK_BYTES);
        tma_load_5d(a_smem + s * L::STAGE_BYTES, &in_map, &full[s], 0, tx * CONV_TILE_W - 1,
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
      constexpr uint32_t idesc = idesc_f16_f32(128, COUT);
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
          const uint32_t d = tmem_base + (uint32_t)(a * 64);
          const uint32_t abase = abase0 + (uint32_t)(s * L::STAGE_BYTES);
#pragma unroll
          for (int tap = 0; tap < 9; tap++) {
            const uint32_t off = (uint32_t)(((tap / 3) * CONV_HALO_W + (tap % 3)) * 16);
#pragma unroll
            for (int ks = 0; ks < KCH / 2; ks++) {
              const uint64_t adesc =
                  smem_desc(abase + (uint32_t)(2 * ks * CONV_CHUNK_BYTES) + off, CONV_CHUNK_BYTES, CONV_HALO_W * 16);
              const uint64_t bdesc =
                  smem_desc(wbase + (uint32_t)((tap * KCH + 2 * ks) * COUT * 16), COUT * 16, 128);
              umma_f16(d, adesc, bdesc, idesc, (tap | ks) != 0);
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
    const int row = quarter * 32 + lane;     // M row = pixel of the tile
    const int my = row >> 3, mx = row & 7;
    int i = 0;
    for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, i++) {
      const int a = i & 1;
      const uint32_t acc_phase = (uint32_t)(i >> 1) & 1;
      if (!mbar_wait(&acc_full[a], acc_phase, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_FULL)) break;
      tc_fence_after();
      uint32_t v[COUT];
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * 64);
#pragma unroll
      for (int c = 0; c < COUT; c += 16) tmem_ld16(taddr + (uint32_t)c, v + c);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);

      const int img = tile / tiles_per_img;
      const int rem = tile - img * tiles_per_img;
      const int ty = rem / p.tiles_x, tx = rem - ty * p.tiles_x;
      const int y = ty * CONV_TILE_H + my, x = tx * CONV_TILE_W + mx;
      if (y >= p.H || x >= p.W) continue;

      if constexpr (MODE == CONV_PRELU) {
        const size_t plane = (size_t)p.MH * p.MW;
        __half* base = p.out + ((size_t)img * (COUT / 8) * plane + (size_t)y * p.MW + x) * 8;
#pragma unroll
        for (int g = 0; g < COUT / 8; g++) {
          uint32_t packed[4];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const int c = g * 8 + 2 * e;
            float v0 = __uint_as_float(v[c]) + s_bias[c];
            float v1 = __uint_as_float(v[c + 1]) + s_bias[c + 1];
            v0 = v0 < 0.0f ? v0 * s_slope[c] : v0;
            v1 = v1 < 0.0f ? v1 * s_slope[c + 1] : v1;
            __half2 h = __floats2half2_rn(v0, v1);
            packed[e] = *reinterpret_cast<uint32_t*>(&h);
          }
          *reinterpret_cast<uint4*>(base + (size_t)g * plane * 8) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
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
#pragma unroll
        for (int ii = 0; ii < 4; ii++) {
          float o[12];
#pragma unroll
          for (int j = 0; j < 4; j++)
#pragma unroll
            for (int c = 0; c < 3; c++) {
              const int k = 16 * c + 4 * ii + j;
              o[j * 3 + c] = (__uint_as_float(v[k]) + s_bias[k]) + in[c];
            }
          const size_t opix = ((size_t)img * so.src_h * 4 + (size_t)gy * 4 + ii) * ow + (size_t)gx * 4;
          if (so.dst_u8) {
            uint8_t b[12];
#pragma unroll
            for (int e = 0; e < 12; e++) b[e] = (uint8_t)roundf(fminf(fmaxf(o[e], 0.0f), 1.0f) * 255.0f);
            uint8_t* d = reinterpret_cast<uint8_t*>(so.dst) + opix * 3;
#pragma unroll
            for (int e = 0; e < 12; e++) d[e] = b[e];
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
