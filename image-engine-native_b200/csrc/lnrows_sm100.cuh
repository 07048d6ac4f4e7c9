// LayerNorm and the shifted-window partition folded into the staged A
// operand of one tcgen05 product, on sm_100a:
//
//   out[r] = LayerNorm(map[pixel(r)]) x W + b
//
// the window attention's first product (crates/scunet-native/src/swin.rs:
// 124-181: LN1, the partition into 8 x 8 windows shifted by 4, and the qkv
// layer; crates/birefnet-native/src/swin.rs:219-251 with 7 x 7 windows in
// 64-row slots, whose padding rows and tokens past the map are zero rows,
// not normalised). Row r of the output is token r % 64 of window r / 64 in
// the order layer_norm_planar's window mode writes (gemm.h WindowMap).
// Per tile of 128 output rows:
//   * two groups of four loader warps (each group every other tile), one
//     row per thread, gather the row's C channels
//     (16-byte pixel groups of the planar map; consecutive tokens of a window
//     row are consecutive pixels), take its mean and mean squared deviation,
//     and write the normalised f16 row into one of two shared-memory A tiles
//     in the K-major core-matrix layout [C / 8][128][8]; fence.proxy.async;
//   * one thread issues the MMAs (M 128 x N x K C; N above 256 as two halves)
//     into one of two TMEM accumulators (one when 2 N exceeds 512 columns),
//     the weights resident in shared memory for the whole launch;
//   * eight epilogue warps add the bias and store the f16 rows, planar
//     [N / 8][rows][8], while the next tile is gathered and multiplied.
// Every wait is bounded (sm100.cuh).
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "gemm.h"
#include "igemm_sm100.cuh"
#include "sm100.cuh"

namespace iec {

struct LnRowsParams {
  int rows;                // output rows (windows x 64)
  int tiles;               // ceil(rows / 128)
  const __half* src;       // the map's first channel plane, planar [C / 8][pixels][8]
  long long src_plane;     // elements per plane
  WindowMap wm;
  const uint8_t* w;        // [C / 8][N][8] f16: the B operand's core-matrix image
  const float* params;     // gamma [C], beta [C], bias [N]
  __half* out;             // planar [N / 8][rows][8]
  long long out_plane;
  int* dev_err;
};

template <int C, int N>
struct LnRowsSmem {
  // Eight loader warps in two groups of four (one row per thread), each
  // group owning every other tile and one of the two A tiles, so that two
  // tiles' gathers and LayerNorms are in flight; eight epilogue warps.
  static constexpr int LOADERS = 8, GROUP = 4, EPI = 8, THREADS = 32 * (2 + LOADERS + EPI);
  static constexpr int ACCS = 2 * N <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = ACCS * N <= 256 ? 256 : 512;
  static constexpr int NSPLIT = N > 256 ? 2 : 1, NPART = N / NSPLIT;
  static constexpr int A_BYTES = (C / 8) * 128 * 16;
  static constexpr int W_BYTES = (C / 8) * N * 16;
  static constexpr int W_OFF = 2 * A_BYTES;
  static constexpr int PAR_FLOATS = 2 * C + N;
  static constexpr int PAR_OFF = W_OFF + W_BYTES;
  static constexpr int BAR_OFF = PAR_OFF + PAR_FLOATS * 4;
  static constexpr int TOTAL = BAR_OFF + 16 * 8 + 16;
  static_assert(C % 16 == 0 && N % 48 == 0 && NPART % 16 == 0 && NPART <= 256, "product shape");
  static_assert(TOTAL <= 227 * 1024, "shared memory");
};

enum : int { LB_W = 0, LB_A_FULL = 1, LB_A_EMPTY = 3, LB_ACC_FULL = 5, LB_ACC_EMPTY = 7, LB_COUNT = 9 };

template <int C, int N>
__global__ void __launch_bounds__(LnRowsSmem<C, N>::THREADS, 1)
    lnrows_sm100(const LnRowsParams p) {
  using L = LnRowsSmem<C, N>;
  extern __shared__ __align__(128) uint8_t ln_smem[];
  uint8_t* A = ln_smem;
  uint8_t* Wm = ln_smem + L::W_OFF;
  float* par = reinterpret_cast<float*>(ln_smem + L::PAR_OFF);
  const float* gamma = par;
  const float* beta = par + C;
  const float* bias = par + 2 * C;
  uint64_t* bar = reinterpret_cast<uint64_t*>(ln_smem + L::BAR_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ln_smem + L::BAR_OFF + 16 * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(ln_smem + L::BAR_OFF + 16 * 8 + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bar[LB_W], 1);
    for (int b = 0; b < 2; b++) {
      mbar_init(&bar[LB_A_FULL + b], L::GROUP);
      mbar_init(&bar[LB_A_EMPTY + b], 1);
      mbar_init(&bar[LB_ACC_FULL + b], 1);
      mbar_init(&bar[LB_ACC_EMPTY + b], L::EPI);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  for (int i = (int)threadIdx.x; i < L::PAR_FLOATS; i += L::THREADS) par[i] = p.params[i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // The weights do not depend on the previous kernel: fetched before the wait.
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bar[LB_W], (uint32_t)L::W_BYTES);
    bulk_load(Wm, p.w, (uint32_t)L::W_BYTES, &bar[LB_W]);
  }
  griddep_launch_dependents();
  griddep_wait();

  if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = idesc_f16_f32(128, L::NPART);
      const uint32_t aa = smem_u32(A), wa = smem_u32(Wm);
      bool ok = mbar_wait(&bar[LB_W], 0, abort_flag, p.dev_err, DEV_ERR_WAIT_WEIGHTS);
      int i = 0, last = -1;
      for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, i++) {
        const int b = i & 1, a = i % L::ACCS;
        const uint32_t ph = (uint32_t)(i >> 1) & 1, aph = (uint32_t)(i / L::ACCS) & 1;
        if (!mbar_wait(&bar[LB_A_FULL + b], ph, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL)) break;
        if (!mbar_wait(&bar[LB_ACC_EMPTY + a], aph ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_EMPTY)) break;
        tc_fence_after();
        const uint32_t ab = aa + (uint32_t)(b * L::A_BYTES);
#pragma unroll
        for (int k = 0; k < C / 16; k++)
#pragma unroll
          for (int s = 0; s < L::NSPLIT; s++) {
            const uint64_t ad = smem_desc(ab + (uint32_t)(2 * k * 128 * 16), 128 * 16, 128);
            const uint64_t bd = smem_desc(wa + (uint32_t)(2 * k * N * 16 + s * L::NPART * 16), N * 16, 128);
            umma_f16(tmem + (uint32_t)(a * N + s * L::NPART), ad, bd, idesc, k > 0 ? 1u : 0u);
          }
        umma_commit(&bar[LB_A_EMPTY + b]);
        umma_commit(&bar[LB_ACC_FULL + a]);
        last = i;
      }
      if (last >= 0)
        mbar_wait(&bar[LB_ACC_FULL + last % L::ACCS], (uint32_t)(last / L::ACCS) & 1, abort_flag, p.dev_err, 0);
    }
  } else if (warp >= 2 && warp < 2 + L::LOADERS) {
    // ------------------------------------------------ gather + LayerNorm
    const int group = (warp - 2) / L::GROUP;            // tiles i = group, group + 2, ...
    const int row = ((warp - 2) % L::GROUP) * 32 + lane;  // row of the tile
    const WindowMap wm = p.wm;
    const int cols = wm.pad_w / wm.ws;
    // The token row `row` of a tile holds (layer_norm_rows' window order):
    // whether it is a zero row, and its pixel.
    auto locate = [&](int tile, bool& zero, long long& pix) {
      const int r = tile * 128 + row;
      const int win = r >> 6, t = r & 63;
      const int wy = win / cols, wx = win - wy * cols;
      const int y = (wy * wm.ws + t / wm.ws + wm.shift) % wm.pad_h, x = (wx * wm.ws + t % wm.ws + wm.shift) % wm.pad_w;
      zero = r >= p.rows || t >= wm.ws * wm.ws || y >= wm.map_h || x >= wm.map_w;
      pix = zero ? 0 : (long long)y * wm.map_w + x;
    };
    // Narrow rows stay in registers across the three passes, and the next
    // tile's row is loaded before this one is normalised; wide ones are read
    // again (L1 hits) in each pass, the next tile's row prefetched towards
    // L1, which keeps the loaders unspilled. Either way the row's global
    // latency overlaps the previous tile's work.
    constexpr bool HOLD = C <= 32;
    uint4 v[HOLD ? C / 8 : 1], vn[HOLD ? C / 8 : 1];
    auto fetch = [&](bool z, long long px, uint4* dst) {
#pragma unroll
      for (int g = 0; g < C / 8; g++) {
        const __half* at = p.src + (long long)g * p.src_plane + px * 8;
        if constexpr (HOLD)
          dst[g] = z ? make_uint4(0u, 0u, 0u, 0u) : *reinterpret_cast<const uint4*>(at);
        else if (!z)
          prefetch_l1(at);
      }
    };
    bool zero = true;
    long long pix = 0;
    const int first = (int)blockIdx.x + group * (int)gridDim.x, step = 2 * (int)gridDim.x;
    if (first < p.tiles) {
      locate(first, zero, pix);
      fetch(zero, pix, v);
    }
    // the CTA's tile sequence i = group, group + 2, ...: A tile b = group
    for (int tile = first, i = group; tile < p.tiles; tile += step, i += 2) {
      const int b = i & 1;
      const uint32_t ph = (uint32_t)(i >> 1) & 1;
      bool zero_n = true;
      long long pix_n = 0;
      if (tile + step < p.tiles) {
        locate(tile + step, zero_n, pix_n);
        fetch(zero_n, pix_n, vn);
      }
      if (!mbar_wait(&bar[LB_A_EMPTY + b], ph ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_EMPTY)) break;
      auto group = [&](int g) -> uint4 {
        if (zero) return make_uint4(0u, 0u, 0u, 0u);
        if constexpr (HOLD) return v[g];
        return *reinterpret_cast<const uint4*>(p.src + (long long)g * p.src_plane + pix * 8);
      };
      float sum = 0.0f;
#pragma unroll
      for (int g = 0; g < C / 8; g++) {
        const uint4 u = group(g);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float2 f = __half22float2(h[e]);
          sum += f.x + f.y;
        }
      }
      const float mean = sum / (float)C;
      float var = 0.0f;
#pragma unroll
      for (int g = 0; g < C / 8; g++) {
        const uint4 u = group(g);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float2 f = __half22float2(h[e]);
          var += (f.x - mean) * (f.x - mean) + (f.y - mean) * (f.y - mean);
        }
      }
      const float inv = 1.0f / sqrtf(var / (float)C + 1e-5f);
      uint8_t* ab = A + b * L::A_BYTES;
#pragma unroll
      for (int g = 0; g < C / 8; g++) {
        float o[8];
        const uint4 u = group(g);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float2 f = __half22float2(h[e]);
          o[2 * e] = zero ? 0.0f : (f.x - mean) * inv * gamma[8 * g + 2 * e] + beta[8 * g + 2 * e];
          o[2 * e + 1] = zero ? 0.0f : (f.y - mean) * inv * gamma[8 * g + 2 * e + 1] + beta[8 * g + 2 * e + 1];
        }
        *reinterpret_cast<uint4*>(ab + (g * 128 + row) * 16) = pack_half8(o);
      }
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[LB_A_FULL + b]);
      zero = zero_n;
      pix = pix_n;
      if constexpr (HOLD) {
#pragma unroll
        for (int g = 0; g < C / 8; g++) v[g] = vn[g];
      }
    }
  } else if (warp >= 2 + L::LOADERS) {
    // ------------------------------------------------------------- epilogue
    const int e = warp - 2 - L::LOADERS;  // 0 .. EPI - 1
    const int quarter = warp & 3, part = e >> 2;  // EPI / 4 column parts per lane quarter
    const int row = quarter * 32 + lane;
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    constexpr int COLS = N / (L::EPI / 4);
    static_assert(COLS % 16 == 0, "epilogue columns");
    int i = 0;
    for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, i++) {
      const int a = i % L::ACCS;
      const uint32_t aph = (uint32_t)(i / L::ACCS) & 1;
      if (!mbar_wait(&bar[LB_ACC_FULL + a], aph, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_FULL)) break;
      tc_fence_after();
      const int r = tile * 128 + row;
#pragma unroll 1
      for (int c0 = part * COLS; c0 < (part + 1) * COLS; c0 += 16) {
        uint32_t acc[16];
        tmem_ld16(tmem + lanes + (uint32_t)(a * N + c0), acc);
        tmem_wait_ld();
        if (r >= p.rows) continue;
#pragma unroll
        for (int q = 0; q < 2; q++) {
          float o[8];
#pragma unroll
          for (int k = 0; k < 8; k++) o[k] = __uint_as_float(acc[8 * q + k]) + bias[c0 + 8 * q + k];
          *reinterpret_cast<uint4*>(p.out + (long long)((c0 + 8 * q) / 8) * p.out_plane + (long long)r * 8) =
              pack_half8(o);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[LB_ACC_EMPTY + a]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, L::TMEM_COLS);
  // (the weight copy landed: the MMA issuer waited for it, or every role
  // gave up after the bounded wait)
}

}  // namespace iec
