// The transformer MLP of SCUNet and BiRefNet as one sm_100a kernel:
//
//   x += fc2(GELU(fc1(LayerNorm(x))))
//
// (crates/scunet-native/src/swin.rs:222-254, crates/birefnet-native/src/
// swin.rs:308-346) over planar f16 rows [C / 8][rows][8], C channels, hidden
// width 4 C. Per tile of 128 rows:
//   * the tile arrives by TMA in the K-major core-matrix layout
//     [C / 8][128][8] (the A_ROWS box of igemm_sm100.cuh);
//   * LayerNorm (eps 1e-5, two passes: mean, then the mean square deviation)
//     normalises it in place in shared memory: the epilogue warps (16, or 8
//     for 32 and 64 channels), four or two per TMEM lane quarter; each thread
//     takes its row's statistics over all channels and
//     normalises a quarter of the row's channel groups once the four warps
//     of its quarter have read the row; then fence.proxy.async, so that the
//     tensor core reads the normalised tile;
//   * the hidden layer in chunks of NH columns: fc1 (M 128 x N NH x K C) into
//     one of two TMEM accumulators, bias and GELU (the erf form of
//     igemm_sm100.cuh) by the epilogue warps into one of two f16 shared-memory
//     tiles [NH / 8][128][8], fc2 (M 128 x N C x K NH) accumulated into a
//     third TMEM accumulator; the MMA issuer runs fc1 of chunk j + 1 before
//     fc2 of chunk j, so the tensor core works while GELU runs;
//   * the final epilogue adds fc2's bias and the tile's old rows (read back
//     from global memory) and stores the f16 result over them.
// The weights stream through a ring of two stages, one chunk (W1 columns and
// W2 rows of NH hidden units) per stage. The hidden layer never leaves the
// SM. Every wait is bounded as in the other kernels (sm100.cuh): on expiry
// the kernel sets the device error word and every role leaves its loop.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "igemm_sm100.cuh"
#include "sm100.cuh"

namespace iec {


struct MlpParams {
  int M;                  // rows
  int tiles;              // ceil(M / 128)
  __half* x;              // planar [C / 8][rows][8], plane stride plane_elems (halves)
  long long plane_elems;
  const uint8_t* w;       // per chunk: W1 [C / 8][NH][8] f16, then W2 [NH / 8][C][8] f16
  const float* params;    // gamma [C], beta [C], b1 [4 C], b2 [C]
  int* dev_err;
};

// Hidden columns per chunk: 64, or 32 where shared memory is short.
__host__ __device__ constexpr int mlp_nh(int c) { return c <= 192 ? 64 : 32; }

template <int C>
struct MlpSmem {
  // Narrow MLPs take 8 epilogue warps and half of TMEM, so that two CTAs
  // share an SM and hide each other's hand-offs; wider ones take 16 warps.
  static constexpr int EW = C <= 64 ? 8 : 16, PARTS = EW / 4, THREADS = 64 + 32 * EW, CTAS = EW == 8 ? 2 : 1;
  static constexpr int TMEM_COLS = C <= 64 ? 256 : 512;
  static constexpr int NH = mlp_nh(C);
  static constexpr int HID = 4 * C, CHUNKS = HID / NH;
  static constexpr int X_BYTES = (C / 8) * 128 * 16;
  static constexpr int W1_BYTES = (C / 8) * NH * 16, W2_BYTES = (NH / 8) * C * 16;
  static constexpr int STAGE = W1_BYTES + W2_BYTES;
  static constexpr int H_BYTES = (NH / 8) * 128 * 16;
  static constexpr int PAR_FLOATS = 3 * C + HID;
  static constexpr int NBAR = 24;
  // Shared memory per CTA (two CTAs per SM share 228 KB). The weights stay
  // resident (every chunk loaded once per CTA) where they fit beside two
  // row tiles; else they stream through a ring of two chunks. The row tile
  // is double-buffered where that fits, so the next tile's rows land while
  // this one is in the hidden layer.
  static constexpr int BUDGET = (CTAS == 2 ? 112 : 224) * 1024;
  static constexpr int FIXED = 2 * H_BYTES + PAR_FLOATS * 4 + NBAR * 8 + 16;
  static constexpr bool RES = CHUNKS * STAGE + 2 * X_BYTES + FIXED <= BUDGET;
  static constexpr int WS = RES ? CHUNKS : 2;  // weight stages
  static constexpr int XB = WS * STAGE + 2 * X_BYTES + FIXED <= BUDGET ? 2 : 1;
  static constexpr int W_OFF = XB * X_BYTES;
  static constexpr int H_OFF = W_OFF + WS * STAGE;
  static constexpr int PAR_OFF = H_OFF + 2 * H_BYTES;
  static constexpr int BAR_OFF = PAR_OFF + PAR_FLOATS * 4;
  static constexpr int TOTAL = BAR_OFF + NBAR * 8 + 16;
  // TMEM: fc2's accumulator at column 0 (C columns), fc1's two at D1 and D1 + NH.
  static constexpr int D1 = C <= 64 ? 64 : C <= 256 ? 256 : 384;
  static constexpr int N2_SPLIT = C > 256 ? 2 : 1, N2 = C / N2_SPLIT;  // fc2's MMA width
  static_assert(C % 32 == 0 && C <= 384, "MLP width");
  static_assert(TOTAL <= 227 * 1024 && (CTAS == 1 || TOTAL <= 113 * 1024), "MLP shared memory");
  static_assert(D1 + 2 * NH <= TMEM_COLS, "MLP tensor memory");
};

// Barrier slots.
enum : int {
  MB_X_FULL = 0, MB_X_READY = 2, MB_X_EMPTY = 4,  // per row-tile buffer
  MB_W_FULL = 6, MB_W_EMPTY = MB_W_FULL + 2, MB_D1_FULL = MB_W_EMPTY + 2,
  MB_H_FULL = MB_D1_FULL + 2, MB_H_EMPTY = MB_H_FULL + 2, MB_D2_FULL = MB_H_EMPTY + 2, MB_D2_EMPTY,
  MB_LN_READ,  // four: the warps of one lane quarter have read their rows
  MB_COUNT = MB_LN_READ + 4
};

template <int C>
__global__ void __launch_bounds__(MlpSmem<C>::THREADS, MlpSmem<C>::CTAS)
    mlp_sm100(const __grid_constant__ CUtensorMap x_map, const MlpParams p) {
  using L = MlpSmem<C>;
  constexpr int NH = L::NH, CHUNKS = L::CHUNKS;
  static_assert(MB_COUNT <= L::NBAR, "barrier slots");
  extern __shared__ __align__(128) uint8_t mlp_smem[];
  uint8_t* X = mlp_smem;
  uint8_t* Wst = mlp_smem + L::W_OFF;
  uint8_t* Hb = mlp_smem + L::H_OFF;
  float* par = reinterpret_cast<float*>(mlp_smem + L::PAR_OFF);
  const float* gamma = par;
  const float* beta = par + C;
  const float* b1 = par + 2 * C;
  const float* b2 = par + 2 * C + L::HID;
  uint64_t* bar = reinterpret_cast<uint64_t*>(mlp_smem + L::BAR_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mlp_smem + L::BAR_OFF + L::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(mlp_smem + L::BAR_OFF + L::NBAR * 8 + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bar[MB_D2_FULL], 1);
    mbar_init(&bar[MB_D2_EMPTY], L::EW);
    for (int b = 0; b < 2; b++) {
      mbar_init(&bar[MB_X_FULL + b], 1);
      mbar_init(&bar[MB_X_READY + b], L::EW);
      mbar_init(&bar[MB_X_EMPTY + b], 1);
      mbar_init(&bar[MB_W_FULL + b], 1);
      mbar_init(&bar[MB_W_EMPTY + b], 1);
      mbar_init(&bar[MB_D1_FULL + b], 1);
      mbar_init(&bar[MB_H_FULL + b], L::EW);
      mbar_init(&bar[MB_H_EMPTY + b], 1);
    }
    for (int q = 0; q < 4; q++) mbar_init(&bar[MB_LN_READ + q], L::PARTS);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  // The LayerNorm and bias parameters are weights: staged before waiting for
  // the previous kernel.
  for (int i = (int)threadIdx.x; i < L::PAR_FLOATS; i += L::THREADS) par[i] = p.params[i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Resident weights do not depend on the previous kernel: every chunk
  // once, on the first weight barrier, before the wait.
  if (L::RES && threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bar[MB_W_FULL], (uint32_t)(CHUNKS * L::STAGE));
    for (int j = 0; j < CHUNKS; j++)
      bulk_load(Wst + j * L::STAGE, p.w + (size_t)j * L::STAGE, (uint32_t)L::STAGE, &bar[MB_W_FULL]);
  }
  griddep_launch_dependents();
  griddep_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      prefetch_tensor_map(&x_map);
      bool ok = true;
      int i = 0;
      for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, i++) {
        const int xb = i % L::XB;
        const uint32_t xph = (uint32_t)(i / L::XB) & 1;
        if (!mbar_wait(&bar[MB_X_EMPTY + xb], xph ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(&bar[MB_X_FULL + xb], (uint32_t)L::X_BYTES);
        tma_load_3d(X + xb * L::X_BYTES, &x_map, &bar[MB_X_FULL + xb], 0, tile * 8, 0);
        for (int j = 0; j < CHUNKS && !L::RES; j++) {
          const int c = i * CHUNKS + j, b = c & 1;
          const uint32_t ph = (uint32_t)(c >> 1) & 1;
          if (!mbar_wait(&bar[MB_W_EMPTY + b], ph ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_WEIGHTS)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bar[MB_W_FULL + b], (uint32_t)L::STAGE);
          bulk_load(Wst + b * L::STAGE, p.w + (size_t)j * L::STAGE, (uint32_t)L::STAGE, &bar[MB_W_FULL + b]);
        }
      }
      // let the copies in flight land before the CTA may leave
      const int n = L::RES ? 0 : i * CHUNKS;
      for (int t = i - L::XB; t < i; t++)
        if (t >= 0) mbar_wait(&bar[MB_X_FULL + t % L::XB], (uint32_t)(t / L::XB) & 1, abort_flag, p.dev_err, 0);
      if (L::RES) mbar_wait(&bar[MB_W_FULL], 0, abort_flag, p.dev_err, 0);
      for (int c = n - 2; c < n; c++)
        if (c >= 0) mbar_wait(&bar[MB_W_FULL + (c & 1)], (uint32_t)(c >> 1) & 1, abort_flag, p.dev_err, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc1 = idesc_f16_f32(128, NH);
      constexpr uint32_t idesc2 = idesc_f16_f32(128, L::N2);
      const uint32_t xa0 = smem_u32(X), wa = smem_u32(Wst), ha = smem_u32(Hb);
      bool ok = true;
      int i = 0;
      // fc2 of chunk c (global chunk count), accumulating over the tile's chunks
      auto fc2 = [&](int c, int j, int tile_i) -> bool {
        const int b = c & 1;
        const uint32_t ph = (uint32_t)(c >> 1) & 1;
        if (!mbar_wait(&bar[MB_H_FULL + b], ph, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_FULL)) return false;
        if (j == 0 && !mbar_wait(&bar[MB_D2_EMPTY], (uint32_t)(tile_i & 1) ^ 1, abort_flag, p.dev_err,
                                 DEV_ERR_WAIT_ACC_EMPTY))
          return false;
        tc_fence_after();
        const uint32_t hb = ha + (uint32_t)(b * L::H_BYTES);
        const uint32_t w2 = wa + (uint32_t)((L::RES ? j : b) * L::STAGE + L::W1_BYTES);
#pragma unroll
        for (int k = 0; k < NH / 16; k++)
#pragma unroll
          for (int s = 0; s < L::N2_SPLIT; s++) {
            const uint64_t ad = smem_desc(hb + (uint32_t)(2 * k * 128 * 16), 128 * 16, 128);
            const uint64_t bd = smem_desc(w2 + (uint32_t)(2 * k * C * 16 + s * L::N2 * 16), C * 16, 128);
            umma_f16(tmem + (uint32_t)(s * L::N2), ad, bd, idesc2, (j > 0 || k > 0) ? 1u : 0u);
          }
        umma_commit(&bar[MB_H_EMPTY + b]);
        if (!L::RES) umma_commit(&bar[MB_W_EMPTY + b]);
        return true;
      };
      if (L::RES) {
        ok = mbar_wait(&bar[MB_W_FULL], 0, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL);
        tc_fence_after();
      }
      for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, i++) {
        const int xb = i % L::XB;
        if (!mbar_wait(&bar[MB_X_READY + xb], (uint32_t)(i / L::XB) & 1, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL))
          break;
        tc_fence_after();
        const uint32_t xa = xa0 + (uint32_t)(xb * L::X_BYTES);
        for (int j = 0; j < CHUNKS && ok; j++) {
          const int c = i * CHUNKS + j, b = c & 1;
          const uint32_t ph = (uint32_t)(c >> 1) & 1;
          if (!L::RES) {
            if (!mbar_wait(&bar[MB_W_FULL + b], ph, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          // fc1 of chunk c: D1[b] = X (128 x C) x W1 chunk (C x NH). D1[b]
          // was last read by the epilogue of chunk c - 2, whose h_full this
          // thread waited for before issuing fc2 of c - 2.
          const uint32_t w1 = wa + (uint32_t)((L::RES ? j : b) * L::STAGE);
#pragma unroll
          for (int k = 0; k < C / 16; k++) {
            const uint64_t ad = smem_desc(xa + (uint32_t)(2 * k * 128 * 16), 128 * 16, 128);
            const uint64_t bd = smem_desc(w1 + (uint32_t)(2 * k * NH * 16), NH * 16, 128);
            umma_f16(tmem + (uint32_t)(L::D1 + b * NH), ad, bd, idesc1, k > 0 ? 1u : 0u);
          }
          umma_commit(&bar[MB_D1_FULL + b]);
          if (j == CHUNKS - 1) umma_commit(&bar[MB_X_EMPTY + xb]);  // every fc1 of the tile has read X
          if (j > 0 && !fc2(c - 1, j - 1, i)) ok = false;
        }
        if (!ok) break;
        if (!fc2(i * CHUNKS + CHUNKS - 1, CHUNKS - 1, i)) break;
        umma_commit(&bar[MB_D2_FULL]);
      }
      if (i > 0 && ok) mbar_wait(&bar[MB_D2_FULL], (uint32_t)((i - 1) & 1), abort_flag, p.dev_err, 0);
    }
  } else {
    // -------------------------------------------- LayerNorm, GELU, epilogue
    // Warp w serves TMEM lane quarter w % 4 (rows 32 q .. 32 q + 31, one row
    // per lane) and part (w - 2) / 4 of the columns.
    const int quarter = warp & 3, part = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    constexpr int G = C / 8 / L::PARTS;  // channel groups this part normalises (part, part + PARTS, ...)
    // LayerNorm of tile `tile` (the CTA's i-th) in place, then X_READY; false
    // when a bounded wait gave up.
    auto layer_norm = [&](int tile, int i) -> bool {
        const int xb = i % L::XB;
        uint8_t* Xt = X + xb * L::X_BYTES;
        if (!mbar_wait(&bar[MB_X_FULL + xb], (uint32_t)(i / L::XB) & 1, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL))
          return false;
        // LayerNorm of the row in place (gemm.cu layer_norm_rows' formula:
        // mean, the mean squared deviation, (v - mean) / sqrt(var + 1e-5)).
        // Every part computes its row's statistics over all C channels itself
        // (no exchange between warps, so no barrier an aborted warp could
        // leave waiting), then normalises its own groups.
        float sum = 0.0f;
#pragma unroll 4
        for (int g = 0; g < C / 8; g++) {
          const uint4 u = *reinterpret_cast<const uint4*>(Xt + (g * 128 + row) * 16);
          const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const float2 f = __half22float2(h[e]);
            sum += f.x + f.y;
          }
        }
        const float mean = sum / (float)C;
        float var = 0.0f;
#pragma unroll 4
        for (int g = 0; g < C / 8; g++) {
          const uint4 u = *reinterpret_cast<const uint4*>(Xt + (g * 128 + row) * 16);
          const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const float2 f = __half22float2(h[e]);
            var += (f.x - mean) * (f.x - mean) + (f.y - mean) * (f.y - mean);
          }
        }
        // every part has read the whole row before any part overwrites its
        // groups: the four warps of a quarter meet on an mbarrier (bounded)
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[MB_LN_READ + quarter]);
        if (!mbar_wait(&bar[MB_LN_READ + quarter], (uint32_t)(i & 1), abort_flag, p.dev_err, DEV_ERR_WAIT_FULL)) return false;
        const float inv = 1.0f / sqrtf(var / (float)C + 1e-5f);
#pragma unroll
        for (int k = 0; k < G; k++) {
          const int g = part + L::PARTS * k;
          uint4* at = reinterpret_cast<uint4*>(Xt + (g * 128 + row) * 16);
          const uint4 u = *at;
          const __half2* h = reinterpret_cast<const __half2*>(&u);
          float v[8];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const float2 f = __half22float2(h[e]);
            v[2 * e] = (f.x - mean) * inv * gamma[8 * g + 2 * e] + beta[8 * g + 2 * e];
            v[2 * e + 1] = (f.y - mean) * inv * gamma[8 * g + 2 * e + 1] + beta[8 * g + 2 * e + 1];
          }
          *at = pack_half8(v);
        }
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[MB_X_READY + xb]);
      return true;
    };
    // Per tile: the hidden layer; then the next tile's LayerNorm, which
    // fills the wait for this tile's last fc2 and lets the next fc1 run
    // under this tile's final epilogue; then the final epilogue.
    bool ln_ok = (int)blockIdx.x >= p.tiles || layer_norm(blockIdx.x, 0);
    int i = 0;
    for (int tile = blockIdx.x; tile < p.tiles && ln_ok; tile += gridDim.x, i++) {

      // The hidden layer, chunk by chunk: bias, GELU, f16 into H[b].
      bool ok = true;
      for (int j = 0; j < CHUNKS; j++) {
        const int c = i * CHUNKS + j, b = c & 1;
        const uint32_t ph = (uint32_t)(c >> 1) & 1;
        if (!mbar_wait(&bar[MB_D1_FULL + b], ph, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_FULL)) {
          ok = false;
          break;
        }
        tc_fence_after();
        constexpr int COLS = NH / L::PARTS;  // this part's columns of the chunk: 32, 16 or 8
        uint32_t r[32];
        const uint32_t d1 = tmem + lanes + (uint32_t)(L::D1 + b * NH + part * COLS);
        if constexpr (COLS == 32) {
          tmem_ld16(d1, r);
          tmem_ld16(d1 + 16, r + 16);
        } else if constexpr (COLS == 16) {
          tmem_ld16(d1, r);
        } else {
          tmem_ld8(d1, r);
        }
        tmem_wait_ld();
        float v[COLS];
        const float4* bias4 = reinterpret_cast<const float4*>(b1 + j * NH + part * COLS);
#pragma unroll
        for (int e = 0; e < COLS; e += 4) {
          const float4 b = bias4[e / 4];
          const float2 g0 = gemm_gelu2(
              fadd2(make_float2(__uint_as_float(r[e]), __uint_as_float(r[e + 1])), make_float2(b.x, b.y)));
          const float2 g1 = gemm_gelu2(
              fadd2(make_float2(__uint_as_float(r[e + 2]), __uint_as_float(r[e + 3])), make_float2(b.z, b.w)));
          v[e] = g0.x;
          v[e + 1] = g0.y;
          v[e + 2] = g1.x;
          v[e + 3] = g1.y;
        }
        if (!mbar_wait(&bar[MB_H_EMPTY + b], ph ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_EMPTY)) {
          ok = false;
          break;
        }
        uint8_t* hb = Hb + b * L::H_BYTES;
#pragma unroll
        for (int q = 0; q < COLS / 8; q++)
          *reinterpret_cast<uint4*>(hb + ((part * (COLS / 8) + q) * 128 + row) * 16) = pack_half8(v + 8 * q);
        fence_proxy_async_shared();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[MB_H_FULL + b]);
      }
      if (!ok) break;

      if (tile + (int)gridDim.x < p.tiles && !layer_norm(tile + gridDim.x, i + 1)) break;

      // x += fc2 + b2 over this part's C / PARTS columns. Their old values
      // are read before the wait for fc2 (into registers for up to four
      // groups, else towards L1), so that the read overlaps the MMAs.
      constexpr int PG = C / 8 / L::PARTS;  // this part's channel groups
      constexpr bool HOLD = PG <= 4;
      const int m = tile * 128 + row;
      const bool live = m < p.M;
      __half* row_at = p.x + (long long)(part * PG) * p.plane_elems + (long long)m * 8;
      uint4 olds[HOLD ? PG : 1];
      if (live) {
#pragma unroll
        for (int q = 0; q < PG; q++) {
          if constexpr (HOLD)
            olds[q] = *reinterpret_cast<const uint4*>(row_at + (long long)q * p.plane_elems);
          else
            prefetch_l1(row_at + (long long)q * p.plane_elems);
        }
      }
      if (!mbar_wait(&bar[MB_D2_FULL], (uint32_t)(i & 1), abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_FULL)) break;
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < PG; q++) {
        const int c0 = (part * PG + q) * 8;
        uint32_t r[8];
        tmem_ld8(tmem + lanes + (uint32_t)c0, r);
        tmem_wait_ld();
        if (!live) continue;
        __half* at = row_at + (long long)q * p.plane_elems;
        uint4 old;
        if constexpr (HOLD)
          old = olds[q];
        else
          old = *reinterpret_cast<const uint4*>(at);
        float w[8];
#pragma unroll
        for (int e = 0; e < 8; e++) w[e] = __uint_as_float(r[e]) + b2[c0 + e];
        add_half8(w, old);
        *reinterpret_cast<uint4*>(at) = pack_half8(w);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[MB_D2_EMPTY]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, L::TMEM_COLS);
}

}  // namespace iec
