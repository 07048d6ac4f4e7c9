// SCUNet's block boundary as one sm_100a kernel: the join 1x1 of block b
// accumulated into the residual stream, then the split 1x1 of block b + 1,
//
//   x += y Wj + bj;   y = x Ws + bs
//
// (crates/scunet-native/src/network.rs:190-212: conv1_2 of one
// ConvTransBlock, the residual add, conv1_1 of the next) over planar f16 rows
// [C / 8][rows][8], C channels in and out of both products. Per tile of 128
// rows:
//   * the producer brings the tile's y rows and old x rows by TMA, both in
//     the K-major core-matrix layout [C / 8][128][8] (the A_ROWS box of
//     igemm_sm100.cuh);
//   * the MMA issuer runs the join (M 128 x N C x K C) from the y tile into
//     a TMEM accumulator;
//   * the epilogue warps add bj and the old x rows, round to f16, store the
//     new x rows to global memory and over the old ones in shared memory;
//   * the MMA issuer runs the split from that tile (the rounded x, as the
//     separate launches read it back) into a second accumulator;
//   * the epilogue warps add bs and store the new y rows over the tile's.
// The issuer runs the join of tile i + 1 before the split of tile i, and the
// epilogue finishes the split of tile i - 1 after the join of tile i, so the
// tensor core works under both epilogues. Up to 128 channels both weight
// matrices stay resident in shared memory, and the row tiles and both
// accumulators are double-buffered; at 256 channels (two 128 KB matrices)
// the weights stream through a ring of two 64-row chunks, in the order the
// issuer takes them (the join's chunks of tile i + 1, then the split's of
// tile i), with one buffer per row tile and one accumulator each (512 TMEM
// columns). The y and x rows are read once and written once: a tile's rows
// are read by TMA before its epilogue overwrites them, and no other tile
// touches them. Every wait is bounded as in the other kernels (sm100.cuh).
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "igemm_sm100.cuh"
#include "sm100.cuh"

namespace iec {

struct JoinSplitParams {
  int M;                  // rows
  int tiles;              // ceil(M / 128)
  __half* x;              // planar [C / 8][rows][8], plane stride plane_elems (halves)
  __half* y;
  long long plane_elems;
  const uint8_t* w;       // Wj [C / 8][C][8] f16, then Ws [C / 8][C][8] f16
  const float* bias;      // bj [C], bs [C]
  int* dev_err;
};

template <int C>
struct JoinSplitSmem {
  // 8 epilogue warps: two per TMEM lane quarter, each over half the columns.
  static constexpr int EW = 8, PARTS = 2, THREADS = 64 + 32 * EW;
  static constexpr bool RES = C <= 128;             // weights resident, else streamed
  static constexpr int TILE = (C / 8) * 128 * 16;  // one row tile, either map
  static constexpr int W_BYTES = (C / 8) * C * 16;  // one weight matrix
  static constexpr int CHUNK = 8 * C * 16;          // 64 of its rows, [8][C][8]
  static constexpr int CHUNKS = C / 64, WS = 2;     // chunks per matrix, ring stages
  static constexpr int NB = RES ? 2 : 1;            // row-tile buffers per map
  static constexpr int ACCS = RES ? 2 : 1;          // accumulators per product
  static constexpr int Y_OFF = 0, X_OFF = NB * TILE, W_OFF = 2 * NB * TILE;
  static constexpr int BIAS_OFF = W_OFF + (RES ? 2 * W_BYTES : WS * CHUNK);
  static constexpr int NBAR = 24;
  static constexpr int BAR_OFF = BIAS_OFF + 2 * C * 4;
  static constexpr int TOTAL = BAR_OFF + NBAR * 8 + 16;
  static constexpr int CTAS = TOTAL <= 113 * 1024 ? 2 : 1;
  // TMEM: the join's accumulators from column 0, the split's from ACCS C.
  static constexpr int TMEM_COLS = 2 * ACCS * C <= 128 ? 128 : 2 * ACCS * C <= 256 ? 256 : 512;
  static_assert(C == 64 || C == 128 || C == 256, "join-split width");
  static_assert(2 * ACCS * C <= 512, "join-split tensor memory");
  static_assert(TOTAL <= 227 * 1024, "join-split shared memory");
  static_assert(CTAS == 1 || 2 * TMEM_COLS <= 512, "join-split tensor memory per SM");
};

// Barrier slots (two of each, per buffer, accumulator or ring stage).
enum : int {
  JS_Y_FULL = 0, JS_Y_EMPTY = 2, JS_X_FULL = 4, JS_X_READY = 6, JS_X_EMPTY = 8,
  JS_D1_FULL = 10, JS_D1_EMPTY = 12, JS_D2_FULL = 14, JS_D2_EMPTY = 16, JS_W_FULL = 18, JS_W_EMPTY = 20, JS_COUNT = 22
};

template <int C>
__global__ void __launch_bounds__(JoinSplitSmem<C>::THREADS, JoinSplitSmem<C>::CTAS)
    joinsplit_sm100(const __grid_constant__ CUtensorMap y_map, const __grid_constant__ CUtensorMap x_map,
                    const JoinSplitParams p) {
  using L = JoinSplitSmem<C>;
  constexpr int NB = L::NB, ACCS = L::ACCS, WS = L::WS;
  static_assert(JS_COUNT <= L::NBAR, "barrier slots");
  extern __shared__ __align__(128) uint8_t js_smem[];
  uint8_t* Y = js_smem + L::Y_OFF;
  uint8_t* X = js_smem + L::X_OFF;
  uint8_t* Wt = js_smem + L::W_OFF;
  float* sbias = reinterpret_cast<float*>(js_smem + L::BIAS_OFF);
  uint64_t* bar = reinterpret_cast<uint64_t*>(js_smem + L::BAR_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(js_smem + L::BAR_OFF + L::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(js_smem + L::BAR_OFF + L::NBAR * 8 + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; b++) {
      mbar_init(&bar[JS_Y_FULL + b], 1);
      mbar_init(&bar[JS_Y_EMPTY + b], 1);
      mbar_init(&bar[JS_X_FULL + b], 1);
      mbar_init(&bar[JS_X_READY + b], L::EW);
      mbar_init(&bar[JS_X_EMPTY + b], 1);
      mbar_init(&bar[JS_D1_FULL + b], 1);
      mbar_init(&bar[JS_D1_EMPTY + b], L::EW);
      mbar_init(&bar[JS_D2_FULL + b], 1);
      mbar_init(&bar[JS_D2_EMPTY + b], L::EW);
      mbar_init(&bar[JS_W_FULL + b], 1);
      mbar_init(&bar[JS_W_EMPTY + b], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  // The biases and weights are not written by any kernel: staged before the
  // wait for the previous one (resident weights all, streamed ones the
  // ring's first chunks).
  for (int i = (int)threadIdx.x; i < 2 * C; i += L::THREADS) sbias[i] = p.bias[i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool any = (int)blockIdx.x < p.tiles;
  if (threadIdx.x == 0 && any) {
    if constexpr (L::RES) {
      mbar_arrive_expect_tx(&bar[JS_W_FULL], (uint32_t)(2 * L::W_BYTES));
      bulk_load(Wt, p.w, (uint32_t)(2 * L::W_BYTES), &bar[JS_W_FULL]);
    } else {
      for (int s = 0; s < WS; s++) {
        mbar_arrive_expect_tx(&bar[JS_W_FULL + s], (uint32_t)L::CHUNK);
        bulk_load(Wt + s * L::CHUNK, p.w + (size_t)s * L::CHUNK, (uint32_t)L::CHUNK, &bar[JS_W_FULL + s]);
      }
    }
  }
  griddep_launch_dependents();
  griddep_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      prefetch_tensor_map(&y_map);
      prefetch_tensor_map(&x_map);
      // Streamed weights: chunk c of the issuer's order (the first WS are
      // already in flight); each tile's join chunks (matrix 0), then the
      // previous tile's split chunks (matrix 1).
      int c = WS;
      auto chunks = [&](int m, int first) -> bool {
        for (int j = first; j < L::CHUNKS; j++, c++) {
          const int s = c % WS;
          if (!mbar_wait(&bar[JS_W_EMPTY + s], ((uint32_t)(c / WS) & 1) ^ 1, abort_flag, p.dev_err,
                         DEV_ERR_WAIT_WEIGHTS))
            return false;
          mbar_arrive_expect_tx(&bar[JS_W_FULL + s], (uint32_t)L::CHUNK);
          bulk_load(Wt + s * L::CHUNK, p.w + (size_t)m * L::W_BYTES + (size_t)j * L::CHUNK, (uint32_t)L::CHUNK,
                    &bar[JS_W_FULL + s]);
        }
        return true;
      };
      bool ok = true;
      int i = 0;
      for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, i++) {
        const int b = i % NB;
        const uint32_t ph = (uint32_t)(i / NB) & 1;
        if (!mbar_wait(&bar[JS_Y_EMPTY + b], ph ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(&bar[JS_Y_FULL + b], (uint32_t)L::TILE);
        tma_load_3d(Y + b * L::TILE, &y_map, &bar[JS_Y_FULL + b], 0, tile * 8, 0);
        if constexpr (!L::RES) {
          ok = chunks(0, i == 0 ? WS : 0) && (i == 0 || chunks(1, 0));
          if (!ok) break;
        }
        if (!mbar_wait(&bar[JS_X_EMPTY + b], ph ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(&bar[JS_X_FULL + b], (uint32_t)L::TILE);
        tma_load_3d(X + b * L::TILE, &x_map, &bar[JS_X_FULL + b], 0, tile * 8, 0);
      }
      if constexpr (!L::RES) {
        if (ok && i > 0) chunks(1, 0);
      }
      // let the copies in flight land before the CTA may leave
      for (int t = i - NB; t < i; t++)
        if (t >= 0) {
          mbar_wait(&bar[JS_Y_FULL + t % NB], (uint32_t)(t / NB) & 1, abort_flag, p.dev_err, 0);
          mbar_wait(&bar[JS_X_FULL + t % NB], (uint32_t)(t / NB) & 1, abort_flag, p.dev_err, 0);
        }
      if (any) {
        if constexpr (L::RES) {
          mbar_wait(&bar[JS_W_FULL], 0, abort_flag, p.dev_err, 0);
        } else {
          for (int k = c - WS; k < c; k++) mbar_wait(&bar[JS_W_FULL + k % WS], (uint32_t)(k / WS) & 1, abort_flag, p.dev_err, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t idesc = idesc_f16_f32(128, C);
      const uint32_t ya = smem_u32(Y), xa = smem_u32(X), wa = smem_u32(Wt);
      int c = 0;  // streamed chunks taken
      // One product of a tile: D = A (128 x C, [C / 8][128][8]) x W_m (C x C,
      // [C / 8][C][8]), unrolled with constant descriptor offsets.
      auto product = [&](uint32_t a, int m, uint32_t d) -> bool {
        if constexpr (L::RES) {
          const uint32_t w = wa + (uint32_t)(m * L::W_BYTES);
#pragma unroll
          for (int k = 0; k < C / 16; k++) {
            const uint64_t ad = smem_desc(a + (uint32_t)(2 * k * 128 * 16), 128 * 16, 128);
            const uint64_t bd = smem_desc(w + (uint32_t)(2 * k * C * 16), C * 16, 128);
            umma_f16(d, ad, bd, idesc, k > 0 ? 1u : 0u);
          }
        } else {
          for (int j = 0; j < L::CHUNKS; j++, c++) {
            const int s = c % WS;
            if (!mbar_wait(&bar[JS_W_FULL + s], (uint32_t)(c / WS) & 1, abort_flag, p.dev_err, DEV_ERR_WAIT_WEIGHTS))
              return false;
            tc_fence_after();
            const uint32_t w = wa + (uint32_t)(s * L::CHUNK), aj = a + (uint32_t)(j * 8 * 128 * 16);
#pragma unroll
            for (int k = 0; k < 4; k++) {
              const uint64_t ad = smem_desc(aj + (uint32_t)(2 * k * 128 * 16), 128 * 16, 128);
              const uint64_t bd = smem_desc(w + (uint32_t)(2 * k * C * 16), C * 16, 128);
              umma_f16(d, ad, bd, idesc, (j > 0 || k > 0) ? 1u : 0u);
            }
            umma_commit(&bar[JS_W_EMPTY + s]);
          }
        }
        return true;
      };
      // The split of the CTA's j-th tile, once the epilogue has written its
      // new x rows.
      auto split = [&](int j) -> bool {
        const int b = j % NB, d = j % ACCS;
        if (!mbar_wait(&bar[JS_X_READY + b], (uint32_t)(j / NB) & 1, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL))
          return false;
        if (!mbar_wait(&bar[JS_D2_EMPTY + d], ((uint32_t)(j / ACCS) & 1) ^ 1, abort_flag, p.dev_err,
                       DEV_ERR_WAIT_ACC_EMPTY))
          return false;
        tc_fence_after();
        if (!product(xa + (uint32_t)(b * L::TILE), 1, tmem + (uint32_t)((ACCS + d) * C))) return false;
        umma_commit(&bar[JS_X_EMPTY + b]);
        umma_commit(&bar[JS_D2_FULL + d]);
        return true;
      };
      bool ok = true;
      if constexpr (L::RES) {
        ok = mbar_wait(&bar[JS_W_FULL], 0, abort_flag, p.dev_err, DEV_ERR_WAIT_WEIGHTS);
        tc_fence_after();
      }
      int i = 0;
      for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, i++) {
        const int b = i % NB, d = i % ACCS;
        if (!mbar_wait(&bar[JS_Y_FULL + b], (uint32_t)(i / NB) & 1, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL)) break;
        if (!mbar_wait(&bar[JS_D1_EMPTY + d], ((uint32_t)(i / ACCS) & 1) ^ 1, abort_flag, p.dev_err,
                       DEV_ERR_WAIT_ACC_EMPTY))
          break;
        tc_fence_after();
        if (!product(ya + (uint32_t)(b * L::TILE), 0, tmem + (uint32_t)(d * C))) break;
        umma_commit(&bar[JS_Y_EMPTY + b]);
        umma_commit(&bar[JS_D1_FULL + d]);
        if (i > 0 && !split(i - 1)) ok = false;
      }
      if (ok && i > 0 && split(i - 1))
        mbar_wait(&bar[JS_D2_FULL + (i - 1) % ACCS], (uint32_t)((i - 1) / ACCS) & 1, abort_flag, p.dev_err, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp w serves TMEM lane quarter w % 4 (rows 32 q .. 32 q + 31, one row
    // per lane) and columns [part C / 2, part C / 2 + C / 2), in batches of
    // up to 32 columns; the accumulator is released after its last batch is
    // loaded.
    const int quarter = warp & 3, part = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    constexpr int PG = C / 8 / L::PARTS;  // this part's channel groups
    constexpr int BG = PG < 4 ? PG : 4;   // groups per batch
    const float* bj = sbias;
    const float* bs = sbias + C;
    // x += y Wj + bj over this part's groups of the CTA's i-th tile: into
    // global memory and over the old rows in shared memory.
    auto join = [&](int tile, int i) -> bool {
      const int b = i % NB, d = i % ACCS;
      if (!mbar_wait(&bar[JS_X_FULL + b], (uint32_t)(i / NB) & 1, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL))
        return false;
      if (!mbar_wait(&bar[JS_D1_FULL + d], (uint32_t)(i / ACCS) & 1, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_FULL))
        return false;
      tc_fence_after();
      const int m = tile * 128 + row;
      uint8_t* xt = X + b * L::TILE;
#pragma unroll
      for (int q0 = 0; q0 < PG; q0 += BG) {
        uint32_t r[BG * 8];
#pragma unroll
        for (int q = 0; q < BG; q += 2)
          tmem_ld16(tmem + lanes + (uint32_t)(d * C + (part * PG + q0 + q) * 8), r + 8 * q);
        tmem_wait_ld();
        if (q0 + BG >= PG) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar[JS_D1_EMPTY + d]);
        }
#pragma unroll
        for (int q = 0; q < BG; q++) {
          const int g = part * PG + q0 + q;
          uint4* at = reinterpret_cast<uint4*>(xt + (g * 128 + row) * 16);
          float w[8];
#pragma unroll
          for (int e = 0; e < 8; e++) w[e] = __uint_as_float(r[8 * q + e]) + bj[8 * g + e];
          add_half8(w, *at);
          const uint4 v = pack_half8(w);
          *at = v;
          if (m < p.M) *reinterpret_cast<uint4*>(p.x + (long long)g * p.plane_elems + (long long)m * 8) = v;
        }
      }
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[JS_X_READY + b]);
      return true;
    };
    // y = x Ws + bs over this part's groups of the CTA's j-th tile.
    auto split = [&](int tile, int j) -> bool {
      const int d = j % ACCS;
      if (!mbar_wait(&bar[JS_D2_FULL + d], (uint32_t)(j / ACCS) & 1, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_FULL))
        return false;
      tc_fence_after();
      const int m = tile * 128 + row;
#pragma unroll
      for (int q0 = 0; q0 < PG; q0 += BG) {
        uint32_t r[BG * 8];
#pragma unroll
        for (int q = 0; q < BG; q += 2)
          tmem_ld16(tmem + lanes + (uint32_t)((ACCS + d) * C + (part * PG + q0 + q) * 8), r + 8 * q);
        tmem_wait_ld();
        if (q0 + BG >= PG) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar[JS_D2_EMPTY + d]);
        }
        if (m < p.M) {
#pragma unroll
          for (int q = 0; q < BG; q++) {
            const int g = part * PG + q0 + q;
            float w[8];
#pragma unroll
            for (int e = 0; e < 8; e++) w[e] = __uint_as_float(r[8 * q + e]) + bs[8 * g + e];
            *reinterpret_cast<uint4*>(p.y + (long long)g * p.plane_elems + (long long)m * 8) = pack_half8(w);
          }
        }
      }
      return true;
    };
    int i = 0, prev = -1;
    bool ok = true;
    for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, i++) {
      ok = join(tile, i) && (prev < 0 || split(prev, i - 1));
      prev = tile;
    }
    if (ok && prev >= 0) split(prev, i - 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, L::TMEM_COLS);
}

}  // namespace iec
