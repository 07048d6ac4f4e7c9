// The network's body — every 64 -> 64 PReLU convolution — as one persistent
// launch with tile-level dataflow between the layers.
//
// Each layer computes exactly what conv3x3_sm100<64, 64, CONV_PRELU> does
// (same tile shape, halo box, N = 3 x 64 tap folding, epilogue); what changes
// is the schedule. A launch per layer pays a fill and a drain (the first
// halo loads, the weights, the last tile's epilogue) of several
// microseconds, and each layer's 100+ MB of maps round-trips through HBM,
// whose power pulls the SM clock down. Here the work items are (layer,
// image, 4 x 30 tile), ordered group by group of `group` images, layer by layer
// within a group, tiles in row order; CTA c takes items c, c + grid, ...
// A group's two maps (group x 2 x 12.6 MB for 256 x 384 images) stay in L2
// while its layers run, and no CTA ever waits for a whole layer: before
// loading a tile's halo, the producer waits only until the previous layer
// has finished the (up to) three tile rows the halo reads, which per-row
// completion counters in global memory report. Two warps keep that
// bookkeeping off the critical path (a fence or an L2 round trip per tile in
// the producer or the epilogue costs more than the tile's math):
//  * the tracker polls the counters for the next eight items of its CTA at
//    once (a lane per item, the items' words from a table), fences acquire,
//    and publishes in shared memory how many items are ready; the producer
//    only reads that word (then orders the async proxy behind it before its
//    TMA load);
//  * the signaller takes the epilogue warps' per-warp progress words (each
//    stored with release after the warp's global stores), and for every tile
//    all sixteen have stored, fences once and bumps its row's counter.
//
// Hazards. Layer l reads maps[l & 1] and writes maps[(l + 1) & 1], the map
// layer l - 1 read. A tile of layer l waits for the rows of layer l - 1
// around it; those rows' tiles are the only readers of the region it
// overwrites, and they had loaded their halos before they counted as done.
// Deadlock freedom: every item depends only on items of lower index, each
// CTA's producer, MMA issuer and epilogue walk their items in index order,
// and every CTA is resident at once (a cooperative launch, one CTA per SM),
// so the lowest unfinished item can always proceed. Every wait is bounded.
//
// Weights: two 72 KB buffers; the producer loads layer l's weights into
// buffer (n & 1) for this CTA's n-th layer change once the MMA issuer has
// released that buffer (a tcgen05.commit when it moved past the layer that
// used it before), so the next layer's weights arrive while the current
// one runs. Three 24 KB halo stages fit beside them.
#pragma once

#include "conv3x3_sm100.cuh"

namespace iec {

constexpr int BODY_NSTAGE = 3;
constexpr int BODY_MAX_LAYERS = 32;
constexpr int BODY_LOOKAHEAD = 8;                          // items the tracker checks per poll
constexpr int BODY_SIGNAL_WARP = 2 + CONV_EPI_WARPS;       // 18
constexpr int BODY_TRACK_WARP = BODY_SIGNAL_WARP + 1;      // 19
constexpr int BODY_THREADS = 32 * (BODY_TRACK_WARP + 1);   // 640

struct BodyParams {
  int H, W, MH, MW;                   // valid and allocated map size
  int tiles_x, tiles_y, tiles_img;    // tile grid of one image
  int count, layers, group;           // images, body layers, images per layer sweep
  int items;                          // layers * count * tiles_img (< 2^24)
  int group_items;                    // layers * group * tiles_img
  int last_group;                     // index of the last (possibly smaller) group
  FastDiv div_tiles_x, div_tiles_img, div_group_items, div_group_tiles, div_last_tiles;
  uint32_t slope_unit;                // bit l: every PReLU slope of layer l is in [0, 1]
  const uint16_t* weights[BODY_MAX_LAYERS];  // [3 ky][8][3 kx][64][8] f16 each
  const float* bias[BODY_MAX_LAYERS];
  const float* slope[BODY_MAX_LAYERS];
  __half* maps[2];                    // layer l reads maps[l & 1], writes maps[(l + 1) & 1]
  int* rows;                          // [layers][count][tiles_y] finished tiles, zero at launch
  const uint32_t* item_words;         // [items] body_item(k) packed by body_pack (epilogue,
                                      // signaller and tracker read it instead of dividing)
  int* dev_err;
};

struct BodyItem {
  int layer, img, ty, tx;
};

__device__ __forceinline__ BodyItem body_item(const BodyParams& p, int k) {
  int grp = (int)p.div_group_items.div((uint32_t)k);
  if (grp > p.last_group) grp = p.last_group;
  const int r = k - grp * p.group_items;
  const FastDiv& per_layer = grp == p.last_group ? p.div_last_tiles : p.div_group_tiles;
  const int l = (int)per_layer.div((uint32_t)r);
  const int t = r - l * (int)per_layer.d;
  const int gi = (int)p.div_tiles_img.div((uint32_t)t);
  const int tt = t - gi * p.tiles_img;
  const int ty = (int)p.div_tiles_x.div((uint32_t)tt);
  BodyItem it;
  it.layer = l;
  it.img = grp * p.group + gi;
  it.ty = ty;
  it.tx = tt - ty * p.tiles_x;
  return it;
}

// One item in a word (the epilogue warps read it instead of dividing):
// layer 5 bits, image 8, tile row 10, tile column 9.
__host__ __device__ constexpr uint32_t body_pack(int layer, int img, int ty, int tx) {
  return ((uint32_t)layer << 27) | ((uint32_t)img << 19) | ((uint32_t)ty << 9) | (uint32_t)tx;
}

__device__ __forceinline__ BodyItem body_unpack(uint32_t w) {
  BodyItem it;
  it.layer = (int)(w >> 27);
  it.img = (int)((w >> 19) & 0xff);
  it.ty = (int)((w >> 9) & 0x3ff);
  it.tx = (int)(w & 0x1ff);
  return it;
}

struct BodySmem {
  static constexpr int KCH = 8;
  static constexpr int W_BYTES = 9 * KCH * 64 * 16;             // 73,728
  static constexpr int STAGE_BYTES = KCH * CONV_CHUNK_BYTES;    // 24,576 (a multiple of 1024)
  static_assert(STAGE_BYTES % 1024 == 0, "stages stay 1024-byte aligned");
  static constexpr int A_OFF = 2 * W_BYTES;
  static constexpr int BAR_OFF = A_OFF + BODY_NSTAGE * STAGE_BYTES;
  // full[NSTAGE], empty[NSTAGE], acc_full[2], acc_empty[2], wfull[2], wempty[2]
  static constexpr int NBARS = 2 * BODY_NSTAGE + 8;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;          // tmem slot, abort flag, ready, want
  static constexpr int PROGRESS_OFF = MISC_OFF + 16;              // [16] items stored per epilogue warp
  static constexpr int TOTAL = PROGRESS_OFF + 4 * CONV_EPI_WARPS;
  static constexpr int DYN_BYTES = TOTAL + 1024;                // room to align the base
};

__global__ void __launch_bounds__(BODY_THREADS, 1)
    conv3x3_body_sm100(const __grid_constant__ CUtensorMap map0, const __grid_constant__ CUtensorMap map1,
                       const __grid_constant__ BodyParams p) {
  using L = BodySmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* w_smem = smem;
  uint8_t* a_smem = smem + L::A_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;
  uint64_t* empty = bars + BODY_NSTAGE;
  uint64_t* acc_full = bars + 2 * BODY_NSTAGE;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* wfull = acc_empty + 2;
  uint64_t* wempty = wfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);
  uint32_t* ready = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF + 8);       // items whose inputs are done
  volatile uint32_t* want = reinterpret_cast<volatile uint32_t*>(smem + L::MISC_OFF + 12);  // producer's item
  uint32_t* progress = reinterpret_cast<uint32_t*>(smem + L::PROGRESS_OFF);  // per epilogue warp

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The last layer's launch may take each SM as this grid's CTA there exits.
  griddep_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < BODY_NSTAGE; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], CONV_EPI_WARPS);
      mbar_init(&wfull[a], 1);
      mbar_init(&wempty[a], 1);
    }
    *abort_flag = 0;
    *ready = 0;
    *want = 0;
    for (int w = 0; w < CONV_EPI_WARPS; w++) progress[w] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, CONV_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      prefetch_tensor_map(&map0);
      prefetch_tensor_map(&map1);
      // The first layer's input (the previous launch's output) and the zeroed
      // row counters.
      griddep_wait();
      int s = 0, cur = -1, nw = 0, i = 0;
      uint32_t phase = 0;
      int issued[BODY_NSTAGE], wissued[2] = {-1, -1};
      for (int j = 0; j < BODY_NSTAGE; j++) issued[j] = -1;
      for (int k = blockIdx.x; k < p.items; k += gridDim.x, i++) {
        const BodyItem it = body_item(p, k);
        *want = (uint32_t)i;
        if (it.layer != cur) {
          const int b = nw & 1;
          if (nw >= 2 && !mbar_wait(&wempty[b], (uint32_t)((nw >> 1) - 1) & 1, abort_flag, p.dev_err,
                                    DEV_ERR_WAIT_WEIGHTS))
            break;
          mbar_arrive_expect_tx(&wfull[b], L::W_BYTES);
          const uint8_t* src = reinterpret_cast<const uint8_t*>(p.weights[it.layer]);
          for (int off = 0; off < L::W_BYTES; off += 24576)
            bulk_load(w_smem + b * L::W_BYTES + off, src + off, 24576, &wfull[b]);
          wissued[b] = (nw >> 1) & 1;
          cur = it.layer;
          nw++;
        }
        if (it.layer > 0) {
          // The tracker saw the rows this halo reads finished (and fenced).
          if (!wait_word(ready, (uint32_t)i, abort_flag, p.dev_err, DEV_ERR_WAIT_ROWS)) break;
          fence_proxy_async_global();
        }
        if (!mbar_wait(&empty[s], phase ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(&full[s], L::STAGE_BYTES);
        tma_load_4d(a_smem + s * L::STAGE_BYTES, (it.layer & 1) ? &map1 : &map0, &full[s],
                    (it.tx * CONV_TILE_W - 1) * 8, it.ty * CONV_TILE_H - 1, 0, it.img);
        issued[s] = (int)phase;
        if (++s == BODY_NSTAGE) {
          s = 0;
          phase ^= 1;
        }
      }
      // No copy may still be writing shared memory when the CTA exits.
      for (int j = 0; j < BODY_NSTAGE; j++)
        if (issued[j] >= 0) mbar_wait(&full[j], (uint32_t)issued[j], abort_flag, p.dev_err, 0);
      for (int b = 0; b < 2; b++)
        if (wissued[b] >= 0) mbar_wait(&wfull[b], (uint32_t)wissued[b], abort_flag, p.dev_err, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      constexpr int N = 3 * 64;
      constexpr uint32_t idesc = idesc_f16_f32(128, N);
      const uint32_t abase0 = smem_u32(a_smem), wbase0 = smem_u32(w_smem);
      int last_acc = -1, cur = -1, nw = 0, wb = 0;
      uint32_t last_parity = 0, phase = 0;
      int s = 0, i = 0;
      // The item's layer from its packed word, read one item ahead: the
      // single issuing thread pays for any arithmetic or load latency
      // between its MMAs.
      uint32_t next = (int)blockIdx.x < p.items ? __ldg(p.item_words + blockIdx.x) : 0u;
      for (int k = blockIdx.x; k < p.items; k += gridDim.x, i++) {
        const int layer = (int)(next >> 27);
        if (k + (int)gridDim.x < p.items) next = __ldg(p.item_words + k + gridDim.x);
        if (layer != cur) {
          if (cur >= 0) umma_commit(&wempty[wb]);  // the old layer's weights, once its MMAs are done
          wb = nw & 1;
          if (!mbar_wait(&wfull[wb], (uint32_t)(nw >> 1) & 1, abort_flag, p.dev_err, DEV_ERR_WAIT_WEIGHTS)) break;
          cur = layer;
          nw++;
        }
        const int a = i & 1;
        const uint32_t acc_phase = (uint32_t)(i >> 1) & 1;
        if (!mbar_wait(&acc_empty[a], acc_phase ^ 1, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_EMPTY)) break;
        if (!mbar_wait(&full[s], phase, abort_flag, p.dev_err, DEV_ERR_WAIT_FULL)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(a * CONV_ACC_COLS);
        const uint32_t abase = abase0 + (uint32_t)(s * L::STAGE_BYTES);
        const uint32_t wbase = wbase0 + (uint32_t)(wb * L::W_BYTES);
#pragma unroll
        for (int ky = 0; ky < 3; ky++) {
#pragma unroll
          for (int ks = 0; ks < L::KCH / 2; ks++) {
            const uint64_t adesc = smem_desc(abase + (uint32_t)(2 * ks * CONV_CHUNK_BYTES + ky * CONV_HALO_W * 16),
                                             CONV_CHUNK_BYTES, 128);
            const uint64_t bdesc = smem_desc(wbase + (uint32_t)((ky * L::KCH + 2 * ks) * N * 16), N * 16, 128);
            umma_f16(d, adesc, bdesc, idesc, (ky | ks) != 0);
          }
        }
        umma_commit(&empty[s]);
        umma_commit(&acc_full[a]);
        last_acc = a;
        last_parity = acc_phase;
        const bool wrap = s + 1 == BODY_NSTAGE;
        s = wrap ? 0 : s + 1;
        phase ^= wrap ? 1u : 0u;
      }
      // The accumulators must be written before TMEM is released.
      if (last_acc >= 0) mbar_wait(&acc_full[last_acc], last_parity, abort_flag, p.dev_err, 0);
    }
  } else if (warp < BODY_SIGNAL_WARP) {
    // ------------------------------------------------------------- epilogue
    const int quarter = warp & 3;            // TMEM lanes 32 q .. 32 q + 31
    const int part = (warp - 2) >> 2;        // channels 16 part .. 16 part + 15
    const int row = quarter * 32 + lane;     // M row = partial-sum position (r, c) of the tile
    const int pr = row / CONV_HALO_W, pc = row % CONV_HALO_W;
    const size_t plane8 = (size_t)p.MH * p.MW * 8;         // halves per channel-group plane
    const size_t img_stride = 8 * plane8;                    // halves per image (8 groups)
    const size_t group_off = (size_t)(part * 2) * plane8;    // this warp's first group
    float r_bias[16], r_slope[16];
    bool unit = false;
    int cur = -1, i = 0;
    uint32_t next = (int)blockIdx.x < p.items ? __ldg(p.item_words + blockIdx.x) : 0u;
    for (int k = blockIdx.x; k < p.items; k += gridDim.x, i++) {
      const BodyItem it = body_unpack(next);
      if (k + (int)gridDim.x < p.items) next = __ldg(p.item_words + k + gridDim.x);
      if (it.layer != cur) {
        cur = it.layer;
        const float* bias = p.bias[cur];
        const float* slope = p.slope[cur];
#pragma unroll
        for (int e = 0; e < 16; e++) {
          r_bias[e] = __ldg(bias + part * 16 + e);
          r_slope[e] = __ldg(slope + part * 16 + e);
        }
        unit = ((p.slope_unit >> cur) & 1u) != 0;
      }
      const int a = i & 1;
      const uint32_t acc_phase = (uint32_t)(i >> 1) & 1;
      if (!mbar_wait(&acc_full[a], acc_phase, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_FULL)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * CONV_ACC_COLS);
      // out(r, c) = Q_0(r, c - 1) + Q_1(r, c) + Q_2(r, c + 1) (neighbouring lanes)
      float2 v[8];  // channel pairs
      {
        uint32_t q0[16], q1[16], q2[16];
        const uint32_t col = (uint32_t)(part * 16);
        tmem_ld16(taddr + col, q0);
        tmem_ld16(taddr + 64u + col, q1);
        tmem_ld16(taddr + 128u + col, q2);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const float2 left = make_float2(__shfl_up_sync(0xffffffffu, __uint_as_float(q0[2 * e]), 1),
                                          __shfl_up_sync(0xffffffffu, __uint_as_float(q0[2 * e + 1]), 1));
          const float2 right = make_float2(__shfl_down_sync(0xffffffffu, __uint_as_float(q2[2 * e]), 1),
                                           __shfl_down_sync(0xffffffffu, __uint_as_float(q2[2 * e + 1]), 1));
          v[e] = fadd2(fadd2(left, make_float2(__uint_as_float(q1[2 * e]), __uint_as_float(q1[2 * e + 1]))), right);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);

      const int y = it.ty * CONV_TILE_H + pr, x = it.tx * CONV_TILE_W + pc - 1;
      if (pc >= 1 && pc <= CONV_TILE_W && y < p.H && x < p.W) {
        // this thread's two channel groups of pixel (y, x): plane offsets
        // hoisted out of the item loop, the pixel offset in 32 bits
        __half* base = p.maps[(cur + 1) & 1] + (size_t)it.img * img_stride + group_off +
                       (size_t)(((uint32_t)y * (uint32_t)p.MW + (uint32_t)x) * 8u);
#pragma unroll
        for (int g = 0; g < 2; g++) {
          uint32_t packed[4];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            const int q = g * 8 + 2 * e;
            const float2 w = fadd2(v[q / 2], make_float2(r_bias[q], r_bias[q + 1]));
            float v0, v1;
            if (unit) {
              const float2 sw = fmul2(w, make_float2(r_slope[q], r_slope[q + 1]));
              v0 = fmaxf(w.x, sw.x);
              v1 = fmaxf(w.y, sw.y);
            } else {
              v0 = w.x < 0.0f ? w.x * r_slope[q] : w.x;
              v1 = w.y < 0.0f ? w.y * r_slope[q + 1] : w.y;
            }
            __half2 h = __floats2half2_rn(v0, v1);
            packed[e] = *reinterpret_cast<uint32_t*>(&h);
          }
          *reinterpret_cast<uint4*>(base + (g ? plane8 : 0)) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        }
      }
      // This warp's share of the tile is stored: publish it to the signaller.
      __syncwarp();
      if (lane == 0) st_release_cta(&progress[warp - 2], (uint32_t)(i + 1));
    }
  } else if (warp == BODY_SIGNAL_WARP) {
    if (lane == 0) {
      // -------------------------------------------------------- signaller
      // Tiles every epilogue warp has stored: the progress words seen
      // (relaxed), one fence (acquire for them, release for what follows),
      // then each tile's row counter; the last layer's tiles feed nothing.
      int i = 0, k = blockIdx.x;
      uint64_t start = global_ns();
      for (uint32_t n = 1; k < p.items; n++) {
        uint32_t done = 0xffffffffu;
#pragma unroll
        for (int w = 0; w < CONV_EPI_WARPS; w++) {
          const uint32_t v = *reinterpret_cast<volatile uint32_t*>(&progress[w]);
          done = v < done ? v : done;
        }
        if ((int)done > i) {
          fence_acq_rel_gpu();
          for (; i < (int)done; i++, k += gridDim.x) {
            const BodyItem it = body_unpack(__ldg(p.item_words + k));
            if (it.layer + 1 < p.layers)
              red_add_gpu(p.rows + ((size_t)it.layer * p.count + it.img) * p.tiles_y + it.ty, 1);
          }
          start = global_ns();
        } else {
          if ((n & 63) == 0) {
            if (*abort_flag) break;
            if (global_ns() - start > IEC_WAIT_NS) {
              *abort_flag = 1;
              atomicOr(p.dev_err, DEV_ERR_WAIT_ROWS);
              break;
            }
          }
          __nanosleep(32);
        }
      }
    }
  } else if (warp == BODY_TRACK_WARP) {
    // ------------------------------------------------------------ tracker
    // Lane j checks item i + j (j < LOOKAHEAD): its three input rows (none
    // for layer-0 items, rows past the grid clamped), loaded together. Every
    // lane fences acquire after its loads; after the warp barrier, lane 0
    // publishes the leading run of ready items. It runs at most WINDOW items
    // ahead of the producer and backs off while rows are unfinished, so the
    // counters' few L2 lines are not flooded.
    constexpr int WINDOW = 4 * BODY_LOOKAHEAD;
    int i = 0, k = blockIdx.x;
    uint32_t nap = 32;
    uint64_t start = global_ns();
    for (uint32_t n = 1; k < p.items; n++) {
      if ((uint32_t)i >= *want + WINDOW) {
        if ((n & 63) == 0 && *abort_flag) break;
        __nanosleep(64);
        start = global_ns();
        continue;
      }
      bool ok = true;
      if (lane < BODY_LOOKAHEAD) {
        const int kk = k + lane * (int)gridDim.x;
        if (kk < p.items) {
          const BodyItem it = body_unpack(__ldg(p.item_words + kk));
          if (it.layer > 0) {
            const int* rows = p.rows + ((size_t)(it.layer - 1) * p.count + it.img) * p.tiles_y;
            const int r0 = it.ty > 0 ? it.ty - 1 : 0, r2 = it.ty + 1 < p.tiles_y ? it.ty + 1 : it.ty;
            const int v0 = ld_relaxed_gpu(rows + r0);
            const int v1 = ld_relaxed_gpu(rows + it.ty);
            const int v2 = ld_relaxed_gpu(rows + r2);
            ok = v0 >= p.tiles_x && v1 >= p.tiles_x && v2 >= p.tiles_x;
          }
        } else {
          ok = false;  // past this CTA's items: ends the run
        }
      }
      const uint32_t not_ready = __ballot_sync(0xffffffffu, !ok);
      const int run = not_ready ? __ffs(not_ready) - 1 : BODY_LOOKAHEAD;
      if (run > 0) {
        fence_acq_rel_gpu();
        __syncwarp();
        if (lane == 0) st_release_cta(ready, (uint32_t)(i + run));
        i += run;
        k += run * (int)gridDim.x;
        nap = 32;
        start = global_ns();
      } else {
        if ((n & 15) == 0) {
          if (*abort_flag) break;
          const int late = __shfl_sync(0xffffffffu, global_ns() - start > IEC_WAIT_NS ? 1 : 0, 0);
          if (late) {
            if (lane == 0) {
              *abort_flag = 1;
              atomicOr(p.dev_err, DEV_ERR_WAIT_ROWS);
            }
            break;
          }
        }
        __nanosleep(nap);
        nap = nap < 512 ? 2 * nap : 512;
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
