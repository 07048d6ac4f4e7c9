// Host side of the general implicit GEMM (igemm_sm100.cuh): weight packing,
// tile-shape choice, tensor maps and launches, and the small bandwidth
// kernels around it (layout conversions, layer norm, window partition).
#pragma once

#include <cuda_fp16.h>

#include <algorithm>
#include <vector>

#include "runtime.h"

namespace iec {

// A layer's weights as the GEMM reads them: `ktot` x `n` (row-major, k =
// tap * cin + channel for a 3x3 convolution) re-packed per (N tile, K step)
// into the tensor-core core-matrix image, f16; bias (f32) kept beside.
struct PackedWeights {
  int n = 0, k = 0, ktot = 0, taps = 1, bn = 0, kb = 0, n_tiles = 0, ksteps = 0;
  DeviceBuffer w, bias;
  bool has_bias = false;
  // For an s x s grid of taps (s = 3, 5, 7; s bn <= 256), the same weights
  // packed per kernel row for halo tiles: [n tile][ky][k chunk][kb / 8]
  // [s bn][8], column dx bn + j of row ky holding tap (ky, dx)'s output j.
  DeviceBuffer rt;
  int rt_kw = 0;
};

// `w` is ktot x n row-major (ktot = taps * k), `bias` n floats or null.
void pack_weights(PackedWeights& pw, const std::vector<float>& w, int taps, int k, int n, const float* bias);

// Where a GEMM writes: planar f16 [planes][rows][8].
struct GemmOutSpec {
  int mode = 0;                // GemmOut
  __half* out = nullptr;
  long long plane_elems = 0;   // rows of the destination * 8
  int plane0 = 0;              // destination plane of column 0
  int map_h = 0, map_w = 0, shift = 0;  // OUT_WINDOW_ACCUM
  int win_ws = 0, pad_h = 0, pad_w = 0;  // window side (0: 8), padded map (0: the map)
  int dbl_w = 0, dbl_cout = 0;          // OUT_DOUBLE
  int phase_y = 0, phase_x = 0;         // OUT_PHASE, OUT_MAP
  // OUT_MAP (set by map_out): the stored map's geometry, output step, and
  // the optional sources added before / after the activation.
  int ostep = 1, dst_h = 0, dst_w = 0, dst_pad = 0, dst_split = 1, dst_pw = 0, dst_ph = 0;
  const __half* acc_src = nullptr;
  const __half* resid = nullptr;
};

// One tap of a convolution: the source pixel (y + dy, x + dx) of phase
// `phase` for output pixel (y, x).
struct Tap {
  int dy, dx, phase;
};

// A convolution's source: planar f16, `phases` images of w x h pixels one
// after another in every plane ([k / 8][phases][h][w][8]).
struct TapSource {
  const __half* ptr;
  long long plane_elems;  // elements between channel-group planes
  int w, h, phases;
};

// A map as LaMa's layers store it: h x w pixels reflect-padded by `pad`
// and, with split 2, stored as the four space-to-depth phases of the padded
// map ([k / 8][phase (py, px)][ph][pw][8]), which a stride-2 convolution
// reads as taps of stride 1.
struct MapGeom {
  int h = 0, w = 0, pad = 0, split = 1;
  int ph() const { return (h + 2 * pad + split - 1) / split; }
  int pw() const { return (w + 2 * pad + split - 1) / split; }
  long long plane_elems() const { return (long long)split * split * ph() * pw() * 8; }
  TapSource source(const __half* ptr, int plane0 = 0) const {
    return TapSource{ptr + (long long)plane0 * plane_elems(), plane_elems(), pw(), ph(), split * split};
  }
};

// An OUT_MAP destination: channel planes from `plane0` of `out` stored as `g`.
GemmOutSpec map_out(const MapGeom& g, __half* out, int plane0 = 0);

// out (h x w pixels) = act(sum over taps and channels + bias), the taps'
// weights row-major in tap order (pw packed with taps = taps.size()).
// `halo`: -1 chooses (halo tiles where they fit and fill the GPU), 0 never
// takes them (one box per tap), 1 takes them wherever they fit. Halo tiles
// need the row-tap packing (PackedWeights::rt) and a full grid of taps.
void gemm_taps(Device& dev, const PackedWeights& pw, const TapSource& src, const std::vector<Tap>& taps, int h, int w,
               int act, const GemmOutSpec& out, cudaStream_t s, int halo = -1);

// out = act(A x W + bias) over `m` rows of the planar input `a` (k / 8
// planes of a_plane_elems / 8 >= gemm_rows_alloc(m) rows each; the rows past
// m are read but their results dropped). With OUT_MAP, row m is pixel
// (m / w, m % w) of the output map (w = dst_w / ostep).
void gemm_rows(Device& dev, const PackedWeights& pw, const __half* a, long long a_plane_elems, int m, int act,
               const GemmOutSpec& out, cudaStream_t s);
inline int gemm_rows_alloc(int m) { return (std::max(m, 128) + 15) / 16 * 16; }

// out = act(conv3x3(map) + bias): `map` is planar f16 with k / 8 planes of
// h x w pixels (plane stride map_plane_elems), zero padding.
void gemm_conv3(Device& dev, const PackedWeights& pw, const __half* map, long long map_plane_elems, int h, int w,
                int act, const GemmOutSpec& out, cudaStream_t s);

// ---------------------------------------------------------- bandwidth kernels
// f32 rows [rows][c] <-> planar f16 [c / 8][rows][8] (c a multiple of 8).
void rows_to_planar(const float* src, int rows, int c, __half* dst, long long dst_plane_elems, cudaStream_t s);
void planar_to_rows(const __half* src, long long src_plane_elems, int rows, int c, float* dst, cudaStream_t s);

// A shifted-window partition: windows of ws x ws tokens tiling the map
// padded to pad_h x pad_w, each stored as a slot of 64 rows; token t of
// window (wy, wx) is pixel ((wy ws + t / ws + shift) % pad_h, (wx ws + t % ws
// + shift) % pad_w) (crates/scunet-native/src/swin.rs:170-181, 8 x 8;
// crates/birefnet-native/src/swin.rs:219-251, 7 x 7).
struct WindowMap {
  int ws = 8, pad_h = 0, pad_w = 0, map_h = 0, map_w = 0, shift = 0;
};

// Layer norm (eps 1e-5) of the c channels starting at plane `plane0` of
// `src` for every row, written as c / 8 planes of `dst`. With `window`, the
// rows are written in window order; slot rows past ws * ws and tokens past
// the map's edge are zero rows, not normalised (birefnet swin.rs:236-248).
void layer_norm_planar(const __half* src, long long src_plane_elems, int plane0, int rows, int c,
                       const float* gamma, const float* beta, __half* dst, long long dst_plane_elems,
                       const WindowMap* window, cudaStream_t s);

// Patch merging (crates/birefnet-native/src/swin.rs:366-404): each 2 x 2
// group of the grid x grid map `src` (c channels) concatenated in the order
// (0,0), (1,0), (0,1), (1,1) by (row, column) and layer-normalised over its
// 4c values, as (grid / 2)^2 rows of 4c / 8 planes of `dst`.
void merge_layer_norm_planar(const __half* src, long long src_plane_elems, int grid, int c, const float* gamma,
                             const float* beta, __half* dst, long long dst_plane_elems, cudaStream_t s);

// The fused transformer MLP (mlp_sm100.cuh): x += fc2(GELU(fc1(LN(x)))) over
// `rows` rows of the C channels at `x` (planar, plane stride plane_elems,
// planes of at least gemm_rows_alloc(rows) rows), C in {32, 64, 96, 128, 192,
// 256, 384}; LN eps 1e-5.
struct MlpWeights {
  int c = 0;
  DeviceBuffer w, params;
};
bool mlp_fits(int c);
bool mlp_preferred(int c);  // fused where it is the faster form
// w1: c x 4c (row k, column n), w2: 4c x c; biases and LayerNorm weights f32.
void pack_mlp(MlpWeights& mw, int c, const std::vector<float>& w1, const std::vector<float>& b1,
              const std::vector<float>& w2, const std::vector<float>& b2, const std::vector<float>& gamma,
              const std::vector<float>& beta);
void mlp_planar(Device& dev, const MlpWeights& mw, __half* x, long long plane_elems, int rows, cudaStream_t s);

// SCUNet's block boundary in one kernel (joinsplit_sm100.cuh): x += y Wj +
// bj, then y = x Ws + bs (the rounded f16 x, as separate launches read it
// back), over `rows` rows of the C channels at `x` and `y` (planar, plane
// stride plane_elems, planes of at least gemm_rows_alloc(rows) rows), C in
// {64, 128, 256}.
struct JoinSplitWeights {
  int c = 0;
  DeviceBuffer w, bias;
};
bool joinsplit_fits(int c);
// wj, ws: c x c (row k, column n); bj, bs: c.
void pack_joinsplit(JoinSplitWeights& jw, int c, const std::vector<float>& wj, const std::vector<float>& bj,
                    const std::vector<float>& ws, const std::vector<float>& bs);
void joinsplit_planar(Device& dev, const JoinSplitWeights& jw, __half* x, __half* y, long long plane_elems, int rows,
                      cudaStream_t s);

// LayerNorm and the window partition folded into one product
// (lnrows_sm100.cuh): out row r (window order, as layer_norm_planar's
// window mode writes) = LN(src[pixel(r)]) x W + b over `rows` rows, for the
// (c, n) shapes of the window attention's qkv layer: (32, 96), (64, 192),
// (96, 288), (128, 384).
struct LnRowsWeights {
  int c = 0, n = 0;
  DeviceBuffer w, params;
};
bool lnrows_fits(int c, int n);
// w: c x n (row k, column n); gamma, beta: c; bias: n.
void pack_lnrows(LnRowsWeights& lw, int c, int n, const std::vector<float>& w, const std::vector<float>& bias,
                 const std::vector<float>& gamma, const std::vector<float>& beta);
void lnrows_planar(Device& dev, const LnRowsWeights& lw, const __half* src, long long src_plane, int rows,
                   const WindowMap& wm, __half* out, long long out_plane, cudaStream_t s);

// Fused attention over 8 x 8 windows (attention.cu): `qkv` planar [3c / 8]
// [windows * 64][8], `bias` [classes][c / 32][64][64] f32 (classes 4 when
// `shifted`, else 1), output planar [c / 8][windows * 64][8].
// The bias tables ([n][64][64] f32: position bias plus shift mask per class
// and head) in the order window_attention reads them.
std::vector<float> attention_bias_layout(const std::vector<float>& tables);

void window_attention(const __half* qkv, long long qkv_plane_elems, int c, int windows, const float* bias,
                      bool shifted, int rows_w, int cols_w, __half* out, long long out_plane_elems, int* dev_err,
                      cudaStream_t s);

// A whole window attention half in one kernel, for one or two heads of 32
// channels (c 32 or 64): LN1, the qkv layer, attention with the bias tables
// of the heads (attention_bias_layout), the projection and the residual add
// onto `y` (planar, planes plane0 .. plane0 + c / 8 - 1) at each token's
// pixel under `wm`. In place of lnrows_planar, window_attention and the
// projection GEMM; the qkv rows and the attention output stay on the SM.
struct WindowBlockWeights {
  int c = 0;
  DeviceBuffer w, params;
  bool mlp = false;  // with one head: the block's MLP (LN2, fc1, GELU, fc2, residual) in the same kernel
  DeviceBuffer mlp_w, mlp_params;
};
bool window_block_fits(int c);
// wq: c x 3c (q, k, v columns), wp: c x c (row k, column n); biases, gamma, beta f32.
void pack_window_block(WindowBlockWeights& wb, int c, const std::vector<float>& wq, const std::vector<float>& bq,
                       const std::vector<float>& wp, const std::vector<float>& bp, const std::vector<float>& gamma,
                       const std::vector<float>& beta);
// The block's MLP folded in after the attention (c = 32 only): w1 c x 4c,
// w2 4c x c (row k, column n); biases, gamma, beta (LN2, eps 1e-5) f32.
void pack_window_block_mlp(WindowBlockWeights& wb, const std::vector<float>& w1, const std::vector<float>& b1,
                           const std::vector<float>& w2, const std::vector<float>& b2, const std::vector<float>& gamma,
                           const std::vector<float>& beta);
void window_block(Device& dev, const WindowBlockWeights& wb, const float* bias, bool shifted, int rows_w, int cols_w,
                  __half* y, long long y_plane_elems, int plane0, const WindowMap& wm, cudaStream_t s);

}  // namespace iec
