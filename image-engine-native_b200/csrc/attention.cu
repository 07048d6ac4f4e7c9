// Fused window attention: one CTA per (window, head), softmax(Q K^T / sqrt(32)
// + bias) V over the 64 tokens of an 8 x 8 window, head dimension 32.
//
// Semantics: crates/native-engine/src/attention.rs:25-111 (one head over one
// window: scores = (q / sqrt 32) . k + bias, the bias already holding the
// relative-position bias and the shift mask, -inf where tokens may not
// attend; softmax; weighted sum of values), with the tables of
// crates/scunet-native/src/swin.rs:26-50.
//
// Layout: qkv is the QKV GEMM's output, planar f16 [3c / 8][tokens][8]
// (queries, then keys, then values, head h at channels 32 h .. 32 h + 31 of
// each); the output is planar f16 [c / 8][tokens][8], ready as the
// projection GEMM's A operand. Four warps each own 16 query rows: Q K^T and
// P V run on mma.sync m16n8k16 (f16 in, f32 accumulate), the scores stay in
// registers between the two (the accumulator fragment of S is the A fragment
// of P), and the softmax uses quad shuffles for the row max and sum. The bias
// tables are stored in the order of those fragments (attention_bias_layout):
// a thread's 32 bias values are 8 float4 loads, each warp's load 512
// contiguous bytes (read element by element they kept L1 83 % busy).
#include <cuda_fp16.h>

#include "gemm.h"
#include "igemm_sm100.cuh"
#include "sm100.cuh"

#include <algorithm>
#include <vector>

namespace iec {

namespace {

constexpr int TOK = 64;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// One warp's 16 query rows (q0 .. q0 + 15) of one head over the window's 64
// keys: S = Q K^T (Q as the A fragments of its two k steps of 16 dims),
// scaled by 1 / sqrt(32), plus the bias (tb: the warp's entries of the
// window class's table, attention_bias_layout), softmax with quad shuffles
// for the row max and sum, O = P V (the accumulator fragments of S are the A
// fragments of P). sk, sv: keys and values as [4 dim groups][64][8]. o is
// unnormalised; inv holds the reciprocal sums of rows g and g + 8.
__device__ __forceinline__ void attend16(const uint32_t (&qa)[2][4], const __half* sk, const __half* sv,
                                         const float4* tb, int lane, float (&o)[4][4], float (&inv)[2]) {
  // S = Q K^T: 8 key tiles of 8.
  float s[8][4];
#pragma unroll
  for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
  for (int kk = 0; kk < 2; kk++) {
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      // keys 8j .. 8j + 15, dims 16 kk .. 16 kk + 15: two B fragments
      uint32_t b0, b1, b2, b3;
      const int key = 8 * j + (lane & 7) + ((lane >> 4) << 3);
      const int grp = kk * 2 + ((lane >> 3) & 1);  // dims 8 grp .. 8 grp + 7
      ldsm_x4((uint32_t)__cvta_generic_to_shared(sk + grp * TOK * 8 + key * 8), b0, b1, b2, b3);
      mma16816(s[j], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
      mma16816(s[j + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
    }
  }
  // Scale, bias, softmax (rows g and g + 8 of the warp's 16).
  const float scale = 0.17677669529663688f;  // 1 / sqrt(32)
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const float4 b4 = __ldg(tb + j * 32);
    const float bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
    for (int e = 0; e < 4; e++) {
      s[j][e] = s[j][e] * scale + bv[e];
      mx[e >> 1] = fmaxf(mx[e >> 1], s[j][e]);
    }
  }
#pragma unroll
  for (int h = 0; h < 2; h++) {
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
  }
  float sum[2] = {0.0f, 0.0f};
#pragma unroll
  for (int j = 0; j < 8; j++)
#pragma unroll
    for (int e = 0; e < 4; e++) {
      s[j][e] = __expf(s[j][e] - mx[e >> 1]);
      sum[e >> 1] += s[j][e];
    }
#pragma unroll
  for (int h = 0; h < 2; h++) {
    sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 1);
    sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 2);
  }
  // O = P V: tokens are the reduction, 4 dim tiles of 8.
#pragma unroll
  for (int j = 0; j < 4; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
#pragma unroll
  for (int kk = 0; kk < 4; kk++) {
    const uint32_t a0 = pack_half2(s[2 * kk][0], s[2 * kk][1]);
    const uint32_t a1 = pack_half2(s[2 * kk][2], s[2 * kk][3]);
    const uint32_t a2 = pack_half2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
    const uint32_t a3 = pack_half2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      // tokens 16 kk .. 16 kk + 15, dims 8 j .. 8 j + 15, transposed
      uint32_t b0, b1, b2, b3;
      const int tok = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int grp = j + (lane >> 4);  // dims 8 grp .. 8 grp + 7
      ldsm_x4_t((uint32_t)__cvta_generic_to_shared(sv + grp * TOK * 8 + tok * 8), b0, b1, b2, b3);
      mma16816(o[j], a0, a1, a2, a3, b0, b1);
      mma16816(o[j + 1], a0, a1, a2, a3, b2, b3);
    }
  }
  inv[0] = 1.0f / sum[0];
  inv[1] = 1.0f / sum[1];
}

__global__ void __launch_bounds__(128) window_attention_kernel(const __half* __restrict__ qkv, long long qkv_plane,
                                                               int c, const float* __restrict__ bias, int shifted,
                                                               int rows_w, int cols_w, __half* __restrict__ out,
                                                               long long out_plane, int* dev_err) {
  // Q, K, V of this head as 12 planes of [64 tokens][8]: plane 4 w + g is
  // channel group g of q (w 0), k (1) or v (2). Each is a contiguous 1 KB
  // run of the planar qkv map, brought by one bulk copy (the 8 x 8 blocks
  // ldmatrix reads are then 128 contiguous bytes: no bank conflicts).
  __shared__ __align__(128) __half sm[12 * TOK * 8];
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  const int win = blockIdx.x, head = blockIdx.y, heads = gridDim.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row0 = (long long)win * TOK;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();
  griddep_launch_dependents();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bar, 12 * TOK * 16);
    for (int j = 0; j < 12; j++) {
      const long long plane = (j >> 2) * (c / 8) + head * 4 + (j & 3);
      bulk_load(sm + j * TOK * 8, qkv + plane * qkv_plane + row0 * 8, TOK * 16, &bar);
    }
  }
  if (!mbar_wait(&bar, 0, &abort_flag, dev_err, DEV_ERR_WAIT_FULL)) return;
  const __half* sq = sm;
  const __half* sk = sm + 4 * TOK * 8;
  const __half* sv = sm + 8 * TOK * 8;

  // The bias table of this window's class (swin.rs:154-159).
  int cls = 0;
  if (shifted) cls = (win % cols_w == cols_w - 1 ? 1 : 0) + 2 * (win / cols_w == rows_w - 1 ? 1 : 0);
  const float4* tb = reinterpret_cast<const float4*>(bias + ((long long)cls * heads + head) * TOK * TOK) +
                     (threadIdx.x >> 5) * 8 * 32 + (threadIdx.x & 31);

  const int g = lane >> 2, t = lane & 3;
  const int q0 = warp * 16;
  // This warp's 16 query rows as the A fragments of two k steps.
  uint32_t qa[2][4];
#pragma unroll
  for (int kk = 0; kk < 2; kk++)
    ldsm_x4((uint32_t)__cvta_generic_to_shared(sq + (kk * 2 + (lane >> 4)) * TOK * 8 + (q0 + (lane & 15)) * 8),
            qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
  float o[4][4], inv[2];
  attend16(qa, sk, sv, tb, lane, o, inv);
#pragma unroll
  for (int j = 0; j < 4; j++)
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const long long tok = row0 + q0 + g + 8 * h;
      const int plane = head * 4 + j;
      *reinterpret_cast<uint32_t*>(out + plane * out_plane + tok * 8 + 2 * t) =
          pack_half2(o[j][2 * h] * inv[h], o[j][2 * h + 1] * inv[h]);
    }
}

// A whole window attention half in one persistent kernel, for one or two
// heads of 32 channels (C = 32 HEADS):
//
//   y[tokens] += proj(attention(qkv(LayerNorm(y[tokens]))))
//
// (crates/scunet-native/src/swin.rs:124-220: LN1, the shifted-window
// partition, the qkv layer, attention per head with the position bias and
// shift mask, the projection and the residual add). Each CTA takes windows
// in turn with four warps per head; warp (hd, tb) owns tokens 16 tb .. 16 tb
// + 15 of the window for head hd, two lanes per token:
//   * the token's C channels arrive from its pixel (16-byte groups of the
//     planar map; a window row's tokens are consecutive pixels), the next
//     window's already in registers while this one is computed;
//   * LayerNorm (eps 1e-5; mean, then the mean squared deviation) over the
//     lane pair; the normalised f16 row into the head's own copy of the A
//     tile and the raw row (the head's channels) into shared memory, both
//     rows of this warp only (__syncwarp between the steps); tokens past the
//     map or the window's ws x ws are zero rows and are not stored;
//   * the head's q, k and v = row x Wqkv + b on mma.sync m16n8k16, rounded to
//     f16 where the separate launches store them: Q stays in registers as
//     the attention's A fragments, K and V go to one of two shared-memory
//     buffers (one barrier);
//   * attention (attend16); with one head the f16 output is the
//     projection's A operand in registers, with two each warp writes its
//     head's output to one of two shared-memory buffers (a second barrier)
//     and projects its 16 rows over both heads into its head's 32 output
//     columns;
//   * plus the projection bias and the raw row, stored to the token's pixel.
// A warp is at most one window ahead of another, and only into the other
// buffer of each pair: it writes window i + 1's keys before the barrier that
// no warp passes before all have finished window i.
// The qkv rows and the attention output never reach global memory: per
// window 64 tokens x C channels are read and written once. Weights (qkv and
// projection as [C / 8][N][8] f16, the B operands' core-matrix images) stay
// in shared memory.
struct WindowBlockArgs {
  __half* y;              // planar map, the block's channels in planes plane0 .. plane0 + C / 8 - 1
  long long y_plane;
  int plane0;
  WindowMap wm;
  int windows, rows_w, cols_w, shifted;
  const uint8_t* w;       // Wqkv [C / 8][3 C][8] f16, then Wproj [C / 8][C][8] f16
  const float* params;    // gamma [C], beta [C], qkv bias [3 C], projection bias [C]
  const float* bias;      // attention bias tables (attention_bias_layout), [class][head]
  // One head only, optional: the block's MLP after the attention
  // (mlp_w: W1 [4][128][8] f16, then W2 [16][32][8] f16; mlp_params: gamma2
  // [32], beta2 [32], b1 [128], b2 [32]).
  const uint8_t* mlp_w;
  const float* mlp_params;
};

template <int HEADS, bool MLP>
struct WindowBlockSmem {
  static constexpr int C = 32 * HEADS, NQ = 3 * C, WARPS = 4 * HEADS, THREADS = 32 * WARPS;
  static constexpr int CTAS = HEADS == 1 ? 4 : 2;  // per SM (registers: 128 per thread)
  static constexpr int WQ_BYTES = C * NQ * 2, WP_BYTES = C * C * 2, PAR_FLOATS = 6 * C;
  static constexpr int TILE = C * TOK * 2;         // [C / 8][64][8] f16
  static constexpr int KV = 8 * TOK * 16;          // one head's K and V
  static constexpr int WQ_OFF = 0, WP_OFF = WQ_BYTES, PAR_OFF = WP_OFF + WP_BYTES;
  static constexpr int X_OFF = PAR_OFF + PAR_FLOATS * 4;       // HEADS copies of the normalised rows
  static constexpr int RAW_OFF = X_OFF + HEADS * TILE;         // the rows as read
  static constexpr int KV_OFF = RAW_OFF + TILE;                // [2][HEADS] K and V
  static constexpr int O_OFF = KV_OFF + 2 * HEADS * KV;        // [2] attention outputs (two heads)
  static constexpr int MW_OFF = O_OFF + (HEADS > 1 ? 2 * TILE : 0);  // the MLP's W1, W2 and parameters
  static constexpr int MW_BYTES = MLP ? 2 * C * 4 * C * 2 : 0, MPAR_FLOATS = MLP ? 7 * C : 0;
  static constexpr int MPAR_OFF = MW_OFF + MW_BYTES;
  static constexpr int TOTAL = MPAR_OFF + MPAR_FLOATS * 4;
  static_assert(!MLP || HEADS == 1, "the MLP folds into one-head blocks");
  static_assert(TOTAL * CTAS <= 220 * 1024, "window block shared memory");
};

template <int HEADS, bool MLP>
__global__ void __launch_bounds__(WindowBlockSmem<HEADS, MLP>::THREADS, WindowBlockSmem<HEADS, MLP>::CTAS)
    window_block_kernel(const WindowBlockArgs a) {
  using L = WindowBlockSmem<HEADS, MLP>;
  constexpr int C = L::C, NQ = L::NQ, G = C / 8;  // G: channel groups (planes)
  extern __shared__ __align__(128) uint8_t wb_smem[];
  __half* sw = reinterpret_cast<__half*>(wb_smem + L::WQ_OFF);
  __half* swp = reinterpret_cast<__half*>(wb_smem + L::WP_OFF);
  float* spar = reinterpret_cast<float*>(wb_smem + L::PAR_OFF);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = warp >> 2, tb = warp & 3;  // head, token block
  const int g = lane >> 2, t = lane & 3, q0 = tb * 16;
  __half* sx = reinterpret_cast<__half*>(wb_smem + L::X_OFF + hd * L::TILE);
  __half* sraw = reinterpret_cast<__half*>(wb_smem + L::RAW_OFF);
  // Weights first: no kernel writes them.
  {
    const uint4* src = reinterpret_cast<const uint4*>(a.w);
    uint4* dst = reinterpret_cast<uint4*>(wb_smem + L::WQ_OFF);
    for (int i = (int)threadIdx.x; i < (L::WQ_BYTES + L::WP_BYTES) / 16; i += L::THREADS) dst[i] = __ldg(src + i);
    for (int i = (int)threadIdx.x; i < L::PAR_FLOATS; i += L::THREADS) spar[i] = __ldg(a.params + i);
    if constexpr (MLP) {
      const uint4* msrc = reinterpret_cast<const uint4*>(a.mlp_w);
      uint4* mdst = reinterpret_cast<uint4*>(wb_smem + L::MW_OFF);
      for (int i = (int)threadIdx.x; i < L::MW_BYTES / 16; i += L::THREADS) mdst[i] = __ldg(msrc + i);
      float* mpar = reinterpret_cast<float*>(wb_smem + L::MPAR_OFF);
      for (int i = (int)threadIdx.x; i < L::MPAR_FLOATS; i += L::THREADS) mpar[i] = __ldg(a.mlp_params + i);
    }
  }
  __syncthreads();
  griddep_wait();
  griddep_launch_dependents();
  const float* gamma = spar;
  const float* beta = spar + C;
  const float* bqkv = spar + 2 * C;
  const float* bproj = spar + 5 * C;
  const WindowMap& wm = a.wm;
  const int ws = wm.ws, cols = wm.pad_w / ws;
  // This lane's token and channel half: token q0 + lane / 2, channel groups
  // [GH hp, GH hp + GH).
  constexpr int GH = G / 2;
  const int tk_own = q0 + (lane >> 1), hp = lane & 1;
  // A lane's tokens are the same in every window: their rows and columns
  // within the window once per launch (ty = -1 for the slot's padding
  // tokens past ws x ws); per window only its origin, shifted. The shifted
  // coordinate is below twice the padded size (shift < ws), so one
  // subtraction wraps it.
  struct Tok {
    int ty, tx;
  };
  auto tok = [&](int tk) -> Tok {
    if (tk >= ws * ws) return Tok{-1, 0};
    const int ty = tk / ws;
    return Tok{ty, tk - ty * ws};
  };
  const Tok t_own = tok(tk_own), t_out[2] = {tok(q0 + g), tok(q0 + g + 8)};
  // The pixel of a token of the window with shifted origin (oy, ox), or -1
  // when the token is padding.
  auto pixel = [&](int oy, int ox, Tok k) -> long long {
    int py = oy + k.ty, px = ox + k.tx;
    if (py >= wm.pad_h) py -= wm.pad_h;
    if (px >= wm.pad_w) px -= wm.pad_w;
    if (k.ty < 0 || py >= wm.map_h || px >= wm.map_w) return -1;
    return (long long)py * wm.map_w + px;
  };
  auto origin = [&](int win, int& oy, int& ox) {
    const int wy = win / cols;
    oy = wy * ws + wm.shift;
    ox = (win - wy * cols) * ws + wm.shift;
  };
  auto fetch = [&](int win, uint4 (&u)[GH]) {
#pragma unroll
    for (int q = 0; q < GH; q++) u[q] = make_uint4(0u, 0u, 0u, 0u);
    if (win >= a.windows) return;
    int oy, ox;
    origin(win, oy, ox);
    const long long px = pixel(oy, ox, t_own);
    if (px < 0) return;
    const __half* at = a.y + (long long)(a.plane0 + GH * hp) * a.y_plane + px * 8;
#pragma unroll
    for (int q = 0; q < GH; q++) u[q] = *reinterpret_cast<const uint4*>(at + q * a.y_plane);
  };
  uint4 u[GH];
  fetch(blockIdx.x, u);
  int it = 0;
  for (int win = blockIdx.x; win < a.windows; win += gridDim.x, it++) {
    int oy, ox;
    origin(win, oy, ox);
    const bool valid = pixel(oy, ox, t_own) >= 0;
    // the next window's rows, in flight while this one is computed
    uint4 nu[GH];
    fetch(win + gridDim.x, nu);
    // LayerNorm over the lane pair's C channels (gemm.cu layer_norm_rows'
    // formula), then the normalised and the raw rows into shared memory.
    {
      float v[8 * GH];
#pragma unroll
      for (int q = 0; q < GH; q++) {
        const __half2* h2 = reinterpret_cast<const __half2*>(&u[q]);
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const float2 f = __half22float2(h2[e]);
          v[8 * q + 2 * e] = f.x;
          v[8 * q + 2 * e + 1] = f.y;
        }
      }
      float sum = 0.0f;
#pragma unroll
      for (int e = 0; e < 8 * GH; e++) sum += v[e];
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      const float mean = sum / (float)C;
      float var = 0.0f;
#pragma unroll
      for (int e = 0; e < 8 * GH; e++) var += (v[e] - mean) * (v[e] - mean);
      var += __shfl_xor_sync(0xffffffffu, var, 1);
      const float inv = 1.0f / sqrtf(var / (float)C + 1e-5f);
      uint4* xr = reinterpret_cast<uint4*>(sx);
      uint4* rr = reinterpret_cast<uint4*>(sraw);
#pragma unroll
      for (int q = 0; q < GH; q++) {
        const int grp = GH * hp + q;
        float nv[8];
#pragma unroll
        for (int e = 0; e < 8; e++) nv[e] = valid ? (v[8 * q + e] - mean) * inv * gamma[8 * grp + e] + beta[8 * grp + e] : 0.0f;
        xr[grp * TOK + tk_own] = make_uint4(pack_half2(nv[0], nv[1]), pack_half2(nv[2], nv[3]),
                                            pack_half2(nv[4], nv[5]), pack_half2(nv[6], nv[7]));
        if (grp / 4 == hd) rr[grp * TOK + tk_own] = u[q];  // this head's channels
      }
    }
    __syncwarp();
    // This head's k and v, then its q, for the warp's 16 rows (local column
    // tile jl: q, k or v by jl / 4, the head's dims 8 (jl % 4) ..), the A
    // fragments loaded once: 32 accumulators live at a time, not 48.
    uint32_t xa[C / 16][4];
#pragma unroll
    for (int kk = 0; kk < C / 16; kk++)
      ldsm_x4((uint32_t)__cvta_generic_to_shared(sx + (kk * 2 + (lane >> 4)) * TOK * 8 + (q0 + (lane & 15)) * 8),
              xa[kk][0], xa[kk][1], xa[kk][2], xa[kk][3]);
    // local tiles j0 .. j0 + NT - 1 into acc, then + bias, rounded to f16
    auto qkv_tiles = [&](auto& acc, auto& hq, int j0) {
      constexpr int NT = sizeof(acc) / sizeof(acc[0]);
#pragma unroll
      for (int j = 0; j < NT; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < C / 16; kk++)
#pragma unroll
        for (int j = 0; j < NT; j += 2) {
          uint32_t b0, b1, b2, b3;
          const int jl = j0 + j, nt = (jl / 4) * G + 4 * hd + (jl % 4);  // global column tile
          const int n = 8 * nt + (lane & 7) + ((lane >> 4) << 3);
          const int grp = kk * 2 + ((lane >> 3) & 1);
          ldsm_x4((uint32_t)__cvta_generic_to_shared(sw + grp * NQ * 8 + n * 8), b0, b1, b2, b3);
          mma16816(acc[j], xa[kk][0], xa[kk][1], xa[kk][2], xa[kk][3], b0, b1);
          mma16816(acc[j + 1], xa[kk][0], xa[kk][1], xa[kk][2], xa[kk][3], b2, b3);
        }
#pragma unroll
      for (int j = 0; j < NT; j++) {
        const int jl = j0 + j, nt = (jl / 4) * G + 4 * hd + (jl % 4);
        const float2 b = *reinterpret_cast<const float2*>(bqkv + 8 * nt + 2 * t);
        hq[j][0] = pack_half2(acc[j][0] + b.x, acc[j][1] + b.y);
        hq[j][1] = pack_half2(acc[j][2] + b.x, acc[j][3] + b.y);
      }
    };
    // K and V into the buffer.
    __half* kv = reinterpret_cast<__half*>(wb_smem + L::KV_OFF + ((it & 1) * HEADS + hd) * L::KV);
    {
      float acc[8][4];
      uint32_t hkv[8][2];
      qkv_tiles(acc, hkv, 4);
#pragma unroll
      for (int j = 0; j < 8; j++)
#pragma unroll
        for (int h = 0; h < 2; h++)
          *reinterpret_cast<uint32_t*>(kv + (j * TOK + q0 + g + 8 * h) * 8 + 2 * t) = hkv[j][h];
    }
    // Q as the attention's A fragments.
    uint32_t qa[2][4];
    {
      float acc[4][4];
      uint32_t hq[4][2];
      qkv_tiles(acc, hq, 0);
#pragma unroll
      for (int kk = 0; kk < 2; kk++) {
        qa[kk][0] = hq[2 * kk][0];
        qa[kk][1] = hq[2 * kk][1];
        qa[kk][2] = hq[2 * kk + 1][0];
        qa[kk][3] = hq[2 * kk + 1][1];
      }
    }
    __syncthreads();
    int cls = 0;
    if (a.shifted) cls = (win % a.cols_w == a.cols_w - 1 ? 1 : 0) + 2 * (win / a.cols_w == a.rows_w - 1 ? 1 : 0);
    const float4* tbl =
        reinterpret_cast<const float4*>(a.bias + ((long long)cls * HEADS + hd) * TOK * TOK) + tb * 8 * 32 + lane;
    float o[4][4], inv[2];
    attend16(qa, kv, kv + 4 * TOK * 8, tbl, lane, o, inv);
    // The projection of the warp's 16 rows into this head's 32 output
    // columns (column tiles 4 hd .. 4 hd + 3), the attention output rounded
    // to f16 as the separate projection reads it.
    float pr[4][4];
#pragma unroll
    for (int j = 0; j < 4; j++) pr[j][0] = pr[j][1] = pr[j][2] = pr[j][3] = 0.0f;
    auto project = [&](int kk, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3) {
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t b0, b1, b2, b3;
        const int n = 8 * (4 * hd + j) + (lane & 7) + ((lane >> 4) << 3);
        const int grp = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4((uint32_t)__cvta_generic_to_shared(swp + grp * C * 8 + n * 8), b0, b1, b2, b3);
        mma16816(pr[j], a0, a1, a2, a3, b0, b1);
        mma16816(pr[j + 1], a0, a1, a2, a3, b2, b3);
      }
    };
    if constexpr (HEADS == 1) {
#pragma unroll
      for (int kk = 0; kk < 2; kk++)
        project(kk, pack_half2(o[2 * kk][0] * inv[0], o[2 * kk][1] * inv[0]),
                pack_half2(o[2 * kk][2] * inv[1], o[2 * kk][3] * inv[1]),
                pack_half2(o[2 * kk + 1][0] * inv[0], o[2 * kk + 1][1] * inv[0]),
                pack_half2(o[2 * kk + 1][2] * inv[1], o[2 * kk + 1][3] * inv[1]));
    } else {
      __half* so = reinterpret_cast<__half*>(wb_smem + L::O_OFF + (it & 1) * L::TILE);
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int h = 0; h < 2; h++)
          *reinterpret_cast<uint32_t*>(so + ((4 * hd + j) * TOK + q0 + g + 8 * h) * 8 + 2 * t) =
              pack_half2(o[j][2 * h] * inv[h], o[j][2 * h + 1] * inv[h]);
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < C / 16; kk++) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4((uint32_t)__cvta_generic_to_shared(so + (kk * 2 + (lane >> 4)) * TOK * 8 + (q0 + (lane & 15)) * 8),
                a0, a1, a2, a3);
        project(kk, a0, a1, a2, a3);
      }
    }
    if constexpr (MLP) {
      // The block's MLP on the warp's 16 rows (swin.rs:222-254), all in
      // registers: the rows after the attention, rounded to f16 as the
      // separate launches store them; LN2 over each row's 32 channels (the
      // four lanes of a quad); fc1 in four chunks of 32 hidden columns,
      // + b1, GELU, f16, which are the A fragments of fc2's k steps; fc2
      // accumulated; + b2 + the rows, stored to the pixels. Rounded where
      // mlp_sm100 rounds (normalised rows, hidden layer, sums).
      const __half* mw1 = reinterpret_cast<const __half*>(wb_smem + L::MW_OFF);
      const __half* mw2 = mw1 + 4 * 128 * 8;
      const float* mpar = reinterpret_cast<const float*>(wb_smem + L::MPAR_OFF);
      const float *g2 = mpar, *be2 = mpar + 32, *b1 = mpar + 64, *b2 = mpar + 192;
      float ya[4][4];
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int tk = q0 + g + 8 * h;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int n = 8 * j + 2 * t;
          const float2 old = __half22float2(*reinterpret_cast<const __half2*>(sraw + (j * TOK + tk) * 8 + 2 * t));
          const float2 r = __half22float2(
              __floats2half2_rn((pr[j][2 * h] + bproj[n]) + old.x, (pr[j][2 * h + 1] + bproj[n + 1]) + old.y));
          ya[j][2 * h] = r.x;
          ya[j][2 * h + 1] = r.y;
        }
      }
      // LN2 (mlp_sm100's formula: mean, the mean squared deviation) of rows g
      // (h 0) and g + 8 (h 1)
      float mean[2], inv2[2];
#pragma unroll
      for (int h = 0; h < 2; h++) {
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; j++) sum += ya[j][2 * h] + ya[j][2 * h + 1];
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        mean[h] = sum / 32.0f;
        float var = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; j++)
          var += (ya[j][2 * h] - mean[h]) * (ya[j][2 * h] - mean[h]) +
                 (ya[j][2 * h + 1] - mean[h]) * (ya[j][2 * h + 1] - mean[h]);
        var += __shfl_xor_sync(0xffffffffu, var, 1);
        var += __shfl_xor_sync(0xffffffffu, var, 2);
        inv2[h] = 1.0f / sqrtf(var / 32.0f + 1e-5f);
      }
      auto norm2 = [&](int j, int h) -> uint32_t {
        const int n = 8 * j + 2 * t;
        return pack_half2((ya[j][2 * h] - mean[h]) * inv2[h] * g2[n] + be2[n],
                          (ya[j][2 * h + 1] - mean[h]) * inv2[h] * g2[n + 1] + be2[n + 1]);
      };
      uint32_t la[2][4];
#pragma unroll
      for (int kk = 0; kk < 2; kk++) {
        la[kk][0] = norm2(2 * kk, 0);
        la[kk][1] = norm2(2 * kk, 1);
        la[kk][2] = norm2(2 * kk + 1, 0);
        la[kk][3] = norm2(2 * kk + 1, 1);
      }
      float p2[4][4];
#pragma unroll
      for (int j = 0; j < 4; j++) p2[j][0] = p2[j][1] = p2[j][2] = p2[j][3] = 0.0f;
#pragma unroll 2
      for (int hc = 0; hc < 4; hc++) {
        float a1[4][4];
#pragma unroll
        for (int j = 0; j < 4; j++) a1[j][0] = a1[j][1] = a1[j][2] = a1[j][3] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < 2; kk++)
#pragma unroll
          for (int jj = 0; jj < 4; jj += 2) {
            uint32_t b0, b1r, b2r, b3;
            const int n = 8 * (4 * hc + jj) + (lane & 7) + ((lane >> 4) << 3);
            const int grp = kk * 2 + ((lane >> 3) & 1);
            ldsm_x4((uint32_t)__cvta_generic_to_shared(mw1 + grp * 128 * 8 + n * 8), b0, b1r, b2r, b3);
            mma16816(a1[jj], la[kk][0], la[kk][1], la[kk][2], la[kk][3], b0, b1r);
            mma16816(a1[jj + 1], la[kk][0], la[kk][1], la[kk][2], la[kk][3], b2r, b3);
          }
        uint32_t hv[4][2];
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
          const float2 bb = *reinterpret_cast<const float2*>(b1 + 32 * hc + 8 * jj + 2 * t);
          const float2 h0 = gemm_gelu2(fadd2(make_float2(a1[jj][0], a1[jj][1]), bb));
          const float2 h1 = gemm_gelu2(fadd2(make_float2(a1[jj][2], a1[jj][3]), bb));
          hv[jj][0] = pack_half2(h0.x, h0.y);
          hv[jj][1] = pack_half2(h1.x, h1.y);
        }
#pragma unroll
        for (int kk = 0; kk < 2; kk++) {
          const int ks = 2 * hc + kk;  // fc2's k step (hidden 16 ks ..)
#pragma unroll
          for (int j = 0; j < 4; j += 2) {
            uint32_t b0, b1r, b2r, b3;
            const int n = 8 * j + (lane & 7) + ((lane >> 4) << 3);
            const int grp = ks * 2 + ((lane >> 3) & 1);
            ldsm_x4((uint32_t)__cvta_generic_to_shared(mw2 + grp * 32 * 8 + n * 8), b0, b1r, b2r, b3);
            mma16816(p2[j], hv[2 * kk][0], hv[2 * kk][1], hv[2 * kk + 1][0], hv[2 * kk + 1][1], b0, b1r);
            mma16816(p2[j + 1], hv[2 * kk][0], hv[2 * kk][1], hv[2 * kk + 1][0], hv[2 * kk + 1][1], b2r, b3);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const long long dest = pixel(oy, ox, t_out[h]);
        if (dest < 0) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int n = 8 * j + 2 * t;
          *reinterpret_cast<__half2*>(a.y + (a.plane0 + j) * a.y_plane + dest * 8 + 2 * t) =
              __floats2half2_rn((p2[j][2 * h] + b2[n]) + ya[j][2 * h], (p2[j][2 * h + 1] + b2[n + 1]) + ya[j][2 * h + 1]);
        }
      }
    } else {
      // rows g and g + 8 of the warp's 16: + bias + the raw row, to the pixel
  #pragma unroll
      for (int h = 0; h < 2; h++) {
        const int tk = q0 + g + 8 * h;
        const long long dest = pixel(oy, ox, t_out[h]);
        if (dest < 0) continue;
  #pragma unroll
        for (int j = 0; j < 4; j++) {
          const int grp = 4 * hd + j, n = 8 * grp + 2 * t;
          const float2 old = __half22float2(*reinterpret_cast<const __half2*>(sraw + (grp * TOK + tk) * 8 + 2 * t));
          *reinterpret_cast<__half2*>(a.y + (a.plane0 + grp) * a.y_plane + dest * 8 + 2 * t) =
              __floats2half2_rn((pr[j][2 * h] + bproj[n]) + old.x, (pr[j][2 * h + 1] + bproj[n + 1]) + old.y);
        }
      }
    }
#pragma unroll
    for (int q = 0; q < GH; q++) u[q] = nu[q];
    __syncwarp();
  }
}

}  // namespace

std::vector<float> attention_bias_layout(const std::vector<float>& tables) {
  if (tables.size() % (TOK * TOK) != 0) throw Error(ERR_INPUT, "bias tables are 64 x 64 each");
  std::vector<float> out(tables.size());
  for (size_t n = 0; n < tables.size() / (TOK * TOK); n++) {
    const float* src = tables.data() + n * TOK * TOK;
    float* dst = out.data() + n * TOK * TOK;
    // thread (warp w, lane l = 4 g + t), value (j, e): row 16 w + g + 8 (e / 2),
    // column 8 j + 2 t + e % 2 of the table, at [w][j][l][e]
    for (int w = 0; w < 4; w++)
      for (int j = 0; j < 8; j++)
        for (int l = 0; l < 32; l++)
          for (int e = 0; e < 4; e++) {
            const int r = 16 * w + (l >> 2) + 8 * (e >> 1), col = 8 * j + 2 * (l & 3) + (e & 1);
            dst[((w * 8 + j) * 32 + l) * 4 + e] = src[r * TOK + col];
          }
  }
  return out;
}

void window_attention(const __half* qkv, long long qkv_plane_elems, int c, int windows, const float* bias,
                      bool shifted, int rows_w, int cols_w, __half* out, long long out_plane_elems, int* dev_err,
                      cudaStream_t s) {
  if (c % 32 != 0) throw Error(ERR_INPUT, "attention channels must be a multiple of 32");
  dim3 grid(windows, c / 32);
  if ((qkv_plane_elems * 2) % 16 != 0) throw Error(ERR_INPUT, "attention planes must be 16-byte multiples");
  // per window and head: S = Q K^T and O = P V, 2 x 64 x 64 x 32 MACs;
  // bytes: q, k, v read and the output written once (f16)
  const double heads = (double)windows * (c / 32);
  timed_launch("window_attention_kernel", heads * 4.0 * 64 * 64 * 32, (double)windows * 64 * 4 * c * 2, s, [&] {
    launch_pdl(window_attention_kernel, grid, 128, 0, s, qkv, qkv_plane_elems, c, bias, shifted ? 1 : 0, rows_w, cols_w,
               out, out_plane_elems, dev_err);
    IEC_CUDA(cudaGetLastError());
  });
}

bool window_block_fits(int c) { return c == 32 || c == 64; }

void pack_window_block(WindowBlockWeights& wb, int c, const std::vector<float>& wq, const std::vector<float>& bq,
                       const std::vector<float>& wp, const std::vector<float>& bp, const std::vector<float>& gamma,
                       const std::vector<float>& beta) {
  if (!window_block_fits(c)) throw Error(ERR_INPUT, "fused window block of " + std::to_string(c) + " channels");
  const size_t nq = (size_t)3 * c;
  if (wq.size() != (size_t)c * nq || bq.size() != nq || wp.size() != (size_t)c * c || bp.size() != (size_t)c ||
      gamma.size() != (size_t)c || beta.size() != (size_t)c)
    throw Error(ERR_WEIGHTS, "window block weights of the wrong size");
  // Wqkv as [c / 8][3c][8], then Wproj as [c / 8][c][8]: the B operands'
  // core-matrix images, which ldmatrix reads as mma.sync B fragments
  std::vector<uint16_t> w((size_t)c * nq + (size_t)c * c);
  size_t at = 0;
  for (int g = 0; g < c / 8; g++)
    for (size_t n = 0; n < nq; n++)
      for (int e = 0; e < 8; e++) w[at++] = f32_to_half(wq[(size_t)(8 * g + e) * nq + n]);
  for (int g = 0; g < c / 8; g++)
    for (int n = 0; n < c; n++)
      for (int e = 0; e < 8; e++) w[at++] = f32_to_half(wp[(size_t)(8 * g + e) * c + n]);
  std::vector<float> par;
  for (const std::vector<float>* v : {&gamma, &beta, &bq, &bp}) par.insert(par.end(), v->begin(), v->end());
  wb.c = c;
  wb.w.reserve(w.size() * 2);
  wb.params.reserve(par.size() * 4);
  IEC_CUDA(cudaMemcpy(wb.w.get(), w.data(), w.size() * 2, cudaMemcpyHostToDevice));
  IEC_CUDA(cudaMemcpy(wb.params.get(), par.data(), par.size() * 4, cudaMemcpyHostToDevice));
}

void pack_window_block_mlp(WindowBlockWeights& wb, const std::vector<float>& w1, const std::vector<float>& b1,
                           const std::vector<float>& w2, const std::vector<float>& b2, const std::vector<float>& gamma,
                           const std::vector<float>& beta) {
  const int c = wb.c, hid = 4 * c;
  if (c != 32) throw Error(ERR_INPUT, "the MLP folds into one-head window blocks only");
  if (w1.size() != (size_t)c * hid || w2.size() != (size_t)hid * c || b1.size() != (size_t)hid ||
      b2.size() != (size_t)c || gamma.size() != (size_t)c || beta.size() != (size_t)c)
    throw Error(ERR_WEIGHTS, "window block MLP weights of the wrong size");
  // W1 as [c / 8][4c][8], then W2 as [4c / 8][c][8]: B operands' core-matrix images
  std::vector<uint16_t> w((size_t)2 * c * hid);
  size_t at = 0;
  for (int g = 0; g < c / 8; g++)
    for (int n = 0; n < hid; n++)
      for (int e = 0; e < 8; e++) w[at++] = f32_to_half(w1[(size_t)(8 * g + e) * hid + n]);
  for (int g = 0; g < hid / 8; g++)
    for (int n = 0; n < c; n++)
      for (int e = 0; e < 8; e++) w[at++] = f32_to_half(w2[(size_t)(8 * g + e) * c + n]);
  std::vector<float> par;
  for (const std::vector<float>* v : {&gamma, &beta, &b1, &b2}) par.insert(par.end(), v->begin(), v->end());
  wb.mlp_w.reserve(w.size() * 2);
  wb.mlp_params.reserve(par.size() * 4);
  IEC_CUDA(cudaMemcpy(wb.mlp_w.get(), w.data(), w.size() * 2, cudaMemcpyHostToDevice));
  IEC_CUDA(cudaMemcpy(wb.mlp_params.get(), par.data(), par.size() * 4, cudaMemcpyHostToDevice));
  wb.mlp = true;
}

namespace {

template <int HEADS, bool MLP>
void launch_window_block(int device, int sms, const WindowBlockArgs& a, cudaStream_t s) {
  using L = WindowBlockSmem<HEADS, MLP>;
  static bool prepared[64] = {};
  if (!prepared[device & 63]) {
    IEC_CUDA(cudaFuncSetAttribute(window_block_kernel<HEADS, MLP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  L::TOTAL));
    prepared[device & 63] = true;
  }
  launch_pdl(window_block_kernel<HEADS, MLP>, std::min(a.windows, sms * L::CTAS), L::THREADS, (size_t)L::TOTAL, s, a);
  IEC_CUDA(cudaGetLastError());
}

}  // namespace

void window_block(Device& dev, const WindowBlockWeights& wb, const float* bias, bool shifted, int rows_w, int cols_w,
                  __half* y, long long y_plane_elems, int plane0, const WindowMap& wm, cudaStream_t s) {
  const int c = wb.c;
  if (!window_block_fits(c)) throw Error(ERR_INPUT, "fused window block shape");
  if (wm.ws < 1 || wm.ws > 8 || wm.pad_w % wm.ws || wm.pad_h % wm.ws || wm.pad_h < wm.map_h || wm.pad_w < wm.map_w ||
      wm.shift < 0 || wm.shift >= wm.ws)
    throw Error(ERR_INPUT, "window partition geometry is inconsistent");
  if ((y_plane_elems * 2) % 16 != 0) throw Error(ERR_INPUT, "map planes must be 16-byte multiples");
  WindowBlockArgs a{};
  a.y = y;
  a.y_plane = y_plane_elems;
  a.plane0 = plane0;
  a.wm = wm;
  a.windows = (wm.pad_h / wm.ws) * (wm.pad_w / wm.ws);
  a.rows_w = rows_w;
  a.cols_w = cols_w;
  a.shifted = shifted ? 1 : 0;
  a.w = wb.w.as<uint8_t>();
  a.params = wb.params.as<float>();
  a.bias = bias;
  if (wb.mlp) {
    a.mlp_w = wb.mlp_w.as<uint8_t>();
    a.mlp_params = wb.mlp_params.as<float>();
  }
  const double heads = c / 32;
  char name[48];
  snprintf(name, sizeof name, wb.mlp ? "window_block<%d>+mlp" : "window_block<%d>", c / 32);
  // per window: qkv (64 x 3c x c), attention (2 x 64 x 64 x 32 per head),
  // the projection (64 x c x c) and with the MLP fc1 and fc2 (2 x 64 x c x
  // 4c); bytes: the tokens' rows read and written
  timed_launch(name,
               (double)a.windows * (2.0 * 64 * 3 * c * c + heads * 4.0 * 64 * 64 * 32 + 2.0 * 64 * c * c +
                                    (wb.mlp ? 4.0 * 64 * c * 4 * c : 0.0)),
               (double)a.windows * 64 * c * 2 * 2, s, [&] {
                 if (c == 32 && wb.mlp) return launch_window_block<1, true>(dev.ordinal(), dev.sms(), a, s);
                 if (c == 32) return launch_window_block<1, false>(dev.ordinal(), dev.sms(), a, s);
                 return launch_window_block<2, false>(dev.ordinal(), dev.sms(), a, s);
               });
}

}  // namespace iec
