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
#include "sm100.cuh"

#include <vector>

namespace iec {

namespace {

constexpr int TOK = 64, HD = 32;

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

// The window projection fused after P V (one head, c = 32): the output's
// rows times W (32 x 32, f16, pre-packed as each lane's mma.sync B
// fragments) plus the bias, added onto the map's pixels the window's tokens
// came from (swin.rs:176-181), as the separate projection's window-scatter
// epilogue adds them.
struct AttnProjArgs {
  const uint4* frag;   // [lane][2 k steps][4 n tiles][2] u32: 4 uint4 per lane
  const float* bias;   // [32]
  __half* y;           // planar map, the head's channels from plane plane0
  long long y_plane;
  int plane0;
  WindowMap wm;
};

__global__ void __launch_bounds__(128) window_attention_kernel(const __half* __restrict__ qkv, long long qkv_plane,
                                                               int c, const float* __restrict__ bias, int shifted,
                                                               int rows_w, int cols_w, __half* __restrict__ out,
                                                               long long out_plane, int* dev_err, AttnProjArgs pj) {
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
  // S = Q K^T for this warp's 16 rows: 8 key tiles of 8.
  float s[8][4];
#pragma unroll
  for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
  for (int kk = 0; kk < 2; kk++) {
    uint32_t a0, a1, a2, a3;
    ldsm_x4((uint32_t)__cvta_generic_to_shared(sq + (kk * 2 + (lane >> 4)) * TOK * 8 + (q0 + (lane & 15)) * 8), a0,
            a1, a2, a3);
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      // keys 8j .. 8j + 15, dims 16 kk .. 16 kk + 15: two B fragments
      uint32_t b0, b1, b2, b3;
      const int key = 8 * j + (lane & 7) + ((lane >> 4) << 3);
      const int grp = kk * 2 + ((lane >> 3) & 1);  // dims 8 grp .. 8 grp + 7
      ldsm_x4((uint32_t)__cvta_generic_to_shared(sk + grp * TOK * 8 + key * 8), b0, b1, b2, b3);
      mma16816(s[j], a0, a1, a2, a3, b0, b1);
      mma16816(s[j + 1], a0, a1, a2, a3, b2, b3);
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
  float o[4][4];
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
  const float inv[2] = {1.0f / sum[0], 1.0f / sum[1]};
  if (pj.frag) {
    // O as f16 A fragments (rounded where the separate launch stores it),
    // the head's 32 dims the reduction: two k steps of 16.
    uint32_t oa[2][4];
#pragma unroll
    for (int kk = 0; kk < 2; kk++) {
      oa[kk][0] = pack_half2(o[2 * kk][0] * inv[0], o[2 * kk][1] * inv[0]);
      oa[kk][1] = pack_half2(o[2 * kk][2] * inv[1], o[2 * kk][3] * inv[1]);
      oa[kk][2] = pack_half2(o[2 * kk + 1][0] * inv[0], o[2 * kk + 1][1] * inv[0]);
      oa[kk][3] = pack_half2(o[2 * kk + 1][2] * inv[1], o[2 * kk + 1][3] * inv[1]);
    }
    uint32_t bw[16];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const uint4 u = __ldg(pj.frag + lane * 4 + q);
      bw[4 * q] = u.x;
      bw[4 * q + 1] = u.y;
      bw[4 * q + 2] = u.z;
      bw[4 * q + 3] = u.w;
    }
    float pr[4][4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      pr[j][0] = pr[j][1] = pr[j][2] = pr[j][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < 2; kk++)
        mma16816(pr[j], oa[kk][0], oa[kk][1], oa[kk][2], oa[kk][3], bw[(kk * 4 + j) * 2], bw[(kk * 4 + j) * 2 + 1]);
    }
    // rows g and g + 8 of the warp's 16: window tokens q0 + g + 8 h
    const WindowMap& wm = pj.wm;
    const int ws = wm.ws, cols = wm.pad_w / ws, wy = win / cols, wx = win - wy * cols;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int tk = q0 + g + 8 * h;
      const int py = (wy * ws + tk / ws + wm.shift) % wm.pad_h, px = (wx * ws + tk % ws + wm.shift) % wm.pad_w;
      if (tk >= ws * ws || py >= wm.map_h || px >= wm.map_w) continue;
      const long long dest = (long long)py * wm.map_w + px;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int n = 8 * j + 2 * t;
        __half2* at = reinterpret_cast<__half2*>(pj.y + (pj.plane0 + j) * pj.y_plane + dest * 8 + 2 * t);
        const float2 old = __half22float2(*at);
        *at = __floats2half2_rn((pr[j][2 * h] + __ldg(pj.bias + n)) + old.x,
                                (pr[j][2 * h + 1] + __ldg(pj.bias + n + 1)) + old.y);
      }
    }
    return;
  }
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
               out, out_plane_elems, dev_err, AttnProjArgs{});
    IEC_CUDA(cudaGetLastError());
  });
}

void pack_attn_proj(AttnProj& ap, const std::vector<float>& w, const std::vector<float>& b) {
  if (w.size() != 32 * 32 || b.size() != 32) throw Error(ERR_WEIGHTS, "fused window projection: 32 x 32 weights");
  // lane l = 4 g + t, k step kk, n tile j: b0 = W[16 kk + 2 t (+1)][8 j + g],
  // b1 = W[16 kk + 2 t + 8 (+9)][8 j + g], each a pair of f16 (low = lower k)
  std::vector<uint16_t> frag(32 * 2 * 4 * 2 * 2);
  for (int l = 0; l < 32; l++)
    for (int kk = 0; kk < 2; kk++)
      for (int j = 0; j < 4; j++)
        for (int r = 0; r < 2; r++) {
          const int g = l >> 2, t = l & 3, k = 16 * kk + 2 * t + 8 * r, n = 8 * j + g;
          const size_t at = ((((size_t)l * 2 + kk) * 4 + j) * 2 + r) * 2;
          frag[at] = f32_to_half(w[(size_t)k * 32 + n]);
          frag[at + 1] = f32_to_half(w[(size_t)(k + 1) * 32 + n]);
        }
  ap.frag.reserve(frag.size() * 2);
  IEC_CUDA(cudaMemcpy(ap.frag.get(), frag.data(), frag.size() * 2, cudaMemcpyHostToDevice));
  ap.bias.reserve(32 * 4);
  IEC_CUDA(cudaMemcpy(ap.bias.get(), b.data(), 32 * 4, cudaMemcpyHostToDevice));
}

void window_attention_proj(const __half* qkv, long long qkv_plane_elems, int windows, const float* bias, bool shifted,
                           int rows_w, int cols_w, const AttnProj& ap, __half* y, long long y_plane_elems, int plane0,
                           const WindowMap& wm, int* dev_err, cudaStream_t s) {
  if ((qkv_plane_elems * 2) % 16 != 0) throw Error(ERR_INPUT, "attention planes must be 16-byte multiples");
  if (wm.ws < 1 || wm.ws > 8 || wm.pad_w % wm.ws || wm.pad_h % wm.ws || windows != (wm.pad_h / wm.ws) * (wm.pad_w / wm.ws))
    throw Error(ERR_INPUT, "window partition geometry is inconsistent");
  AttnProjArgs pj;
  pj.frag = ap.frag.as<uint4>();
  pj.bias = ap.bias.as<float>();
  pj.y = y;
  pj.y_plane = y_plane_elems;
  pj.plane0 = plane0;
  pj.wm = wm;
  dim3 grid(windows, 1);
  // attention as above, then the 64 x 32 x 32 projection per window; bytes:
  // q, k, v read once, the map's old values read and written (f16)
  timed_launch("window_attention_proj", (double)windows * (4.0 * 64 * 64 * 32 + 2.0 * 64 * 32 * 32),
               (double)windows * 64 * (3 * 32 + 2 * 32) * 2, s, [&] {
                 launch_pdl(window_attention_kernel, grid, 128, 0, s, qkv, qkv_plane_elems, 32, bias, shifted ? 1 : 0,
                            rows_w, cols_w, static_cast<__half*>(nullptr), 0LL, dev_err, pj);
                 IEC_CUDA(cudaGetLastError());
               });
}

}  // namespace iec
