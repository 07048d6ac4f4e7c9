// BiRefNet-lite on the CUDA backend (see birefnet.h).
//
// lib.rs:134-172: the normalised image and its aligned-corner half-size copy
// go through the Swin-T backbone (swin.rs:162-215); the decoder
// (decoder.rs:790-926) concatenates each level's two runs (the half-size one
// resized), squeezes the four levels at 1/32, and runs blocks 4..1 upwards,
// each fed the previous output (resized and added onto the level's lateral
// 1x1 convolution) and the image cut into patches; the head ends in f32.
//
// Planar f16 maps `[C/8][pixels][8]` throughout (rows y * w + x); every
// concatenation is a plane offset. A Swin block: LayerNorm + window gather
// into 64-row slots (49 tokens, the rest zero rows), qkv GEMM, fused window
// attention (the 64 x 64 bias tables carry the reference's 49 x 49 tables,
// its -100 shift masks, and -inf for the slots' padding keys), projection
// GEMM scattered back onto the tokens, LayerNorm, fc1 + GELU, fc2 added on.
#include "birefnet.h"

#include <algorithm>
#include <cmath>
#include <cstring>

#include "igemm_sm100.cuh"

namespace iec {

namespace {

constexpr int WS = 7, SHIFT = 3, NTOK = 49, INTER = 64, BRANCH = 256;
constexpr int STAGE_C[4] = {96, 192, 384, 768}, STAGE_D[4] = {2, 2, 6, 2};
constexpr int SIZES[4] = {1, 1, 3, 7};
constexpr int LEVELS[4][2] = {{1728, 768}, {960, 384}, {480, 192}, {240, 96}};
constexpr int PATCH_C[4] = {3072, 768, 192, 48};   // patches5..2 input channels
constexpr int PATCH_OUT[4] = {192, 192, 96, 48};
__constant__ float MEAN[3] = {0.485f, 0.456f, 0.406f}, STDV[3] = {0.229f, 0.224f, 0.225f};
// Full-resolution tables: composed 5x5 [75], conv1 [27 * 64], bias1 [64],
// conv_out [9 * 64], then bias_out and the composed bias.
constexpr int FR_COMPOSED = 0, FR_CONV1 = 75, FR_BIAS1 = FR_CONV1 + 27 * 64, FR_OUT = FR_BIAS1 + 64,
              FR_SCALARS = FR_OUT + 9 * 64, FR_TOTAL = FR_SCALARS + 2;

int blocks_for(long long n, int sms) {
  return (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, (long long)sms * 16));
}

long long pe(long long pixels) { return (long long)gemm_rows_alloc((int)pixels) * 8; }

__device__ __forceinline__ void load8(const __half* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int e = 0; e < 4; e++) {
    const float2 f = __half22float2(h[e]);
    v[2 * e] = f.x;
    v[2 * e + 1] = f.y;
  }
}

__device__ __forceinline__ void store8(__half* p, const float* v) {
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; e++) {
    __half2 h2 = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
    w[e] = *reinterpret_cast<uint32_t*>(&h2);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ float sigmoid_f(float v) {
  // math.rs:33-39: from exp(-|x|), so that neither tail cancels.
  const float e = expf(-fabsf(v)), s = e / (e + 1.0f);
  return v > 0.0f ? 1.0f - s : s;
}

// decoder.rs:462-476: source pixels and weights of output coordinate `out`.
__device__ __forceinline__ void axis(int out, int len_in, int len_out, int& i0, int& i1, float& w0, float& w1) {
  float pos = len_out == 1 ? 0.0f : (float)out * (float)(len_in - 1) / (float)(len_out - 1);
  pos = fminf(fmaxf(pos, 0.0f), (float)(len_in - 1));
  i0 = (int)pos;
  i1 = min(i0 + 1, len_in - 1);
  if (i0 == i1) {
    w0 = 0.5f;
    w1 = 0.5f;
  } else {
    w0 = fabsf(pos - (float)i0);
    w1 = fabsf(pos - (float)i1);
  }
}

// lib.rs:116-133: 8-bit RGB through the ImageNet normalisation (or a copy of
// an already normalised image).
__global__ void bir_prep(const void* __restrict__ src, int u8, long long n, float* __restrict__ dst) {
  griddep_wait();
  griddep_launch_dependents();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    if (u8) {
      const int c = (int)(i % 3);
      dst[i] = ((float)static_cast<const uint8_t*>(src)[i] / 255.0f - MEAN[c]) / STDV[c];
    } else {
      dst[i] = static_cast<const float*>(src)[i];
    }
  }
}

// decoder.rs:443-521 on an f32 NHWC map (the half-size image).
__global__ void bir_resize_f32(const float* __restrict__ src, int sh, int sw, int c, float* __restrict__ dst, int dh,
                               int dw) {
  griddep_wait();
  griddep_launch_dependents();
  const long long n = (long long)dh * dw;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int y = (int)(i / dw), x = (int)(i % dw);
    int y1, y2, x1, x2;
    float dy1, dy2, dx1, dx2;
    axis(y, sh, dh, y1, y2, dy1, dy2);
    axis(x, sw, dw, x1, x2, dx1, dx2);
    for (int j = 0; j < c; j++) {
      const float p11 = src[((long long)y1 * sw + x1) * c + j], p21 = src[((long long)y1 * sw + x2) * c + j];
      const float p12 = src[((long long)y2 * sw + x1) * c + j], p22 = src[((long long)y2 * sw + x2) * c + j];
      dst[i * c + j] = dx2 * dy2 * p11 + dx1 * dy2 * p21 + dx2 * dy1 * p12 + dx1 * dy1 * p22;
    }
  }
}

// The same resize on planar f16 maps, `planes` channel groups, optionally
// added onto the destination (decoder.rs:500-519).
__global__ void bir_resize_planar(const __half* __restrict__ src, long long src_plane, int sh, int sw,
                                  __half* __restrict__ dst, long long dst_plane, int dh, int dw, int planes, int add) {
  griddep_wait();
  griddep_launch_dependents();
  const long long n = (long long)dh * dw * planes;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int q = (int)(i / ((long long)dh * dw));
    const long long p = i - (long long)q * dh * dw;
    const int y = (int)(p / dw), x = (int)(p % dw);
    int y1, y2, x1, x2;
    float dy1, dy2, dx1, dx2;
    axis(y, sh, dh, y1, y2, dy1, dy2);
    axis(x, sw, dw, x1, x2, dx1, dx2);
    const __half* s = src + q * src_plane;
    float p11[8], p21[8], p12[8], p22[8], v[8];
    load8(s + ((long long)y1 * sw + x1) * 8, p11);
    load8(s + ((long long)y1 * sw + x2) * 8, p21);
    load8(s + ((long long)y2 * sw + x1) * 8, p12);
    load8(s + ((long long)y2 * sw + x2) * 8, p22);
    __half* d = dst + q * dst_plane + p * 8;
    float old[8];
    if (add) load8(d, old);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float r = dx2 * dy2 * p11[j] + dx1 * dy2 * p21[j] + dx2 * dy1 * p12[j] + dx1 * dy1 * p22[j];
      v[j] = add ? old[j] + r : r;
    }
    store8(d, v);
  }
}

// One bir_resize_planar launch, recorded for launch timing with its bytes:
// the source read once, the destination written (and read when adding).
void launch_resize(const __half* src, long long src_plane, int sh, int sw, __half* dst, long long dst_plane, int dh,
                   int dw, int c8, int add, int sms, cudaStream_t s) {
  const double bytes = ((double)sh * sw + (double)dh * dw * (1 + add)) * c8 * 16;
  timed_launch("bir_resize_planar", 0.0, bytes, s, [&] {
    launch_pdl(bir_resize_planar, blocks_for((long long)dh * dw * c8, sms), 256, 0, s, src, src_plane, sh, sw, dst,
               dst_plane, dh, dw, c8, add);
  });
}

// swin.rs:188-204: each 4 x 4 patch's 48 values, (ky, kx, c) order.
__global__ void bir_embed_gather(const float* __restrict__ img, int side, __half* __restrict__ dst, long long plane) {
  griddep_wait();
  griddep_launch_dependents();
  const int grid = side / 4;
  const long long n = (long long)grid * grid * 6;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int g = (int)(i % 6);
    const long long t = i / 6;
    const int ty = (int)(t / grid), tx = (int)(t % grid);
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const int j = 8 * g + e, ky = j / 12, kx = (j % 12) / 3, c = j % 3;
      v[e] = img[(((long long)ty * 4 + ky) * side + tx * 4 + kx) * 3 + c];
    }
    store8(dst + g * plane + t * 8, v);
  }
}

// decoder.rs:144-150: per-channel sums of a 64-channel map (f32 partials,
// f64 totals).
__global__ void bir_channel_sums(const __half* __restrict__ t, long long plane, long long pixels,
                                 double* __restrict__ sums) {
  griddep_wait();
  griddep_launch_dependents();
  const int q = blockIdx.y;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x; p < pixels;
       p += (long long)gridDim.x * blockDim.x) {
    float v[8];
    load8(t + q * plane + p * 8, v);
#pragma unroll
    for (int e = 0; e < 8; e++) acc[e] += v[e];
  }
#pragma unroll
  for (int e = 0; e < 8; e++) {
    float v = acc[e];
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(&sums[q * 8 + e], (double)v);
  }
}

// decoder.rs:141-165: the pooling branch (mean, 1x1 to 256, ReLU) and its
// share of conv1, as the bias of conv1 for this map. One block of 256
// threads; the 256-term products of the second step are split in four
// quarters of 64 terms (one per 64 threads), added in quarter order.
__global__ void __launch_bounds__(256) bir_aspp_bias(const double* __restrict__ sums, double pixels,
                                                     const float* __restrict__ pool_w, const float* __restrict__ pool_b,
                                                     const float* __restrict__ conv1_pool,
                                                     const float* __restrict__ conv1_bias, float* __restrict__ bias) {
  static_assert(BRANCH == 256 && BRANCH == 4 * INTER, "one thread per pooled channel, four quarters of conv1's");
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float mean[INTER], pooled[BRANCH], part[4][INTER];
  const int t = threadIdx.x;
  if (t < INTER) mean[t] = (float)(sums[t] / pixels);
  __syncthreads();
  {
    float p = pool_b[t];
#pragma unroll 16
    for (int c = 0; c < INTER; c++) p += mean[c] * pool_w[c * BRANCH + t];
    pooled[t] = p > 0.0f ? p : 0.0f;
  }
  __syncthreads();
  {
    const int q = t / INTER, o = t % INTER;
    float b = 0.0f;
#pragma unroll 16
    for (int j = q * INTER; j < (q + 1) * INTER; j++) b += pooled[j] * conv1_pool[j * INTER + o];
    part[q][o] = b;
  }
  __syncthreads();
  if (t < INTER) bias[t] = conv1_bias[t] + part[0][t] + part[1][t] + part[2][t] + part[3][t];
}

// decoder.rs:243-313: the deformable convolution's input: for pixel p and
// tap k of a size x size kernel, the 64 channels of `t` sampled bilinearly
// at the tap moved by its offset, times 2 sigmoid(modulator). `offs` holds
// the offset convolution's 3 taps channels (y, x per tap, then the logits).
// blockIdx.y is (tap, run of GPT of the 8 channel groups): a thread computes
// the sample point, corner weights and modulator of its (pixel, tap) once
// and gathers its run's GPT channel groups with them. The threads of a block take
// consecutive pixels, so a warp's 16-byte stores fill 512 contiguous bytes of
// each output plane and its neighbour loads stay within a few rows.
template <int GPT>
__global__ void bir_deform_sample(const __half* __restrict__ t, long long t_plane, int height, int width, int size,
                                  const __half* __restrict__ offs, long long offs_plane, __half* __restrict__ out,
                                  long long out_plane) {
  griddep_wait();
  griddep_launch_dependents();
  constexpr int PARTS = 8 / GPT;
  const int taps = size * size;
  const int tap = (int)blockIdx.y / PARTS, g0 = ((int)blockIdx.y % PARTS) * GPT;
  const long long n = (long long)height * width;
  const float hs = (float)(size / 2), hf = (float)height, wf = (float)width;
  const float ky = (float)(tap / size), kx = (float)(tap % size);
  auto chan = [&](int c) { return offs + (long long)(c / 8) * offs_plane + (c % 8); };
  // (y, x) of a tap are channels 2 tap and 2 tap + 1: one pixel group, one
  // 4-byte load
  const __half* off_yx = chan(2 * tap);
  const __half* off_m = chan(2 * taps + tap);
  const __half* src = t + g0 * t_plane;
  __half* dst = out + (long long)(tap * 8 + g0) * out_plane;
  for (long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x; p < n; p += (long long)gridDim.x * blockDim.x) {
    const int y = (int)(p / width), x = (int)(p % width);
    const float2 oyx = __half22float2(*reinterpret_cast<const __half2*>(off_yx + p * 8));
    const float py = ((float)y - hs + ky) + oyx.x;
    const float px = ((float)x - hs + kx) + oyx.y;
    const float m = 2.0f * sigmoid_f(__half2float(off_m[p * 8]));
    float acc[GPT][8];
#pragma unroll
    for (int q = 0; q < GPT; q++)
#pragma unroll
      for (int e = 0; e < 8; e++) acc[q][e] = 0.0f;
    if (!(py <= -1.0f || py >= hf || px <= -1.0f || px >= wf)) {
      const float y0f = floorf(py), x0f = floorf(px);
      const float ly = py - y0f, lx = px - x0f, hy = 1.0f - ly, hx = 1.0f - lx;
      const int y0 = (int)y0f, x0 = (int)x0f;
      const int cy[4] = {y0, y0, y0 + 1, y0 + 1}, cx[4] = {x0, x0 + 1, x0, x0 + 1};
      const float cw[4] = {hy * hx, hy * lx, ly * hx, ly * lx};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        if (cy[k] < 0 || cx[k] < 0 || cy[k] >= height || cx[k] >= width) continue;
        const __half* at = src + ((long long)cy[k] * width + cx[k]) * 8;
#pragma unroll
        for (int q = 0; q < GPT; q++) {
          float v[8];
          load8(at + q * t_plane, v);
#pragma unroll
          for (int e = 0; e < 8; e++) acc[q][e] += cw[k] * v[e];
        }
      }
    }
#pragma unroll
    for (int q = 0; q < GPT; q++) {
#pragma unroll
      for (int e = 0; e < 8; e++) acc[q][e] *= m;
      store8(dst + q * out_plane + p * 8, acc[q]);
    }
  }
}

// decoder.rs:382-404: the gate sigmoid(b + w . g16) multiplied onto the
// block's output (`planes` channel groups). Items are (pixel, run of up to 4
// planes), consecutive threads on consecutive pixels; each item recomputes
// its pixel's gate (two 16-byte loads, cache hits) so that its four plane
// loads are in flight together.
__global__ void bir_gate(const __half* __restrict__ g16, long long g_plane, const float* __restrict__ w, float b,
                         __half* __restrict__ out, long long out_plane, int planes, long long pixels) {
  griddep_wait();
  griddep_launch_dependents();
  const int runs = (planes + 3) / 4;
  const long long n = pixels * runs;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int q0 = (int)(i / pixels) * 4;
    const long long p = i % pixels;
    float v[16];
    load8(g16 + p * 8, v);
    load8(g16 + g_plane + p * 8, v + 8);
    float s = b;
    for (int k = 0; k < 16; k++) s = s + v[k] * w[k];
    const float gate = sigmoid_f(s);
    float o[4][8];
#pragma unroll
    for (int j = 0; j < 4; j++)
      if (q0 + j < planes) load8(out + (q0 + j) * out_plane + p * 8, o[j]);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      if (q0 + j >= planes) continue;
#pragma unroll
      for (int e = 0; e < 8; e++) o[j][e] *= gate;
      store8(out + (q0 + j) * out_plane + p * 8, o[j]);
    }
  }
}

// decoder.rs:564-583: the image cut into g x g patches of size x size
// pixels, patch (gy, gx) of colour c as channel (c g + gy) g + gx.
__global__ void bir_patches(const float* __restrict__ img, int side, int size, __half* __restrict__ dst,
                            long long plane, int out_groups) {
  griddep_wait();
  griddep_launch_dependents();
  const int g = side / size, groups = 3 * g * g / 8;
  const long long n = (long long)size * size * out_groups;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int q = (int)(i % out_groups);
    const long long p = i / out_groups;
    const int y = (int)(p / size), x = (int)(p % size);
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const int ch = 8 * q + e, c = ch / (g * g), rem = ch % (g * g), gy = rem / g, gx = rem % g;
      v[e] = q < groups ? img[(((long long)gy * size + y) * side + gx * size + x) * 3 + c] : 0.0f;
    }
    store8(dst + q * plane + p * 8, v);
  }
}

// decoder.rs:882-898: the head's 1x1 convolution to one channel, in f32.
__global__ void bir_head(const __half* __restrict__ x, long long plane, const float* __restrict__ w, long long pixels,
                         float* __restrict__ low) {
  griddep_wait();
  griddep_launch_dependents();
  for (long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x; p < pixels;
       p += (long long)gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int q = 0; q < 12; q++) {
      float v[8];
      load8(x + q * plane + p * 8, v);
#pragma unroll
      for (int e = 0; e < 8; e++) s = fmaf(v[e], w[q * 8 + e], s);
    }
    low[p] = s;
  }
}

// decoder.rs:899-925 and 637-752: logits = head bias + the low-resolution
// logits resized to the image + the full-resolution branch, here as the
// composed 5x5 convolution; border pixels get the branch from bir_edges.
// A thread takes 4 horizontally adjacent pixels: each row of their 5 x 8
// input window is loaded once and serves all four (the per-pixel sums run
// in the same order as one pixel at a time), the 75 weights sit in shared
// memory.
__global__ void __launch_bounds__(256) bir_logits(const float* __restrict__ low, int lg, const float* __restrict__ img,
                                                  int side, const float* __restrict__ fr, float head_b,
                                                  float* __restrict__ logits) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float wk[76];
  if (threadIdx.x < 76) wk[threadIdx.x] = fr[threadIdx.x < 75 ? FR_COMPOSED + threadIdx.x : FR_SCALARS + 1];
  __syncthreads();
  const int quads = (side + 3) / 4;
  const long long n = (long long)side * quads;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int y = (int)(i / quads), x0 = (int)(i % quads) * 4;
    float acc[4] = {wk[75], wk[75], wk[75], wk[75]};
#pragma unroll
    for (int dy = 0; dy < 5; dy++) {
      const int py = y + dy - 2;
      float r[8][3];
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const int px = x0 + k - 2;
        const bool in = py >= 0 && px >= 0 && py < side && px < side;
        const float* q = img + ((long long)py * side + px) * 3;
        r[k][0] = in ? q[0] : 0.0f;
        r[k][1] = in ? q[1] : 0.0f;
        r[k][2] = in ? q[2] : 0.0f;
      }
#pragma unroll
      for (int dx = 0; dx < 5; dx++) {
        const int e = dy * 5 + dx;
        const float w0 = wk[e * 3], w1 = wk[e * 3 + 1], w2 = wk[e * 3 + 2];
#pragma unroll
        for (int j = 0; j < 4; j++) acc[j] += w0 * r[j + dx][0] + w1 * r[j + dx][1] + w2 * r[j + dx][2];
      }
    }
    int y1, y2;
    float dy1, dy2;
    axis(y, lg, side, y1, y2, dy1, dy2);
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int x = x0 + j;
      if (x >= side) break;
      int x1, x2;
      float dx1, dx2;
      axis(x, lg, side, x1, x2, dx1, dx2);
      const float v = dx2 * dy2 * low[y1 * lg + x1] + dx1 * dy2 * low[y1 * lg + x2] + dx2 * dy1 * low[y2 * lg + x1] +
                      dx1 * dy1 * low[y2 * lg + x2];
      const float d = head_b + v;
      const bool border = y == 0 || x == 0 || y == side - 1 || x == side - 1;
      logits[(long long)y * side + x] = border ? d : d + acc[j];
    }
  }
}

// decoder.rs:684-722: at the border the two 3x3 convolutions run as they are
// (the intermediate map's zero padding is reached). One warp per border
// pixel, two of the 64 intermediate channels per lane.
__global__ void bir_edges(const float* __restrict__ img, int side, const float* __restrict__ fr,
                          float* __restrict__ logits) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int e_count = 4 * side - 4;
  for (int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < e_count; w += (gridDim.x * blockDim.x) >> 5) {
    int y, x;
    if (w < side) {
      y = 0;
      x = w;
    } else if (w < 2 * side) {
      y = side - 1;
      x = w - side;
    } else {
      const int j = w - 2 * side;
      y = 1 + j / 2;
      x = (j & 1) ? side - 1 : 0;
    }
    float s = fr[FR_SCALARS];
    for (int dd = 0; dd < 9; dd++) {
      const int qy = y + dd / 3 - 1, qx = x + dd % 3 - 1;
      if (qy < 0 || qx < 0 || qy >= side || qx >= side) continue;
      float part = 0.0f;
      for (int kk = 0; kk < 2; kk++) {
        const int k = lane + 32 * kk;
        float mid = fr[FR_BIAS1 + k];
        for (int e = 0; e < 9; e++) {
          const int py = qy + e / 3 - 1, px = qx + e % 3 - 1;
          if (py < 0 || px < 0 || py >= side || px >= side) continue;
          const float* q = img + ((long long)py * side + px) * 3;
          for (int c = 0; c < 3; c++) mid += q[c] * fr[FR_CONV1 + (e * 3 + c) * INTER + k];
        }
        part += mid * fr[FR_OUT + dd * INTER + k];
      }
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      s += part;
    }
    if (lane == 0) logits[(long long)y * side + x] += s;
  }
}

// A [taps * k, n] matrix packed with its input channels padded to k_pad per
// tap (zero rows), so that the GEMM's K steps are 64 channels wide.
void pack(WeightFile& f, PackedWeights& pw, const std::string& name, int taps, int k, int n, bool bias,
          int k_pad = 0) {
  HostTensor w = f.take_tensor(name + ".weight", {(size_t)taps * k, (size_t)n});
  std::vector<float> b;
  if (bias) b = f.take(name + ".bias", {(size_t)n});
  if (k_pad <= k) {
    pack_weights(pw, w.values, taps, k, n, bias ? b.data() : nullptr);
    return;
  }
  std::vector<float> padded((size_t)taps * k_pad * n, 0.0f);
  for (int t = 0; t < taps; t++)
    for (int c = 0; c < k; c++)
      std::copy(w.values.begin() + ((size_t)t * k + c) * n, w.values.begin() + ((size_t)t * k + c + 1) * n,
                padded.begin() + ((size_t)t * k_pad + c) * n);
  pack_weights(pw, padded, taps, k_pad, n, bias ? b.data() : nullptr);
}

int pad64(int c) { return (c + 63) / 64 * 64; }

void upload(DeviceBuffer& b, const std::vector<float>& v) {
  b.reserve(v.size() * 4);
  IEC_CUDA(cudaMemcpy(b.get(), v.data(), v.size() * 4, cudaMemcpyHostToDevice));
}

// swin.rs:31-51 tables widened to the 64-row window slots: the reference's
// 49 x 49 position bias (plus its -100 masks between the regions a shift
// brought together, per window class), -inf towards the slots' 15 padding
// keys, and zeros in the padding queries' rows (their outputs are dropped).
std::vector<float> slot_tables(const std::vector<float>& position, int heads, bool shifted) {
  const int classes = shifted ? 4 : 1;
  std::vector<float> t((size_t)classes * heads * 64 * 64);
  auto region = [](int v, bool last) { return (last && v >= WS - SHIFT) ? 1 : 0; };
  for (int cls = 0; cls < classes; cls++) {
    const bool last_col = cls & 1, last_row = cls & 2;
    auto id = [&](int i) { return region(i / WS, last_row) * 2 + region(i % WS, last_col); };
    for (int h = 0; h < heads; h++)
      for (int i = 0; i < 64; i++)
        for (int j = 0; j < 64; j++) {
          float v;
          if (j >= NTOK)
            v = -INFINITY;
          else if (i >= NTOK)
            v = 0.0f;
          else
            v = position[((size_t)h * NTOK + i) * NTOK + j] + (shifted && id(i) != id(j) ? -100.0f : 0.0f);
          t[(((size_t)cls * heads + h) * 64 + i) * 64 + j] = v;
        }
  }
  return t;
}

}  // namespace

struct Birefnet::SwinBlock {
  int c = 0, heads = 0;
  bool shifted = false;
  DeviceBuffer n1g, n1b, n2g, n2b, bias;
  PackedWeights qkv, proj, fc1, fc2;
  MlpWeights mlp;  // norm2, fc1, GELU and fc2 fused (mlp_sm100.cuh), where the width fits
  LnRowsWeights lnqkv;  // norm1 + window partition + qkv (lnrows_sm100.cuh), where the width fits
};

struct Birefnet::Stage {
  int c = 0;
  std::vector<SwinBlock> blocks;
  DeviceBuffer ng, nb, mg, mb;
  PackedWeights merge;
  bool has_merge = false;
};

struct Birefnet::DBlock {
  int cin = 0, cout = 0;
  PackedWeights conv_in, conv_out, gdt, offsets[4], branch[4], conv1;
  bool gated = false;
  DeviceBuffer gw, pool_w, pool_b, conv1_pool, conv1_bias;
  float gb = 0.0f;
};

struct Birefnet::Patches {
  PackedWeights conv1, conv_out;
};

Birefnet::Birefnet(const std::string& path, const Options& opt) : dev_(opt) {
  WeightFile f = WeightFile::read(path, "BIREFNET");
  DeviceScope scope(dev_);
  pack(f, embed_, "patch_embed", 1, 48, 96, true);
  upload(embed_g_, f.take("patch_embed.norm.weight", {96}));
  upload(embed_b_, f.take("patch_embed.norm.bias", {96}));
  for (int s = 0; s < 4; s++) {
    auto st = std::make_unique<Stage>();
    const int c = STAGE_C[s], heads = c / 32;
    st->c = c;
    for (int b = 0; b < STAGE_D[s]; b++) {
      const std::string p = "stage" + std::to_string(s) + ".block" + std::to_string(b);
      SwinBlock blk;
      blk.c = c;
      blk.heads = heads;
      blk.shifted = b % 2 == 1;
      {
        // norm1 and qkv: the separate launches' weights, and the same values
        // for the kernel that folds norm1 and the window partition into the
        // product's staged rows
        const std::vector<float> g1 = f.take(p + ".norm1.weight", {(size_t)c});
        const std::vector<float> be1 = f.take(p + ".norm1.bias", {(size_t)c});
        HostTensor wq = f.take_tensor(p + ".qkv.weight", {(size_t)c, (size_t)(3 * c)});
        const std::vector<float> bq = f.take(p + ".qkv.bias", {(size_t)(3 * c)});
        upload(blk.n1g, g1);
        upload(blk.n1b, be1);
        pack_weights(blk.qkv, wq.values, 1, c, 3 * c, bq.data());
        if (lnrows_fits(c, 3 * c)) pack_lnrows(blk.lnqkv, c, 3 * c, wq.values, bq, g1, be1);
      }
      upload(blk.bias, attention_bias_layout(
                           slot_tables(f.take(p + ".position_bias", {(size_t)heads, NTOK, NTOK}), heads, blk.shifted)));
      pack(f, blk.proj, p + ".proj", 1, c, c, true);
      {
        // norm2 and the MLP: the separate launches' weights, and the same
        // values packed for the fused MLP kernel
        const std::vector<float> g2 = f.take(p + ".norm2.weight", {(size_t)c});
        const std::vector<float> be2 = f.take(p + ".norm2.bias", {(size_t)c});
        HostTensor w1 = f.take_tensor(p + ".fc1.weight", {(size_t)c, (size_t)(4 * c)});
        const std::vector<float> bb1 = f.take(p + ".fc1.bias", {(size_t)(4 * c)});
        HostTensor w2 = f.take_tensor(p + ".fc2.weight", {(size_t)(4 * c), (size_t)c});
        const std::vector<float> bb2 = f.take(p + ".fc2.bias", {(size_t)c});
        upload(blk.n2g, g2);
        upload(blk.n2b, be2);
        pack_weights(blk.fc1, w1.values, 1, c, 4 * c, bb1.data());
        pack_weights(blk.fc2, w2.values, 1, 4 * c, c, bb2.data());
        if (mlp_preferred(c)) pack_mlp(blk.mlp, c, w1.values, bb1, w2.values, bb2, g2, be2);
      }
      st->blocks.push_back(std::move(blk));
    }
    const std::string sn = "stage" + std::to_string(s);
    if (s < 3) {
      st->has_merge = true;
      upload(st->mg, f.take(sn + ".merge.norm.weight", {(size_t)4 * c}));
      upload(st->mb, f.take(sn + ".merge.norm.bias", {(size_t)4 * c}));
      pack(f, st->merge, sn + ".merge", 1, 4 * c, 2 * c, false);
    }
    upload(st->ng, f.take(sn + ".norm.weight", {(size_t)c}));
    upload(st->nb, f.take(sn + ".norm.bias", {(size_t)c}));
    stages_.push_back(std::move(st));
  }
  auto load_block = [&](const std::string& p, int cin, int cout, bool gate) {
    auto b = std::make_unique<DBlock>();
    b->cin = cin;
    b->cout = cout;
    pack(f, b->conv_in, p + ".conv_in", 9, cin, INTER, true, pad64(cin));
    pack(f, b->conv_out, p + ".conv_out", 9, INTER, cout, true);
    if (gate) {
      b->gated = true;
      pack(f, b->gdt, p + ".gdt", 9, cout, 16, true);
      upload(b->gw, f.take(p + ".gdt_attn.weight", {16, 1}));
      b->gb = f.take(p + ".gdt_attn.bias", {1})[0];
    }
    for (int i = 0; i < 4; i++) {
      const int taps = SIZES[i] * SIZES[i];
      const std::string br = p + ".aspp.branch" + std::to_string(i);
      pack(f, b->offsets[i], br + ".offset", taps, INTER, 3 * taps, true);
      pack(f, b->branch[i], br, 1, taps * INTER, BRANCH, true);
    }
    upload(b->pool_w, f.take(p + ".aspp.pool.weight", {INTER, BRANCH}));
    upload(b->pool_b, f.take(p + ".aspp.pool.bias", {BRANCH}));
    HostTensor c1 = f.take_tensor(p + ".aspp.conv1.weight", {5 * BRANCH, INTER});
    upload(b->conv1_bias, f.take(p + ".aspp.conv1.bias", {INTER}));
    std::vector<float> rows(c1.values.begin(), c1.values.begin() + 4 * BRANCH * INTER);
    std::vector<float> zero(INTER, 0.0f);
    // conv1's bias is written per run (the pooling branch's share).
    pack_weights(b->conv1, rows, 1, 4 * BRANCH, INTER, zero.data());
    upload(b->conv1_pool, std::vector<float>(c1.values.begin() + 4 * BRANCH * INTER, c1.values.end()));
    return b;
  };
  squeeze_ = load_block("squeeze", 2880, 1536, false);
  for (int i = 0; i < 4; i++)
    blocks_.push_back(load_block("block" + std::to_string(4 - i), LEVELS[i][0], LEVELS[i][1], i < 3));
  const int lat[3][2] = {{4, 768}, {3, 384}, {2, 192}};
  for (int i = 0; i < 3; i++) pack(f, laterals_[i], "lateral" + std::to_string(lat[i][0]), 1, lat[i][1], lat[i][1], true);
  for (int i = 0; i < 4; i++) {
    auto pt = std::make_unique<Patches>();
    const std::string p = "patches" + std::to_string(5 - i);
    pack(f, pt->conv1, p + ".conv1", 9, PATCH_C[i], INTER, true, pad64(PATCH_C[i]));
    pack(f, pt->conv_out, p + ".conv_out", 9, INTER, PATCH_OUT[i], true);
    patches_.push_back(std::move(pt));
  }
  upload(head_w_, f.take("head.weight", {96, 1}));
  head_b_ = f.take("head.bias", {1})[0];
  {
    // decoder.rs:605-633: the composed 5x5 convolution, in double.
    const std::vector<float> conv1 = f.take("patches1.conv1.weight", {27, INTER});
    const std::vector<float> bias1 = f.take("patches1.conv1.bias", {INTER});
    const std::vector<float> conv_out = f.take("patches1.conv_out.weight", {9 * INTER, 1});
    const float bias_out = f.take("patches1.conv_out.bias", {1})[0];
    std::vector<double> comp(75, 0.0);
    double cb = bias_out;
    for (int d = 0; d < 9; d++)
      for (int k = 0; k < INTER; k++) {
        const double w2 = conv_out[d * INTER + k];
        cb += w2 * (double)bias1[k];
        for (int e = 0; e < 9; e++) {
          const int ey = d / 3 + e / 3, ex = d % 3 + e % 3;
          for (int c = 0; c < 3; c++) comp[(ey * 5 + ex) * 3 + c] += w2 * (double)conv1[(e * 3 + c) * INTER + k];
        }
      }
    std::vector<float> fr(FR_TOTAL);
    for (int i = 0; i < 75; i++) fr[FR_COMPOSED + i] = (float)comp[i];
    std::copy(conv1.begin(), conv1.end(), fr.begin() + FR_CONV1);
    std::copy(bias1.begin(), bias1.end(), fr.begin() + FR_BIAS1);
    std::copy(conv_out.begin(), conv_out.end(), fr.begin() + FR_OUT);
    fr[FR_SCALARS] = bias_out;
    fr[FR_SCALARS + 1] = (float)cb;
    upload(full_, fr);
  }
  f.finish();
  sums_.reserve(INTER * sizeof(double));
  for (cudaStream_t* st : {&s_half_, &s_patch_, &s_aspp_}) IEC_CUDA(cudaStreamCreateWithFlags(st, cudaStreamNonBlocking));
  for (cudaEvent_t* e : {&ev_prep_, &ev_half_, &ev_t_, &ev_aspp_, &ev_patch_[0], &ev_patch_[1], &ev_patch_[2],
                         &ev_patch_[3]})
    IEC_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
  IEC_CUDA(cudaDeviceSynchronize());
}

Birefnet::~Birefnet() {
  if (!dev_.poisoned()) {
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(dev_.ordinal());
    for (cudaEvent_t e : {ev_prep_, ev_half_, ev_t_, ev_aspp_, ev_patch_[0], ev_patch_[1], ev_patch_[2], ev_patch_[3]})
      if (e) cudaEventDestroy(e);
    for (cudaStream_t st : {s_half_, s_patch_, s_aspp_})
      if (st) cudaStreamDestroy(st);
    if (prev >= 0) cudaSetDevice(prev);
  }
  if (dev_.poisoned()) {
    graph_.leak();
    for (BackboneBuffers& bb : bb_)
      for (DeviceBuffer* b : {&bb.patch_rows, &bb.x, &bb.tok, &bb.qkv, &bb.att, &bb.ln, &bb.hid, &bb.mrg}) b->leak();
    for (int i = 0; i < 3; i++) {
      offs_b_[i].leak();
      samp_b_[i].leak();
    }
    for (DeviceBuffer* b : {&img_, &himg_, &lev_[0],
                            &lev_[1], &lev_[2], &hf_[0], &hf_[1], &hf_[2], &hf_[3], &x4_, &in_[0], &in_[1], &in_[2],
                            &in_[3], &outb_[0], &outb_[1], &outb_[2], &out1_, &t_, &t2_, &offs_, &samp_, &cat_, &g16_,
                            &sums_, &low_, &stack_, &pmid_, &host_in, &host_out})
      b->leak();
  }
}

void Birefnet::ensure(int side) {
  if (side == alloc_side_) return;
  alloc_gen_++;  // buffers may move: captured passes must not replay
  const long long g0 = side / 4, P0 = g0 * g0;
  auto bytes = [](long long planes, long long elems) { return (size_t)(planes * elems * 2); };
  img_.reserve((size_t)side * side * 3 * 4);
  himg_.reserve((size_t)(side / 2) * (side / 2) * 3 * 4);
  ensure_backbone(bb_[0], side);
  ensure_backbone(bb_[1], side / 2);
  for (int i = 0; i < 3; i++) {
    const long long gi = g0 >> i;
    lev_[i].reserve(bytes(2 * STAGE_C[i] / 8, pe(gi * gi)));
  }
  for (int i = 0; i < 4; i++) {
    const long long hg = (g0 >> i) / 2;
    hf_[i].reserve(bytes(STAGE_C[i] / 8, pe(hg * hg)));
  }
  const long long g3 = g0 >> 3;
  x4_.reserve(bytes(360, pe(g3 * g3)));
  for (int i = 0; i < 4; i++) {
    const long long gi = g0 >> (3 - i);
    // the planes past cin stay zero: conv_in's padded input channels
    in_[i].reserve(bytes(pad64(LEVELS[i][0]) / 8, pe(gi * gi)));
    IEC_CUDA(cudaMemset(in_[i].get(), 0, bytes(pad64(LEVELS[i][0]) / 8, pe(gi * gi))));
    if (i < 3)
      outb_[i].reserve(bytes(LEVELS[i][1] / 8, pe(gi * gi)));
    else
      out1_.reserve(bytes(12, pe(gi * gi)));
  }
  t_.reserve(bytes(8, pe(P0)));
  t2_.reserve(bytes(8, pe(P0)));
  offs_.reserve(bytes(19, pe(P0)));
  samp_.reserve(bytes(49 * 8, pe(P0)));
  for (int i = 0; i < 3; i++) {
    offs_b_[i].reserve(bytes(19, pe(P0)));
    samp_b_[i].reserve(bytes(SIZES[i] * SIZES[i] * 8, pe(P0)));
  }
  cat_.reserve(bytes(128, pe(P0)));
  g16_.reserve(bytes(2, pe(P0)));
  low_.reserve((size_t)P0 * 4);
  size_t bstack = 0;
  for (int i = 0; i < 4; i++) {
    const long long gi = g0 >> (3 - i);
    bstack = std::max(bstack, bytes(pad64(PATCH_C[i]) / 8, pe(gi * gi)));
  }
  stack_.reserve(bstack);
  pmid_.reserve(bytes(8, pe(P0)));
  alloc_side_ = side;
}

void Birefnet::ensure_backbone(BackboneBuffers& bb, int side) {
  const long long g0 = side / 4, P0 = g0 * g0;
  auto bytes = [](long long planes, long long elems) { return (size_t)(planes * elems * 2); };
  bb.patch_rows.reserve(bytes(6, pe(P0)));
  size_t bx = 0, btok = 0, bqkv = 0, bln = 0, bhid = 0, bmrg = 0;
  long long g = g0;
  for (int s = 0; s < 4; s++, g /= 2) {
    const long long c = STAGE_C[s], tokens = g * g, pad = (g + WS - 1) / WS * WS, slots = (pad / WS) * (pad / WS) * 64;
    bx = std::max(bx, bytes(c / 8, pe(tokens)));
    btok = std::max(btok, bytes(c / 8, pe(slots)));
    bqkv = std::max(bqkv, bytes(3 * c / 8, pe(slots)));
    bln = std::max(bln, bytes(c / 8, pe(tokens)));
    bhid = std::max(bhid, bytes(4 * c / 8, pe(tokens)));
    if (s < 3) bmrg = std::max(bmrg, bytes(4 * c / 8, pe(tokens / 4)));
  }
  bb.x.reserve(bx);
  bb.tok.reserve(btok);
  bb.att.reserve(btok);
  bb.qkv.reserve(bqkv);
  bb.ln.reserve(bln);
  bb.hid.reserve(bhid);
  bb.mrg.reserve(bmrg);
}

void Birefnet::backbone(const float* img, int side, __half* const dst[4], const long long dst_plane[4],
                        const int plane0[4], BackboneBuffers& bb, cudaStream_t s) {
  const int sms = dev_.sms();
  int grid = side / 4;
  long long tokens = (long long)grid * grid;
  launch_pdl(bir_embed_gather, blocks_for(tokens * 6, sms), 256, 0, s, img, side, bb.patch_rows.as<__half>(), pe(tokens));
  IEC_CUDA(cudaGetLastError());
  __half* x = bb.x.as<__half>();
  {
    GemmOutSpec o;
    o.mode = OUT_STORE;
    o.out = x;
    o.plane_elems = pe(tokens);
    gemm_rows(dev_, embed_, bb.patch_rows.as<__half>(), pe(tokens), (int)tokens, ACT_NONE, o, s);
    layer_norm_planar(x, pe(tokens), 0, (int)tokens, 96, embed_g_.as<float>(), embed_b_.as<float>(), x, pe(tokens),
                      nullptr, s);
  }
  for (int si = 0; si < 4; si++) {
    const Stage& st = *stages_[si];
    const int c = st.c;
    const long long xp = pe(tokens);
    const int pad = (grid + WS - 1) / WS * WS, wins = pad / WS;
    const long long slots = (long long)wins * wins * 64, sp = pe(slots);
    for (const SwinBlock& B : st.blocks) {
      const int shift = B.shifted ? SHIFT : 0;
      // attention: x += proj(attn(window(LN1(x))))
      const WindowMap wm{WS, pad, pad, grid, grid, shift};
      GemmOutSpec o;
      if (fused_mlp_ && B.lnqkv.c == c) {
        lnrows_planar(dev_, B.lnqkv, x, xp, (int)slots, wm, bb.qkv.as<__half>(), sp, s);
      } else {
        layer_norm_planar(x, xp, 0, (int)slots, c, B.n1g.as<float>(), B.n1b.as<float>(), bb.tok.as<__half>(), sp, &wm,
                          s);
        o.mode = OUT_STORE;
        o.out = bb.qkv.as<__half>();
        o.plane_elems = sp;
        gemm_rows(dev_, B.qkv, bb.tok.as<__half>(), sp, (int)slots, ACT_NONE, o, s);
      }
      window_attention(bb.qkv.as<__half>(), sp, c, (int)(slots / 64), B.bias.as<float>(), B.shifted, wins, wins,
                       bb.att.as<__half>(), sp, dev_.dev_err(), s);
      o.mode = OUT_WINDOW_ACCUM;
      o.out = x;
      o.plane_elems = xp;
      o.map_h = grid;
      o.map_w = grid;
      o.shift = shift;
      o.win_ws = WS;
      o.pad_h = pad;
      o.pad_w = pad;
      gemm_rows(dev_, B.proj, bb.att.as<__half>(), sp, (int)slots, ACT_NONE, o, s);
      // MLP: x += fc2(GELU(fc1(LN2(x))))
      if (fused_mlp_ && B.mlp.c == c) {
        mlp_planar(dev_, B.mlp, x, xp, (int)tokens, s);
      } else {
        layer_norm_planar(x, xp, 0, (int)tokens, c, B.n2g.as<float>(), B.n2b.as<float>(), bb.ln.as<__half>(), xp,
                          nullptr, s);
        GemmOutSpec h;
        h.mode = OUT_STORE;
        h.out = bb.hid.as<__half>();
        h.plane_elems = xp;
        gemm_rows(dev_, B.fc1, bb.ln.as<__half>(), xp, (int)tokens, ACT_GELU, h, s);
        GemmOutSpec a;
        a.mode = OUT_ACCUM;
        a.out = x;
        a.plane_elems = xp;
        gemm_rows(dev_, B.fc2, bb.hid.as<__half>(), xp, (int)tokens, ACT_NONE, a, s);
      }
    }
    // the stage's normalised output
    layer_norm_planar(x, xp, 0, (int)tokens, c, st.ng.as<float>(), st.nb.as<float>(),
                      dst[si] + (long long)plane0[si] * dst_plane[si], dst_plane[si], nullptr, s);
    if (st.has_merge) {
      const long long mt = tokens / 4, mp = pe(mt);
      merge_layer_norm_planar(x, xp, grid, c, st.mg.as<float>(), st.mb.as<float>(), bb.mrg.as<__half>(), mp, s);
      GemmOutSpec o;
      o.mode = OUT_STORE;
      o.out = x;
      o.plane_elems = mp;
      gemm_rows(dev_, st.merge, bb.mrg.as<__half>(), mp, (int)mt, ACT_NONE, o, s);
      grid /= 2;
      tokens = mt;
    }
  }
}

void Birefnet::block(const DBlock& b, const __half* x, long long x_plane, int cin, int g, __half* out,
                     long long out_plane, int plane0, cudaStream_t s) {
  const int sms = dev_.sms();
  const long long P = (long long)g * g, pp = pe(P);
  (void)cin;
  __half* t = t_.as<__half>();
  // t = ReLU(conv_in(x))
  {
    GemmOutSpec o;
    o.mode = OUT_STORE;
    o.out = t;
    o.plane_elems = pp;
    gemm_conv3(dev_, b.conv_in, x, x_plane, g, g, ACT_RELU, o, s);
  }
  // ASPP (decoder.rs:138-236): the pooled bias, four deformable branches
  // into `cat`, conv1 + bias + ReLU.
  IEC_CUDA(cudaMemsetAsync(sums_.get(), 0, INTER * sizeof(double), s));
  launch_pdl(bir_channel_sums, dim3(std::max(1, std::min(64, (int)((P + 255) / 256))), 8), 256, 0, s, t, pp, P,
                                                                                              sums_.as<double>());
  IEC_CUDA(cudaGetLastError());
  launch_pdl(bir_aspp_bias, 1, 256, 0, s, sums_.as<double>(), (double)P, b.pool_w.as<float>(), b.pool_b.as<float>(),
                                  b.conv1_pool.as<float>(), b.conv1_bias.as<float>(), b.conv1.bias.as<float>());
  IEC_CUDA(cudaGetLastError());
  // Branches 0-2 on the side stream (their own offset and sample buffers),
  // beside the 7x7 branch; each writes its 256 planes of `cat`.
  IEC_CUDA(cudaEventRecord(ev_t_, s));
  IEC_CUDA(cudaStreamWaitEvent(s_aspp_, ev_t_, 0));
  for (int i = 0; i < 4; i++) {
    const int k = SIZES[i], taps = k * k;
    cudaStream_t bs = i < 3 ? s_aspp_ : s;
    __half* offs = i < 3 ? offs_b_[i].as<__half>() : offs_.as<__half>();
    __half* samp = i < 3 ? samp_b_[i].as<__half>() : samp_.as<__half>();
    std::vector<Tap> tl;
    for (int ky = 0; ky < k; ky++)
      for (int kx = 0; kx < k; kx++) tl.push_back({ky - k / 2, kx - k / 2, 0});
    GemmOutSpec o;
    o.mode = OUT_STORE;
    o.out = offs;
    o.plane_elems = pp;
    gemm_taps(dev_, b.offsets[i], TapSource{t, pp, g, g, 1}, tl, g, g, ACT_NONE, o, bs);
    // Channel groups per thread: 4 where the (pixel, tap) pairs alone fill
    // the GPU about once over, fewer on the small maps (all 8 in a thread
    // took 127 registers and ran 0.4 % slower on the whole network).
    const long long pairs = P * taps;
    const int gpt = pairs >= 1024LL * sms ? 4 : pairs >= 512LL * sms ? 2 : 1;
    const dim3 grid((unsigned)std::min<long long>((P + 255) / 256, 4LL * sms), (unsigned)(taps * (8 / gpt)));
    // bytes: the offsets and modulators (3 per tap), the 64-channel map read
    // once and the sampled operand (64 channels per tap) written, f16
    timed_launch("bir_deform_sample", 0.0, (double)P * (3 * taps + 64 + 64 * taps) * 2, bs, [&] {
      if (gpt == 4)
        launch_pdl(bir_deform_sample<4>, grid, 256, 0, bs, t, pp, g, g, k, offs, pp, samp, pp);
      else if (gpt == 2)
        launch_pdl(bir_deform_sample<2>, grid, 256, 0, bs, t, pp, g, g, k, offs, pp, samp, pp);
      else
        launch_pdl(bir_deform_sample<1>, grid, 256, 0, bs, t, pp, g, g, k, offs, pp, samp, pp);
      IEC_CUDA(cudaGetLastError());
    });
    GemmOutSpec c;
    c.mode = OUT_STORE;
    c.out = cat_.as<__half>();
    c.plane_elems = pp;
    c.plane0 = i * (BRANCH / 8);
    gemm_rows(dev_, b.branch[i], samp, pp, (int)P, ACT_RELU, c, bs);
    if (i == 2) IEC_CUDA(cudaEventRecord(ev_aspp_, s_aspp_));
  }
  IEC_CUDA(cudaStreamWaitEvent(s, ev_aspp_, 0));
  __half* t2 = t2_.as<__half>();
  {
    GemmOutSpec o;
    o.mode = OUT_STORE;
    o.out = t2;
    o.plane_elems = pp;
    gemm_rows(dev_, b.conv1, cat_.as<__half>(), pp, (int)P, ACT_RELU, o, s);
  }
  // out = conv_out(t2) [* gate]
  GemmOutSpec o;
  o.mode = OUT_STORE;
  o.out = out;
  o.plane_elems = out_plane;
  o.plane0 = plane0;
  gemm_conv3(dev_, b.conv_out, t2, pp, g, g, ACT_NONE, o, s);
  if (b.gated) {
    __half* base = out + (long long)plane0 * out_plane;
    GemmOutSpec go;
    go.mode = OUT_STORE;
    go.out = g16_.as<__half>();
    go.plane_elems = pp;
    gemm_conv3(dev_, b.gdt, base, out_plane, g, g, ACT_RELU, go, s);
    const int planes = b.cout / 8;
    launch_pdl(bir_gate, blocks_for(P * ((planes + 3) / 4), sms), 256, 0, s, g16_.as<__half>(), pp,
               b.gw.as<float>(), b.gb, base, out_plane, planes, P);
    IEC_CUDA(cudaGetLastError());
  }
}

void Birefnet::run(const void* image, bool u8, int side, float* logits, cudaStream_t s) {
  // Replayed as a graph while the same buffers and size repeat (PassGraph).
  graph_.run({(long long)(uintptr_t)image, u8, side, (long long)(uintptr_t)logits, (long long)alloc_gen_,
              (long long)dev_.scratch_generation()},
             s,
             [&](cudaStream_t st) { run_pass(image, u8, side, logits, st); });
}

void Birefnet::run_pass(const void* image, bool u8, int side, float* logits, cudaStream_t s) {
  SerialStreams serial(dev_.timing(), {&s_half_, &s_patch_, &s_aspp_}, s);
  if (side <= 0 || side % 64 != 0)
    throw Error(ERR_INPUT, "side " + std::to_string(side) + " is not a positive multiple of 64");
  ensure(side);
  const int sms = dev_.sms();
  const long long n = (long long)side * side * 3;
  float* img = img_.as<float>();
  launch_pdl(bir_prep, blocks_for(n, sms), 256, 0, s, image, u8 ? 1 : 0, n, img);
  IEC_CUDA(cudaGetLastError());
  const int hs = side / 2;
  launch_pdl(bir_resize_f32, blocks_for((long long)hs * hs, sms), 256, 0, s, img, side, side, 3, himg_.as<float>(), hs, hs);
  IEC_CUDA(cudaGetLastError());

  const int g0 = side / 4, g[4] = {g0, g0 / 2, g0 / 4, g0 / 8};
  const int main_c[4] = {1536, 768, 384, 192};
  // Three concurrent chains from here: the image patches of the four levels
  // (they read only the image; each writes its level's input planes after
  // the main ones), the half-size backbone pass, and the full-size pass.
  IEC_CUDA(cudaEventRecord(ev_prep_, s));
  IEC_CUDA(cudaStreamWaitEvent(s_patch_, ev_prep_, 0));
  IEC_CUDA(cudaStreamWaitEvent(s_half_, ev_prep_, 0));
  for (int i = 0; i < 4; i++) {
    const int level = 3 - i, gi = g[level];
    const Patches& pt = *patches_[i];
    const int groups = pad64(PATCH_C[i]) / 8;  // zero channels past the stack's
    const long long sp = pe((long long)gi * gi), ip = pe((long long)gi * gi);
    launch_pdl(bir_patches, blocks_for((long long)gi * gi * groups, sms), 256, 0, s_patch_, img, side, gi,
               stack_.as<__half>(), sp, groups);
    IEC_CUDA(cudaGetLastError());
    GemmOutSpec o;
    o.mode = OUT_STORE;
    o.out = pmid_.as<__half>();
    o.plane_elems = sp;
    gemm_conv3(dev_, pt.conv1, stack_.as<__half>(), sp, gi, gi, ACT_NONE, o, s_patch_);
    o.out = in_[i].as<__half>();
    o.plane_elems = ip;
    o.plane0 = main_c[i] / 8;
    gemm_conv3(dev_, pt.conv_out, pmid_.as<__half>(), sp, gi, gi, ACT_NONE, o, s_patch_);
    IEC_CUDA(cudaEventRecord(ev_patch_[i], s_patch_));
  }
  // Half-size features into hf (side stream); full-size features straight
  // into their levels (level 3 into x4, after the three resized levels' 168
  // planes).
  {
    __half* dst[4] = {hf_[0].as<__half>(), hf_[1].as<__half>(), hf_[2].as<__half>(), hf_[3].as<__half>()};
    long long dp[4];
    for (int i = 0; i < 4; i++) dp[i] = pe((long long)(g[i] / 2) * (g[i] / 2));
    const int p0[4] = {0, 0, 0, 0};
    backbone(himg_.as<float>(), hs, dst, dp, p0, bb_[1], s_half_);
    IEC_CUDA(cudaEventRecord(ev_half_, s_half_));
  }
  {
    __half* dst[4] = {lev_[0].as<__half>(), lev_[1].as<__half>(), lev_[2].as<__half>(), x4_.as<__half>()};
    const long long dp[4] = {pe((long long)g[0] * g[0]), pe((long long)g[1] * g[1]), pe((long long)g[2] * g[2]),
                             pe((long long)g[3] * g[3])};
    const int p0[4] = {0, 0, 0, 168};
    backbone(img, side, dst, dp, p0, bb_[0], s);
  }
  IEC_CUDA(cudaStreamWaitEvent(s, ev_half_, 0));
  // Each level's second half: the half-size run resized to the level's grid.
  for (int i = 0; i < 4; i++) {
    const int c8 = STAGE_C[i] / 8, hg = g[i] / 2;
    __half* dst = i < 3 ? lev_[i].as<__half>() : x4_.as<__half>();
    const int plane = i < 3 ? c8 : 168 + c8;
    const long long dp = pe((long long)g[i] * g[i]);
    launch_resize(hf_[i].as<__half>(), pe((long long)hg * hg), hg, hg, dst + plane * dp, dp, g[i], g[i], c8, 0, sms, s);
    IEC_CUDA(cudaGetLastError());
  }
  // x4: levels 1-3 resized to 1/32 (planes 0..167), level 4 after them.
  {
    const long long p3 = pe((long long)g[3] * g[3]);
    int plane = 0;
    for (int i = 0; i < 3; i++) {
      const int c8 = 2 * STAGE_C[i] / 8;
      launch_resize(lev_[i].as<__half>(), pe((long long)g[i] * g[i]), g[i], g[i], x4_.as<__half>() + plane * p3, p3,
                    g[3], g[3], c8, 0, sms, s);
      IEC_CUDA(cudaGetLastError());
      plane += c8;
    }
  }
  // squeeze -> block 4's input planes 0..191
  block(*squeeze_, x4_.as<__half>(), pe((long long)g[3] * g[3]), 2880, g[3], in_[0].as<__half>(),
        pe((long long)g[3] * g[3]), 0, s);
  for (int i = 0; i < 4; i++) {
    const int level = 3 - i, gi = g[level], cin = LEVELS[i][0];
    const long long ip = pe((long long)gi * gi);
    __half* in = in_[i].as<__half>();
    if (i > 0) {
      // lateral(level features) + previous output resized
      GemmOutSpec o;
      o.mode = OUT_STORE;
      o.out = in;
      o.plane_elems = ip;
      gemm_rows(dev_, laterals_[i - 1], lev_[level].as<__half>(), ip, gi * gi, ACT_NONE, o, s);
      const int pg = g[level + 1];
      const __half* prev = outb_[i - 1].as<__half>();
      launch_resize(prev, pe((long long)pg * pg), pg, pg, in, ip, gi, gi, main_c[i] / 8, 1, sms, s);
      IEC_CUDA(cudaGetLastError());
    }
    // the level's image patches, through two convolutions (side stream)
    IEC_CUDA(cudaStreamWaitEvent(s, ev_patch_[i], 0));
    __half* out = i < 3 ? outb_[i].as<__half>() : out1_.as<__half>();
    block(*blocks_[i], in, ip, cin, gi, out, ip, 0, s);
  }
  // head
  {
    const long long P0 = (long long)g0 * g0;
    launch_pdl(bir_head, blocks_for(P0, sms), 256, 0, s, out1_.as<__half>(), pe(P0), head_w_.as<float>(), P0,
                                                  low_.as<float>());
    IEC_CUDA(cudaGetLastError());
    launch_pdl(bir_logits, blocks_for((long long)side * ((side + 3) / 4), sms), 256, 0, s, low_.as<float>(), g0, img, side,
                                                                        full_.as<float>(), head_b_, logits);
    IEC_CUDA(cudaGetLastError());
    launch_pdl(bir_edges, blocks_for((long long)(4 * side - 4) * 32, sms), 256, 0, s, img, side, full_.as<float>(), logits);
    IEC_CUDA(cudaGetLastError());
  }
}

}  // namespace iec
