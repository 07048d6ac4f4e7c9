// LaMa's 2-D real Fourier transforms on planar f16 maps (see fft.h).
//
// A transform runs as two passes through an f32 scratch of row spectra, each
// pass a batch of 1-D transforms of "lines": n points of one channel group
// (8 channels, the 16 bytes a pixel holds in one plane), so every load and
// store moves whole 16-byte pixel groups. A CTA holds up to 512 points
// (several short lines, or one long one) in shared memory and transforms them
// in place of fourier.rs's recursive mixed-radix FFT (fourier.rs:16-139):
// radix-2 Stockham passes when n is a power of two, else the direct sum of
// the transform's definition. Twiddles are cos / sin of 2 pi j / n computed
// in double and rounded to f32, as fourier.rs:45-52 makes them.
//   forward: rows  real -> complex (all n outputs, the first w/2 + 1 kept)
//            cols  complex, times 1 / sqrt(h w), to the f16 spectrum
//   inverse: cols  complex from the f16 spectrum
//            rows  the Hermitian row (imaginary parts of columns 0 and w/2
//                  dropped) -> real part, times 1 / sqrt(h w), added on x
// Maps small enough that both passes fit one CTA's shared memory for a few
// channels (64 x 64 for two, LaMa's Fourier units at a 512 x 512 input) run
// both passes in one launch per direction instead (fft2_fwd_small /
// fft2_inv_small: a CTA per channel slice, the row spectra never leave
// shared memory), the same butterflies in the same order.
#include "fft.h"
#include "sm100.cuh"

#include <cmath>

#include <vector>

namespace iec {

namespace {

constexpr int FFT_THREADS = 256;
constexpr int FFT_SMALL_THREADS = 1024;  // the one-launch transforms: a stage's butterflies at once
constexpr int FFT_POINTS = 512;   // points per CTA when lines are short
constexpr int FFT_MAX_N = 1536;   // longest line (shared memory: 2 x 64 n bytes)

struct Line {
  int n, log2n;  // log2n < 0: not a power of two
  const float* cos_t;
  const float* sin_t;
};


__device__ __forceinline__ float4 cmul2(float4 v, float wr, float wi) {
  return make_float4(v.x * wr - v.y * wi, v.x * wi + v.y * wr, v.z * wr - v.w * wi, v.z * wi + v.w * wr);
}
__device__ __forceinline__ float4 add4(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
__device__ __forceinline__ float4 sub4(float4 a, float4 b) { return make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w); }
// v times (s i): (x + i y)(s i) = -s y + i s x, for both complex values of v.
__device__ __forceinline__ float4 mul_si(float4 v, float s) { return make_float4(-s * v.y, s * v.x, -s * v.w, s * v.z); }

// Transforms `lines` lines of f.n points x C channels held in `a`
// ([line][n][C] complex) with `b` as the other buffer, sign -1 forward or +1
// inverse (no scaling); returns the buffer that holds the result. Powers of
// two run Stockham stages of radix 4 (and one of radix 2 for odd log2 n):
// for span m and l m = n / 4, the four points k + j m + q l m of sub-
// transform (j, k) go through a 4-point DFT and out to k + (4 j + q) m
// turned by w^(q j m), w = exp(sign 2 pi i / n). One thread per (line,
// butterfly, channel pair). Other lengths take the direct sum. `ct` / `st`
// are the cos / sin tables in shared memory.
template <int C>
__device__ float2* fft_lines(float2* a, float2* b, int lines, const Line f, const float* ct, const float* st,
                             float sign) {
  static_assert(C == 2 || C == 4 || C == 8, "channel pairs per point");
  constexpr int P = C / 2;  // float4 (channel pairs) per point
  const int n = f.n;
  if (f.log2n >= 0) {
    int sm = 0, rem = f.log2n;
    while (rem > 0) {
      const int m = 1 << sm;
      const float4* src4 = reinterpret_cast<const float4*>(a);
      float4* dst4 = reinterpret_cast<float4*>(b);
      if (rem >= 2) {
        const int lq = f.log2n - 2, quarter = n >> 2;
        const int total = (lines << lq) * P;
        for (int t = threadIdx.x; t < total; t += blockDim.x) {
          const int cc = t % P, rest = t / P, line = rest >> lq, r = rest & (quarter - 1);
          const int j = r >> sm, k = r & (m - 1);
          const int base = (line * n) * P + cc;
          const float4 c0 = src4[base + r * P], c1 = src4[base + (r + quarter) * P];
          const float4 c2 = src4[base + (r + 2 * quarter) * P], c3 = src4[base + (r + 3 * quarter) * P];
          const float4 t0 = add4(c0, c2), t1 = sub4(c0, c2), t2 = add4(c1, c3), t3 = mul_si(sub4(c1, c3), sign);
          const int o = base + (k + 4 * j * m) * P, jm = j * m;
          dst4[o] = add4(t0, t2);
          dst4[o + m * P] = cmul2(add4(t1, t3), ct[jm], sign * st[jm]);
          dst4[o + 2 * m * P] = cmul2(sub4(t0, t2), ct[2 * jm], sign * st[2 * jm]);
          dst4[o + 3 * m * P] = cmul2(sub4(t1, t3), ct[3 * jm], sign * st[3 * jm]);
        }
        sm += 2;
        rem -= 2;
      } else {
        const int lh = f.log2n - 1, half = n >> 1;
        const int total = (lines << lh) * P;
        for (int t = threadIdx.x; t < total; t += blockDim.x) {
          const int cc = t % P, rest = t / P, line = rest >> lh, r = rest & (half - 1);
          const int j = r >> sm, k = r & (m - 1);
          const int base = (line * n) * P + cc;
          const float4 c0 = src4[base + r * P], c1 = src4[base + (r + half) * P];
          const int o = base + (k + 2 * j * m) * P, jm = j * m;
          dst4[o] = add4(c0, c1);
          dst4[o + m * P] = cmul2(sub4(c0, c1), ct[jm], sign * st[jm]);
        }
        sm += 1;
        rem -= 1;
      }
      __syncthreads();
      float2* tmp = a;
      a = b;
      b = tmp;
    }
    return a;
  }
  const int total = lines * n * C;
  for (int t = threadIdx.x; t < total; t += blockDim.x) {
    const int c = t % C, r = t / C;
    const int line = r / n, k = r - line * n;
    const float2* src = a + (size_t)line * n * C;
    float re = 0.0f, im = 0.0f;
    int idx = 0;
    for (int j = 0; j < n; j++) {
      const float2 x = src[j * C + c];
      const float wr = ct[idx], wi = sign * st[idx];
      re += x.x * wr - x.y * wi;
      im += x.x * wi + x.y * wr;
      idx += k;
      if (idx >= n) idx -= n;
    }
    b[((size_t)line * n + k) * C + c] = make_float2(re, im);
  }
  __syncthreads();
  return b;
}

// The twiddle table of `f` copied into shared memory after the two buffers.
__device__ __forceinline__ void load_twiddles(const Line f, float* ct, float* st) {
  for (int j = threadIdx.x; j < f.n; j += blockDim.x) {
    ct[j] = f.cos_t[j];
    st[j] = f.sin_t[j];
  }
}

struct Dims {
  int h, w, half, groups, lines_rows, lines_cols;
  float scale;
};

// One thread moves one point of a line: the 8 channels of a pixel group,
// 16 bytes of f16 or 64 bytes of complex f32, in vector loads and stores.
__device__ __forceinline__ void load_half8(const __half* src, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(src);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int e = 0; e < 4; e++) {
    const float2 f = __half22float2(h[e]);
    v[2 * e] = f.x;
    v[2 * e + 1] = f.y;
  }
}

__device__ __forceinline__ void store_half8(__half* dst, const float* v) {
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; e++) {
    __half2 h2 = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
    w[e] = *reinterpret_cast<uint32_t*>(&h2);
  }
  *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ void copy_point(float2* dst, const float2* src) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  float4 r[4];
#pragma unroll
  for (int e = 0; e < 4; e++) r[e] = s4[e];
#pragma unroll
  for (int e = 0; e < 4; e++) d4[e] = r[e];
}

// Forward rows: x (real) -> scratch row spectra.
__global__ void __launch_bounds__(FFT_THREADS) fft_rows_fwd(const __half* __restrict__ x, long long x_plane,
                                                           float2* __restrict__ T, Dims d, Line f) {
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ float4 fft_smem4[];
  float2* fft_smem = reinterpret_cast<float2*>(fft_smem4);
  const int g = blockIdx.y, y0 = blockIdx.x * d.lines_rows;
  const int lines = min(d.lines_rows, d.h - y0), n = d.w;
  float2* a = fft_smem;
  float2* b = fft_smem + (size_t)d.lines_rows * n * 8;
  float* ct = reinterpret_cast<float*>(b + (size_t)d.lines_rows * n * 8);
  float* st = ct + n;
  load_twiddles(f, ct, st);
  const __half* src = x + g * x_plane + (size_t)y0 * n * 8;
  for (int t = threadIdx.x; t < lines * n; t += blockDim.x) {
    float v[8];
    load_half8(src + (size_t)t * 8, v);
#pragma unroll
    for (int c = 0; c < 8; c++) a[(size_t)t * 8 + c] = make_float2(v[c], 0.0f);
  }
  __syncthreads();
  const float2* r = fft_lines<8>(a, b, lines, f, ct, st, -1.0f);
  for (int t = threadIdx.x; t < lines * d.half; t += blockDim.x) {
    const int line = t / d.half, k = t - line * d.half;
    copy_point(T + (((size_t)g * d.h + y0 + line) * d.half + k) * 8, r + ((size_t)line * n + k) * 8);
  }
}

// Forward columns: scratch -> f16 spectrum (real planes, then imaginary).
__global__ void __launch_bounds__(FFT_THREADS) fft_cols_fwd(const float2* __restrict__ T, __half* __restrict__ spec,
                                                           long long spec_plane, Dims d, Line f) {
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ float4 fft_smem4[];
  float2* fft_smem = reinterpret_cast<float2*>(fft_smem4);
  const int g = blockIdx.y, k0 = blockIdx.x * d.lines_cols;
  const int lines = min(d.lines_cols, d.half - k0), n = d.h;
  float2* a = fft_smem;
  float2* b = fft_smem + (size_t)d.lines_cols * n * 8;
  float* ct = reinterpret_cast<float*>(b + (size_t)d.lines_cols * n * 8);
  float* st = ct + n;
  load_twiddles(f, ct, st);
  for (int t = threadIdx.x; t < lines * n; t += blockDim.x) {
    const int line = t % lines, y = t / lines;
    copy_point(a + ((size_t)line * n + y) * 8, T + (((size_t)g * d.h + y) * d.half + k0 + line) * 8);
  }
  __syncthreads();
  const float2* r = fft_lines<8>(a, b, lines, f, ct, st, -1.0f);
  __half* re = spec + g * spec_plane;
  __half* im = spec + (g + d.groups) * spec_plane;
  for (int t = threadIdx.x; t < lines * n; t += blockDim.x) {
    const int line = t % lines, ky = t / lines;
    const float2* v = r + ((size_t)line * n + ky) * 8;
    float vr[8], vi[8];
#pragma unroll
    for (int c = 0; c < 8; c++) {
      vr[c] = v[c].x * d.scale;
      vi[c] = v[c].y * d.scale;
    }
    const size_t at = ((size_t)ky * d.half + k0 + line) * 8;
    store_half8(re + at, vr);
    store_half8(im + at, vi);
  }
}

// Inverse columns: f16 spectrum -> scratch.
__global__ void __launch_bounds__(FFT_THREADS) fft_cols_inv(const __half* __restrict__ spec, long long spec_plane,
                                                           float2* __restrict__ T, Dims d, Line f) {
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ float4 fft_smem4[];
  float2* fft_smem = reinterpret_cast<float2*>(fft_smem4);
  const int g = blockIdx.y, k0 = blockIdx.x * d.lines_cols;
  const int lines = min(d.lines_cols, d.half - k0), n = d.h;
  float2* a = fft_smem;
  float2* b = fft_smem + (size_t)d.lines_cols * n * 8;
  float* ct = reinterpret_cast<float*>(b + (size_t)d.lines_cols * n * 8);
  float* st = ct + n;
  load_twiddles(f, ct, st);
  const __half* re = spec + g * spec_plane;
  const __half* im = spec + (g + d.groups) * spec_plane;
  for (int t = threadIdx.x; t < lines * n; t += blockDim.x) {
    const int line = t % lines, ky = t / lines;
    const size_t at = ((size_t)ky * d.half + k0 + line) * 8;
    float vr[8], vi[8];
    load_half8(re + at, vr);
    load_half8(im + at, vi);
    float2* dst = a + ((size_t)line * n + ky) * 8;
#pragma unroll
    for (int c = 0; c < 8; c++) dst[c] = make_float2(vr[c], vi[c]);
  }
  __syncthreads();
  const float2* r = fft_lines<8>(a, b, lines, f, ct, st, 1.0f);
  for (int t = threadIdx.x; t < lines * n; t += blockDim.x) {
    const int line = t % lines, y = t / lines;
    copy_point(T + (((size_t)g * d.h + y) * d.half + k0 + line) * 8, r + ((size_t)line * n + y) * 8);
  }
}

// Inverse rows: scratch -> the Hermitian row -> real part, added on x.
__global__ void __launch_bounds__(FFT_THREADS) fft_rows_inv(const float2* __restrict__ T, __half* __restrict__ x,
                                                           long long x_plane, Dims d, Line f) {
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ float4 fft_smem4[];
  float2* fft_smem = reinterpret_cast<float2*>(fft_smem4);
  const int g = blockIdx.y, y0 = blockIdx.x * d.lines_rows;
  const int lines = min(d.lines_rows, d.h - y0), n = d.w;
  float2* a = fft_smem;
  float2* b = fft_smem + (size_t)d.lines_rows * n * 8;
  float* ct = reinterpret_cast<float*>(b + (size_t)d.lines_rows * n * 8);
  float* st = ct + n;
  load_twiddles(f, ct, st);
  for (int t = threadIdx.x; t < lines * n; t += blockDim.x) {
    const int line = t / n, j = t - line * n;
    const float2* row = T + (((size_t)g * d.h + y0 + line) * d.half) * 8;
    float2* dst = a + (size_t)t * 8;
    if (j < d.half) {
      copy_point(dst, row + (size_t)j * 8);
      if (j == 0 || 2 * j == n) {
#pragma unroll
        for (int c = 0; c < 8; c++) dst[c].y = 0.0f;
      }
    } else {
      copy_point(dst, row + (size_t)(n - j) * 8);
#pragma unroll
      for (int c = 0; c < 8; c++) dst[c].y = -dst[c].y;
    }
  }
  __syncthreads();
  const float2* r = fft_lines<8>(a, b, lines, f, ct, st, 1.0f);
  __half* dst = x + g * x_plane + (size_t)y0 * n * 8;
  for (int t = threadIdx.x; t < lines * n; t += blockDim.x) {
    float v[8];
    load_half8(dst + (size_t)t * 8, v);
#pragma unroll
    for (int c = 0; c < 8; c++) v[c] += r[(size_t)t * 8 + c].x * d.scale;
    store_half8(dst + (size_t)t * 8, v);
  }
}

// C of a pixel group's 8 channels, from channel c0 on (aligned to C halves).
template <int C>
__device__ __forceinline__ void load_halves(const __half* src, float* v) {
  if constexpr (C == 8) {
    load_half8(src, v);
  } else if constexpr (C == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(src);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
  } else {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(src));
    v[0] = a.x, v[1] = a.y;
  }
}

template <int C>
__device__ __forceinline__ void store_halves(__half* dst, const float* v) {
  if constexpr (C == 8) {
    store_half8(dst, v);
  } else if constexpr (C == 4) {
    __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(dst) = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
  } else {
    *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(v[0], v[1]);
  }
}

// Both forward passes for C channels of one group (blockIdx.x = group x
// 8 / C + slice): rows of the real map, the first w/2 + 1 columns kept in
// shared memory column by column, columns, the scaled f16 spectrum.
template <int C>
__global__ void __launch_bounds__(FFT_SMALL_THREADS) fft2_fwd_small(const __half* __restrict__ x, long long x_plane,
                                                             __half* __restrict__ spec, long long spec_plane, Dims d,
                                                             Line fr, Line fc) {
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ float4 fft_smem4[];
  constexpr int SLICES = 8 / C;
  const int g = blockIdx.x / SLICES, c0 = (blockIdx.x % SLICES) * C;
  const int h = d.h, w = d.w, half = d.half, pts = max(h * w, half * h);
  float2* a = reinterpret_cast<float2*>(fft_smem4);
  float2* b = a + (size_t)pts * C;
  float* ctw = reinterpret_cast<float*>(b + (size_t)pts * C);
  float* stw = ctw + w;
  float* cth = stw + w;
  float* sth = cth + h;
  load_twiddles(fr, ctw, stw);
  load_twiddles(fc, cth, sth);
  const __half* src = x + g * x_plane + c0;
  for (int t = threadIdx.x; t < h * w; t += blockDim.x) {
    float v[C];
    load_halves<C>(src + (size_t)t * 8, v);
#pragma unroll
    for (int c = 0; c < C; c++) a[(size_t)t * C + c] = make_float2(v[c], 0.0f);
  }
  __syncthreads();
  float2* r = fft_lines<C>(a, b, h, fr, ctw, stw, -1.0f);  // [y][k][c]
  float2* o = r == a ? b : a;
  for (int t = threadIdx.x; t < half * h; t += blockDim.x) {
    const int k = t / h, y = t - k * h;
#pragma unroll
    for (int c = 0; c < C; c++) o[(size_t)t * C + c] = r[((size_t)y * w + k) * C + c];
  }
  __syncthreads();
  const float2* q = fft_lines<C>(o, r, half, fc, cth, sth, -1.0f);  // [k][ky][c]
  __half* re = spec + g * spec_plane + c0;
  __half* im = spec + (g + d.groups) * spec_plane + c0;
  for (int t = threadIdx.x; t < half * h; t += blockDim.x) {
    const int ky = t / half, k = t - ky * half;
    const float2* v = q + ((size_t)k * h + ky) * C;
    float vr[C], vi[C];
#pragma unroll
    for (int c = 0; c < C; c++) {
      vr[c] = v[c].x * d.scale;
      vi[c] = v[c].y * d.scale;
    }
    store_halves<C>(re + (size_t)t * 8, vr);
    store_halves<C>(im + (size_t)t * 8, vi);
  }
}

// Both inverse passes for C channels of one group: columns of the f16
// spectrum, the Hermitian rows built in shared memory, rows, the scaled real
// part added on x.
template <int C>
__global__ void __launch_bounds__(FFT_SMALL_THREADS) fft2_inv_small(const __half* __restrict__ spec, long long spec_plane,
                                                             __half* __restrict__ x, long long x_plane, Dims d,
                                                             Line fr, Line fc) {
  griddep_wait();
  griddep_launch_dependents();
  extern __shared__ float4 fft_smem4[];
  constexpr int SLICES = 8 / C;
  const int g = blockIdx.x / SLICES, c0 = (blockIdx.x % SLICES) * C;
  const int h = d.h, w = d.w, half = d.half, pts = max(h * w, half * h);
  float2* a = reinterpret_cast<float2*>(fft_smem4);
  float2* b = a + (size_t)pts * C;
  float* ctw = reinterpret_cast<float*>(b + (size_t)pts * C);
  float* stw = ctw + w;
  float* cth = stw + w;
  float* sth = cth + h;
  load_twiddles(fr, ctw, stw);
  load_twiddles(fc, cth, sth);
  const __half* re = spec + g * spec_plane + c0;
  const __half* im = spec + (g + d.groups) * spec_plane + c0;
  for (int t = threadIdx.x; t < half * h; t += blockDim.x) {
    const int ky = t / half, k = t - ky * half;
    float vr[C], vi[C];
    load_halves<C>(re + (size_t)t * 8, vr);
    load_halves<C>(im + (size_t)t * 8, vi);
    float2* dst = a + ((size_t)k * h + ky) * C;
#pragma unroll
    for (int c = 0; c < C; c++) dst[c] = make_float2(vr[c], vi[c]);
  }
  __syncthreads();
  float2* r = fft_lines<C>(a, b, half, fc, cth, sth, 1.0f);  // [k][y][c]
  float2* o = r == a ? b : a;
  for (int t = threadIdx.x; t < h * w; t += blockDim.x) {
    const int y = t / w, j = t - y * w;
    float2* dst = o + (size_t)t * C;
    if (j < half) {
      const float2* v = r + ((size_t)j * h + y) * C;
      const bool real_only = j == 0 || 2 * j == w;
#pragma unroll
      for (int c = 0; c < C; c++) dst[c] = make_float2(v[c].x, real_only ? 0.0f : v[c].y);
    } else {
      const float2* v = r + ((size_t)(w - j) * h + y) * C;
#pragma unroll
      for (int c = 0; c < C; c++) dst[c] = make_float2(v[c].x, -v[c].y);
    }
  }
  __syncthreads();
  const float2* q = fft_lines<C>(o, r, h, fr, ctw, stw, 1.0f);  // [y][j][c]
  __half* dst = x + g * x_plane + c0;
  for (int t = threadIdx.x; t < h * w; t += blockDim.x) {
    float v[C];
    load_halves<C>(dst + (size_t)t * 8, v);
#pragma unroll
    for (int c = 0; c < C; c++) v[c] += q[(size_t)t * C + c].x * d.scale;
    store_halves<C>(dst + (size_t)t * 8, v);
  }
}

// Shared memory of the one-launch transforms for C channels per CTA.
size_t small_smem(const FourierPlan& p, int c) {
  const size_t pts = std::max((size_t)p.h * p.w, (size_t)p.half * p.h);
  return 2 * pts * c * sizeof(float2) + (size_t)2 * (p.w + p.h) * sizeof(float);
}

constexpr size_t SMALL_SMEM_MAX = 200 * 1024;

// Channels per CTA of the one-launch transforms (the most that fit), or 0.
int small_channels(const FourierPlan& p) {
  for (int c : {8, 4, 2})
    if (small_smem(p, c) <= SMALL_SMEM_MAX) return c;
  return 0;
}

int log2_exact(int n) {
  int l = 0;
  while ((1 << l) < n) l++;
  return (1 << l) == n ? l : -1;
}

Dims dims_of(const FourierPlan& p) {
  Dims d;
  d.h = p.h;
  d.w = p.w;
  d.half = p.half;
  d.groups = p.channels / 8;
  d.lines_rows = std::max(1, FFT_POINTS / p.w);
  d.lines_cols = std::max(1, FFT_POINTS / p.h);
  d.scale = (float)(1.0 / std::sqrt((double)p.h * (double)p.w));
  return d;
}

Line line_of(const FourierPlan& p, bool rows) {
  const float* t = p.twiddles.as<float>();
  if (rows) return Line{p.w, log2_exact(p.w), t, t + p.w};
  return Line{p.h, log2_exact(p.h), t + 2 * p.w, t + 2 * p.w + p.h};
}

size_t smem_for(int lines, int n) { return (size_t)2 * lines * n * 8 * sizeof(float2) + (size_t)2 * n * sizeof(float); }

template <class K>
void prepare(K kernel, size_t bytes) {
  if (bytes > 48 * 1024) IEC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

}  // namespace

void fourier_plan(FourierPlan& plan, int h, int w, int channels) {
  if (h < 1 || w < 1 || h > FFT_MAX_N || w > FFT_MAX_N || channels % 8 != 0)
    throw Error(ERR_INPUT, "Fourier transform of " + std::to_string(h) + " x " + std::to_string(w) +
                               ": sides up to " + std::to_string(FFT_MAX_N));
  plan.h = h;
  plan.w = w;
  plan.half = w / 2 + 1;
  plan.channels = channels;
  std::vector<float> t(2 * (size_t)w + 2 * (size_t)h);
  for (int j = 0; j < w; j++) {
    const double a = 2.0 * M_PI * j / w;
    t[j] = (float)std::cos(a);
    t[w + j] = (float)std::sin(a);
  }
  for (int j = 0; j < h; j++) {
    const double a = 2.0 * M_PI * j / h;
    t[2 * w + j] = (float)std::cos(a);
    t[2 * w + h + j] = (float)std::sin(a);
  }
  plan.twiddles.reserve(t.size() * sizeof(float));
  IEC_CUDA(cudaMemcpy(plan.twiddles.get(), t.data(), t.size() * sizeof(float), cudaMemcpyHostToDevice));
  plan.scratch.reserve((size_t)channels / 8 * h * plan.half * 8 * sizeof(float2));
}

template <int C>
void launch_fwd_small(const FourierPlan& plan, const Dims& d, const __half* x, long long x_plane, __half* spec,
                      long long spec_plane, cudaStream_t s) {
  const size_t bytes = small_smem(plan, C);
  prepare(fft2_fwd_small<C>, bytes);
  launch_pdl(fft2_fwd_small<C>, dim3(d.groups * (8 / C)), FFT_SMALL_THREADS, bytes, s, x, x_plane, spec, spec_plane, d,
             line_of(plan, true), line_of(plan, false));
  IEC_CUDA(cudaGetLastError());
}

template <int C>
void launch_inv_small(const FourierPlan& plan, const Dims& d, const __half* spec, long long spec_plane, __half* x,
                      long long x_plane, cudaStream_t s) {
  const size_t bytes = small_smem(plan, C);
  prepare(fft2_inv_small<C>, bytes);
  launch_pdl(fft2_inv_small<C>, dim3(d.groups * (8 / C)), FFT_SMALL_THREADS, bytes, s, spec, spec_plane, x, x_plane, d,
             line_of(plan, true), line_of(plan, false));
  IEC_CUDA(cudaGetLastError());
}

void rfft2_planar(const FourierPlan& plan, const __half* x, long long x_plane_elems, __half* spec,
                  long long spec_plane_elems, cudaStream_t s) {
  const Dims d = dims_of(plan);
  switch (plan.two_pass ? 0 : small_channels(plan)) {
    case 8: return launch_fwd_small<8>(plan, d, x, x_plane_elems, spec, spec_plane_elems, s);
    case 4: return launch_fwd_small<4>(plan, d, x, x_plane_elems, spec, spec_plane_elems, s);
    case 2: return launch_fwd_small<2>(plan, d, x, x_plane_elems, spec, spec_plane_elems, s);
    default: break;
  }
  float2* T = plan.scratch.as<float2>();
  const size_t sr = smem_for(d.lines_rows, d.w), sc = smem_for(d.lines_cols, d.h);
  prepare(fft_rows_fwd, sr);
  prepare(fft_cols_fwd, sc);
  launch_pdl(fft_rows_fwd, dim3((d.h + d.lines_rows - 1) / d.lines_rows, d.groups), FFT_THREADS, sr, s, 
      x, x_plane_elems, T, d, line_of(plan, true));
  IEC_CUDA(cudaGetLastError());
  launch_pdl(fft_cols_fwd, dim3((d.half + d.lines_cols - 1) / d.lines_cols, d.groups), FFT_THREADS, sc, s, 
      T, spec, spec_plane_elems, d, line_of(plan, false));
  IEC_CUDA(cudaGetLastError());
}

void irfft2_add_planar(const FourierPlan& plan, const __half* spec, long long spec_plane_elems, __half* x,
                       long long x_plane_elems, cudaStream_t s) {
  const Dims d = dims_of(plan);
  switch (plan.two_pass ? 0 : small_channels(plan)) {
    case 8: return launch_inv_small<8>(plan, d, spec, spec_plane_elems, x, x_plane_elems, s);
    case 4: return launch_inv_small<4>(plan, d, spec, spec_plane_elems, x, x_plane_elems, s);
    case 2: return launch_inv_small<2>(plan, d, spec, spec_plane_elems, x, x_plane_elems, s);
    default: break;
  }
  float2* T = plan.scratch.as<float2>();
  const size_t sr = smem_for(d.lines_rows, d.w), sc = smem_for(d.lines_cols, d.h);
  prepare(fft_cols_inv, sc);
  prepare(fft_rows_inv, sr);
  launch_pdl(fft_cols_inv, dim3((d.half + d.lines_cols - 1) / d.lines_cols, d.groups), FFT_THREADS, sc, s, 
      spec, spec_plane_elems, T, d, line_of(plan, false));
  IEC_CUDA(cudaGetLastError());
  launch_pdl(fft_rows_inv, dim3((d.h + d.lines_rows - 1) / d.lines_rows, d.groups), FFT_THREADS, sr, s, 
      T, x, x_plane_elems, d, line_of(plan, true));
  IEC_CUDA(cudaGetLastError());
}

}  // namespace iec
