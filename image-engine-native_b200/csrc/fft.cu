// LaMa's 2-D real Fourier transforms on planar f16 maps (see fft.h).
//
// A transform runs as two passes through an f32 scratch of row spectra, each
// pass a batch of 1-D transforms of "lines": n points of one channel group
// (8 channels, the 16 bytes a pixel holds in one plane), so every load and
// store moves whole 16-byte pixel groups. A CTA holds up to 512 points
// (several short lines, or one long one) in shared memory and transforms them
// in place of fourier.rs's recursive mixed-radix FFT (fourier.rs:16-139):
// radix-4 (and one radix-2) Stockham passes when n is a power of two, else
// mixed-radix Stockham passes over n's factors in fourier.rs's order (4 while
// it divides n, then 2, then the odd primes ascending; radices 3, 5 and 7
// unrolled, any other prime as its own r-point sum). Twiddles are cos / sin
// of 2 pi j / n computed in double and rounded to f32, as fourier.rs:45-52
// makes them.
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
constexpr int FFT_POINTS = 256;   // points per CTA when lines are short (measured: 512 and 128 slower)
constexpr int FFT_MAX_N = 1536;   // longest line (shared memory: 2 x 64 n bytes)

__device__ __forceinline__ float4 cmul2(float4 v, float wr, float wi) {
  return make_float4(v.x * wr - v.y * wi, v.x * wi + v.y * wr, v.z * wr - v.w * wi, v.z * wi + v.w * wr);
}
__device__ __forceinline__ float4 add4(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
__device__ __forceinline__ float4 sub4(float4 a, float4 b) { return make_float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w); }
// v times (s i): (x + i y)(s i) = -s y + i s x, for both complex values of v.
__device__ __forceinline__ float4 mul_si(float4 v, float s) { return make_float4(-s * v.y, s * v.x, -s * v.w, s * v.z); }

struct Line {
  int n, log2n;  // log2n < 0: not a power of two
  const float* cos_t;
  const float* sin_t;
  int nf;        // other lengths: the radices of the stages, in order
  int fac[12];
};

// One Stockham stage of radix r for lines of n points x C channels:
// for span m (the product of the earlier radices) the r points
// k + j m + q n / r (q < r) of sub-transform (j, k) go through an r-point
// DFT (its roots of unity w^(n / r (p q mod r)) from the n-point table) and
// out to k + (r j + p) m turned by w^(p j m), w = exp(sign 2 pi i / n): the
// radix-2 and radix-4 stages of the power-of-two path, for any radix.
template <int C, int R>
__device__ __forceinline__ void radix_stage(const float4* __restrict__ src4, float4* __restrict__ dst4, int lines,
                                            int n, int r, int m, const float* ct, const float* st, float sign) {
  constexpr int P = C / 2;
  const int rr = R > 0 ? R : r, stride = n / rr, total = lines * stride * P;
  for (int t = threadIdx.x; t < total; t += blockDim.x) {
    const int cc = t % P, rest = t / P, line = rest / stride, i = rest - line * stride;
    const int j = i / m, k = i - j * m;
    const int base = line * n * P + cc;
    if constexpr (R > 0) {
      float4 x[R];
#pragma unroll
      for (int q = 0; q < R; q++) x[q] = src4[base + (k + j * m + q * stride) * P];
#pragma unroll
      for (int p = 0; p < R; p++) {
        float4 acc = x[0];
#pragma unroll
        for (int q = 1; q < R; q++) {
          const int idx = stride * ((p * q) % R);
          acc = add4(acc, cmul2(x[q], ct[idx], sign * st[idx]));
        }
        const int tw = p * j * m;
        dst4[base + (k + (R * j + p) * m) * P] = p == 0 ? acc : cmul2(acc, ct[tw], sign * st[tw]);
      }
    } else {
      for (int p = 0; p < rr; p++) {
        float4 acc = src4[base + (k + j * m) * P];
        for (int q = 1; q < rr; q++) {
          const int idx = stride * ((p * q) % rr);
          acc = add4(acc, cmul2(src4[base + (k + j * m + q * stride) * P], ct[idx], sign * st[idx]));
        }
        const int tw = p * j * m;
        dst4[base + (k + (rr * j + p) * m) * P] = p == 0 ? acc : cmul2(acc, ct[tw], sign * st[tw]);
      }
    }
  }
}



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
  static_assert(C % 2 == 0 && C >= 2 && C <= 24, "channel pairs per point");
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
  // Other lengths: mixed-radix stages (radix 4 while it divides n, then 2,
  // then the odd primes ascending, as fourier.rs:34-50 factors n).
  int m = 1;
  for (int s = 0; s < f.nf; s++) {
    const int r = f.fac[s];
    const float4* src4 = reinterpret_cast<const float4*>(a);
    float4* dst4 = reinterpret_cast<float4*>(b);
    switch (r) {
      case 2: radix_stage<C, 2>(src4, dst4, lines, n, r, m, ct, st, sign); break;
      case 3: radix_stage<C, 3>(src4, dst4, lines, n, r, m, ct, st, sign); break;
      case 4: radix_stage<C, 4>(src4, dst4, lines, n, r, m, ct, st, sign); break;
      case 5: radix_stage<C, 5>(src4, dst4, lines, n, r, m, ct, st, sign); break;
      case 7: radix_stage<C, 7>(src4, dst4, lines, n, r, m, ct, st, sign); break;
      default: radix_stage<C, 0>(src4, dst4, lines, n, r, m, ct, st, sign); break;
    }
    m *= r;
    __syncthreads();
    float2* tmp = a;
    a = b;
    b = tmp;
  }
  return a;
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

// ---------------------------------------------------------------- Fourier unit
// The spectral 1x1 convolution fused between the column transforms
// (fft.h, fourier_unit_planar). A cluster of FU_Q CTAs owns the spectrum
// columns 2 p and 2 p + 1 (MMA rows l * 64 + ky, l the column of the pair);
// CTA q of the cluster transforms the columns of complex channels
// 48 q .. 48 q + 47 and puts their f16 spectrum (real parts at K = channel,
// imaginary parts at K = 192 + channel) into its own A operand; after a
// cluster barrier each CTA copies the other three quarters of K from its
// peers' shared memory, issues the 24 K16 MMAs of its output quarter
// (N = 96: the real and imaginary parts of channels 48 q .. 48 q + 47) and
// runs bias, ReLU, the f16 rounding and the inverse column transforms of
// those channels into the row-spectrum scratch.
constexpr int FU_CH = FOURIER_UNIT_CHANNELS;  // complex channels
constexpr int FU_K = 2 * FU_CH;               // MMA K: real parts, then imaginary parts
constexpr int FU_Q = 4;                       // CTAs per cluster: output quarters
constexpr int FU_QCH = FU_CH / FU_Q;          // 48 complex channels per CTA
constexpr int FU_N = 2 * FU_QCH;              // 96 MMA columns per CTA
constexpr int FU_CC = 24;                     // channels per transform chunk
constexpr int FU_CHUNKS = FU_QCH / FU_CC;     // 2
constexpr int FU_THREADS = 384;
constexpr int FU_MAXH = 64;                   // spectrum rows per column (MMA rows per column)
constexpr int FU_A_BYTES = (FU_K / 8) * 128 * 16;             // 98304
constexpr int FU_B_BYTES = (FU_K / 8) * FU_N * 16;            // 73728
constexpr int FU_F_BYTES = 2 * FU_MAXH * FU_CC * 8;           // 24576 per buffer
constexpr int FU_B_OFF = FU_A_BYTES;
constexpr int FU_F_OFF = FU_B_OFF + FU_B_BYTES;
constexpr int FU_TW_OFF = FU_F_OFF + 2 * FU_F_BYTES;
constexpr int FU_BIAS_OFF = FU_TW_OFF + 2 * FU_MAXH * 4;
constexpr int FU_BAR_OFF = FU_BIAS_OFF + FU_N * 4;
constexpr int FU_SMEM = FU_BAR_OFF + 64;
constexpr uint32_t FU_TMEM_COLS = 128;
static_assert(FU_SMEM <= 227 * 1024, "Fourier unit shared memory");
static_assert(FU_CH % (8 * FU_Q) == 0 && FU_QCH % FU_CC == 0 && FU_CC % 8 == 0, "channel split");

struct FuParams {
  float2* T;             // row spectra [c / 8][h][half][8] complex: read, then overwritten
  const uint16_t* b;     // [FU_Q][FU_K / 8][FU_N][8] f16
  const float* bias;     // [FU_Q][FU_N]
  Dims d;
  Line f;                // the column transform (n = h)
  int* dev_err;
};

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// 16 bytes of CTA `rank`'s shared memory at the offset of `local` in ours.
__device__ __forceinline__ uint4 ld_peer16(const void* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(remote));
  return v;
}


__global__ void __launch_bounds__(FU_THREADS, 1) fourier_unit_cols(const FuParams p) {
  extern __shared__ __align__(128) uint8_t fu_smem[];
  uint8_t* A = fu_smem;
  uint8_t* B = fu_smem + FU_B_OFF;
  float2* fa = reinterpret_cast<float2*>(fu_smem + FU_F_OFF);
  float2* fb = reinterpret_cast<float2*>(fu_smem + FU_F_OFF + FU_F_BYTES);
  float* ct = reinterpret_cast<float*>(fu_smem + FU_TW_OFF);
  float* st = ct + FU_MAXH;
  float* sbias = reinterpret_cast<float*>(fu_smem + FU_BIAS_OFF);
  uint64_t* bbar = reinterpret_cast<uint64_t*>(fu_smem + FU_BAR_OFF);
  uint64_t* mbar = bbar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fu_smem + FU_BAR_OFF + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(fu_smem + FU_BAR_OFF + 20);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t q = cluster_rank();
  const int pair = blockIdx.x / FU_Q;
  const int h = p.d.h, half = p.d.half;
  const int k0 = 2 * pair;  // first spectrum column of the pair
  const uint8_t* bsrc = reinterpret_cast<const uint8_t*>(p.b) + (size_t)q * FU_B_BYTES;

  if (tid == 0) {
    mbar_init(bbar, 1);
    mbar_init(mbar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, FU_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // The weights and bias do not depend on the previous kernel: fetch them
  // while it drains.
  if (tid == 0) {
    mbar_arrive_expect_tx(bbar, (uint32_t)FU_B_BYTES);
    bulk_load(B, bsrc, (uint32_t)FU_B_BYTES, bbar);
  }
  if (tid < FU_N) sbias[tid] = p.bias[q * FU_N + tid];
  griddep_launch_dependents();
  griddep_wait();
  load_twiddles(p.f, ct, st);

  // ---- forward column transforms of this CTA's 48 channels, in chunks.
  // Every thread's row-spectrum points of both chunks are loaded at once
  // (one latency), then each chunk is transformed in shared memory.
  const float scale = p.d.scale;
  constexpr int TASKS = 2 * FU_MAXH * (FU_CC / 8);  // points of a chunk (lines x rows x groups)
  constexpr int PER = (TASKS + FU_THREADS - 1) / FU_THREADS;
  float4 pts[FU_CHUNKS][PER][4];
#pragma unroll
  for (int c = 0; c < FU_CHUNKS; c++) {
    const int g0 = (int)q * (FU_QCH / 8) + c * (FU_CC / 8);
#pragma unroll
    for (int i = 0; i < PER; i++) {
      const int t = tid + i * FU_THREADS;
      const int l = t / (h * (FU_CC / 8)), r = t - l * (h * (FU_CC / 8));
      const int y = r / (FU_CC / 8), j = r - y * (FU_CC / 8);
      const bool live = t < 2 * h * (FU_CC / 8) && k0 + l < half;
      const float4* src = reinterpret_cast<const float4*>(p.T + (((size_t)(g0 + j) * h + y) * half + k0 + l) * 8);
#pragma unroll
      for (int e = 0; e < 4; e++) pts[c][i][e] = live ? src[e] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
  }
#pragma unroll
  for (int c = 0; c < FU_CHUNKS; c++) {
    const int g0 = (int)q * (FU_QCH / 8) + c * (FU_CC / 8);
#pragma unroll
    for (int i = 0; i < PER; i++) {
      const int t = tid + i * FU_THREADS;
      if (t < 2 * h * (FU_CC / 8)) {
        const int l = t / (h * (FU_CC / 8)), r = t - l * (h * (FU_CC / 8));
        const int y = r / (FU_CC / 8), j = r - y * (FU_CC / 8);
        float4* dst = reinterpret_cast<float4*>(fa + ((size_t)l * h + y) * FU_CC + 8 * j);
#pragma unroll
        for (int e = 0; e < 4; e++) dst[e] = pts[c][i][e];
      }
    }
    __syncthreads();
    const float2* r = fft_lines<FU_CC>(fa, fb, 2, p.f, ct, st, -1.0f);
    for (int t = tid; t < 2 * h * (FU_CC / 8); t += FU_THREADS) {
      const int l = t / (h * (FU_CC / 8)), rr = t - l * (h * (FU_CC / 8));
      const int ky = rr / (FU_CC / 8), j = rr - ky * (FU_CC / 8);
      const float2* v = r + ((size_t)l * h + ky) * FU_CC + 8 * j;
      float vr[8], vi[8];
#pragma unroll
      for (int e = 0; e < 8; e++) {
        vr[e] = v[e].x * scale;
        vi[e] = v[e].y * scale;
      }
      const int row = l * FU_MAXH + ky, kg = g0 + j;
      store_half8(reinterpret_cast<__half*>(A + ((size_t)kg * 128 + row) * 16), vr);
      store_half8(reinterpret_cast<__half*>(A + ((size_t)(FU_CH / 8 + kg) * 128 + row) * 16), vi);
    }
    __syncthreads();
  }

  // ---- the other quarters of K from the cluster's peers: every load of a
  // thread issued before its stores
  cluster_sync_all();
  {
    constexpr int COPIES = (FU_Q - 1) * 2 * (FU_QCH / 8) * 128;
    constexpr int CPER = (COPIES + FU_THREADS - 1) / FU_THREADS;
    uint4 v[CPER];
    uint8_t* at[CPER];
#pragma unroll
    for (int i = 0; i < CPER; i++) {
      const int t = tid + i * FU_THREADS;
      const int tt = t < COPIES ? t : 0;
      const int peer_i = tt / (2 * (FU_QCH / 8) * 128), rest = tt - peer_i * (2 * (FU_QCH / 8) * 128);
      const uint32_t peer = ((uint32_t)peer_i + q + 1) % FU_Q;
      const int which = rest / ((FU_QCH / 8) * 128), rr = rest - which * ((FU_QCH / 8) * 128);
      const int kg = which * (FU_CH / 8) + (int)peer * (FU_QCH / 8) + rr / 128, row = rr % 128;
      at[i] = t < COPIES ? A + ((size_t)kg * 128 + row) * 16 : nullptr;
      if (at[i]) v[i] = ld_peer16(at[i], peer);
    }
#pragma unroll
    for (int i = 0; i < CPER; i++)
      if (at[i]) *reinterpret_cast<uint4*>(at[i]) = v[i];
  }
  fence_proxy_async_shared();
  cluster_sync_all();  // every peer has read our quarter: we may leave at any time from here

  // ---- the 1x1 product: D[128 rows][96] = A[128][384] x B[384][96]
  if (tid == 0) {
    if (mbar_wait(bbar, 0, abort_flag, p.dev_err, DEV_ERR_WAIT_WEIGHTS)) {
      tc_fence_after();
      constexpr uint32_t idesc = idesc_f16_f32(128, FU_N);
      const uint32_t abase = smem_u32(A), bbase = smem_u32(B);
#pragma unroll 4
      for (int j = 0; j < FU_K / 16; j++) {
        const uint64_t adesc = smem_desc(abase + (uint32_t)(2 * j * 128 * 16), 128 * 16, 128);
        const uint64_t bdesc = smem_desc(bbase + (uint32_t)(2 * j * FU_N * 16), FU_N * 16, 128);
        umma_f16(tmem, adesc, bdesc, idesc, j > 0 ? 1u : 0u);
      }
      umma_commit(mbar);
    }
  }
  const bool have = mbar_wait(mbar, 0, abort_flag, p.dev_err, DEV_ERR_WAIT_ACC_FULL);
  tc_fence_after();

  // ---- bias, ReLU, f16, inverse column transforms, chunk by chunk
  const int quarter = warp & 3, part = warp >> 2;  // TMEM lanes 32 quarter.., 8 channels each
  const int row = quarter * 32 + lane, l = row / FU_MAXH, ky = row % FU_MAXH;
  for (int c = 0; c < FU_CHUNKS; c++) {
    const int cl = c * FU_CC + part * 8;  // this warp's first channel (of the CTA's 48)
    uint32_t re[8], im[8];
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    tmem_ld8(tmem + lanes + (uint32_t)cl, re);
    tmem_ld8(tmem + lanes + (uint32_t)(FU_QCH + cl), im);
    tmem_wait_ld();
    if (ky < h) {
      float2 val[8];
#pragma unroll
      for (int e = 0; e < 8; e++) {
        float vr = __uint_as_float(re[e]) + sbias[cl + e], vi = __uint_as_float(im[e]) + sbias[FU_QCH + cl + e];
        vr = vr > 0.0f ? vr : 0.0f;
        vi = vi > 0.0f ? vi : 0.0f;
        const float2 rounded = __half22float2(__floats2half2_rn(vr, vi));
        val[e] = have ? rounded : make_float2(0.0f, 0.0f);
      }
      float2* dst = fa + ((size_t)l * h + ky) * FU_CC + part * 8;
#pragma unroll
      for (int e = 0; e < 8; e++) dst[e] = val[e];
    }
    __syncthreads();
    const float2* r = fft_lines<FU_CC>(fa, fb, 2, p.f, ct, st, 1.0f);
    const int g0 = (int)q * (FU_QCH / 8) + c * (FU_CC / 8);
    for (int t = tid; t < 2 * h * (FU_CC / 8); t += FU_THREADS) {
      const int ll = t / (h * (FU_CC / 8)), rr = t - ll * (h * (FU_CC / 8));
      const int y = rr / (FU_CC / 8), j = rr - y * (FU_CC / 8);
      if (k0 + ll < half)
        copy_point(p.T + (((size_t)(g0 + j) * h + y) * half + k0 + ll) * 8, r + ((size_t)ll * h + y) * FU_CC + 8 * j);
    }
    __syncthreads();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, FU_TMEM_COLS);
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
  Line f{};
  f.n = rows ? p.w : p.h;
  f.log2n = log2_exact(f.n);
  f.cos_t = rows ? t : t + 2 * p.w;
  f.sin_t = rows ? t + p.w : t + 2 * p.w + p.h;
  if (f.log2n < 0) {
    int left = f.n;
    for (int r : {4, 2})
      while (left % r == 0) {
        f.fac[f.nf++] = r;
        left /= r;
      }
    for (int r = 3; left > 1; r += 2)
      while (left % r == 0) {
        f.fac[f.nf++] = r;
        left /= r;
      }
  }
  return f;
}

size_t smem_for(int lines, int n) { return (size_t)2 * lines * n * 8 * sizeof(float2) + (size_t)2 * n * sizeof(float); }

template <class K>
void prepare(K kernel, size_t bytes) {
  if (bytes > 48 * 1024) IEC_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

// The row passes of the two-launch transforms: x -> row spectra, and row
// spectra -> added on x.
void launch_rows_fwd(const FourierPlan& plan, const Dims& d, const __half* x, long long x_plane_elems, cudaStream_t s) {
  const size_t sr = smem_for(d.lines_rows, d.w);
  prepare(fft_rows_fwd, sr);
  // bytes: the map read (f16), the row spectra written (complex f32)
  const double io = (double)plan.h * plan.w * plan.channels * 2 + (double)plan.h * plan.half * plan.channels * 8;
  timed_launch("fft_rows_fwd", 0.0, io, s, [&] {
    launch_pdl(fft_rows_fwd, dim3((d.h + d.lines_rows - 1) / d.lines_rows, d.groups), FFT_THREADS, sr, s, x,
               x_plane_elems, plan.scratch.as<float2>(), d, line_of(plan, true));
    IEC_CUDA(cudaGetLastError());
  });
}

void launch_rows_inv(const FourierPlan& plan, const Dims& d, __half* x, long long x_plane_elems, cudaStream_t s) {
  const size_t sr = smem_for(d.lines_rows, d.w);
  prepare(fft_rows_inv, sr);
  // bytes: the row spectra read, the map read and written
  const double io = (double)plan.h * plan.half * plan.channels * 8 + (double)plan.h * plan.w * plan.channels * 4;
  timed_launch("fft_rows_inv", 0.0, io, s, [&] {
    launch_pdl(fft_rows_inv, dim3((d.h + d.lines_rows - 1) / d.lines_rows, d.groups), FFT_THREADS, sr, s,
               (const float2*)plan.scratch.as<float2>(), x, x_plane_elems, d, line_of(plan, true));
    IEC_CUDA(cudaGetLastError());
  });
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
  // bytes: the map read (f16) and the spectrum written (f16, real and imaginary)
  const double io = (double)plan.h * plan.w * plan.channels * 2 + (double)plan.h * plan.half * plan.channels * 4;
  timed_launch("fft2_fwd_small", 0.0, io, s, [&] {
    launch_pdl(fft2_fwd_small<C>, dim3(d.groups * (8 / C)), FFT_SMALL_THREADS, bytes, s, x, x_plane, spec, spec_plane,
               d, line_of(plan, true), line_of(plan, false));
    IEC_CUDA(cudaGetLastError());
  });
}

template <int C>
void launch_inv_small(const FourierPlan& plan, const Dims& d, const __half* spec, long long spec_plane, __half* x,
                      long long x_plane, cudaStream_t s) {
  const size_t bytes = small_smem(plan, C);
  prepare(fft2_inv_small<C>, bytes);
  // bytes: the spectrum read, the map read and written
  const double io = (double)plan.h * plan.half * plan.channels * 4 + (double)plan.h * plan.w * plan.channels * 4;
  timed_launch("fft2_inv_small", 0.0, io, s, [&] {
    launch_pdl(fft2_inv_small<C>, dim3(d.groups * (8 / C)), FFT_SMALL_THREADS, bytes, s, spec, spec_plane, x, x_plane,
               d, line_of(plan, true), line_of(plan, false));
    IEC_CUDA(cudaGetLastError());
  });
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
  const size_t sc = smem_for(d.lines_cols, d.h);
  launch_rows_fwd(plan, d, x, x_plane_elems, s);
  prepare(fft_cols_fwd, sc);
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
  const size_t sc = smem_for(d.lines_cols, d.h);
  prepare(fft_cols_inv, sc);
  launch_pdl(fft_cols_inv, dim3((d.half + d.lines_cols - 1) / d.lines_cols, d.groups), FFT_THREADS, sc, s, 
      spec, spec_plane_elems, T, d, line_of(plan, false));
  IEC_CUDA(cudaGetLastError());
  launch_rows_inv(plan, d, x, x_plane_elems, s);
}

void pack_fourier_weights(FourierWeights& fw, const std::vector<float>& w, const std::vector<float>& bias) {
  if (w.size() != (size_t)FU_K * FU_K || bias.size() != (size_t)FU_K)
    throw Error(ERR_WEIGHTS, "Fourier unit weights of the wrong size");
  // CTA q's MMA column n: the real part (n < 48) or the imaginary part of
  // complex channel 48 q + n % 48, whose planar column is that channel or
  // 192 + that channel.
  auto column = [](int quarter, int n) { return (n < FU_QCH ? 0 : FU_CH) + quarter * FU_QCH + n % FU_QCH; };
  std::vector<uint16_t> b((size_t)FU_Q * FU_K * FU_N);
  std::vector<float> bb((size_t)FU_Q * FU_N);
  for (int q = 0; q < FU_Q; q++)
    for (int n = 0; n < FU_N; n++) {
      const int col = column(q, n);
      bb[(size_t)q * FU_N + n] = bias[col];
      for (int k = 0; k < FU_K; k++)
        b[(((size_t)q * (FU_K / 8) + k / 8) * FU_N + n) * 8 + k % 8] = f32_to_half(w[(size_t)k * FU_K + col]);
    }
  fw.b.reserve(b.size() * 2);
  fw.bias.reserve(bb.size() * 4);
  IEC_CUDA(cudaMemcpy(fw.b.get(), b.data(), b.size() * 2, cudaMemcpyHostToDevice));
  IEC_CUDA(cudaMemcpy(fw.bias.get(), bb.data(), bb.size() * 4, cudaMemcpyHostToDevice));
}

bool fourier_unit_fits(const FourierPlan& plan) {
  return plan.channels == FU_CH && plan.h <= FU_MAXH && plan.w >= 1 && !plan.two_pass;
}

void fourier_unit_planar(const FourierPlan& plan, const FourierWeights& fw, __half* x, long long x_plane_elems,
                         int* dev_err, cudaStream_t s, int only) {
  if (!fourier_unit_fits(plan)) throw Error(ERR_INPUT, "the fused Fourier unit takes 192 channels and up to 64 rows");
  const Dims d = dims_of(plan);
  if (only == 0 || only == 1) launch_rows_fwd(plan, d, x, x_plane_elems, s);
  if (only == 1 || only == 3) {
    if (only == 3) launch_rows_inv(plan, d, x, x_plane_elems, s);
    return;
  }
  static bool prepared[64] = {};
  int dev = 0;
  IEC_CUDA(cudaGetDevice(&dev));
  if (!prepared[dev & 63]) {
    IEC_CUDA(cudaFuncSetAttribute(fourier_unit_cols, cudaFuncAttributeMaxDynamicSharedMemorySize, FU_SMEM));
    prepared[dev & 63] = true;
  }
  FuParams fp;
  fp.T = plan.scratch.as<float2>();
  fp.b = fw.b.as<uint16_t>();
  fp.bias = fw.bias.as<float>();
  fp.d = d;
  fp.f = line_of(plan, false);
  fp.dev_err = dev_err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(FU_Q * ((d.half + 1) / 2));
  cfg.blockDim = dim3(FU_THREADS);
  cfg.dynamicSmemBytes = FU_SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = FU_Q;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  // FLOPs: the 1x1 product over the spectrum (h half rows, K = N = 2c);
  // bytes: the row spectra read and written (complex f32) and the weights
  const double rows = (double)plan.h * plan.half;
  timed_launch("fourier_unit_cols", 2.0 * rows * FU_K * FU_K, rows * plan.channels * 16 + (double)FU_K * FU_K * 2, s,
               [&] { IEC_CUDA(cudaLaunchKernelEx(&cfg, fourier_unit_cols, fp)); });
  if (only == 0) launch_rows_inv(plan, d, x, x_plane_elems, s);
}

}  // namespace iec
