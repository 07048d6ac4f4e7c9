// The 2-D real Fourier transforms of LaMa's Fourier units
// (crates/lama-native/src/fourier.rs): rfftn / irfftn over the two spatial
// axes with "ortho" scaling, on planar f16 maps, computed in f32.
#pragma once

#include <cuda_fp16.h>

#include "runtime.h"

namespace iec {

// Twiddles and scratch for transforms of h x w maps of `channels` channels.
struct FourierPlan {
  int h = 0, w = 0, half = 0, channels = 0;
  DeviceBuffer twiddles;  // cos / sin of 2 pi j / w, then of 2 pi j / h (f32, from double)
  DeviceBuffer scratch;   // row spectra [channels / 8][h][half][8] complex f32
  bool two_pass = false;  // always the two-launch transforms (for comparisons)
};

void fourier_plan(FourierPlan& plan, int h, int w, int channels);

// spec = rfft2(x): x planar [c / 8][>= h w rows][8] f16 (pixel y w + x);
// spec planar [2 c / 8][>= h half rows][8] f16, row ky half + k, the real
// parts in planes 0 .. c / 8 - 1 and the imaginary parts after them
// (fourier.rs:1-9: a spectrum pixel holds its channels' real parts, then
// their imaginary parts).
void rfft2_planar(const FourierPlan& plan, const __half* x, long long x_plane_elems, __half* spec,
                  long long spec_plane_elems, cudaStream_t s);

// x += irfft2(spec), reading only the real part of column 0 and, for an even
// width, of column w / 2 after the column transforms, as irfftn does.
void irfft2_add_planar(const FourierPlan& plan, const __half* spec, long long spec_plane_elems, __half* x,
                       long long x_plane_elems, cudaStream_t s);

}  // namespace iec
