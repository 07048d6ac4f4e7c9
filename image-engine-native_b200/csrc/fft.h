// The 2-D real Fourier transforms of LaMa's Fourier units
// (crates/lama-native/src/fourier.rs): rfftn / irfftn over the two spatial
// axes with "ortho" scaling, on planar f16 maps, computed in f32.
#pragma once

#include <cuda_fp16.h>

#include <vector>

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

// LaMa's whole Fourier unit (crates/lama-native/src/network.rs:174-248 and
// fourier.rs:291-400, the "fourier" step of the spectral transform) on a map
// of FOURIER_UNIT_CHANNELS channels:
//   x += irfft2(relu(rfft2(x) W + b))
// with W the 2c x 2c matrix over the spectrum's planar channels (real parts,
// then imaginary parts) and b its bias. Three launches: the row transforms
// into the f32 row-spectrum scratch; one kernel in which a cluster of four
// CTAs owns two spectrum columns: column transforms in shared memory, the
// f16 spectrum exchanged through distributed shared memory, the 1x1 product
// on tcgen05 into TMEM (each CTA a quarter of the output channels), bias and
// ReLU, the inverse column transforms back into the scratch; and the inverse
// row transforms added on x. Same roundings as rfft2_planar, the GEMM and
// irfft2_add_planar one after another (f16 spectrum, f32 sums, f16 filtered
// spectrum). For maps of at most 64 rows.
constexpr int FOURIER_UNIT_CHANNELS = 192;

struct FourierWeights {
  DeviceBuffer b;     // [4 quarters][2c / 8 k groups][96 columns][8] f16
  DeviceBuffer bias;  // [4 quarters][96] f32
};

// `w` is the 2c x 2c matrix (row k, column n, planar order), `bias` 2c floats.
void pack_fourier_weights(FourierWeights& fw, const std::vector<float>& w, const std::vector<float>& bias);

bool fourier_unit_fits(const FourierPlan& plan);

// `only` (timing diagnostics): 0 the whole unit, 1 the row transforms, 2 the
// column kernel, 3 the inverse row transforms.
void fourier_unit_planar(const FourierPlan& plan, const FourierWeights& fw, __half* x, long long x_plane_elems,
                         int* dev_err, cudaStream_t s, int only = 0);

}  // namespace iec
