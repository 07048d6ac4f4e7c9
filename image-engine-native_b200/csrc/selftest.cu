// Diagnostics entry points (no counterpart in the reference): single kernels
// of the backend on host buffers, so the tests can check each against the
// CPU oracle in isolation.
#include <cuda_runtime.h>

#include <algorithm>
#include <memory>
#include <string>

#include "../../include/iec_cuda.h"
#include "gemm.h"
#include "igemm_sm100.cuh"

using namespace iec;

extern "C" iec_status iec_selftest_gemm(int device, int conv, int rows_or_h, int w, int k, int n, const float* a,
                                        const float* weights, const float* bias, int act, int accumulate,
                                        float* out) {
  try {
    Options opt;
    opt.device = device;
    Device dev(opt);
    DeviceScope scope(dev);
    const int rows = conv ? rows_or_h * w : rows_or_h;
    const int taps = conv ? 9 : 1;
    std::vector<float> wv(weights, weights + (size_t)taps * k * n);
    PackedWeights pw;
    pack_weights(pw, wv, taps, k, n, bias);
    const long long in_plane = (long long)rows * 8, out_plane = (long long)rows * 8;
    const int out_groups = (n + 7) / 8;
    DeviceBuffer d_a32, d_a16, d_o32, d_o16;
    d_a32.reserve((size_t)rows * k * 4);
    d_a16.reserve((size_t)rows * k * 2);
    d_o32.reserve((size_t)rows * out_groups * 8 * 4);
    d_o16.reserve((size_t)rows * out_groups * 8 * 2);
    cudaStream_t s = dev.stream();
    IEC_CUDA(cudaMemcpyAsync(d_a32.get(), a, (size_t)rows * k * 4, cudaMemcpyHostToDevice, s));
    rows_to_planar(d_a32.as<float>(), rows, k, d_a16.as<__half>(), in_plane, s);
    IEC_CUDA(cudaMemsetAsync(d_o32.get(), 0, (size_t)rows * out_groups * 8 * 4, s));
    if (accumulate) {
      IEC_CUDA(cudaMemcpy2DAsync(d_o32.get(), (size_t)out_groups * 8 * 4, out, (size_t)n * 4, (size_t)n * 4, rows,
                                 cudaMemcpyHostToDevice, s));
    }
    rows_to_planar(d_o32.as<float>(), rows, out_groups * 8, d_o16.as<__half>(), out_plane, s);
    GemmOutSpec o;
    o.mode = accumulate ? OUT_ACCUM : OUT_STORE;
    o.out = d_o16.as<__half>();
    o.plane_elems = out_plane;
    if (conv)
      gemm_conv3(dev, pw, d_a16.as<__half>(), in_plane, rows_or_h, w, act, o, s);
    else
      gemm_rows(dev, pw, d_a16.as<__half>(), in_plane, rows, act, o, s);
    planar_to_rows(d_o16.as<__half>(), out_plane, rows, out_groups * 8, d_o32.as<float>(), s);
    IEC_CUDA(cudaMemcpy2DAsync(out, (size_t)n * 4, d_o32.get(), (size_t)out_groups * 8 * 4, (size_t)n * 4, rows,
                               cudaMemcpyDeviceToHost, s));
    dev.sync(s);
    return IEC_OK;
  } catch (const Error& e) {
    return (iec_status)e.code;
  }
}

extern "C" iec_status iec_selftest_attention(int device, const float* qkv, int windows, int c, const float* bias,
                                             int shifted, int rows_w, int cols_w, float* out) {
  try {
    Options opt;
    opt.device = device;
    Device dev(opt);
    DeviceScope scope(dev);
    const int rows = windows * 64, classes = shifted ? 4 : 1;
    const long long plane = (long long)std::max(rows, 128) * 8;
    DeviceBuffer d32, dq, db, dout, do32;
    d32.reserve((size_t)rows * 3 * c * 4);
    dq.reserve((size_t)plane * (3 * c / 8) * 2);
    db.reserve((size_t)classes * (c / 32) * 64 * 64 * 4);
    dout.reserve((size_t)plane * (c / 8) * 2);
    do32.reserve((size_t)rows * c * 4);
    cudaStream_t s = dev.stream();
    IEC_CUDA(cudaMemcpyAsync(d32.get(), qkv, (size_t)rows * 3 * c * 4, cudaMemcpyHostToDevice, s));
    IEC_CUDA(cudaMemcpyAsync(db.get(), bias, (size_t)classes * (c / 32) * 64 * 64 * 4, cudaMemcpyHostToDevice, s));
    rows_to_planar(d32.as<float>(), rows, 3 * c, dq.as<__half>(), plane, s);
    window_attention(dq.as<__half>(), plane, c, windows, db.as<float>(), shifted != 0, rows_w, cols_w,
                     dout.as<__half>(), plane, s);
    planar_to_rows(dout.as<__half>(), plane, rows, c, do32.as<float>(), s);
    IEC_CUDA(cudaMemcpyAsync(out, do32.get(), (size_t)rows * c * 4, cudaMemcpyDeviceToHost, s));
    dev.sync(s);
    return IEC_OK;
  } catch (const Error& e) {
    return (iec_status)e.code;
  }
}
