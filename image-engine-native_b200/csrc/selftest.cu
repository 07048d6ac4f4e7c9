// Diagnostics entry points (no counterpart in the reference): single kernels
// of the backend on host buffers, so the tests can check each against the
// CPU oracle in isolation.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <functional>
#include <vector>
#include <memory>
#include <string>

#include "../../include/iec_cuda.h"
#include "fft.h"
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

extern "C" iec_status iec_selftest_joinsplit(int device, int rows, int c, const float* wj, const float* bj,
                                             const float* ws, const float* bs, int fused, float* x, float* y,
                                             int iters, float* us) {
  try {
    Options opt;
    opt.device = device;
    Device dev(opt);
    DeviceScope scope(dev);
    const size_t cc = (size_t)c * c;
    const std::vector<float> vwj(wj, wj + cc), vws(ws, ws + cc), vbj(bj, bj + c), vbs(bs, bs + c);
    PackedWeights pj, ps;
    pack_weights(pj, vwj, 1, c, c, bj);
    pack_weights(ps, vws, 1, c, c, bs);
    JoinSplitWeights jw;
    if (fused) pack_joinsplit(jw, c, vwj, vbj, vws, vbs);
    const long long plane = (long long)gemm_rows_alloc(rows) * 8;
    DeviceBuffer d32, dx, dy;
    d32.reserve((size_t)rows * c * 4);
    dx.reserve((size_t)plane * c / 8 * 2);
    dy.reserve((size_t)plane * c / 8 * 2);
    cudaStream_t s = dev.stream();
    for (int v = 0; v < 2; v++) {
      IEC_CUDA(cudaMemcpyAsync(d32.get(), v ? y : x, (size_t)rows * c * 4, cudaMemcpyHostToDevice, s));
      rows_to_planar(d32.as<float>(), rows, c, (v ? dy : dx).as<__half>(), plane, s);
    }
    auto run = [&] {
      if (fused) {
        joinsplit_planar(dev, jw, dx.as<__half>(), dy.as<__half>(), plane, rows, s);
        return;
      }
      GemmOutSpec o;
      o.plane_elems = plane;
      o.mode = OUT_ACCUM;
      o.out = dx.as<__half>();
      gemm_rows(dev, pj, dy.as<__half>(), plane, rows, ACT_NONE, o, s);
      o.mode = OUT_STORE;
      o.out = dy.as<__half>();
      gemm_rows(dev, ps, dx.as<__half>(), plane, rows, ACT_NONE, o, s);
    };
    run();
    for (int v = 0; v < 2; v++) {
      planar_to_rows((v ? dy : dx).as<__half>(), plane, rows, c, d32.as<float>(), s);
      IEC_CUDA(cudaMemcpyAsync(v ? y : x, d32.get(), (size_t)rows * c * 4, cudaMemcpyDeviceToHost, s));
    }
    dev.sync(s);
    if (iters > 0 && us) {
      // the timed launches keep rewriting the buffers; their values are not read
      cudaEvent_t e0, e1;
      IEC_CUDA(cudaEventCreate(&e0));
      IEC_CUDA(cudaEventCreate(&e1));
      IEC_CUDA(cudaEventRecord(e0, s));
      for (int i = 0; i < iters; i++) run();
      IEC_CUDA(cudaEventRecord(e1, s));
      IEC_CUDA(cudaEventSynchronize(e1));
      float ms = 0.0f;
      IEC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
      us[0] = ms * 1000.0f / (float)iters;
      IEC_CUDA(cudaEventDestroy(e0));
      IEC_CUDA(cudaEventDestroy(e1));
    }
    return IEC_OK;
  } catch (const Error& e) {
    return (iec_status)e.code;
  }
}

extern "C" iec_status iec_selftest_conv(int device, int h, int w, int k, int n, int size, int halo, const float* a,
                                        const float* weights, const float* bias, int act, float* out, int iters,
                                        float* us) {
  try {
    if (h < 1 || w < 1 || size < 1 || size > 7 || k % 8 != 0 || n < 1) throw Error(ERR_INPUT, "bad convolution");
    Options opt;
    opt.device = device;
    Device dev(opt);
    DeviceScope scope(dev);
    const int rows = h * w, taps = size * size;
    std::vector<float> wv(weights, weights + (size_t)taps * k * n);
    PackedWeights pw;
    pack_weights(pw, wv, taps, k, n, bias);
    std::vector<Tap> tt;
    for (int t = 0; t < taps; t++) tt.push_back(Tap{t / size - size / 2, t % size - size / 2, 0});
    const long long plane = (long long)gemm_rows_alloc(rows) * 8;
    const int out_groups = (n + 7) / 8;
    DeviceBuffer d_a32, d_a16, d_o32, d_o16;
    d_a32.reserve((size_t)rows * k * 4);
    d_a16.reserve((size_t)plane * (k / 8) * 2);
    d_o32.reserve((size_t)rows * out_groups * 8 * 4);
    d_o16.reserve((size_t)plane * out_groups * 2);
    cudaStream_t s = dev.stream();
    IEC_CUDA(cudaMemcpyAsync(d_a32.get(), a, (size_t)rows * k * 4, cudaMemcpyHostToDevice, s));
    rows_to_planar(d_a32.as<float>(), rows, k, d_a16.as<__half>(), plane, s);
    GemmOutSpec o;
    o.mode = OUT_STORE;
    o.out = d_o16.as<__half>();
    o.plane_elems = plane;
    const TapSource src{d_a16.as<__half>(), plane, w, h, 1};
    gemm_taps(dev, pw, src, tt, h, w, act, o, s, halo);
    planar_to_rows(d_o16.as<__half>(), plane, rows, out_groups * 8, d_o32.as<float>(), s);
    IEC_CUDA(cudaMemcpy2DAsync(out, (size_t)n * 4, d_o32.get(), (size_t)out_groups * 8 * 4, (size_t)n * 4, rows,
                               cudaMemcpyDeviceToHost, s));
    if (iters > 0 && us) {
      cudaEvent_t e0, e1;
      IEC_CUDA(cudaEventCreate(&e0));
      IEC_CUDA(cudaEventCreate(&e1));
      IEC_CUDA(cudaEventRecord(e0, s));
      for (int i = 0; i < iters; i++) gemm_taps(dev, pw, src, tt, h, w, act, o, s, halo);
      IEC_CUDA(cudaEventRecord(e1, s));
      dev.sync(s);
      float ms = 0.0f;
      IEC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
      us[0] = ms * 1000.0f / (float)iters;
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
    }
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
    const std::vector<float> tables =
        attention_bias_layout(std::vector<float>(bias, bias + (size_t)classes * (c / 32) * 64 * 64));
    IEC_CUDA(cudaMemcpyAsync(db.get(), tables.data(), tables.size() * 4, cudaMemcpyHostToDevice, s));
    dev.sync(s);  // the host vector goes out of scope
    rows_to_planar(d32.as<float>(), rows, 3 * c, dq.as<__half>(), plane, s);
    window_attention(dq.as<__half>(), plane, c, windows, db.as<float>(), shifted != 0, rows_w, cols_w,
                     dout.as<__half>(), plane, dev.dev_err(), s);
    planar_to_rows(dout.as<__half>(), plane, rows, c, do32.as<float>(), s);
    IEC_CUDA(cudaMemcpyAsync(out, do32.get(), (size_t)rows * c * 4, cudaMemcpyDeviceToHost, s));
    dev.sync(s);
    return IEC_OK;
  } catch (const Error& e) {
    return (iec_status)e.code;
  }
}

namespace {

// A wait that nothing ends: an mbarrier no thread arrives on (which 0), or a
// shared word no warp publishes (which 1, the fused body's wait for ready
// items). The bounded wait gives up after IEC_WAIT_NS, sets the error word
// and returns; the kernel then exits normally.
__global__ void selftest_wait_kernel(int which, int* dev_err) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  __shared__ uint32_t word;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    word = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    volatile int* flag = &abort_flag;
    if (which == 0)
      mbar_wait(&bar, 0, flag, dev_err, DEV_ERR_WAIT_FULL);
    else
      wait_word(&word, 0, flag, dev_err, DEV_ERR_WAIT_ROWS);
  }
}

}  // namespace

namespace {

// Issue rate of tcgen05.mma kind::f16 128 x N x 16 from zeroed shared
// memory (no-swizzle K-major operands as the GEMMs lay them out), one CTA
// per SM, `iters` x 4 MMAs into one accumulator. V 0: the four MMAs of an
// iteration unrolled with descriptors computed before the loop; V 1: the
// same MMAs issued through an inner loop whose trip count is only known at
// run time (2 x 2). cycles[cta] = SM cycles from the first issue to the
// completion of the last MMA.
template <int N, int V>
__global__ void __launch_bounds__(128, 1) selftest_mma_rate_kernel(int iters, int inner, unsigned long long* cycles,
                                                                   int* dev_err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t tslot;
  __shared__ int abort_flag;
  constexpr int A_BYTES = 128 * 64 * 2, B_BYTES = N * 64 * 2;
  for (int i = threadIdx.x; i < (A_BYTES + B_BYTES) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  fence_proxy_async_shared();
  if (threadIdx.x < 32) tmem_alloc(&tslot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tslot;
  if (threadIdx.x == 0) {
    const uint32_t a = smem_u32(smem), b = a + A_BYTES;
    constexpr uint32_t idesc = idesc_f16_f32(128, N);
    const unsigned long long t0 = clock64();
    if (V == 0) {
      uint64_t ad[4], bd[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        ad[j] = smem_desc(a + (uint32_t)(2 * j * 128 * 16), 128 * 16, 128);
        bd[j] = smem_desc(b + (uint32_t)(2 * j * N * 16), N * 16, 128);
      }
      for (int it = 0; it < iters; it++) {
#pragma unroll
        for (int j = 0; j < 4; j++) umma_f16(tmem, ad[j], bd[j], idesc, (it | j) != 0);
      }
    } else {
      for (int it = 0; it < iters; it++)
        for (int o = 0; o < 2; o++)
          for (int j = 0; j < inner; j++) {
            const int q = 2 * o + j;
            umma_f16(tmem, smem_desc(a + (uint32_t)(2 * q * 128 * 16), 128 * 16, 128),
                     smem_desc(b + (uint32_t)(2 * q * N * 16), N * 16, 128), idesc, (it | q) != 0);
          }
    }
    umma_commit(&bar);
    volatile int* flag = &abort_flag;
    mbar_wait(&bar, 0, flag, dev_err, DEV_ERR_WAIT_FULL);
    cycles[blockIdx.x] = clock64() - t0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(tmem, 256);
}

template <int N>
void mma_rate_launch(Device& dev, int variant, int iters, unsigned long long* cycles, cudaStream_t s) {
  // 120 KB of shared memory: one CTA per SM
  const int smem = 120 * 1024;
  auto k = variant == 0 ? selftest_mma_rate_kernel<N, 0> : selftest_mma_rate_kernel<N, 1>;
  IEC_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  k<<<dev.sms(), 128, smem, s>>>(iters, 2, cycles, dev.dev_err());
  IEC_CUDA(cudaGetLastError());
}

}  // namespace

extern "C" iec_status iec_selftest_mma_rate(int device, int n, int variant, float* cycles_per_mma) {
  try {
    if (variant != 0 && variant != 1) throw Error(ERR_INPUT, "mma rate: variant is 0 or 1");
    Options opt;
    opt.device = device;
    Device dev(opt);
    DeviceScope scope(dev);
    cudaStream_t s = dev.stream();
    const int iters = 4096, ctas = dev.sms();
    DeviceBuffer cyc;
    cyc.reserve((size_t)ctas * 8);
    for (int rep = 0; rep < 2; rep++) {  // the first launch warms up
      switch (n) {
        case 32: mma_rate_launch<32>(dev, variant, iters, cyc.as<unsigned long long>(), s); break;
        case 64: mma_rate_launch<64>(dev, variant, iters, cyc.as<unsigned long long>(), s); break;
        case 96: mma_rate_launch<96>(dev, variant, iters, cyc.as<unsigned long long>(), s); break;
        case 128: mma_rate_launch<128>(dev, variant, iters, cyc.as<unsigned long long>(), s); break;
        case 192: mma_rate_launch<192>(dev, variant, iters, cyc.as<unsigned long long>(), s); break;
        case 224: mma_rate_launch<224>(dev, variant, iters, cyc.as<unsigned long long>(), s); break;
        case 256: mma_rate_launch<256>(dev, variant, iters, cyc.as<unsigned long long>(), s); break;
        default: throw Error(ERR_INPUT, "mma rate: n is 32, 64, 96, 128, 192, 224 or 256");
      }
    }
    std::vector<unsigned long long> host(ctas);
    IEC_CUDA(cudaMemcpyAsync(host.data(), cyc.get(), (size_t)ctas * 8, cudaMemcpyDeviceToHost, s));
    dev.sync(s);
    double sum = 0;
    for (unsigned long long c : host) sum += (double)c;
    *cycles_per_mma = (float)(sum / ctas / (iters * 4.0));
    return IEC_OK;
  } catch (const Error& e) {
    return (iec_status)e.code;
  }
}

extern "C" iec_status iec_selftest_wait_timeout(int device, int which) {
  try {
    if (which != 0 && which != 1) throw Error(ERR_INPUT, "wait self-test: which is 0 or 1");
    Options opt;
    opt.device = device;
    Device dev(opt);
    DeviceScope scope(dev);
    cudaStream_t s = dev.stream();
    selftest_wait_kernel<<<1, 32, 0, s>>>(which, dev.dev_err());
    IEC_CUDA(cudaGetLastError());
    dev.sync(s);  // reads the error word back: IEC_ERR_TIMEOUT
    return IEC_OK;
  } catch (const Error& e) {
    return (iec_status)e.code;
  }
}

extern "C" iec_status iec_selftest_rfft2(int device, const float* x, int h, int w, int c, int two_pass, float* spec,
                                         float* back) {
  try {
    if (c % 8 != 0 || h < 1 || w < 1) throw Error(ERR_INPUT, "rfft2 self-test: c a multiple of 8");
    Options opt;
    opt.device = device;
    Device dev(opt);
    DeviceScope scope(dev);
    FourierPlan plan;
    fourier_plan(plan, h, w, c);
    plan.two_pass = two_pass != 0;
    const int half = w / 2 + 1, rows = h * w, frows = h * half;
    const long long xp = (long long)rows * 8, fp = (long long)frows * 8;
    DeviceBuffer d32, dx, dspec, dout;
    d32.reserve((size_t)std::max(rows * c, frows * 2 * c) * 4);
    dx.reserve((size_t)xp * (c / 8) * 2);
    dspec.reserve((size_t)fp * (2 * c / 8) * 2);
    cudaStream_t s = dev.stream();
    IEC_CUDA(cudaMemcpyAsync(d32.get(), x, (size_t)rows * c * 4, cudaMemcpyHostToDevice, s));
    rows_to_planar(d32.as<float>(), rows, c, dx.as<__half>(), xp, s);
    rfft2_planar(plan, dx.as<__half>(), xp, dspec.as<__half>(), fp, s);
    planar_to_rows(dspec.as<__half>(), fp, frows, 2 * c, d32.as<float>(), s);
    IEC_CUDA(cudaMemcpyAsync(spec, d32.get(), (size_t)frows * 2 * c * 4, cudaMemcpyDeviceToHost, s));
    IEC_CUDA(cudaMemsetAsync(dx.get(), 0, (size_t)xp * (c / 8) * 2, s));
    irfft2_add_planar(plan, dspec.as<__half>(), fp, dx.as<__half>(), xp, s);
    planar_to_rows(dx.as<__half>(), xp, rows, c, d32.as<float>(), s);
    IEC_CUDA(cudaMemcpyAsync(back, d32.get(), (size_t)rows * c * 4, cudaMemcpyDeviceToHost, s));
    dev.sync(s);
    return IEC_OK;
  } catch (const Error& e) {
    return (iec_status)e.code;
  }
}

// Diagnostics: LaMa's Fourier unit (x += irfft2(relu(rfft2(x) W + b))) on an
// h x w map of 192 channels, zero weights and a seeded map, `iters` times
// back to back after 3 warm-up runs: us[0] the fused unit, us[1] its row
// transforms alone, us[2] its column kernel alone, us[3] its inverse row
// transforms alone, us[4] rfft2, the GEMM and irfft2 as separate launches;
// device microseconds per run (CUDA events on the launch stream).
extern "C" iec_status iec_selftest_fourier_unit_time(int device, int h, int w, int iters, float* us) {
  try {
    Options opt;
    opt.device = device;
    Device dev(opt);
    DeviceScope scope(dev);
    const int c = FOURIER_UNIT_CHANNELS, half = w / 2 + 1;
    FourierPlan plan;
    fourier_plan(plan, h, w, c);
    if (!fourier_unit_fits(plan)) throw Error(ERR_INPUT, "Fourier unit timing: up to 64 rows");
    std::vector<float> wm((size_t)2 * c * 2 * c, 0.0f), bias((size_t)2 * c, 0.0f);
    FourierWeights fw;
    pack_fourier_weights(fw, wm, bias);
    PackedWeights pw;
    pack_weights(pw, wm, 1, 2 * c, 2 * c, bias.data());
    const long long xp = (long long)gemm_rows_alloc(h * w) * 8, fp = (long long)gemm_rows_alloc(h * half) * 8;
    DeviceBuffer x, spec, filt;
    x.reserve((size_t)xp * (c / 8) * 2);
    spec.reserve((size_t)fp * (2 * c / 8) * 2);
    filt.reserve((size_t)fp * (2 * c / 8) * 2);
    cudaStream_t s = dev.stream();
    IEC_CUDA(cudaMemsetAsync(x.get(), 0, (size_t)xp * (c / 8) * 2, s));
    IEC_CUDA(cudaMemsetAsync(spec.get(), 0, (size_t)fp * (2 * c / 8) * 2, s));
    cudaEvent_t e0, e1;
    IEC_CUDA(cudaEventCreate(&e0));
    IEC_CUDA(cudaEventCreate(&e1));
    auto timed = [&](const std::function<void()>& run) {
      for (int i = 0; i < 3; i++) run();
      IEC_CUDA(cudaEventRecord(e0, s));
      for (int i = 0; i < iters; i++) run();
      IEC_CUDA(cudaEventRecord(e1, s));
      dev.sync(s);
      float ms = 0;
      IEC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
      return ms * 1000.0f / (float)iters;
    };
    for (int only = 0; only < 4; only++)
      us[only] = timed([&] { fourier_unit_planar(plan, fw, x.as<__half>(), xp, dev.dev_err(), s, only); });
    us[4] = timed([&] {
      rfft2_planar(plan, x.as<__half>(), xp, spec.as<__half>(), fp, s);
      GemmOutSpec fo;
      fo.mode = OUT_STORE;
      fo.out = filt.as<__half>();
      fo.plane_elems = fp;
      gemm_rows(dev, pw, spec.as<__half>(), fp, h * half, ACT_RELU, fo, s);
      irfft2_add_planar(plan, filt.as<__half>(), fp, x.as<__half>(), xp, s);
    });
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    dev.sync(s);
    return IEC_OK;
  } catch (const Error& e) {
    return (iec_status)e.code;
  }
}

// Diagnostics: per launch of the general GEMM on zero-filled device buffers,
// `iters` launches back to back after 3 warm-up ones: us[0] device
// microseconds, us[1] host microseconds to enqueue, us[2] device microseconds
// when the launches replay from a CUDA graph. mode 0: rows (m x k); mode 1: 3x3 taps over an h x w map (K = k per
// tap); mode 2: one tap over an h x w map. out_map: store through OUT_MAP
// (unpadded map) with `sources` old-value sources (0..2) instead of OUT_STORE.
extern "C" iec_status iec_selftest_gemm_time(int device, int mode, int m_or_h, int w, int k, int n, int out_map,
                                             int sources, int act, int iters, float* us) {
  try {
    Options opt;
    opt.device = device;
    Device dev(opt);
    DeviceScope scope(dev);
    const int taps = mode == 1 ? 9 : 1;
    // rows stored through the map epilogue: a map of rows / 64 x 64 pixels
    const int h = mode == 0 ? (out_map ? m_or_h / 64 : 1) : m_or_h, width = mode == 0 ? (out_map ? 64 : 1) : w;
    const int rows = mode == 0 ? m_or_h : h * width;
    if (mode == 0 && out_map && m_or_h % 64 != 0) throw Error(ERR_INPUT, "map rows: a multiple of 64");
    std::vector<float> wv((size_t)taps * k * n, 0.0f);
    std::vector<float> bias(n, 0.0f);
    PackedWeights pw;
    pack_weights(pw, wv, taps, k, n, bias.data());
    const MapGeom src_geom{h, width, 1, 1};
    const long long in_plane = mode == 0 ? (long long)gemm_rows_alloc(rows) * 8 : src_geom.plane_elems();
    const long long out_plane = out_map ? (long long)h * width * 8 : (long long)gemm_rows_alloc(rows) * 8;
    DeviceBuffer a, o, s1, s2;
    const size_t abytes = (size_t)in_plane * (k / 8) * 2, obytes = (size_t)out_plane * ((n + 7) / 8) * 2;
    a.reserve(abytes);
    o.reserve(obytes);
    s1.reserve(obytes);
    s2.reserve(obytes);
    cudaStream_t s = dev.stream();
    IEC_CUDA(cudaMemsetAsync(a.get(), 0, abytes, s));
    IEC_CUDA(cudaMemsetAsync(o.get(), 0, obytes, s));
    IEC_CUDA(cudaMemsetAsync(s1.get(), 0, obytes, s));
    IEC_CUDA(cudaMemsetAsync(s2.get(), 0, obytes, s));
    GemmOutSpec spec;
    if (out_map) {
      spec = map_out(MapGeom{h, width, 0, 1}, o.as<__half>());
      if (sources >= 1) spec.acc_src = s1.as<__half>();
      if (sources >= 2) spec.resid = s2.as<__half>();
    } else {
      spec.mode = OUT_STORE;
      spec.out = o.as<__half>();
      spec.plane_elems = out_plane;
    }
    std::vector<Tap> tl;
    if (mode == 1)
      for (int t = 0; t < 9; t++) tl.push_back({t / 3, t % 3, 0});
    else
      tl.push_back({1, 1, 0});
    auto launch = [&]() {
      if (mode == 0)
        gemm_rows(dev, pw, a.as<__half>(), in_plane, rows, act, spec, s);
      else
        gemm_taps(dev, pw, src_geom.source(a.as<__half>()), tl, h, width, act, spec, s);
    };
    for (int i = 0; i < 3; i++) launch();
    cudaEvent_t e0, e1;
    IEC_CUDA(cudaEventCreate(&e0));
    IEC_CUDA(cudaEventCreate(&e1));
    dev.sync(s);
    const auto h0 = std::chrono::steady_clock::now();
    IEC_CUDA(cudaEventRecord(e0, s));
    for (int i = 0; i < iters; i++) launch();
    IEC_CUDA(cudaEventRecord(e1, s));
    const auto h1 = std::chrono::steady_clock::now();
    dev.sync(s);
    float ms = 0;
    IEC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    us[0] = ms * 1000.0f / (float)iters;
    us[1] = (float)std::chrono::duration<double, std::micro>(h1 - h0).count() / (float)iters;
    // The same launches replayed from a CUDA graph: no host work between them.
    cudaGraph_t graph;
    cudaGraphExec_t exec;
    IEC_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    for (int i = 0; i < iters; i++) launch();
    IEC_CUDA(cudaStreamEndCapture(s, &graph));
    IEC_CUDA(cudaGraphInstantiate(&exec, graph, 0));
    IEC_CUDA(cudaGraphLaunch(exec, s));
    IEC_CUDA(cudaEventRecord(e0, s));
    IEC_CUDA(cudaGraphLaunch(exec, s));
    IEC_CUDA(cudaEventRecord(e1, s));
    dev.sync(s);
    IEC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    us[2] = ms * 1000.0f / (float)iters;
    cudaGraphExecDestroy(exec);
    cudaGraphDestroy(graph);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return IEC_OK;
  } catch (const Error& e) {
    return (iec_status)e.code;
  }
}
