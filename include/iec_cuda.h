/*
 * iec_cuda.h - C ABI of the B200 (sm_100a) CUDA backend for the image models
 * of image-engine-native.
 *
 * Each entry point replaces one call of a reference model crate's public API
 * (crates/<model>-native/src/lib.rs), with the same argument meaning and
 * errors, so that a native-cuda backend crate binds it with plain `extern
 * "C"` declarations. Images are NHWC (row by row, channels interleaved), as
 * everywhere in the reference.
 *
 * Errors (crates/native-engine/src/lib.rs:62-85, Error): every call returns
 * an iec_status; the message of the last failure on the calling thread is
 * iec_last_error(). A GPU failure or a wait that timed out poisons the
 * handle, as the reference's Vulkan backend refuses work after a failed
 * wait (crates/native-vulkan/src/lib.rs:443-480, usable): every later call
 * on it returns IEC_ERR_GPU. Handles are not thread-safe: one handle per
 * host thread (the reference's Model takes &mut self).
 */
#ifndef IEC_CUDA_H
#define IEC_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum iec_status {
  IEC_OK = 0,
  IEC_ERR_IO = 1,       /* Error::Io: a file could not be read */
  IEC_ERR_WEIGHTS = 2,  /* Error::Weights: the weights file is not this model's */
  IEC_ERR_INPUT = 3,    /* Error::Input: bad sizes or arguments */
  IEC_CANCELLED = 4,    /* Error::Cancelled: the progress callback asked to stop */
  IEC_ERR_GPU = 5,      /* Error::Gpu: no usable GPU, or a CUDA failure */
  IEC_ERR_TIMEOUT = 6   /* a bounded wait on the GPU ran out (also poisons) */
} iec_status;

/* Load options; a NULL pointer means all defaults. */
typedef struct iec_options {
  int device;       /* CUDA device ordinal; -1: $IEC_CUDA_DEVICE, else 0 */
  int timeout_ms;   /* bound on every host wait; 0: $IEC_TIMEOUT_MS, else 120000 */
  int batch_chunk;  /* images per launch in batched runs; 0: chosen by the backend */
} iec_options;

/* Called with the share of the work done (0..1] after each layer; a nonzero
 * return stops the run with IEC_CANCELLED (the reference's progress closure
 * returning ControlFlow::Break, crates/realesrgan-native/src/lib.rs:181-191). */
typedef int (*iec_progress_fn)(float done, void* user);

/* Message of the last failure on this thread ("" when none). */
const char* iec_last_error(void);

/* Number of CUDA devices the backend can use (0 without a GPU). */
int iec_device_count(void);

/* ------------------------------------------------------------------ Real-ESRGAN
 * crates/realesrgan-native/src/lib.rs: realesr-general-x4v3 (SRVGGNetCompact),
 * output 4x larger on each side. */
typedef struct iec_realesrgan iec_realesrgan;

/* Model::load (lib.rs:120-137) with IMAGE_ENGINE_NATIVE_GPU=1 semantics: a
 * missing or unsuitable GPU is IEC_ERR_GPU, never a CPU fallback. Reads the
 * "REALESRG" weights file export_weights.py writes (f32 or f16 matrices). */
iec_status iec_realesrgan_load(const char* weights_path, const iec_options* options,
                               iec_realesrgan** out);

/* Drop a model (frees its device memory). NULL is ignored. */
void iec_realesrgan_free(iec_realesrgan* model);

/* Model::gpu (lib.rs:153-159): the device's name. */
const char* iec_realesrgan_device_name(const iec_realesrgan* model);

/* Model::run_float (lib.rs:197-219): width x height x 3 floats in 0..=1 to
 * (4 width) x (4 height) x 3 floats, neither clamped nor rounded. Runs in
 * tiles of 768 with a 34-pixel margin, which give the whole image's result
 * bit for bit (each output pixel is computed the same way wherever its tile
 * is). */
iec_status iec_realesrgan_run_float(iec_realesrgan* model, const float* image, size_t width,
                                    size_t height, float* out);

/* Model::run_float_tiled (lib.rs:221-232): a grid of equal tiles at most
 * `tile` input pixels on a side, each run with up to `margin` pixels of its
 * surroundings (SIZE_MAX: unbounded). `progress` (may be NULL) is called 34
 * times per tile. */
iec_status iec_realesrgan_run_float_tiled(iec_realesrgan* model, const float* image, size_t width,
                                          size_t height, size_t tile, size_t margin, float* out,
                                          iec_progress_fn progress, void* user);

/* Model::run / run_with_progress (lib.rs:161-191): 8-bit RGB in and out
 * (v / 255 in, clamp(0, 1) * 255 rounded out), tiles of 768 with margin 34. */
iec_status iec_realesrgan_run(iec_realesrgan* model, const uint8_t* rgb, size_t width,
                              size_t height, uint8_t* out, iec_progress_fn progress, void* user);

/* Batched Model::run_float over `count` images of one size, HOST buffers
 * (count x height x width x 3 in, count x 4 height x 4 width x 3 out). The
 * copies and kernels are queued on `stream` (a cudaStream_t; NULL: the
 * model's own stream) and the call returns when the outputs are in `out`.
 * Page-locked host buffers let the copies overlap the kernels. */
iec_status iec_realesrgan_run_batch(iec_realesrgan* model, const float* images, size_t count,
                                    size_t width, size_t height, float* out, void* stream);

/* Batched Model::run (lib.rs:161-191) over `count` images of one size:
 * 8-bit RGB in (v / 255) and out (clamp(0, 1) * 255 rounded), HOST buffers,
 * each image run whole, which gives the tiled run's pixels bit for bit. The
 * host link carries a quarter of iec_realesrgan_run_batch's bytes. Queued on
 * `stream` (NULL: the model's stream); returns when the outputs are in
 * `out`. */
iec_status iec_realesrgan_run_batch_u8(iec_realesrgan* model, const uint8_t* images, size_t count,
                                       size_t width, size_t height, uint8_t* out, void* stream);

/* Part of Model::run_float_tiled for sharding one large image over GPUs: of
 * the grid of tiles run_float_tiled would cut (row-major order), only tiles
 * first .. last - 1 run, and only their own output windows of `out` (the
 * whole 4x image, width x height x 48 floats) are written; the rest of `out`
 * is left as it was. Host buffers; returns when the windows are in `out`.
 * Every tile's pixels come out exactly as in run_float_tiled. */
iec_status iec_realesrgan_run_float_tiles(iec_realesrgan* model, const float* image,
                                          size_t width, size_t height, size_t tile,
                                          size_t margin, size_t first, size_t last, float* out);

/* As iec_realesrgan_run_float_tiles on DEVICE pointers of the model's
 * device (the whole image in, the whole 4x output); queued on `stream`
 * (NULL: the model's stream), no wait. */
iec_status iec_realesrgan_run_tiles_device(iec_realesrgan* model, const float* image,
                                           size_t width, size_t height, size_t tile,
                                           size_t margin, size_t first, size_t last, float* out,
                                           void* stream);

/* As iec_realesrgan_run_batch on DEVICE pointers of the model's device; the
 * work is queued on `stream` and the call returns without waiting for it. */
iec_status iec_realesrgan_run_device(iec_realesrgan* model, const float* images, size_t count,
                                     size_t width, size_t height, float* out, void* stream);

/* iec_realesrgan_run_device without any allocation. This entry point has no
 * counterpart in the reference. It is for callers that cannot allocate device
 * memory while they run: a process that hands all device memory to its own
 * pool allocator at start-up and forbids raw cudaMalloc afterwards, or a
 * real-time frame pipeline that cannot absorb the device-wide
 * synchronisation cudaMalloc and cudaFree imply. The other entry points grow
 * their feature maps with cudaMalloc on demand; this one keeps them in a
 * fixed scratch array built into the library, 31.5 MiB that every GPU which
 * loads the library holds until the process exits.
 *  - Limit: count x max(width, 32) x max(height, 6) <= 114688 pixels (for
 *    example one 384 x 256 image; 32 x 6 is the input box one tile of the
 *    convolution reads, so narrower or shorter images are counted at that
 *    size); a larger call returns IEC_ERR_INPUT before any work is queued.
 *  - The model itself is loaded beforehand with iec_realesrgan_load, which
 *    does allocate; the call only uses `images`, `out` and the scratch.
 *  - The first call on a device looks up the scratch array's device address
 *    (once per device); make that first call before any stream capture.
 *  - Every call on a device shares the one scratch array: calls whose work
 *    overlaps on the GPU (other streams, other models on the same device)
 *    race and corrupt each other's results. Order them on one stream.
 *  - Work is queued on `stream` (NULL: the model's stream); no wait. */
iec_status iec_realesrgan_run_device_noalloc(iec_realesrgan* model, const float* images,
                                             size_t count, size_t width, size_t height,
                                             float* out, void* stream);

/* Kernel launches one run_device call of this size makes (for accounting). */
size_t iec_realesrgan_launches(const iec_realesrgan* model, size_t count, size_t width,
                               size_t height);

/* Measurement hooks (no counterpart in the reference, which has no GPU
 * timestamps). iec_realesrgan_set_timing(model, capacity) makes every later
 * run record a CUDA event before each kernel launch and after the last one,
 * on the stream the kernel runs on, for up to `capacity` launches (0 turns
 * it off). iec_realesrgan_timing then waits for those events, writes each
 * launch's kind (0 input prep, 1 conv 16->64, 2 conv 64->64, 3 conv 64->48
 * with the pixel-shuffle store, 4 the 32 fused 64->64 layers) and duration in
 * ms, returns how many it wrote (at most `n`) and starts a new record. */
iec_status iec_realesrgan_set_timing(iec_realesrgan* model, size_t capacity);
size_t iec_realesrgan_timing(iec_realesrgan* model, int* kinds, float* ms, size_t n);

/* The 32 64->64 layers run as fused persistent launches (the default, `on` =
 * 1: one per pass, or four of 8 layers in passes with progress reports, each
 * launch's layers reported when it completes) or, with `on` = 0, as 32
 * launches. The outputs are identical; this switch exists to compare the
 * two. */
iec_status iec_realesrgan_set_fused(iec_realesrgan* model, int on);

/* ------------------------------------------------------------------ SCUNet
 * crates/scunet-native/src/lib.rs: SCUNet denoising, output the size of the
 * input. */
typedef struct iec_scunet iec_scunet;

/* Model::load (lib.rs:82-100) with IMAGE_ENGINE_NATIVE_GPU=1 semantics; the
 * "SCUNET\0\0" weights file of export_weights.py (f16 matrices). */
iec_status iec_scunet_load(const char* weights_path, const iec_options* options, iec_scunet** out);
void iec_scunet_free(iec_scunet* model);
const char* iec_scunet_device_name(const iec_scunet* model);

/* Model::run_float (lib.rs:148-162): the whole image at once (padded to a
 * multiple of 64 inside), neither clamped nor rounded. */
iec_status iec_scunet_run_float(iec_scunet* model, const float* image, size_t width, size_t height,
                                float* out);

/* Model::run_float_tiled (lib.rs:164-183); `progress` called 28 times per
 * tile. */
iec_status iec_scunet_run_float_tiled(iec_scunet* model, const float* image, size_t width,
                                      size_t height, size_t tile, size_t margin, float* out,
                                      iec_progress_fn progress, void* user);

/* Model::run / run_with_progress (lib.rs:121-146): 8-bit RGB in and out,
 * tiles of 896 with a 64-pixel margin. */
iec_status iec_scunet_run(iec_scunet* model, const uint8_t* rgb, size_t width, size_t height,
                          uint8_t* out, iec_progress_fn progress, void* user);

/* Model::run_float on DEVICE pointers of the model's device (width x height
 * x 3 floats in and out); queued on `stream` (NULL: the model's stream), no
 * wait. */
iec_status iec_scunet_run_device(iec_scunet* model, const float* image, size_t width, size_t height,
                                 float* out, void* stream);

/* Batched Model::run_float over `count` images of one size (each run whole,
 * as run_device runs it), HOST buffers: count x height x width x 3 in and
 * out. The H2D copy of the next image and the D2H copy of the previous one
 * overlap each image's kernels (page-locked buffers let them); queued on
 * `stream` (NULL: the model's stream), returns when the outputs are in
 * `out`. For sharding a batch of images over GPUs, one handle per GPU. */
iec_status iec_scunet_run_batch(iec_scunet* model, const float* images, size_t count, size_t width,
                                size_t height, float* out, void* stream);

/* Each transformer block runs its LayerNorms fused (the default, `on` = 1:
 * LN1 and the window partition folded into the qkv product's staged rows;
 * LN2, fc1, GELU and fc2 in one kernel with the hidden layer kept in shared
 * memory, for the widths those kernels take; with one head, LN1, qkv,
 * attention, the projection and the residual add in one kernel; a block's
 * join with the next block's split in one kernel) or, with `on` = 0, as LayerNorm
 * launches and GEMM launches through device buffers (for comparisons; no
 * counterpart in the reference). The two agree to f16 rounding (the
 * LayerNorm and product sums run in another order). */
iec_status iec_scunet_set_fused(iec_scunet* model, int on);

/* -------------------------------------------------------------------- LaMa
 * crates/lama-native/src/lib.rs: Big LaMa inpainting, output the size of the
 * input. Sides of at least 9 pixels (lib.rs:180-194); at most 12288 here. */
typedef struct iec_lama iec_lama;

/* Model::load (lib.rs:76-94) with IMAGE_ENGINE_NATIVE_GPU=1 semantics; the
 * "LAMA\0\0\0\0" weights file of tools/lama/export_weights.py. */
iec_status iec_lama_load(const char* weights_path, const iec_options* options, iec_lama** out);
void iec_lama_free(iec_lama* model);
const char* iec_lama_device_name(const iec_lama* model);

/* Model::run_float (lib.rs:163-172): the network's prediction for every
 * pixel, width x height x 3 floats, given the image (values in 0..=1) and a
 * mask of width x height floats (1 to fill, 0 to keep). */
iec_status iec_lama_run_float(iec_lama* model, const float* image, const float* mask, size_t width,
                              size_t height, float* out);

/* Model::run / run_with_progress (lib.rs:118-156): 8-bit RGB with the pixels
 * whose mask byte is not zero filled in; `progress` after each of the 26
 * steps, non-zero cancels (IEC_CANCELLED). */
iec_status iec_lama_run(iec_lama* model, const uint8_t* rgb, const uint8_t* mask, size_t width,
                        size_t height, uint8_t* out, iec_progress_fn progress, void* user);

/* Model::run_float on DEVICE pointers of the model's device; queued on
 * `stream` (NULL: the model's stream), no wait. */
iec_status iec_lama_run_device(iec_lama* model, const float* image, const float* mask, size_t width,
                               size_t height, float* out, void* stream);

/* Batched Model::run_float over `count` images of one size: images count x
 * height x width x 3 and masks count x height x width (1 fills) in, count x
 * height x width x 3 predictions out, HOST buffers, copies overlapped with
 * the kernels as in iec_scunet_run_batch. */
iec_status iec_lama_run_batch(iec_lama* model, const float* images, const float* masks, size_t count,
                              size_t width, size_t height, float* out, void* stream);

/* Each Fourier unit runs fused (the default, `on` = 1: rfft2, the spectral
 * 1x1 convolution and irfft2 in three launches, the spectrum kept in shared
 * memory and TMEM) or, with `on` = 0, as a forward transform, a GEMM and an
 * inverse transform through device buffers. The outputs are identical; this
 * switch exists to compare the two (no counterpart in the reference). */
iec_status iec_lama_set_fused(iec_lama* model, int on);

/* ---------------------------------------------------------------- BiRefNet
 * crates/birefnet-native/src/lib.rs: BiRefNet-lite background removal. The
 * side must be a positive multiple of 64 (lib.rs:175-187); at most 8192 here. */
typedef struct iec_birefnet iec_birefnet;

/* Model::load (lib.rs:62-80) with IMAGE_ENGINE_NATIVE_GPU=1 semantics; the
 * "BIREFNET" weights file of tools/birefnet/export_weights.py (f16 matrices). */
iec_status iec_birefnet_load(const char* weights_path, const iec_options* options, iec_birefnet** out);
void iec_birefnet_free(iec_birefnet* model);
const char* iec_birefnet_device_name(const iec_birefnet* model);

/* Model::run (lib.rs:116-133): the foreground logit of every pixel of a
 * side x side 8-bit RGB image (side * side floats); the sigmoid of a logit is
 * the pixel's opacity. */
iec_status iec_birefnet_run(iec_birefnet* model, const uint8_t* rgb, size_t side, float* logits);

/* Model::run_normalized (lib.rs:134-172): the same for an image already
 * normalised with the ImageNet mean and deviation (side x side x 3 floats). */
iec_status iec_birefnet_run_normalized(iec_birefnet* model, const float* image, size_t side, float* logits);

/* run / run_normalized on DEVICE pointers of the model's device (`image_u8`
 * selects 8-bit RGB or normalised floats); queued on `stream` (NULL: the
 * model's stream), no wait. */
iec_status iec_birefnet_run_device(iec_birefnet* model, const void* image, int image_u8, size_t side,
                                   float* logits, void* stream);

/* Batched Model::run over `count` 8-bit RGB images of side x side (HOST
 * buffers, count x side x side x 3 in), count x side x side logits out,
 * copies overlapped with the kernels as in iec_scunet_run_batch. */
iec_status iec_birefnet_run_batch(iec_birefnet* model, const uint8_t* images, size_t count, size_t side,
                                  float* logits, void* stream);

/* The backbone blocks run their LayerNorms fused (the default, `on` = 1:
 * norm1 and the window partition folded into the qkv product's staged rows
 * at width 96; norm2, fc1, GELU and fc2 in one kernel at widths 96 and 192)
 * or, with `on` = 0, as LayerNorm launches and GEMM launches (for
 * comparisons; no counterpart in the reference). The two agree to f16
 * rounding. */
iec_status iec_birefnet_set_fused(iec_birefnet* model, int on);

/* Launch timing (measurement hooks, no counterpart in the reference).
 * iec_set_launch_timing(model, 1) on any model handle (SCUNet, LaMa,
 * BiRefNet; Real-ESRGAN has its own hooks above) starts a new record: every
 * later launch of the general GEMM, its split-K reduce, the layer norms,
 * the window attention, the Fourier transforms and BiRefNet's deformable
 * sampling and resizes records a CUDA event before and after itself on the
 * stream it runs on, with its algorithmic FLOPs and bytes (the inputs read
 * once, the outputs written once); meanwhile passes run eagerly instead of
 * as CUDA graphs, with the work of their side streams on the pass's own
 * stream, so that each event pair times one kernel alone. iec_launch_timing waits for the events and writes up to
 * `n` records in launch order, returning how many; 0 turns recording off. */
typedef struct iec_launch_record {
  char name[64];  /* kernel, with the product's M x N x K for the GEMM */
  double flop;    /* algorithmic FLOPs of the launch (0 for data movement) */
  double bytes;   /* algorithmic bytes */
  float ms;       /* CUDA-event duration */
} iec_launch_record;

iec_status iec_set_launch_timing(void* model, int on);
size_t iec_launch_timing(void* model, iec_launch_record* records, size_t n);

/* Diagnostics (no counterpart in the reference): one launch of the general
 * GEMM on host arrays. conv = 0: `a` rows_or_h x k, `weights` k x n; conv = 1:
 * `a` rows_or_h x w x k, `weights` 9k x n (3x3, zero padding). act 0 none,
 * 1 ReLU, 2 GELU; accumulate adds onto `out` (rows x n). */
iec_status iec_selftest_gemm(int device, int conv, int rows_or_h, int w, int k, int n,
                             const float* a, const float* weights, const float* bias, int act,
                             int accumulate, float* out);

/* Diagnostics: a size x size convolution (zero padding size / 2) through the
 * general GEMM on host arrays: `a` h x w x k, `weights` size^2 k x n (tap-
 * major), out h x w x n. halo -1 lets the GEMM choose its A operand, 0 takes
 * one box per tap, 1 the halo tiles wherever they fit. With iters > 0 and
 * `us` non-null, us[0] gets the device microseconds per launch over `iters`
 * launches after the checked one. */
iec_status iec_selftest_conv(int device, int h, int w, int k, int n, int size, int halo, const float* a,
                             const float* weights, const float* bias, int act, float* out, int iters, float* us);

/* Diagnostics: SCUNet's block boundary on host arrays `x` and `y` (rows x c
 * each, rounded to f16 on the way in, overwritten with the results): x += y wj
 * + bj, then y = x ws + bs (wj, ws c x c row-major, row k column n). fused
 * non-zero runs the one-kernel form (c 64, 128 or 256), 0 two GEMM launches. With
 * iters > 0 and `us` non-null, us[0] gets the device microseconds per pass
 * over `iters` passes after the checked one. */
iec_status iec_selftest_joinsplit(int device, int rows, int c, const float* wj, const float* bj, const float* ws,
                                  const float* bs, int fused, float* x, float* y, int iters, float* us);

/* Diagnostics: the issue rate of tcgen05.mma kind::f16 128 x n x 16 (n 32,
 * 64, 96, 128, 192, 224 or 256) on zeroed no-swizzle operands, one CTA per
 * SM: *cycles_per_mma = SM cycles per MMA. variant 0 issues unrolled MMAs
 * with precomputed descriptors; 1 issues the same MMAs through an inner
 * loop whose trip count is known only at run time. */
iec_status iec_selftest_mma_rate(int device, int n, int variant, float* cycles_per_mma);

/* Diagnostics: LaMa's planar Fourier transforms on host arrays: `x` h x w x c
 * floats (c a multiple of 8, rounded to f16 on the way in); `spec` gets
 * rfft2(x) as h x (w / 2 + 1) x 2c floats (real parts of the c channels, then
 * imaginary), `back` gets irfft2 of that spectrum (h x w x c). `two_pass`
 * non-zero takes the two-launch transforms even where the one-launch ones
 * for small maps apply (the results are the same). */
iec_status iec_selftest_rfft2(int device, const float* x, int h, int w, int c, int two_pass, float* spec,
                              float* back);

/* Diagnostics: per launch of the general GEMM on zero-filled buffers (mode
 * 0: m x k rows; 1: 3x3 taps over an h x w map; 2: one tap over an h x w
 * map), `iters` launches back to back; out_map stores through the map
 * epilogue with `sources` (0..2) old-value sources; act 0 none, 1 ReLU, 2 GELU,
 * 3 sigmoid. us[0] device
 * microseconds, us[1] host microseconds to enqueue, us[2] device
 * microseconds replayed from a CUDA graph. */
iec_status iec_selftest_gemm_time(int device, int mode, int m_or_h, int w, int k, int n, int out_map,
                                  int sources, int act, int iters, float* us);

/* Diagnostics: LaMa's Fourier unit (x += irfft2(relu(rfft2(x) W + b)), 192
 * channels, h <= 64) on device buffers, `iters` runs back to back: us[0] the
 * fused unit, us[1] its row transforms alone, us[2] its column kernel alone,
 * us[3] its inverse row transforms alone, us[4] rfft2, the GEMM and irfft2
 * as separate launches; device microseconds per run. */
iec_status iec_selftest_fourier_unit_time(int device, int h, int w, int iters, float* us);

/* Diagnostics: the fused window attention on host arrays: `qkv` windows * 64
 * rows of 3c (q | k | v), `bias` classes x (c / 32) x 64 x 64, `out` windows *
 * 64 rows of c. */
iec_status iec_selftest_attention(int device, const float* qkv, int windows, int c, const float* bias,
                                  int shifted, int rows_w, int cols_w, float* out);

/* Diagnostics: failure detection without a fault. One kernel waits on
 * something nothing provides (`which` 0: an mbarrier no thread arrives on;
 * 1: a shared word no warp publishes, as the fused Real-ESRGAN body's
 * producer waits for ready items); its bounded wait gives up after about 2 s,
 * sets the device error word and returns, and the call returns
 * IEC_ERR_TIMEOUT. The CUDA context stays usable. */
iec_status iec_selftest_wait_timeout(int device, int which);

#ifdef __cplusplus
}
#endif

#endif /* IEC_CUDA_H */
