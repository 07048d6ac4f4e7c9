"""Python mirror of the reference models' public API over the CUDA backend.

The C ABI (include/iec_cuda.h, implemented by libiec_cuda.so next to this
file) is the product's boundary; this module is a thin ctypes binding with
the reference's method names and error kinds (crates/<model>-native/src/
lib.rs, crates/native-engine/src/lib.rs:62-85), used by the tests and the
benchmark. There is no CPU fallback: without the library or a B200 every
call fails loudly.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libiec_cuda.so")

OK, ERR_IO, ERR_WEIGHTS, ERR_INPUT, CANCELLED, ERR_GPU, ERR_TIMEOUT = range(7)
_KIND = {ERR_IO: "io", ERR_WEIGHTS: "weights", ERR_INPUT: "input", CANCELLED: "cancelled",
         ERR_GPU: "gpu", ERR_TIMEOUT: "timeout"}

PROGRESS = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_float, ctypes.c_void_p)


class IecError(RuntimeError):
    """A failed call: `code` is the iec_status, `kind` its Error variant."""

    def __init__(self, code: int, message: str):
        self.code = code
        self.kind = _KIND.get(code, "unknown")
        super().__init__(f"{self.kind}: {message}")


class Cancelled(IecError):
    pass


class Options(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("timeout_ms", ctypes.c_int), ("batch_chunk", ctypes.c_int)]


class LaunchRecord(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 64), ("flop", ctypes.c_double), ("bytes", ctypes.c_double),
                ("ms", ctypes.c_float)]


_lib = None


def lib():
    """The backend library, loaded once; raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        sz, vp, f32p = ctypes.c_size_t, ctypes.c_void_p, ctypes.POINTER(ctypes.c_float)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        L.iec_last_error.restype = ctypes.c_char_p
        L.iec_device_count.restype = ctypes.c_int
        L.iec_realesrgan_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(Options), ctypes.POINTER(vp)]
        L.iec_realesrgan_free.argtypes = [vp]
        L.iec_realesrgan_device_name.argtypes = [vp]
        L.iec_realesrgan_device_name.restype = ctypes.c_char_p
        L.iec_realesrgan_run_float.argtypes = [vp, f32p, sz, sz, f32p]
        L.iec_realesrgan_run_float_tiled.argtypes = [vp, f32p, sz, sz, sz, sz, f32p, PROGRESS, vp]
        L.iec_realesrgan_run.argtypes = [vp, u8p, sz, sz, u8p, PROGRESS, vp]
        L.iec_realesrgan_run_float_tiles.argtypes = [vp, f32p, sz, sz, sz, sz, sz, sz, f32p]
        L.iec_realesrgan_run_tiles_device.argtypes = [vp, vp, sz, sz, sz, sz, sz, sz, vp, vp]
        L.iec_realesrgan_run_batch.argtypes = [vp, vp, sz, sz, sz, vp, vp]
        L.iec_realesrgan_run_batch_u8.argtypes = [vp, vp, sz, sz, sz, vp, vp]
        L.iec_realesrgan_run_device.argtypes = [vp, vp, sz, sz, sz, vp, vp]
        L.iec_realesrgan_set_fused.argtypes = [vp, ctypes.c_int]
        L.iec_realesrgan_set_fused.restype = ctypes.c_int
        L.iec_scunet_run_batch.argtypes = [vp, vp, sz, sz, sz, vp, vp]
        L.iec_lama_run_batch.argtypes = [vp, vp, vp, sz, sz, sz, vp, vp]
        L.iec_birefnet_run_batch.argtypes = [vp, vp, sz, sz, vp, vp]
        L.iec_set_launch_timing.argtypes = [vp, ctypes.c_int]
        L.iec_launch_timing.argtypes = [vp, ctypes.POINTER(LaunchRecord), sz]
        L.iec_launch_timing.restype = sz
        L.iec_scunet_set_fused.argtypes = [vp, ctypes.c_int]
        L.iec_scunet_set_fused.restype = ctypes.c_int
        L.iec_birefnet_set_fused.argtypes = [vp, ctypes.c_int]
        L.iec_birefnet_set_fused.restype = ctypes.c_int
        L.iec_lama_set_fused.argtypes = [vp, ctypes.c_int]
        L.iec_selftest_fourier_unit_time.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                     ctypes.POINTER(ctypes.c_float)]
        L.iec_lama_set_fused.restype = ctypes.c_int
        L.iec_realesrgan_launches.argtypes = [vp, sz, sz, sz]
        L.iec_realesrgan_launches.restype = sz
        i32 = ctypes.c_int
        L.iec_selftest_gemm.argtypes = [i32, i32, i32, i32, i32, i32, f32p, f32p, f32p, i32, i32, f32p]
        L.iec_selftest_joinsplit.argtypes = [i32, i32, i32, f32p, f32p, f32p, f32p, i32, f32p, f32p, i32, f32p]
        L.iec_selftest_mma_rate.argtypes = [i32, i32, i32, f32p]
        L.iec_selftest_conv.argtypes = [i32, i32, i32, i32, i32, i32, i32, f32p, f32p, f32p, i32, f32p, i32, f32p]
        L.iec_selftest_rfft2.argtypes = [ctypes.c_int, f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         f32p, f32p]
        L.iec_selftest_wait_timeout.argtypes = [ctypes.c_int, ctypes.c_int]
        L.iec_selftest_wait_timeout.restype = ctypes.c_int
        L.iec_selftest_gemm_time.argtypes = [i32, i32, i32, i32, i32, i32, i32, i32, i32, i32, ctypes.POINTER(ctypes.c_float)]
        L.iec_selftest_attention.argtypes = [i32, f32p, i32, i32, f32p, i32, i32, i32, f32p]
        L.iec_scunet_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(Options), ctypes.POINTER(vp)]
        L.iec_scunet_free.argtypes = [vp]
        L.iec_scunet_device_name.argtypes = [vp]
        L.iec_scunet_device_name.restype = ctypes.c_char_p
        L.iec_scunet_run_float.argtypes = [vp, f32p, sz, sz, f32p]
        L.iec_scunet_run_float_tiled.argtypes = [vp, f32p, sz, sz, sz, sz, f32p, PROGRESS, vp]
        L.iec_scunet_run.argtypes = [vp, u8p, sz, sz, u8p, PROGRESS, vp]
        L.iec_scunet_run_device.argtypes = [vp, vp, sz, sz, vp, vp]
        L.iec_lama_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(Options), ctypes.POINTER(vp)]
        L.iec_lama_free.argtypes = [vp]
        L.iec_lama_device_name.argtypes = [vp]
        L.iec_lama_device_name.restype = ctypes.c_char_p
        L.iec_lama_run_float.argtypes = [vp, f32p, f32p, sz, sz, f32p]
        L.iec_lama_run.argtypes = [vp, u8p, u8p, sz, sz, u8p, PROGRESS, vp]
        L.iec_lama_run_device.argtypes = [vp, vp, vp, sz, sz, vp, vp]
        L.iec_birefnet_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(Options), ctypes.POINTER(vp)]
        L.iec_birefnet_free.argtypes = [vp]
        L.iec_birefnet_device_name.argtypes = [vp]
        L.iec_birefnet_device_name.restype = ctypes.c_char_p
        L.iec_birefnet_run.argtypes = [vp, u8p, sz, f32p]
        L.iec_birefnet_run_normalized.argtypes = [vp, f32p, sz, f32p]
        L.iec_birefnet_run_device.argtypes = [vp, vp, i32, sz, vp, vp]
        L.iec_realesrgan_set_timing.argtypes = [vp, sz]
        L.iec_realesrgan_timing.argtypes = [vp, ctypes.POINTER(ctypes.c_int), f32p, sz]
        L.iec_realesrgan_timing.restype = sz
        _lib = L
    return _lib


def _check(status: int):
    if status != OK:
        msg = lib().iec_last_error().decode(errors="replace")
        raise (Cancelled if status == CANCELLED else IecError)(status, msg)


def device_count() -> int:
    return lib().iec_device_count()


def _progress(progress):
    """The reference's progress closure (returns ControlFlow::Break to stop)
    as a C callback: `progress(done)` returning True stops the run."""
    if progress is None:
        return PROGRESS()
    return PROGRESS(lambda done, _user: 1 if progress(done) else 0)


def _f32(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


class RealEsrgan:
    """crates/realesrgan-native/src/lib.rs Model, on the CUDA backend."""

    SCALE = 4
    GPU_TILE = 768
    MARGIN = 34
    STEPS = 34

    def __init__(self, path, device: int = -1, timeout_ms: int = 0, batch_chunk: int = 0):
        self._h = ctypes.c_void_p()
        opt = Options(device, timeout_ms, batch_chunk)
        _check(lib().iec_realesrgan_load(os.fsencode(path), ctypes.byref(opt), ctypes.byref(self._h)))

    load = classmethod(lambda cls, path, **kw: cls(path, **kw))

    def close(self):
        if getattr(self, "_h", None):
            lib().iec_realesrgan_free(self._h)
            self._h = None

    __del__ = close

    def gpu(self) -> str:
        """Model::gpu: the device's name."""
        return lib().iec_realesrgan_device_name(self._h).decode()

    def run_float(self, image: np.ndarray) -> np.ndarray:
        """Model::run_float: HxWx3 floats in 0..=1 to 4Hx4Wx3, unclamped."""
        image = np.ascontiguousarray(image, np.float32)
        h, w, c = image.shape
        assert c == 3
        out = np.empty((4 * h, 4 * w, 3), np.float32)
        _check(lib().iec_realesrgan_run_float(self._h, _f32(image), w, h, _f32(out)))
        return out

    def run_float_tiled(self, image: np.ndarray, tile: int, margin: int, progress=None) -> np.ndarray:
        """Model::run_float_tiled; `progress(done)` returning True cancels."""
        image = np.ascontiguousarray(image, np.float32)
        h, w, _ = image.shape
        out = np.empty((4 * h, 4 * w, 3), np.float32)
        cb = _progress(progress)
        margin = min(margin, 2**64 - 1)
        _check(lib().iec_realesrgan_run_float_tiled(self._h, _f32(image), w, h, tile, margin, _f32(out), cb, None))
        return out

    def run(self, rgb: np.ndarray, progress=None) -> np.ndarray:
        """Model::run / run_with_progress: 8-bit RGB in and out."""
        rgb = np.ascontiguousarray(rgb, np.uint8)
        h, w, _ = rgb.shape
        out = np.empty((4 * h, 4 * w, 3), np.uint8)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        _check(lib().iec_realesrgan_run(self._h, rgb.ctypes.data_as(u8p), w, h, out.ctypes.data_as(u8p),
                                        _progress(progress), None))
        return out

    run_with_progress = run


    def run_float_tiles(self, image: np.ndarray, tile: int, margin: int, first: int, last: int, out=None):
        """Tiles first .. last - 1 of run_float_tiled's grid into `out` (the
        whole 4x output; the other tiles' windows are left untouched)."""
        image = np.ascontiguousarray(image, np.float32)
        h, w, _ = image.shape
        if out is None:
            out = np.zeros((4 * h, 4 * w, 3), np.float32)
        assert out.flags.c_contiguous and out.dtype == np.float32
        _check(lib().iec_realesrgan_run_float_tiles(self._h, _f32(image), w, h, tile, min(margin, 2**64 - 1),
                                                    first, last, _f32(out)))
        return out

    def run_tiles_device(self, image_ptr: int, width: int, height: int, tile: int, margin: int, first: int,
                         last: int, out_ptr: int, stream: int = 0):
        """run_float_tiles on device pointers, queued on `stream`."""
        _check(lib().iec_realesrgan_run_tiles_device(self._h, image_ptr, width, height, tile, margin, first, last,
                                                     out_ptr, stream or None))

    def run_batch(self, images, out=None, stream: int = 0):
        """Batched run_float on host arrays (N x H x W x 3). `images` and
        `out` may be page-locked torch tensors or numpy arrays."""
        n, h, w, _ = images.shape
        if out is None:
            out = np.empty((n, 4 * h, 4 * w, 3), np.float32)
        _check(lib().iec_realesrgan_run_batch(self._h, _addr(images), n, w, h, _addr(out), stream or None))
        return out

    def run_batch_u8(self, images, out=None, stream: int = 0):
        """Batched run (8-bit RGB in and out) on host arrays (N x H x W x 3);
        page-locked torch tensors or numpy arrays."""
        n, h, w, _ = images.shape
        if out is None:
            out = np.empty((n, 4 * h, 4 * w, 3), np.uint8)
        _check(lib().iec_realesrgan_run_batch_u8(self._h, _addr(images), n, w, h, _addr(out), stream or None))
        return out

    def run_device(self, images_ptr: int, count: int, width: int, height: int, out_ptr: int, stream: int = 0):
        """Batched run_float on device pointers; queued on `stream`, no wait."""
        _check(lib().iec_realesrgan_run_device(self._h, images_ptr, count, width, height, out_ptr, stream or None))

    def launches(self, count: int, width: int, height: int) -> int:
        return lib().iec_realesrgan_launches(self._h, count, width, height)

    def set_fused(self, on: bool):
        """Fused 32-layer body launch (default) or one launch per layer."""
        _check(lib().iec_realesrgan_set_fused(self._h, 1 if on else 0))

    # Measurement hooks (see iec_cuda.h): kinds 0 prep, 1 conv 16->64,
    # 2 conv 64->64, 3 conv 64->48 + pixel shuffle, 4 the fused 32 layers.
    def set_timing(self, capacity: int):
        _check(lib().iec_realesrgan_set_timing(self._h, capacity))

    def timing(self, n: int):
        kinds = (ctypes.c_int * n)()
        ms = np.zeros(n, np.float32)
        k = lib().iec_realesrgan_timing(self._h, kinds, _f32(ms), n)
        return np.array(kinds[:k], np.int32), ms[:k]


def _addr(a) -> int:
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


def selftest_gemm(a, w, bias=None, *, conv=False, shape=None, act=0, accumulate_onto=None, device=0):
    """Diagnostics: one general-GEMM launch on host arrays. Rows: `a` is
    rows x k, `w` k x n. conv: `a` is h x w x k (shape=(h, w)), `w` 9k x n,
    3x3 zero padding. act 0 none, 1 ReLU, 2 GELU. Returns rows x n float32."""
    a = np.ascontiguousarray(a, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    n = w.shape[1]
    if conv:
        h, wd = shape
        k = a.shape[-1]
        rows_or_h, width, rows = h, wd, h * wd
    else:
        rows, k = a.shape
        rows_or_h, width = rows, 0
    out = (np.zeros((rows, n), np.float32) if accumulate_onto is None
           else np.ascontiguousarray(accumulate_onto, np.float32).copy())
    b = np.ascontiguousarray(bias, np.float32) if bias is not None else None
    st = lib().iec_selftest_gemm(device, int(conv), rows_or_h, width, k, n, _f32(a), _f32(w),
                                 _f32(b) if b is not None else None, act, int(accumulate_onto is not None), _f32(out))
    _check(st)
    return out


def selftest_joinsplit(x, y, wj, bj, ws, bs, *, fused=True, iters=0, device=0):
    """Diagnostics: SCUNet's block boundary x += y wj + bj; y = x ws + bs on
    host arrays (rows x c, c x c, c). fused runs the one-kernel form (c 64,
    128 or 256), else two GEMM launches. Returns (x, y, microseconds per pass or
    None)."""
    x = np.ascontiguousarray(x, np.float32).copy()
    y = np.ascontiguousarray(y, np.float32).copy()
    rows, c = x.shape
    us = np.zeros(1, np.float32)
    args = [np.ascontiguousarray(v, np.float32) for v in (wj, bj, ws, bs)]
    _check(lib().iec_selftest_joinsplit(device, rows, c, *[_f32(v) for v in args], int(fused), _f32(x), _f32(y),
                                        iters, _f32(us) if iters > 0 else None))
    return x, y, (float(us[0]) if iters > 0 else None)


def selftest_conv(a, w, bias=None, *, size=3, halo=-1, act=0, iters=0, device=0):
    """Diagnostics: a size x size convolution with zero padding through the
    general GEMM: `a` h x w x k, `w` (size^2 k) x n tap-major. halo -1 lets
    the GEMM choose its A operand, 0 one box per tap, 1 halo tiles wherever
    they fit. Returns (h w x n float32, microseconds per launch or None)."""
    a = np.ascontiguousarray(a, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    h, wd, k = a.shape
    n = w.shape[1]
    out = np.zeros((h * wd, n), np.float32)
    us = np.zeros(1, np.float32)
    b = np.ascontiguousarray(bias, np.float32) if bias is not None else None
    _check(lib().iec_selftest_conv(device, h, wd, k, n, size, halo, _f32(a), _f32(w),
                                   _f32(b) if b is not None else None, act, _f32(out), iters,
                                   _f32(us) if iters > 0 else None))
    return out, (float(us[0]) if iters > 0 else None)


def selftest_mma_rate(n: int, variant: int = 0, device: int = 0) -> float:
    """Diagnostics: SM cycles per tcgen05.mma kind::f16 128 x n x 16 (see
    iec_selftest_mma_rate); variant 0 unrolled, 1 through a run-time loop."""
    out = np.zeros(1, np.float32)
    _check(lib().iec_selftest_mma_rate(device, n, variant, _f32(out)))
    return float(out[0])


def selftest_attention(qkv, windows, c, bias, shifted, rows_w, cols_w, device=0):
    """Diagnostics: the fused window attention on host arrays (see
    iec_selftest_attention)."""
    qkv = np.ascontiguousarray(qkv, np.float32)
    bias = np.ascontiguousarray(bias, np.float32)
    out = np.zeros((windows * 64, c), np.float32)
    _check(lib().iec_selftest_attention(device, _f32(qkv), windows, c, _f32(bias), int(shifted), rows_w, cols_w,
                                        _f32(out)))
    return out


class Scunet:
    """crates/scunet-native/src/lib.rs Model, on the CUDA backend."""

    TILE = 896
    MARGIN = 64
    STEPS = 28

    def __init__(self, path, device: int = -1, timeout_ms: int = 0):
        self._h = ctypes.c_void_p()
        opt = Options(device, timeout_ms, 0)
        _check(lib().iec_scunet_load(os.fsencode(path), ctypes.byref(opt), ctypes.byref(self._h)))

    def close(self):
        if getattr(self, "_h", None):
            lib().iec_scunet_free(self._h)
            self._h = None

    __del__ = close

    def gpu(self) -> str:
        return lib().iec_scunet_device_name(self._h).decode()

    def run_float(self, image: np.ndarray) -> np.ndarray:
        """Model::run_float: HxWx3 floats to HxWx3, the whole image at once."""
        image = np.ascontiguousarray(image, np.float32)
        h, w, _ = image.shape
        out = np.empty_like(image)
        _check(lib().iec_scunet_run_float(self._h, _f32(image), w, h, _f32(out)))
        return out

    def run_float_tiled(self, image: np.ndarray, tile: int, margin: int, progress=None) -> np.ndarray:
        image = np.ascontiguousarray(image, np.float32)
        h, w, _ = image.shape
        out = np.empty_like(image)
        _check(lib().iec_scunet_run_float_tiled(self._h, _f32(image), w, h, tile, min(margin, 2**64 - 1), _f32(out),
                                                _progress(progress), None))
        return out

    def run_device(self, image_ptr: int, width: int, height: int, out_ptr: int, stream: int = 0):
        """run_float on device pointers, queued on `stream`."""
        _check(lib().iec_scunet_run_device(self._h, image_ptr, width, height, out_ptr, stream or None))

    def set_fused(self, on: bool):
        """Fused transformer MLPs (default) or LayerNorm + two GEMMs apart."""
        _check(lib().iec_scunet_set_fused(self._h, 1 if on else 0))

    def run_batch(self, images, out=None, stream: int = 0):
        """Batched run_float on host arrays (N x H x W x 3 float32; numpy or
        page-locked torch tensors), copies overlapped with the kernels."""
        n, h, w, _ = images.shape
        if out is None:
            out = np.empty((n, h, w, 3), np.float32)
        _check(lib().iec_scunet_run_batch(self._h, _addr(images), n, w, h, _addr(out), stream or None))
        return out

    def run(self, rgb: np.ndarray, progress=None) -> np.ndarray:
        rgb = np.ascontiguousarray(rgb, np.uint8)
        h, w, _ = rgb.shape
        out = np.empty_like(rgb)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        _check(lib().iec_scunet_run(self._h, rgb.ctypes.data_as(u8p), w, h, out.ctypes.data_as(u8p),
                                    _progress(progress), None))
        return out

    run_with_progress = run


class Lama:
    """crates/lama-native/src/lib.rs Model, on the CUDA backend."""

    MIN_SIDE = 9
    STEPS = 26

    def __init__(self, path, device: int = -1, timeout_ms: int = 0):
        self._h = ctypes.c_void_p()
        opt = Options(device, timeout_ms, 0)
        _check(lib().iec_lama_load(os.fsencode(path), ctypes.byref(opt), ctypes.byref(self._h)))

    def close(self):
        if getattr(self, "_h", None):
            lib().iec_lama_free(self._h)
            self._h = None

    __del__ = close

    def gpu(self) -> str:
        return lib().iec_lama_device_name(self._h).decode()

    def run_batch(self, images, masks, out=None, stream: int = 0):
        """Batched run_float on host arrays: images N x H x W x 3, masks
        N x H x W (float32; numpy or page-locked torch tensors)."""
        n, h, w, _ = images.shape
        if out is None:
            out = np.empty((n, h, w, 3), np.float32)
        _check(lib().iec_lama_run_batch(self._h, _addr(images), _addr(masks), n, w, h, _addr(out), stream or None))
        return out

    def set_fused(self, on: bool):
        """Fused Fourier units (default) or rfft2, GEMM and irfft2 apart."""
        _check(lib().iec_lama_set_fused(self._h, 1 if on else 0))

    def run_float(self, image: np.ndarray, mask: np.ndarray) -> np.ndarray:
        """Model::run_float: the prediction (HxWx3) for an HxWx3 image in
        0..=1 and an HxW mask (1 fills)."""
        image = np.ascontiguousarray(image, np.float32)
        mask = np.ascontiguousarray(mask, np.float32)
        h, w, _ = image.shape
        if mask.shape != (h, w):
            raise ValueError("mask must be height x width")
        out = np.empty_like(image)
        _check(lib().iec_lama_run_float(self._h, _f32(image), _f32(mask), w, h, _f32(out)))
        return out

    def run(self, rgb: np.ndarray, mask: np.ndarray, progress=None) -> np.ndarray:
        """Model::run: 8-bit RGB with the pixels where `mask` (u8) is not
        zero filled in."""
        rgb = np.ascontiguousarray(rgb, np.uint8)
        mask = np.ascontiguousarray(mask, np.uint8)
        h, w, _ = rgb.shape
        if mask.shape != (h, w):
            raise ValueError("mask must be height x width")
        out = np.empty_like(rgb)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        _check(lib().iec_lama_run(self._h, rgb.ctypes.data_as(u8p), mask.ctypes.data_as(u8p), w, h,
                                  out.ctypes.data_as(u8p), _progress(progress), None))
        return out

    run_with_progress = run

    def run_device(self, image_ptr: int, mask_ptr: int, width: int, height: int, out_ptr: int, stream: int = 0):
        """run_float on device pointers, queued on `stream`."""
        _check(lib().iec_lama_run_device(self._h, image_ptr, mask_ptr, width, height, out_ptr, stream or None))


class Birefnet:
    """crates/birefnet-native/src/lib.rs Model, on the CUDA backend."""

    def __init__(self, path, device: int = -1, timeout_ms: int = 0):
        self._h = ctypes.c_void_p()
        opt = Options(device, timeout_ms, 0)
        _check(lib().iec_birefnet_load(os.fsencode(path), ctypes.byref(opt), ctypes.byref(self._h)))

    def close(self):
        if getattr(self, "_h", None):
            lib().iec_birefnet_free(self._h)
            self._h = None

    __del__ = close

    def gpu(self) -> str:
        return lib().iec_birefnet_device_name(self._h).decode()

    def run(self, rgb: np.ndarray) -> np.ndarray:
        """Model::run: side x side logits of a side x side x 3 8-bit image."""
        rgb = np.ascontiguousarray(rgb, np.uint8)
        side = rgb.shape[0]
        out = np.empty((side, side), np.float32)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        _check(lib().iec_birefnet_run(self._h, rgb.ctypes.data_as(u8p), side, _f32(out)))
        return out

    def run_normalized(self, image: np.ndarray) -> np.ndarray:
        """Model::run_normalized: logits of an ImageNet-normalised image."""
        image = np.ascontiguousarray(image, np.float32)
        side = image.shape[0]
        out = np.empty((side, side), np.float32)
        _check(lib().iec_birefnet_run_normalized(self._h, _f32(image), side, _f32(out)))
        return out

    def set_fused(self, on: bool):
        """Fused backbone MLPs (default) or LayerNorm + two GEMMs apart."""
        _check(lib().iec_birefnet_set_fused(self._h, 1 if on else 0))

    def run_batch(self, images, out=None, stream: int = 0):
        """Batched run on host arrays: N x side x side x 3 uint8 images to
        N x side x side float32 logits."""
        n, side, _, _ = images.shape
        if out is None:
            out = np.empty((n, side, side), np.float32)
        _check(lib().iec_birefnet_run_batch(self._h, _addr(images), n, side, _addr(out), stream or None))
        return out

    def run_device(self, image_ptr: int, image_u8: bool, side: int, logits_ptr: int, stream: int = 0):
        """run / run_normalized on device pointers, queued on `stream`."""
        _check(lib().iec_birefnet_run_device(self._h, image_ptr, int(image_u8), side, logits_ptr, stream or None))


def selftest_rfft2(x: np.ndarray, device: int = -1, two_pass: bool = False):
    """LaMa's planar rfft2 / irfft2 on an h x w x c array (c % 8 == 0):
    returns (spectrum h x (w/2+1) x 2c, irfft2 of it h x w x c); `two_pass`
    forces the two-launch transforms."""
    x = np.ascontiguousarray(x, np.float32)
    h, w, c = x.shape
    spec = np.empty((h, w // 2 + 1, 2 * c), np.float32)
    back = np.empty_like(x)
    _check(lib().iec_selftest_rfft2(device, _f32(x), h, w, c, 1 if two_pass else 0, _f32(spec), _f32(back)))
    return spec, back


def selftest_fourier_unit_time(h: int = 64, w: int = 64, iters: int = 50, device: int = -1):
    """Device microseconds per run of LaMa's Fourier unit on an h x w map of
    192 channels: (fused unit, its row transforms, its column kernel, its
    inverse row transforms, rfft2 + GEMM + irfft2 as separate launches)."""
    us = (ctypes.c_float * 5)()
    _check(lib().iec_selftest_fourier_unit_time(device, h, w, iters, us))
    return tuple(us)


def set_launch_timing(model, on: bool):
    """Record CUDA events around every instrumented launch of `model` (a
    Scunet, Lama or Birefnet), passes eager meanwhile (iec_set_launch_timing)."""
    _check(lib().iec_set_launch_timing(model._h, 1 if on else 0))


def launch_timing(model, n: int = 100000):
    """The launches recorded since set_launch_timing(model, True), in order:
    dicts of name, flop, bytes (algorithmic) and ms (CUDA events)."""
    recs = (LaunchRecord * n)()
    k = lib().iec_launch_timing(model._h, recs, n)
    return [{"name": r.name.decode(), "flop": r.flop, "bytes": r.bytes, "ms": r.ms} for r in recs[:k]]


def selftest_wait_timeout(which: int, device: int = -1) -> int:
    """Status of a kernel whose bounded wait nothing ends (0: an mbarrier,
    1: a shared word); IEC_ERR_TIMEOUT when the bound works."""
    return lib().iec_selftest_wait_timeout(device, which)


def selftest_gemm_time(mode: int, m_or_h: int, w: int, k: int, n: int, out_map: bool = False, sources: int = 0,
                       iters: int = 50, device: int = -1, act: int = 1):
    """(device us, host enqueue us, graph-replay device us) per launch of
    one GEMM shape (iec_selftest_gemm_time)."""
    us = (ctypes.c_float * 3)()
    _check(lib().iec_selftest_gemm_time(device, mode, m_or_h, w, k, n, int(out_map), sources, act, iters, us))
    return tuple(us)
