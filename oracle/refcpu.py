"""Test infrastructure: ctypes access to the CPU oracle (oracle/librefcpu.so).

The oracle restates the reference's CPU f32 path (crates/native-engine and
the model crates) in C++; see oracle/refcpu/engine.h for the file:line map.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it,
and only as the checker or the timed CPU baseline, never as the product.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librefcpu.so")

_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
PROGRESS = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_float, ctypes.c_void_p)


class OracleError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(f"status {code}: {message}")
        self.code = code


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.refcpu_last_error.restype = ctypes.c_char_p
        L.refcpu_f32_to_half.restype = ctypes.c_uint16
        L.refcpu_f32_to_half.argtypes = [ctypes.c_float]
        L.refcpu_half_to_f32.restype = ctypes.c_float
        L.refcpu_half_to_f32.argtypes = [ctypes.c_uint16]
        L.refcpu_parse_weights.argtypes = [ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p]
        sz = ctypes.c_size_t
        L.refcpu_multiply.argtypes = [
            ctypes.c_int, _f32p, sz, sz, sz, sz, sz, sz, ctypes.c_int, ctypes.POINTER(sz), sz,
            sz, sz, _f32p, sz, sz, _f32p, ctypes.c_int, _f32p, sz, ctypes.c_int, ctypes.c_int,
        ]
        L.refcpu_conv3.argtypes = [
            _f32p, sz, sz, sz, sz, ctypes.c_int, _f32p, sz, _f32p, ctypes.c_int, _f32p, sz,
            ctypes.c_int, ctypes.c_int,
        ]
        L.refcpu_realesrgan_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
        L.refcpu_realesrgan_free.argtypes = [ctypes.c_void_p]
        L.refcpu_realesrgan_run_float.argtypes = [ctypes.c_void_p, _f32p, sz, sz, _f32p]
        L.refcpu_realesrgan_run_tiled.argtypes = [
            ctypes.c_void_p, _f32p, sz, sz, sz, sz, _f32p, PROGRESS, ctypes.c_void_p,
        ]
        L.refcpu_scunet_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
        L.refcpu_scunet_free.argtypes = [ctypes.c_void_p]
        L.refcpu_scunet_run_float.argtypes = [ctypes.c_void_p, _f32p, sz, sz, _f32p]
        L.refcpu_scunet_run_tiled.argtypes = [
            ctypes.c_void_p, _f32p, sz, sz, sz, sz, _f32p, PROGRESS, ctypes.c_void_p,
        ]
        L.refcpu_lama_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
        L.refcpu_lama_free.argtypes = [ctypes.c_void_p]
        L.refcpu_lama_run_float.argtypes = [
            ctypes.c_void_p, _f32p, _f32p, sz, sz, _f32p, PROGRESS, ctypes.c_void_p,
        ]
        L.refcpu_rfft2.argtypes = [_f32p, sz, sz, sz, _f32p]
        L.refcpu_irfft2_add.argtypes = [_f32p, sz, sz, sz, _f32p]
        L.refcpu_birefnet_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
        L.refcpu_birefnet_free.argtypes = [ctypes.c_void_p]
        L.refcpu_birefnet_run_normalized.argtypes = [ctypes.c_void_p, _f32p, sz, _f32p]
        L.refcpu_birefnet_run.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint8), sz, _f32p]
        L.refcpu_resize.argtypes = [_f32p, sz, sz, sz, _f32p, sz, sz, ctypes.c_int]
        L.refcpu_attention.argtypes = [_f32p, sz, sz, _f32p, sz, _f32p]
        L.refcpu_layer_norm.argtypes = [_f32p, sz, sz, _f32p, _f32p]
        L.refcpu_gelu.argtypes = [_f32p, sz]
        L.refcpu_sigmoid.argtypes = [_f32p, sz]
        L.refcpu_set_threads.argtypes = [ctypes.c_int]
        L.refcpu_set_direct.argtypes = [ctypes.c_int]
        _lib = L
    return _lib


def _check(status):
    if status != 0:
        raise OracleError(status, lib().refcpu_last_error().decode())


def _ptr(a):
    return a.ctypes.data_as(_f32p)


def set_threads(n: int):
    lib().refcpu_set_threads(n)


def threads() -> int:
    return lib().refcpu_threads()


def set_direct(direct: bool):
    lib().refcpu_set_direct(int(direct))


def f32_to_half(v: float) -> int:
    return lib().refcpu_f32_to_half(v)


def half_to_f32(h: int) -> float:
    return lib().refcpu_half_to_f32(h)


def parse_weights(data: bytes, magic: bytes):
    _check(lib().refcpu_parse_weights(data, len(data), magic))


def multiply(a, w, bias=None, *, kind="rows", shape=None, stride=None, size=1, step=1,
             reflect=False, offsets=(), rows=None, out=None, out_stride=None, act=0,
             accumulate=False, half=False):
    """gemm.rs multiply. `a` is float32 (rows x stride, or an image's pixels);
    `w` k x n. For kind "conv"/"phase", shape = (height, width, channels)."""
    a = np.ascontiguousarray(a, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    k, n = w.shape
    h = wd = ch = 0
    if kind == "rows":
        kcode, in_stride = 0, stride or k
        m = a.size // in_stride
    else:
        h, wd, ch = shape
        in_stride = stride or ch
        kcode = 1 if kind == "conv" else 2
        if kind == "conv":
            m = ((h - 1) // step + 1) * ((wd - 1) // step + 1)
        else:
            m = h * wd
    r0, r1 = rows if rows is not None else (0, m)
    out_stride = out_stride or n
    if out is None:
        out = np.zeros(((r1 - r0 - 1) * out_stride + n) if r1 > r0 else 0, np.float32)
    offs = (ctypes.c_size_t * 8)(*[v for o in offsets for v in o], *([0] * (8 - 2 * len(offsets))))
    b = np.ascontiguousarray(bias, np.float32) if bias is not None else None
    _check(lib().refcpu_multiply(
        kcode, _ptr(a), h, wd, ch, in_stride, size, step, int(reflect), offs, len(offsets),
        r0, r1, _ptr(w), k, n, _ptr(b) if b is not None else None, int(half), _ptr(out),
        out_stride, act, int(accumulate)))
    return out


def conv3(data, shape, w, bias, *, stride=None, reflect=False, half=False, out=None,
          out_stride=None, accumulate=False, double_first=False):
    h, wd, ch = shape
    data = np.ascontiguousarray(data, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    n = w.shape[1]
    out_stride = out_stride or n
    if out is None:
        out = np.zeros(h * wd * out_stride, np.float32)
    b = np.ascontiguousarray(bias, np.float32) if bias is not None else None
    _check(lib().refcpu_conv3(
        _ptr(data), h, wd, ch, stride or ch, int(reflect), _ptr(w), n,
        _ptr(b) if b is not None else None, int(half), _ptr(out), out_stride, int(accumulate),
        int(double_first)))
    return out


class RealEsrgan:
    """The reference's CPU Real-ESRGAN (Model::load_cpu) as restated."""

    SCALE = 4

    def __init__(self, path):
        self._h = ctypes.c_void_p()
        _check(lib().refcpu_realesrgan_load(os.fsencode(path), ctypes.byref(self._h)))

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.refcpu_realesrgan_free(self._h)
            self._h = None

    def run_float(self, image: np.ndarray) -> np.ndarray:
        image = np.ascontiguousarray(image, np.float32)
        h, w, _ = image.shape
        out = np.empty((h * 4, w * 4, 3), np.float32)
        _check(lib().refcpu_realesrgan_run_float(self._h, _ptr(image), w, h, _ptr(out)))
        return out

    def run_float_tiled(self, image: np.ndarray, tile: int, margin: int, progress=None):
        image = np.ascontiguousarray(image, np.float32)
        h, w, _ = image.shape
        out = np.empty((h * 4, w * 4, 3), np.float32)
        cb = PROGRESS(lambda f, _u: int(bool(progress(f)))) if progress else PROGRESS()
        _check(lib().refcpu_realesrgan_run_tiled(self._h, _ptr(image), w, h, tile, margin,
                                                 _ptr(out), cb, None))
        return out


class Scunet:
    """The reference's CPU SCUNet (Model::load_cpu) as restated."""

    def __init__(self, path):
        self._h = ctypes.c_void_p()
        _check(lib().refcpu_scunet_load(os.fsencode(path), ctypes.byref(self._h)))

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.refcpu_scunet_free(self._h)
            self._h = None

    def run_float(self, image: np.ndarray) -> np.ndarray:
        image = np.ascontiguousarray(image, np.float32)
        h, w, _ = image.shape
        out = np.empty((h, w, 3), np.float32)
        _check(lib().refcpu_scunet_run_float(self._h, _ptr(image), w, h, _ptr(out)))
        return out

    def run_float_tiled(self, image: np.ndarray, tile: int, margin: int, progress=None):
        image = np.ascontiguousarray(image, np.float32)
        h, w, _ = image.shape
        out = np.empty((h, w, 3), np.float32)
        cb = PROGRESS(lambda f, _u: int(bool(progress(f)))) if progress else PROGRESS()
        _check(lib().refcpu_scunet_run_tiled(self._h, _ptr(image), w, h, tile, margin, _ptr(out), cb, None))
        return out


class Lama:
    """The reference's CPU Big LaMa (Model::load_cpu) as restated."""

    MIN_SIDE = 9
    STEPS = 26

    def __init__(self, path):
        self._h = ctypes.c_void_p()
        _check(lib().refcpu_lama_load(os.fsencode(path), ctypes.byref(self._h)))

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.refcpu_lama_free(self._h)
            self._h = None

    def run_float(self, image: np.ndarray, mask: np.ndarray, progress=None) -> np.ndarray:
        """lib.rs:163-172: the prediction for every pixel (image h x w x 3,
        mask h x w, both in 0..=1)."""
        image = np.ascontiguousarray(image, np.float32)
        mask = np.ascontiguousarray(mask, np.float32)
        h, w, _ = image.shape
        if mask.shape != (h, w):
            raise ValueError("mask shape")
        out = np.empty((h, w, 3), np.float32)
        cb = PROGRESS(lambda f, _u: int(bool(progress(f)))) if progress else PROGRESS()
        _check(lib().refcpu_lama_run_float(self._h, _ptr(image), _ptr(mask), w, h, _ptr(out), cb, None))
        return out

    def run(self, rgb: np.ndarray, mask: np.ndarray) -> np.ndarray:
        """lib.rs:128-160: 8-bit image with the pixels where `mask` (u8) is
        non-zero filled from the prediction."""
        rgb = np.ascontiguousarray(rgb, np.uint8)
        mask = np.ascontiguousarray(mask, np.uint8)
        pred = self.run_float(rgb.astype(np.float32) / np.float32(255.0), (mask != 0).astype(np.float32))
        v = (np.clip(pred, np.float32(0.0), np.float32(1.0)) * np.float32(255.0)).astype(np.float64)
        fill = np.floor(v + 0.5).astype(np.uint8)  # f32::round: half away from zero
        out = rgb.copy()
        out[mask != 0] = fill[mask != 0]
        return out


class Birefnet:
    """The reference's CPU BiRefNet-lite (Model::load_cpu) as restated."""

    def __init__(self, path):
        self._h = ctypes.c_void_p()
        _check(lib().refcpu_birefnet_load(os.fsencode(path), ctypes.byref(self._h)))

    def __del__(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.refcpu_birefnet_free(self._h)
            self._h = None

    def run_normalized(self, image: np.ndarray) -> np.ndarray:
        """lib.rs:134-172: side x side logits of a normalised NHWC image."""
        image = np.ascontiguousarray(image, np.float32)
        side = image.shape[0]
        out = np.empty((side, side), np.float32)
        _check(lib().refcpu_birefnet_run_normalized(self._h, _ptr(image), side, _ptr(out)))
        return out

    def run(self, rgb: np.ndarray) -> np.ndarray:
        """lib.rs:116-133: logits of an 8-bit side x side image."""
        rgb = np.ascontiguousarray(rgb, np.uint8)
        side = rgb.shape[0]
        out = np.empty((side, side), np.float32)
        _check(lib().refcpu_birefnet_run(self._h, rgb.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), side,
                                         _ptr(out)))
        return out


def resize(src, dh, dw, out=None, add=False):
    """decoder.rs:443-521: aligned-corner bilinear resize of an h x w x c map."""
    src = np.ascontiguousarray(src, np.float32)
    sh, sw, c = src.shape
    dst = np.zeros((dh, dw, c), np.float32) if out is None else np.array(out, np.float32, copy=True, order="C")
    _check(lib().refcpu_resize(_ptr(src), sh, sw, c, _ptr(dst), dh, dw, int(add)))
    return dst


def rfft2(x, h, w, c):
    """fourier.rs forward: ortho rfft2 of an h x w x c map; h x (w/2+1) x 2c."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty((h, w // 2 + 1, 2 * c), np.float32)
    _check(lib().refcpu_rfft2(_ptr(x), h, w, c, _ptr(out)))
    return out


def irfft2_add(spec, h, w, c, out):
    """fourier.rs inverse: adds the ortho inverse of `spec` onto `out`."""
    spec = np.ascontiguousarray(spec, np.float32)
    out = np.array(out, np.float32, copy=True, order="C")
    _check(lib().refcpu_irfft2_add(_ptr(spec), h, w, c, _ptr(out)))
    return out


def attention(qkv, c, head, bias, tokens):
    qkv = np.ascontiguousarray(qkv, np.float32)
    bias = np.ascontiguousarray(bias, np.float32)
    out = np.zeros((tokens, c), np.float32)
    _check(lib().refcpu_attention(_ptr(qkv), c, head, _ptr(bias), tokens, _ptr(out)))
    return out


def layer_norm(x, gamma, beta):
    x = np.array(x, np.float32, copy=True, order="C")
    g = np.ascontiguousarray(gamma, np.float32)
    b = np.ascontiguousarray(beta, np.float32)
    _check(lib().refcpu_layer_norm(_ptr(x), x.shape[0], x.shape[1], _ptr(g), _ptr(b)))
    return x


def gelu(x):
    x = np.array(x, np.float32, copy=True)
    lib().refcpu_gelu(_ptr(x), x.size)
    return x


def sigmoid(x):
    x = np.array(x, np.float32, copy=True)
    lib().refcpu_sigmoid(_ptr(x), x.size)
    return x
