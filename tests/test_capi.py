"""The C ABI library on the CPU: it loads, exports every entry point the
header declares, and without a GPU refuses to load a model with IEC_ERR_GPU
(never a CPU fallback)."""

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "iec_cuda.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(iec_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_model_api():
    names = declared()
    for n in ["iec_realesrgan_load", "iec_realesrgan_free", "iec_realesrgan_device_name", "iec_realesrgan_run",
              "iec_realesrgan_run_float", "iec_realesrgan_run_float_tiled", "iec_realesrgan_run_batch",
              "iec_realesrgan_run_device", "iec_last_error"]:
        assert n in names


def test_library_exports_every_declared_symbol():
    import iec

    lib = iec.lib()
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing


def test_no_gpu_is_a_gpu_error(realesrgan_weights):
    import iec

    if iec.device_count() > 0:
        pytest.skip("a GPU is present")
    with pytest.raises(iec.IecError) as e:
        iec.RealEsrgan(realesrgan_weights)
    assert e.value.code == iec.ERR_GPU
    assert "no CUDA device" in str(e.value)


def test_null_arguments_are_input_errors():
    import iec

    L = iec.lib()
    out = ctypes.c_void_p()
    assert L.iec_realesrgan_load(None, None, ctypes.byref(out)) == iec.ERR_INPUT
    assert b"null" in L.iec_last_error()
    assert L.iec_realesrgan_run_float(None, None, 4, 4, None) == iec.ERR_INPUT


def test_seeded_weights_parse_in_the_oracle(realesrgan_weights):
    from oracle import refcpu

    with open(realesrgan_weights, "rb") as f:
        refcpu.parse_weights(f.read(), b"REALESRG")
