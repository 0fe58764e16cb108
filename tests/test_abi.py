"""The C-ABI library: it loads, exports every entry point include/voxtral_cuda.h
declares, and reports 'unavailable' cleanly where there is no GPU.  CPU only."""
import ctypes
import os
import subprocess

import pytest

import voxcuda as V


def test_library_exports_every_declared_symbol():
    assert os.path.exists(V.LIB_PATH), "libvoxtral_cuda.so not built"
    lib = ctypes.CDLL(V.LIB_PATH)
    declared = V.header_symbols()
    assert len(declared) >= 20
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing


def test_header_is_plain_c():
    # the boundary header compiles as C with no CUDA / C++ headers
    hdr = os.path.dirname(V.HEADER)
    src = '#include "voxtral_cuda.h"\nint main(void){return VOX_CUDA_OK;}\n'
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only", "-I", hdr, "-x", "c", "-"],
                       input=src, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def _gpu_present():
    return os.path.exists("/dev/nvidia0") and os.environ.get("CUDA_VISIBLE_DEVICES", "x") != ""


@pytest.mark.skipif(_gpu_present(), reason="needs a host without a GPU")
def test_init_reports_unavailable_without_gpu():
    lib = V.lib()
    assert lib.vox_cuda_init() == 0
    assert lib.vox_cuda_available() == 0
    assert V.last_error()
    # every entry point refuses cleanly instead of touching a device
    import numpy as np
    x = np.zeros((1, 8), np.float32)
    W = np.zeros((8, 8), np.uint16)
    y = np.zeros((1, 8), np.float32)
    rc = lib.vox_cuda_sgemm_bf16(1, 8, 8, V._f(x), V._u16(W), None, V._f(y))
    assert rc == V.ERR_UNAVAILABLE


def test_argument_errors_are_reported_before_device_use():
    import numpy as np
    lib = V.lib()
    x = np.zeros((1, 12), np.float32)
    W = np.zeros((8, 12), np.uint16)
    y = np.zeros((1, 8), np.float32)
    # bad shapes / NULL operands -> VOX_CUDA_ERR_ARG regardless of the device
    assert lib.vox_cuda_sgemm_bf16(1, 8, 12, None, V._u16(W), None, V._f(y)) == V.ERR_ARG
    assert lib.vox_cuda_sgemm_bf16(0, 8, 8, V._f(x), V._u16(W), None, V._f(y)) == V.ERR_ARG
    assert lib.vox_cuda_sgemm_bf16(1, 8, -8, V._f(x), V._u16(W), None, V._f(y)) == V.ERR_ARG
    assert lib.vox_cuda_decoder_step_batch(None, 9, None, None) == V.ERR_ARG
