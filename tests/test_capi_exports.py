"""CPU-side checks of the C-ABI library: it loads, exports every symbol that
include/tpt_cuda.h declares, and reports errors without a GPU."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if h.endswith(".h"):
            src = open(os.path.join(ROOT, "include", h)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(tpt_cuda_\w+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol():
    from tpt_infer_b200 import _capi

    declared = _declared_symbols()
    assert len(declared) > 30
    missing = [n for n in sorted(declared) if not hasattr(_capi.lib, n)]
    assert not missing, missing
    # and the Python binding covers every declared symbol
    assert declared <= set(_capi.SIGNATURES), sorted(declared - set(_capi.SIGNATURES))


def test_backend_name_and_status_strings():
    from tpt_infer_b200._capi import lib

    assert lib.tpt_cuda_backend_name() == b"cuda"
    assert lib.tpt_cuda_status_str(1) == b"size mismatch"
    assert lib.tpt_cuda_status_str(2) == b"shape mismatch"
    assert lib.tpt_cuda_status_str(3) == b"operation not supported by this backend"


def test_no_device_means_no_backend():
    # Like WebGpuBackend::new() -> Option (webgpu.rs:272): no sm_100 device, no backend.
    import torch

    from tpt_infer_b200 import CudaBackend

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert CudaBackend.new(0) is None


def test_null_context_is_invalid():
    from tpt_infer_b200._capi import lib

    assert lib.tpt_cuda_relu(None, None, 0, None, 0) == 4
