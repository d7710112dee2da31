"""The C-ABI library builds, loads and exports every entry point declared in
include/vc_cuda.h; without a GPU it reports itself unavailable and every
compute entry point fails loudly (no CPU fallback). CPU only."""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import has_nvidia_device

pytestmark = pytest.mark.skipif(has_nvidia_device(), reason="checks the no-GPU behaviour")


def test_library_exports_every_header_symbol():
    from vectorcore_b200 import _abi

    declared = _abi.header_symbols()
    assert len(declared) >= 30
    missing = [s for s in declared if not hasattr(_abi.lib, s)]
    assert not missing, f"declared but not exported: {missing}"
    # every declared symbol has a ctypes signature in the binding
    unbound = [s for s in declared if s not in _abi._SIGS]
    assert not unbound, f"declared but not bound: {unbound}"


def test_no_gpu_means_unavailable_and_loud_failures():
    from vectorcore_b200 import _abi

    assert not _abi.available()
    assert "no CUDA device" in _abi.last_error() or "CUDA" in _abi.last_error()
    out = np.zeros(4, np.float32)
    st = _abi.lib.vc_cuda_unary(0, ctypes.c_void_p(out.ctypes.data), ctypes.c_void_p(out.ctypes.data),
                                ctypes.c_size_t(4))
    assert st == _abi.VC_ERR_RUNTIME
    with pytest.raises(RuntimeError):
        _abi.alloc(16)
    from vectorcore_b200.backend import CudaBackend

    assert CudaBackend.instance().available() is False


def test_missing_library_fails_import(tmp_path):
    # A product path with no CUDA library must not import (no CPU fallback).
    code = "import vectorcore_b200"
    env = dict(os.environ, PYTHONPATH=os.getcwd(), VECTORCORE_B200_LIB=str(tmp_path / "libvc_cuda.so"))
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env)
    assert res.returncode != 0
    assert "not built" in res.stderr
