"""The C-ABI library without a GPU: it loads, exports every symbol the header
declares, and rejects bad arguments with the documented status codes before
touching a device."""
import ctypes
import os
import re

import pytest

from chelis_b200 import lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    inc = os.path.join(ROOT, "include")
    for h in sorted(os.listdir(inc)):
        if not h.endswith(".h"):
            continue
        text = open(os.path.join(inc, h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(chelis_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_loads_and_exports_every_declared_symbol():
    lib = L.load()
    names = declared_functions()
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # every declared entry point has a ctypes signature in the binding
    assert set(names) <= set(L.SIGNATURES), set(names) - set(L.SIGNATURES)


def test_descriptor_layout_matches_reference():
    # chelis_device_descriptor.h:8-18 on LP64
    assert ctypes.sizeof(L.GpuTensor) == 48
    assert L.GpuTensor.count.offset == 24
    assert L.GpuTensor.rank.offset == 40
    assert L.GpuTensor.dtype.offset == 44
    assert L.GpuTensor.ownership.offset == 45


def test_status_codes_without_device():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    lib = L.load()
    assert lib.chelis_cuda_init(0) == 6  # NO_DEVICE
    assert "no CUDA device" in L.last_error()
    # argument validation happens before any device work
    assert lib.chelis_cuda_sgemm(0, 0, -1, 4, 4, None, 4, 0, None, 4, 0, None, 4, 0, 1) == 1
    assert lib.chelis_cuda_dgemm(0, 0, 4, 4, 4, None, 2, 0, None, 4, 0, None, 4, 0, 1) == 1
    assert lib.chelis_cuda_dropout_f32(None, None, 10, 42, 1.5, 0) == 1
    assert "dropout" in L.last_error()
    assert lib.chelis_cuda_portfolio_f64(None, None, 1, 252, 63, None, None, None) == 4
    assert lib.chelis_cuda_chain_fwd(None, None, None, 1e-5, 42, 0.1, 4, 1 << 20, 0, None, None) == 4
    assert lib.chelis_cuda_set_gemm_mode(7) == 1
    assert lib.chelis_cuda_set_rows_mode(7) == 1
    # empty work is a successful no-op (emit.rs:4806 count == 0 skip)
    assert lib.chelis_cuda_sgemm(0, 0, 0, 4, 4, None, 4, 0, None, 4, 0, None, 4, 0, 1) == 0
    assert lib.chelis_device_tensor_alloc_shape(0, 1, (ctypes.c_int64 * 1)(4)) is None


def test_error_raises_with_message():
    with pytest.raises(L.ChelisCudaError, match="DOMAIN"):
        L.call("chelis_cuda_set_gemm_mode", 99)
