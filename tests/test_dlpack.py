"""DLPack exchange (chelis_b200/dlpack.py; the reference's
crates/chelis-python/src/dlpack.rs): struct layouts on CPU; zero-copy import
and export with torch, lifetimes and refusals on the GPU."""
import ctypes
import gc

import pytest

from chelis_b200 import dlpack as D
from chelis_b200 import lib as L


def test_dlpack_struct_layouts():
    # dlpack.h (v1.0) on LP64
    assert ctypes.sizeof(D.DLTensor) == 48
    assert D.DLTensor.ndim.offset == 16 and D.DLTensor.dtype.offset == 20
    assert D.DLTensor.shape.offset == 24 and D.DLTensor.byte_offset.offset == 40
    assert ctypes.sizeof(D.DLManagedTensor) == 64
    assert ctypes.sizeof(D.DLManagedTensorVersioned) == 80
    assert D.DLManagedTensorVersioned.dl_tensor.offset == 32


@pytest.mark.gpu
def test_import_export_round_trip_with_torch(cuda):
    import torch
    x = torch.randn(64, 48, device="cuda")
    t = D.DeviceTensor.from_dlpack(x)
    assert t.shape == (64, 48) and t.__dlpack_device__() == (D.KDL_CUDA, 0)
    assert t.view().data == x.data_ptr()
    y = torch.utils.dlpack.from_dlpack(t)
    assert y.data_ptr() == x.data_ptr() and torch.equal(y, x)
    # a strided producer keeps its strides through the round trip
    xt = x.t()
    tt = D.DeviceTensor.from_dlpack(xt)
    v = tt.view()
    assert (v.strides[0], v.strides[1]) == (1, 48)
    yt = torch.utils.dlpack.from_dlpack(tt)
    assert torch.equal(yt, xt)
    # the versioned protocol
    cap = t.__dlpack__(max_version=(1, 0))
    assert ctypes.pythonapi.PyCapsule_IsValid(ctypes.py_object(cap), b"dltensor_versioned")
    del cap
    # refusals (dlpack.rs:103-130)
    with pytest.raises(BufferError):
        t.__dlpack__(copy=True)
    with pytest.raises(BufferError):
        t.__dlpack__(dl_device=(D.KDL_CUDA, 7))
    del y, yt
    t.release()
    tt.release()


@pytest.mark.gpu
def test_library_output_exported_to_torch(cuda):
    """An owner the library allocated (a program output) is read by torch
    without a copy and stays alive until torch lets go of it."""
    import numpy as np
    import torch
    lib = L.load()
    a = torch.randn(32, 40, device="cuda", dtype=torch.float64)
    b = torch.randn(40, 24, device="cuda", dtype=torch.float64)
    ta, tb = D.DeviceTensor.from_dlpack(a), D.DeviceTensor.from_dlpack(b)
    ins = (ctypes.c_void_p * 2)(ta.owner, tb.owner)
    outs = (ctypes.c_void_p * 1)()
    L.call("chelis_matmul_device", ins, 2, outs, 1)
    out = D.DeviceTensor(outs[0])
    c = torch.utils.dlpack.from_dlpack(out)
    del out
    gc.collect()
    ref = a @ b
    assert float(((c - ref).abs() / (a.abs() @ b.abs())).max()) <= 1e-12
    assert np.isfinite(c.cpu().numpy()).all()


def test_capsule_lifetimes_on_the_host():
    """An unconsumed capsule releases its managed tensor when it dies; a
    consumed one (renamed "used_dltensor") leaves that to the consumer."""
    m = D.DLManagedTensor()
    addr = ctypes.addressof(m)
    D._exported[addr] = (m, None, None, None)
    cap = D._api.PyCapsule_New(addr, b"dltensor", ctypes.cast(D._DESTROY_LEGACY, ctypes.c_void_p))
    del cap
    gc.collect()
    assert addr not in D._exported
    m2 = D.DLManagedTensor()
    a2 = ctypes.addressof(m2)
    D._exported[a2] = (m2, None, None, None)
    cap = D._api.PyCapsule_New(a2, b"dltensor", ctypes.cast(D._DESTROY_LEGACY, ctypes.c_void_p))
    D._api.PyCapsule_SetName(cap, b"used_dltensor")
    del cap
    gc.collect()
    assert a2 in D._exported
    D._legacy_deleter(ctypes.pointer(m2))   # the consumer's deleter call
    assert a2 not in D._exported
