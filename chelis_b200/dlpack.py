"""DLPack exchange of device tensors: zero-copy interop with torch, CuPy, JAX
and any other DLPack producer or consumer.

The reference's Python bindings export Chelis tensors through DLPack
(crates/chelis-python/src/dlpack.rs: `__dlpack__(stream, max_version,
dl_device, copy)`, `__dlpack_device__()`, legacy "dltensor" and versioned
"dltensor_versioned" capsules, cross-device export and copy requests
refused with BufferError).  Here the tensor is a device owner of the
library (chelis_device_tensor_owner, include/chelis_cuda.h) on a CUDA
device (kDLCUDA = 2):

    t = DeviceTensor.from_dlpack(torch_tensor)     # borrows torch's memory
    out = torch.utils.dlpack.from_dlpack(t)         # borrows t's memory

A borrowed tensor keeps its producer alive (the producer's deleter runs when
the DeviceTensor is released); an exported capsule keeps the DeviceTensor
alive until the consumer calls the capsule's deleter.  Export synchronises
the library's stream of this thread unless the consumer passes stream=-1.
"""
from __future__ import annotations

import ctypes

from . import lib as L

KDL_CUDA = 2
_CODE_INT, _CODE_UINT, _CODE_FLOAT, _CODE_BFLOAT, _CODE_BOOL = 0, 1, 2, 4, 6
# chelis dtype id -> DLPack (code, bits)
_TO_DL = {L.DTYPE_F32: (_CODE_FLOAT, 32), L.DTYPE_F64: (_CODE_FLOAT, 64), L.DTYPE_I32: (_CODE_INT, 32),
          L.DTYPE_BOOL: (_CODE_BOOL, 8), L.DTYPE_I64: (_CODE_INT, 64), L.DTYPE_BF16: (_CODE_BFLOAT, 16),
          L.DTYPE_F16: (_CODE_FLOAT, 16), 7: (_CODE_INT, 8), 8: (_CODE_INT, 16)}
_FROM_DL = {v: k for k, v in _TO_DL.items()}
_FROM_DL[(_CODE_UINT, 8)] = L.DTYPE_BOOL  # a uint8 mask imports as bool storage


class DLDevice(ctypes.Structure):
    _fields_ = [("device_type", ctypes.c_int32), ("device_id", ctypes.c_int32)]


class DLDataType(ctypes.Structure):
    _fields_ = [("code", ctypes.c_uint8), ("bits", ctypes.c_uint8), ("lanes", ctypes.c_uint16)]


class DLTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("device", DLDevice), ("ndim", ctypes.c_int32),
                ("dtype", DLDataType), ("shape", ctypes.POINTER(ctypes.c_int64)),
                ("strides", ctypes.POINTER(ctypes.c_int64)), ("byte_offset", ctypes.c_uint64)]


class DLManagedTensor(ctypes.Structure):
    pass


_LEGACY_DELETER = ctypes.CFUNCTYPE(None, ctypes.POINTER(DLManagedTensor))
DLManagedTensor._fields_ = [("dl_tensor", DLTensor), ("manager_ctx", ctypes.c_void_p),
                            ("deleter", _LEGACY_DELETER)]


class DLPackVersion(ctypes.Structure):
    _fields_ = [("major", ctypes.c_uint32), ("minor", ctypes.c_uint32)]


class DLManagedTensorVersioned(ctypes.Structure):
    pass


_VERSIONED_DELETER = ctypes.CFUNCTYPE(None, ctypes.POINTER(DLManagedTensorVersioned))
DLManagedTensorVersioned._fields_ = [("version", DLPackVersion), ("manager_ctx", ctypes.c_void_p),
                                     ("deleter", _VERSIONED_DELETER), ("flags", ctypes.c_uint64),
                                     ("dl_tensor", DLTensor)]

_api = ctypes.pythonapi
_api.PyCapsule_New.restype = ctypes.py_object
_api.PyCapsule_New.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p]
_api.PyCapsule_GetPointer.restype = ctypes.c_void_p
_api.PyCapsule_GetPointer.argtypes = [ctypes.py_object, ctypes.c_char_p]
_api.PyCapsule_IsValid.restype = ctypes.c_int
_api.PyCapsule_IsValid.argtypes = [ctypes.py_object, ctypes.c_char_p]
_api.PyCapsule_SetName.restype = ctypes.c_int
_api.PyCapsule_SetName.argtypes = [ctypes.py_object, ctypes.c_char_p]
# The destructor runs while the capsule is being deallocated: it takes the raw
# object pointer (a py_object argument would take a new reference to an object
# whose count already reached zero) and queries it through raw-pointer calls.
_CAPSULE_DESTRUCTOR = ctypes.CFUNCTYPE(None, ctypes.c_void_p)
_raw = ctypes.PyDLL(None)
_raw_is_valid = _raw.PyCapsule_IsValid
_raw_is_valid.restype = ctypes.c_int
_raw_is_valid.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
_raw_get_pointer = _raw.PyCapsule_GetPointer
_raw_get_pointer.restype = ctypes.c_void_p
_raw_get_pointer.argtypes = [ctypes.c_void_p, ctypes.c_char_p]

# exported managed tensors still owned by a capsule or a consumer:
# address -> (struct, shape array, strides array, the DeviceTensor)
_exported: dict[int, tuple] = {}


def _release_export(address: int) -> None:
    _exported.pop(address, None)


@_LEGACY_DELETER
def _legacy_deleter(managed):
    _release_export(ctypes.cast(managed, ctypes.c_void_p).value)


@_VERSIONED_DELETER
def _versioned_deleter(managed):
    _release_export(ctypes.cast(managed, ctypes.c_void_p).value)


def _capsule_destructor_for(name: bytes):
    # an unconsumed capsule (name unchanged) still owns its managed tensor
    @_CAPSULE_DESTRUCTOR
    def destroy(capsule):
        if _raw_is_valid(capsule, name):
            _release_export(_raw_get_pointer(capsule, name))
    return destroy


_DESTROY_LEGACY = _capsule_destructor_for(b"dltensor")
_DESTROY_VERSIONED = _capsule_destructor_for(b"dltensor_versioned")


class DeviceTensor:
    """A device owner of the library, exchangeable through DLPack."""

    def __init__(self, owner: int, keep=None, on_release=None):
        self._owner = owner
        self._keep = keep              # the producer object a borrowed tensor reads
        self._on_release = on_release  # the producer's deleter (imported tensors)

    # ---- construction
    @classmethod
    def from_dlpack(cls, obj) -> "DeviceTensor":
        """Borrow the memory of any DLPack producer on the current CUDA device
        (zero-copy).  The producer stays alive as long as this tensor."""
        lib = L.load()
        if hasattr(obj, "__dlpack__"):
            try:
                capsule = obj.__dlpack__(stream=None, max_version=(1, 0))
            except TypeError:
                capsule = obj.__dlpack__(stream=None)
        else:
            capsule = obj
        if _api.PyCapsule_IsValid(capsule, b"dltensor_versioned"):
            ptr = _api.PyCapsule_GetPointer(capsule, b"dltensor_versioned")
            managed = ctypes.cast(ptr, ctypes.POINTER(DLManagedTensorVersioned)).contents
            _api.PyCapsule_SetName(capsule, b"used_dltensor_versioned")
            dl = managed.dl_tensor
            release = (lambda m=managed, p=ptr: m.deleter(ctypes.cast(p, ctypes.POINTER(DLManagedTensorVersioned)))
                       if m.deleter else None)
        elif _api.PyCapsule_IsValid(capsule, b"dltensor"):
            ptr = _api.PyCapsule_GetPointer(capsule, b"dltensor")
            managed = ctypes.cast(ptr, ctypes.POINTER(DLManagedTensor)).contents
            _api.PyCapsule_SetName(capsule, b"used_dltensor")
            dl = managed.dl_tensor
            release = (lambda m=managed, p=ptr: m.deleter(ctypes.cast(p, ctypes.POINTER(DLManagedTensor)))
                       if m.deleter else None)
        else:
            raise TypeError("not a DLPack capsule or producer")
        try:
            if dl.device.device_type != KDL_CUDA:
                raise BufferError("DLPack import takes CUDA device memory (kDLCUDA)")
            key = (dl.dtype.code, dl.dtype.bits)
            if dl.dtype.lanes != 1 or key not in _FROM_DL:
                raise BufferError(f"unsupported DLPack dtype {key}")
            dt = _FROM_DL[key]
            rank = dl.ndim
            shape = [dl.shape[i] for i in range(rank)]
            if dl.strides:
                strides = [dl.strides[i] for i in range(rank)]
            else:  # compact row-major
                strides, run = [0] * rank, 1
                for d in range(rank - 1, -1, -1):
                    strides[d], run = run, run * shape[d]
            width = dl.dtype.bits // 8
            count = 1
            for e in shape:
                count *= e
            reach = 1 + sum((e - 1) * s for e, s in zip(shape, strides)) if count else 0
            sh = (ctypes.c_int64 * max(rank, 1))(*shape)
            st = (ctypes.c_int64 * max(rank, 1))(*strides)
            packet = L.GpuTensor()
            packet.data = (dl.data or 0) + dl.byte_offset
            packet.shape, packet.strides = sh, st
            packet.count, packet.byte_capacity = count, reach * width
            packet.rank, packet.dtype, packet.ownership = rank, dt, 0
            owner = lib.chelis_device_tensor_import(ctypes.byref(packet))
            if not owner:
                raise BufferError(f"DLPack import refused: {L.last_error()}")
        except BaseException:
            release()
            raise
        return cls(owner, keep=(capsule, obj), on_release=release)

    # ---- metadata
    def view(self) -> L.GpuTensor:
        return L.load().chelis_device_tensor_view(self._owner).contents

    @property
    def owner(self) -> int:
        return self._owner

    @property
    def shape(self) -> tuple:
        v = self.view()
        return tuple(v.shape[i] for i in range(v.rank))

    @property
    def device(self) -> int:
        return L.load().chelis_device_tensor_device(self._owner)

    # ---- DLPack export (dlpack.rs:95-170 request rules)
    def __dlpack_device__(self):
        return (KDL_CUDA, self.device)

    def __dlpack__(self, stream=None, max_version=None, dl_device=None, copy=None):
        if dl_device is not None and tuple(dl_device) != self.__dlpack_device__():
            raise BufferError("cross-device DLPack export is unsupported")
        if copy is True:
            raise BufferError("DLPack copying is unsupported; no copy was made")
        if stream is not None and stream != -1:
            if stream in (0,):
                raise ValueError("CUDA DLPack stream 0 is disallowed")
        if stream != -1:
            L.call("chelis_cuda_synchronize")  # the data is ready for any consumer stream
        v = self.view()
        if v.dtype not in _TO_DL:
            raise BufferError(f"dtype {v.dtype} has no DLPack form")
        code, bits = _TO_DL[v.dtype]
        shape = (ctypes.c_int64 * max(v.rank, 1))(*[v.shape[i] for i in range(v.rank)])
        strides = (ctypes.c_int64 * max(v.rank, 1))(*[v.strides[i] for i in range(v.rank)])
        dl = DLTensor(v.data, DLDevice(KDL_CUDA, self.device), v.rank, DLDataType(code, bits, 1),
                      shape, strides, 0)
        versioned = max_version is not None and tuple(max_version) >= (1, 0)
        if versioned:
            managed = DLManagedTensorVersioned(DLPackVersion(1, 0), None, _versioned_deleter, 0, dl)
            name, destroy = b"dltensor_versioned", _DESTROY_VERSIONED
        else:
            managed = DLManagedTensor(dl, None, _legacy_deleter)
            name, destroy = b"dltensor", _DESTROY_LEGACY
        address = ctypes.addressof(managed)
        _exported[address] = (managed, shape, strides, self)
        return _api.PyCapsule_New(address, name, ctypes.cast(destroy, ctypes.c_void_p))

    # ---- lifetime
    def release(self) -> None:
        if self._owner:
            L.load().chelis_device_tensor_release(self._owner)
            self._owner = 0
            if self._on_release is not None:
                self._on_release()
                self._on_release = None
            self._keep = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass
