"""Device fields: the tack ``Field`` interface over CUDA device memory.

Mirrors packages/tack-core/src/tack/lang/field.py (``tack.field``,
``Field.from_numpy/to_numpy/fill/sum/min/max/mean``, ``field_from_ptr``) and
the ``_buffer.device_ptr`` attribute of its CUDA buffer
(packages/tack-core/src/tack/runtime/cuda_backend.py:121-171), so code written
against tack's CUDA backend finds the same surface.  Storage is a PyTorch
CUDA tensor: PyTorch provides allocation, streams and host copies; all
compute goes through libtackmc.so.
"""

import ctypes

import numpy as np
import torch

from . import _lib
from .runtime import current_device, current_stream, workspace


class ScalarType:
    """A field element type (tack.f32, tack.i32, ...)."""

    def __init__(self, name, numpy_dtype, torch_dtype):
        self.name = name
        self.numpy_dtype = np.dtype(numpy_dtype)
        self.torch_dtype = torch_dtype

    @property
    def size(self):
        return self.numpy_dtype.itemsize

    def __repr__(self):
        return f"tack_b200.{self.name}"


f32 = ScalarType("f32", np.float32, torch.float32)
f64 = ScalarType("f64", np.float64, torch.float64)
i32 = ScalarType("i32", np.int32, torch.int32)
i64 = ScalarType("i64", np.int64, torch.int64)
u8 = ScalarType("u8", np.uint8, torch.uint8)
_BY_NUMPY = {t.numpy_dtype: t for t in (f32, f64, i32, i64, u8)}
_BY_TORCH = {t.torch_dtype: t for t in (f32, f64, i32, i64, u8)}


def from_numpy_dtype(dt):
    return _BY_NUMPY[np.dtype(dt)]


class CUDABuffer:
    """Field storage; ``device_ptr`` is the raw CUDA device address."""

    def __init__(self, tensor, owner=None):
        self.tensor = tensor
        self._owner = owner  # keeps an external allocation alive, if any

    @property
    def device_ptr(self):
        return self.tensor.data_ptr()

    @property
    def nbytes(self):
        return self.tensor.numel() * self.tensor.element_size()


class Field:
    """An n-dimensional array in CUDA device memory."""

    def __init__(self, dtype, shape, buffer, writable=True):
        self.dtype = dtype
        self.shape = tuple(shape)
        self._buffer = buffer
        self._writable = writable

    # -- plumbing ------------------------------------------------------
    @property
    def tensor(self):
        """The storage as a flat torch tensor (zero-copy)."""
        return self._buffer.tensor

    @property
    def size(self):
        return int(np.prod(self.shape, dtype=np.int64)) if self.shape else 1

    def _check_writable(self):
        if not self._writable:
            raise RuntimeError(
                "Field is read-only (created from an external pointer). "
                "Use writable=True in field_from_ptr() to enable writes.")

    # -- tack Field API ----------------------------------------------------
    def from_numpy(self, arr):
        """Copy a numpy array into the field (host -> device)."""
        self._check_writable()
        arr = np.asarray(arr)
        if arr.dtype != self.dtype.numpy_dtype:
            arr = arr.astype(self.dtype.numpy_dtype)
        if arr.shape != self.shape:
            raise ValueError(f"Shape mismatch: field is {self.shape}, got {arr.shape}")
        src = torch.from_numpy(np.ascontiguousarray(arr).reshape(-1))
        self.tensor.copy_(src, non_blocking=False)

    def to_numpy(self):
        """Copy the field into a new numpy array (device -> host)."""
        return self.tensor.detach().cpu().numpy().reshape(self.shape)

    def fill(self, value):
        self._check_writable()
        self.tensor.fill_(value)

    def sum(self):
        return reduce_field(self, "sum")

    def min(self):
        return reduce_field(self, "min")

    def max(self):
        return reduce_field(self, "max")

    def mean(self):
        return self.sum() / self.size

    def __repr__(self):
        return f"Field({self.dtype!r}, shape={self.shape}, device_ptr=0x{self._buffer.device_ptr:x})"


def field(dtype, shape):
    """Allocate a zero-filled field on the current CUDA device."""
    if isinstance(shape, int):
        shape = (shape,)
    n = int(np.prod(shape, dtype=np.int64)) if len(shape) else 1
    t = torch.zeros(n, dtype=dtype.torch_dtype, device=current_device())
    return Field(dtype, shape, CUDABuffer(t))


def from_torch(tensor, shape=None, writable=True):
    """Wrap a contiguous CUDA tensor as a field without copying."""
    if not tensor.is_cuda:
        raise ValueError("from_torch() needs a CUDA tensor")
    if not tensor.is_contiguous():
        raise ValueError("from_torch() needs a contiguous tensor")
    dt = _BY_TORCH[tensor.dtype]
    shape = tuple(tensor.shape) if shape is None else tuple(shape)
    return Field(dt, shape, CUDABuffer(tensor.reshape(-1)), writable=writable)


class _CudaArray:
    """__cuda_array_interface__ view of external device memory.

    Always exported as writable (PyTorch rejects read-only interfaces);
    read-only fields are enforced by Field._check_writable instead.
    """

    def __init__(self, ptr, n, dtype):
        self.__cuda_array_interface__ = {
            "shape": (n,), "typestr": dtype.numpy_dtype.str, "data": (int(ptr), False),
            "version": 3, "strides": None,
        }


def field_from_ptr(ptr, dtype, shape, writable=False):
    """Wrap an existing device pointer as a field without copying.

    The field does not own the memory.  Read-only unless writable=True
    (field.py:379-424 of the reference).
    """
    if isinstance(shape, int):
        shape = (shape,)
    n = int(np.prod(shape, dtype=np.int64)) if len(shape) else 1
    t = torch.as_tensor(_CudaArray(ptr, n, dtype), device=current_device())
    return Field(dtype, shape, CUDABuffer(t), writable=writable)


def device_tensor(obj, dtype=f32):
    """Resolve a field-like object to a flat contiguous CUDA tensor.

    Accepts a tack_b200 Field, a torch CUDA tensor, a reference tack field on
    its CUDA backend (anything with ``_buffer.device_ptr`` and ``shape``), a
    CPU tensor (copied on the current stream; without a host wait when it is
    pinned) or a numpy array (copied to the device).
    """
    if isinstance(obj, Field):
        t = obj.tensor
    elif isinstance(obj, torch.Tensor):
        t = obj if obj.is_cuda else obj.to(current_device(), non_blocking=obj.is_pinned())
        t = t.reshape(-1)
        if not t.is_contiguous():
            t = t.contiguous()
    elif isinstance(obj, np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(obj, dtype.numpy_dtype).reshape(-1)).to(
            current_device())
    elif hasattr(obj, "_buffer") and hasattr(obj._buffer, "device_ptr"):
        n = int(np.prod(obj.shape, dtype=np.int64))
        t = field_from_ptr(int(obj._buffer.device_ptr), dtype, (n,)).tensor
    else:
        raise TypeError(f"cannot use {type(obj).__name__} as a device field")
    if t.dtype != dtype.torch_dtype:
        raise TypeError(f"expected a {dtype.name} field, got {t.dtype}")
    return t


def reduce_field(fld, op):
    """sum / min / max of a field on the device (tkmc_reduce_f32 for f32).

    Replaces CUDABackend.reduce_field (cuda_backend.py:576-615); like it,
    non-f32 fields are reduced on the host.
    """
    if op not in ("sum", "min", "max"):
        raise ValueError(f"unknown reduction {op!r}")
    if fld.dtype is not f32:
        return float(getattr(fld.to_numpy(), op)())
    out = reduce_f32(fld.tensor)
    return {"min": out[0], "max": out[1], "sum": out[2]}[op]


def reduce_f32(t):
    """(min, max, sum, nan_count) of a flat f32 CUDA tensor in one read."""
    lib = _lib.load()
    n = t.numel()
    ws = workspace("reduce", lib.tkmc_reduce_workspace_bytes(n), t.device)
    out = (ctypes.c_double * 4)()
    _lib.check(lib.tkmc_reduce_f32(t.data_ptr(), n, ws.data_ptr(), ws.numel(), out,
                                   current_stream(t.device)), "tkmc_reduce_f32")
    return float(out[0]), float(out[1]), float(out[2]), int(out[3])
