"""Device selection, streams and workspace caching.

Mirrors ``tack.init(tack.cuda)`` (packages/tack-core/src/tack/runtime/
dispatch.py:36-80): selecting the backend checks that a CUDA device and the
compiled library are present, and fails loudly otherwise.  Unlike the
reference's CUDA backend, which binds device 0 only
(runtime/cuda_backend.py:443), the device is LOCAL_RANK (one process per GPU)
or an explicit index.  Work is issued on PyTorch's current stream of that
device, so callers can order it with their own torch work.
"""

import os
import threading

import torch

from . import _lib

cuda = "cuda"  # the only architecture: tack_b200.init(tack_b200.cuda)

_state = {"device": None}
_tls = threading.local()


def init(arch=cuda, device=None):
    """Select the CUDA device and load libtackmc.so.

    device: index; defaults to $LOCAL_RANK or 0.  Raises RuntimeError when
    no CUDA device or no library is available (there is no CPU fallback).
    """
    if arch not in (cuda, "cuda", None):
        raise RuntimeError(f"tack_b200 runs on CUDA (sm_100a) only, not {arch!r}")
    if not torch.cuda.is_available():
        raise RuntimeError("tack_b200.init: no CUDA device is visible")
    _lib.load()
    if device is None:
        device = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(device)
    _state["device"] = torch.device("cuda", device)
    return _state["device"]


def current_device():
    if _state["device"] is None:
        init()
    return _state["device"]


def current_stream(device=None):
    """Raw cudaStream_t (as int) of torch's current stream on `device`."""
    return torch.cuda.current_stream(device or current_device()).cuda_stream


def workspace(tag, nbytes, device):
    """A cached device byte buffer of at least nbytes, per thread and device.

    Each thread gets its own buffers, so concurrent calls from different
    threads never share scratch memory.  The buffer is reused across calls
    on the same stream; PyTorch's caching allocator backs it.
    """
    cache = getattr(_tls, "ws", None)
    if cache is None:
        cache = _tls.ws = {}
    key = (tag, device.index if device.index is not None else torch.cuda.current_device())
    buf = cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        cache[key] = buf
    return buf


def release_workspaces():
    """Drop this thread's cached workspaces."""
    _tls.ws = {}
