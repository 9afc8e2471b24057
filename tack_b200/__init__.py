"""tack_b200 -- B200-native (sm_100a) isosurface extraction with tack's API.

A drop-in for tack-vis's flying-edges isosurface filter
(``tack.algorithms.flying_edges``) and the tack-core pieces it is used with
(fields, scan, field reductions).  Hand-written CUDA kernels in
libtackmc.so do all compute; PyTorch provides device memory, streams and
``torch.distributed``.

    import tack_b200 as tack
    tack.init(tack.cuda)
    f = tack.field(dtype=tack.f32, shape=(n,)); f.from_numpy(values)
    result = tack.algorithms.flying_edges(f, grid, isovalue)
"""

from . import algorithms  # noqa: F401
from .algorithms import (UniformGrid, compute_normals, flying_edges,  # noqa: F401
                         flying_edges_multiblock)
from .field import (Field, ScalarType, f32, f64, field, field_from_ptr,  # noqa: F401
                    from_torch, i32, i64, reduce_f32, u8)
from .runtime import cuda, current_device, init  # noqa: F401

__version__ = "0.1.0"
