"""Algorithms on device fields: the flying-edges isosurface, its helpers, and
vertex normals of the surface.

Mirrors the names tack exports from ``tack.algorithms`` for this path
(packages/tack-core/src/tack/algorithms/__init__.py:29-76).
"""

from .compute_normals import compute_normals  # noqa: F401
from .flying_edges import (MCTables, UniformGrid, flying_edges,  # noqa: F401
                           flying_edges_multiblock)
from .marching_cubes import classify_cells, marching_cubes_soup  # noqa: F401
from .scan import exclusive_scan, inclusive_scan  # noqa: F401
