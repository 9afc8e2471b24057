"""Shared pytest configuration.

Markers:
  gpu  -- needs a CUDA device (a B200); runs the libtackmc.so kernels.
Tests without the marker run on CPU only (oracle pins, host logic, ABI
symbol checks, gloo multi-process tests).
"""

import glob
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


def golden_fe_cases():
    """Names of the single-block fe fixtures made by tests/golden/make_golden.py."""
    out = []
    for p in sorted(glob.glob(os.path.join(GOLDEN, "fe_*.npz"))):
        name = os.path.basename(p)[3:-4]
        if name.startswith("multiblock"):
            continue
        out.append(name)
    return out


def load_fe_case(name):
    z = np.load(os.path.join(GOLDEN, f"fe_{name}.npz"))
    d = {k: z[k] for k in z.files}
    g = d["grid"]
    d["grid_tuple"] = (int(g[0]), int(g[1]), int(g[2]), float(g[3]), float(g[4]),
                       float(g[5]), float(g[6]), float(g[7]), float(g[8]))
    d["mask"] = d["mask"] if int(d["has_mask"]) else None
    d["isovalue"] = float(d["isovalue"])
    return d


@pytest.fixture(scope="session")
def tack():
    """The product package, initialised on cuda:0 (GPU tests only)."""
    import tack_b200
    tack_b200.init(tack_b200.cuda)
    return tack_b200


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O
