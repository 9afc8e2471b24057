"""Concurrent calls from several host threads, as the reference allows
(test_concurrent_dispatch.py:115-175 calls kernels from many threads).

Each thread runs flying_edges on its own volume and isovalue, on its own
CUDA stream or on the default one; every result must equal the same call
made alone.  Workspaces are per thread, output buffers per call, and the
library keeps no mutable state between calls except per-device caches
filled under a lock.
"""

import threading

import numpy as np
import pytest
import torch

from tack_b200 import workloads

pytestmark = pytest.mark.gpu


def _cases(tack):
    out = []
    for i, (name, shape, iso) in enumerate([("blobs", (96, 80, 72), 0.5),
                                            ("gyroid", (64, 64, 64), 0.0),
                                            ("sines", (100, 64, 40), 0.25),
                                            ("noise", (64, 96, 48), 0.3),
                                            ("blobs", (128, 64, 64), 0.8),
                                            ("gyroid", (33, 47, 61), 0.1)]):
        v = workloads.generate(name, shape)
        g = tack.UniformGrid(shape[0] - 1, shape[1] - 1, shape[2] - 1, 0.5 * i, 0.0, -1.0,
                             1.0, 0.5, 0.25)
        out.append((tack.from_torch(v), g, iso))
    return out


@pytest.mark.parametrize("own_streams", [True, False])
def test_threads_match_sequential(tack, own_streams):
    cases = _cases(tack)
    ref = [tack.flying_edges(f, g, iso) for f, g, iso in cases]
    torch.cuda.synchronize()
    results = [None] * (2 * len(cases))
    errors = []
    start = threading.Barrier(len(results))

    def work(i):
        try:
            f, g, iso = cases[i % len(cases)]
            start.wait()
            if own_streams:
                s = torch.cuda.Stream()
                with torch.cuda.stream(s):
                    results[i] = tack.flying_edges(f, g, iso)
            else:
                results[i] = tack.flying_edges(f, g, iso)
        except Exception as e:  # reported below
            errors.append(e)

    threads = [threading.Thread(target=work, args=(i,)) for i in range(len(results))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not errors, errors
    for i, r in enumerate(results):
        want = ref[i % len(cases)]
        assert r is not None and want is not None
        assert (r["total_points"], r["total_tris"]) == (want["total_points"], want["total_tris"])
        np.testing.assert_array_equal(r["conn"], want["conn"])
        np.testing.assert_array_equal(r["points"].view(np.uint32), want["points"].view(np.uint32))
