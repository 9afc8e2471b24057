"""Host-side helpers of bench.py: the CPU sample and the reference copy.

Both CPU legs (the reference arm and the GPU arm's cpu_baseline) time the
same sample, so its bounds must be deterministic and stay inside the
volume; the reference copy must take exactly the two source trees.
"""

import os

import pytest

import bench


@pytest.mark.parametrize("shape,niso", [((64, 64, 64), 1), ((256, 256, 256), 1),
                                        ((1024, 1024, 1024), 1), ((2048, 2048, 1024), 4),
                                        ((100, 90, 12), 2)])
def test_cpu_sample_bounds_inside_volume_and_sized(shape, niso):
    nx, ny, nz = shape
    b = bench.cpu_sample_bounds(shape, niso)
    assert b == bench.cpu_sample_bounds(shape, niso)  # deterministic
    for k0, k1 in b:
        assert 0 <= k0 < k1 <= nz and k1 - k0 >= 2
    cells = sum((nx - 1) * (ny - 1) * (k1 - k0 - 1) for k0, k1 in b) * niso
    if b == [(0, nz)]:
        assert (nx - 1) * (ny - 1) * (nz - 1) * niso <= bench.CPU_SAMPLE_CELLS
    else:
        assert len(b) == bench.CPU_SAMPLE_SLABS
        # spread over the depth: increasing, non-overlapping, first in the
        # first eighth and last in the last eighth
        assert all(b[i][1] <= b[i + 1][0] for i in range(len(b) - 1))
        assert b[0][0] < nz // 8 and b[-1][1] > nz - nz // 8
        assert cells <= 3 * bench.CPU_SAMPLE_CELLS


def test_install_reference_copies_the_two_source_trees(tmp_path, monkeypatch):
    checkout = tmp_path / "checkout"
    for pkg, mod in (("tack-core", "core.py"), ("tack-vis", "vis.py")):
        d = checkout / "packages" / pkg / "src" / "tack"
        d.mkdir(parents=True)
        (d / mod).write_text("x = 1\n")
        (d / "__pycache__").mkdir()
        (d / "__pycache__" / "junk.pyc").write_bytes(b"\0")
    dest = tmp_path / "ref"
    monkeypatch.setattr(bench, "REF_DIR", str(dest))
    assert bench.install_reference(str(checkout)) == str(dest)
    assert (dest / "tack-core" / "src" / "tack" / "core.py").read_text() == "x = 1\n"
    assert (dest / "tack-vis" / "src" / "tack" / "vis.py").exists()
    assert not os.path.exists(dest / "tack-core" / "src" / "tack" / "__pycache__")
    with pytest.raises(FileNotFoundError):
        bench.install_reference(str(tmp_path / "missing"))


def test_slab_split_arguments(monkeypatch):
    """N>1 slabs default to measured balancing; --balance-slabs means the
    surface split; the JSON wording names the split that ran."""
    monkeypatch.setattr("sys.argv", ["bench.py"])
    assert bench.parse_args().slabs == "measured"
    monkeypatch.setattr("sys.argv", ["bench.py", "--balance-slabs"])
    assert bench.parse_args().slabs == "surface"
    monkeypatch.setattr("sys.argv", ["bench.py", "--slabs", "equal"])
    assert bench.parse_args().slabs == "equal"
    assert bench.slab_words("measured", None) == "equal plane runs"
    assert "surface" in bench.slab_words("surface", [0, 3, 8])
    assert "measured" in bench.slab_words("measured", [0, 3, 8])
