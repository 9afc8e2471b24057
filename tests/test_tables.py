"""Marching-cubes tables: the library's tables equal the reference's.

Invariants follow packages/tack-vis/tests/test_flying_edges.py:48-89; the
equality check is against the reference's own tables dumped into
tests/golden/mc_tables.npz.
"""

import numpy as np

from conftest import GOLDEN


def _lib_tables():
    from tack_b200.algorithms.flying_edges import _EDGE_CORNERS, _NUM_TRIS, _TRI_TABLE
    return _TRI_TABLE, _NUM_TRIS, _EDGE_CORNERS


def test_tables_equal_reference():
    z = np.load(f"{GOLDEN}/mc_tables.npz")
    tri, num, edges = _lib_tables()
    np.testing.assert_array_equal(tri, z["tri_table"])
    np.testing.assert_array_equal(num, z["num_tris"])
    np.testing.assert_array_equal(edges, z["edge_corners"])


def test_num_tris_matches_tri_table():
    tri, num, _ = _lib_tables()
    for case in range(256):
        row = tri[case * 16:(case + 1) * 16]
        assert num[case] == sum(1 for t in range(0, 16, 3) if row[t] >= 0)


def test_tri_table_triples_are_complete():
    tri, _, _ = _lib_tables()
    for case in range(256):
        row = tri[case * 16:(case + 1) * 16]
        for t in range(0, 15, 3):
            triple = row[t:t + 3]
            assert (triple >= 0).all() or (triple < 0).all()
        assert row[15] == -1


def test_tri_table_edges_in_range():
    tri, _, _ = _lib_tables()
    valid = tri[tri >= 0]
    assert valid.min() >= 0 and valid.max() <= 11


def test_only_uniform_cases_are_empty():
    _, num, _ = _lib_tables()
    assert num[0] == 0 and num[255] == 0
    assert (num == 0).sum() == 2
    assert num.max() == 5


def test_edges_join_adjacent_corners():
    """Each edge joins two corners that differ in exactly one coordinate."""
    _, _, edges = _lib_tables()
    corner = [(0, 0, 0), (1, 0, 0), (1, 1, 0), (0, 1, 0), (0, 0, 1), (1, 0, 1), (1, 1, 1), (0, 1, 1)]
    for e in range(12):
        a, b = corner[edges[2 * e]], corner[edges[2 * e + 1]]
        assert sum(x != y for x, y in zip(a, b)) == 1


def test_closed_form_triangle_count():
    """The count pass computes a cell's triangle count without the table:
    ntri = V - 2F - 4*belt + 4*full, V = corners above, F = faces whose four
    corners are above, belt = exactly two antipodal corners below, full = all
    eight above.  It must equal the table's count for every case."""
    _, num, _ = _lib_tables()
    corner = [(0, 0, 0), (1, 0, 0), (1, 1, 0), (0, 1, 0), (0, 0, 1), (1, 0, 1), (1, 1, 1), (0, 1, 1)]
    faces = [[c for c in range(8) if corner[c][ax] == side] for ax in range(3) for side in (0, 1)]
    antipodal = [(a, b) for a in range(8) for b in range(a + 1, 8)
                 if all(corner[a][d] != corner[b][d] for d in range(3))]
    assert len(antipodal) == 4
    for case in range(256):
        above = [(case >> c) & 1 for c in range(8)]
        v = sum(above)
        f = sum(all(above[c] for c in face) for face in faces)
        below = {c for c in range(8) if not above[c]}
        belt = int(len(below) == 2 and tuple(sorted(below)) in antipodal)
        full = int(v == 8)
        assert v - 2 * f - 4 * belt + 4 * full == num[case], case
