"""The C ABI library loads and exports every declared entry point (no GPU).

Also checks the host-side argument validation paths, which return a status
before touching the device.
"""

import ctypes
import os
import re

import pytest

from conftest import REPO
from tack_b200 import _lib

HEADER = os.path.join(REPO, "include", "tackmc.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tkmc_\w+)\s*\(", src)))


def test_header_declares_the_api():
    names = declared_functions()
    for must in ("tkmc_fe_count", "tkmc_fe_emit", "tkmc_scan_i32", "tkmc_reduce_f32",
                 "tkmc_fe_workspace_bytes", "tkmc_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_library_loads_and_reports_version():
    lib = _lib.load()
    assert lib.tkmc_version() == 100
    assert lib.tkmc_launch_count() >= 0


def test_workspace_sizes():
    lib = _lib.load()
    a = lib.tkmc_fe_workspace_bytes(63, 63, 63, 1)
    b = lib.tkmc_fe_workspace_bytes(63, 63, 63, 4)
    c = lib.tkmc_fe_workspace_bytes(1023, 1023, 1023, 1)
    assert 0 < a < b < c
    # 1024^3: unit list (32 B for every 32-node word: 1 GiB) + bitmask 128 MiB
    # + per-word counts 128 MiB + row offsets 32 MiB + row counts 16 MiB +
    # word summaries, activity masks, row lists (~24 MiB)
    assert 1300 << 20 < c < 1400 << 20
    assert lib.tkmc_fe_workspace_bytes(-1, 4, 4, 1) == 0
    assert lib.tkmc_fe_workspace_bytes(4, 4, 4, 0) == 0
    assert lib.tkmc_fe_workspace_bytes(4, 4, 4, 9) == 0
    assert lib.tkmc_scan_workspace_bytes(10) > 0


def test_argument_errors_return_status_without_a_device():
    lib = _lib.load()
    isos = (ctypes.c_float * 1)(0.0)
    counts = (ctypes.c_int64 * 4)()
    rc = lib.tkmc_fe_count(None, 4, 4, 4, 0, isos, 0, None, None, 0, counts, None)
    assert rc == _lib.TKMC_ERR_INVALID_ARG
    assert b"niso" in lib.tkmc_last_error()
    rc = lib.tkmc_fe_count(None, -2, 4, 4, 0, isos, 1, None, None, 0, counts, None)
    assert rc == _lib.TKMC_ERR_INVALID_ARG
    rc = lib.tkmc_fe_count(0x1000, 4, 4, 4, 0, isos, 1, None, 0x100000, 16, counts, None)
    assert rc == _lib.TKMC_ERR_WORKSPACE
    rc = lib.tkmc_fe_count(0x1000, 4, 4, 4, 0, isos, 1, None, 0x100010, 1 << 20, counts, None)
    assert rc == _lib.TKMC_ERR_INVALID_ARG  # workspace not 256-byte aligned
    with pytest.raises(_lib.TkmcError) as e:
        _lib.check(_lib.TKMC_ERR_INVALID_ARG, "x")
    assert e.value.code == _lib.TKMC_ERR_INVALID_ARG


def test_tables_are_host_only():
    lib = _lib.load()
    num = (ctypes.c_int32 * 256)()
    assert lib.tkmc_mc_tables(None, num, None) == 0
    assert max(num) == 5
