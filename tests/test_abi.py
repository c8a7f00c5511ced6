"""The C ABI: the library loads, exports every entry point the headers declare, and rejects bad
arguments with a status (CPU only: no call here reaches a kernel)."""
import ctypes
import re

import pytest

from conftest import ROOT


def _declared():
    names = []
    for header in sorted((ROOT / "include").glob("*.h")):
        names += re.findall(r"^FMD_API\s+[\w\s\*]+?\b(fmd_\w+)\s*\(", header.read_text(), flags=re.M)
    return names


def test_headers_declare_entry_points():
    names = _declared()
    assert len(names) >= 10
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    from fastmd_b200 import _lib

    lib = _lib.lib()
    missing = [name for name in _declared() if not hasattr(lib, name)]
    assert not missing, missing


def test_python_binding_covers_every_symbol():
    from fastmd_b200 import _lib

    import fastmd_b200  # noqa: F401  (modules that register extra signatures)
    missing = [name for name in _declared() if name not in _lib._SIGNATURES]
    assert not missing, missing


def test_status_strings_and_version():
    from fastmd_b200 import _lib

    lib = _lib.lib()
    assert lib.fmd_version() >= 100
    assert lib.fmd_status_string(0) == b"ok"
    assert lib.fmd_status_string(1) == b"invalid argument"
    assert lib.fmd_status_string(99) == b"unknown status"


def test_invalid_arguments_are_rejected_before_any_launch():
    from fastmd_b200 import _lib

    lib = _lib.lib()
    assert lib.fmd_gather_cat(None, 0, 0, None, 0, None, None) == 1
    assert lib.fmd_copy_rows(None, 0, None, 0, 1, 1, None) == 1
    assert lib.fmd_csr_segment_sum(None, 0, None, 0, None, None, 1, 1, -1, None, 0, None) == 1
    assert lib.fmd_nhc_pre_force(None, None, None, 1, 1, 3, 1, 0, None, None) == 1
    assert lib.fmd_nhc_post_force(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 1, 1, 3, 1, 0,
                                  None, None, None, None) == 1  # neither force dtype
    p16 = ctypes.c_void_p(1 << 20)
    assert lib.fmd_gemm_tf32x3(None, 8, p16, p16, 8, None, None, 0, p16, 8, 1, 8, 8, 0, 0, None, None) == 1
    assert lib.fmd_gemm_tf32x3(p16, 8, p16, p16, 8, None, None, 0, p16, 8, 1, 8, 8, 2, 0, None, None) == 1  # gate: c
    assert lib.fmd_gemm_tf32x3(p16, 8, p16, p16, 8, None, None, 0, p16, 8, 1, 8, 8, 3, 0, None, None) == 1  # act
    assert lib.fmd_gemm_tf32x3(p16, 8, p16, p16, 8, None, None, 0, p16, 8, 1, 8, 8, 32, 0, None, None) == 1
    # TMA operands: unaligned base or a row stride that is not a multiple of 16 bytes -> unsupported
    assert lib.fmd_gemm_tf32x3(ctypes.c_void_p((1 << 20) + 4), 8, p16, p16, 8, None, None, 0, p16, 8, 1, 8, 8, 0, 0,
                               None, None) == 3
    assert lib.fmd_gemm_tf32x3(p16, 9, p16, p16, 8, None, None, 0, p16, 8, 1, 8, 8, 0, 0, None, None) == 3
    assert lib.fmd_tf32_split(None, 2, 2, 2, 0, None, None, 2, None) == 1
    assert lib.fmd_pair_aggregate(4, p16, 8, p16, 1, 8, p16, None, None) == 1  # no such op
    assert lib.fmd_pair_aggregate(0, p16, 4, p16, 1, 8, p16, None, None) == 1  # row stride below the width
    assert lib.fmd_pair_aggregate(0, None, 8, None, 0, 8, None, None, None) == 0  # no pairs: nothing to do
    assert lib.fmd_residual_add(2, p16, 8, p16, 8, p16, 1, 8, p16, 8, None) == 1  # no such op
    nb = ctypes.c_size_t(0)
    assert lib.fmd_bond_graph_workspace_bytes(0, 2100, ctypes.byref(nb)) == 1
    cell = (ctypes.c_float * 9)(*[10, 0, 0, 0, 10, 0, 0, 0, 10])
    image = (ctypes.c_int32 * 3)(1, 0, 0)
    args = [p16, cell, 8, p16, p16, p16, 16, 32, ctypes.c_float(4.5), 0, 4, None, p16, 1 << 20, p16, p16, p16, p16,
            p16, None]
    bad = list(args)
    bad[9] = 2  # no such padding rule
    assert lib.fmd_bond_graph(*bad) == 1
    bad = list(args)
    bad[10] = 0  # sink padding needs sink atoms
    assert lib.fmd_bond_graph(*bad) == 1
    bad = list(args)
    bad[9], bad[11] = 1, None  # far self-loops need the loop image
    assert lib.fmd_bond_graph(*bad) == 1
    bad = list(args)
    bad[8] = ctypes.c_float(-1.0)  # negative line cutoff
    assert lib.fmd_bond_graph(*bad) == 1
    del image
    assert lib.fmd_residual_add(0, p16, 4, p16, 8, p16, 1, 8, p16, 8, None) == 1  # delta stride below the width
    assert lib.fmd_residual_add(0, None, 8, p16, 8, p16, 1, 8, p16, 8, None) == 1  # forward needs delta
    assert lib.fmd_residual_add(1, None, 0, None, 8, None, 0, 8, None, 8, None) == 0  # no rows: nothing to do


def test_no_cpu_fallback():
    import torch

    from fastmd_b200 import ops
    from fastmd_b200._lib import FastMDLibraryError

    x = torch.zeros(4, 8)
    idx = torch.zeros(4, dtype=torch.int64)
    with pytest.raises(FastMDLibraryError):
        ops.aligned_gather_cat3(x, x, idx, idx)
    with pytest.raises(FastMDLibraryError):
        ops.csr_segment_sum(x, idx, 2)
    from fastmd_b200 import wide_gemm

    with pytest.raises(FastMDLibraryError):
        wide_gemm.linear(x, torch.zeros(16, 8))
