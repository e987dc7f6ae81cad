"""The C-ABI library builds for sm_100a, loads without a GPU and exports every
symbol that include/scacchi_b200.h declares; host-only helpers agree with the
oracle's key schedule."""

import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "scacchi_b200.h")).read()
    return sorted(set(re.findall(r"^(?:int|size_t|uint64_t)\s+(scacchi_\w+)\(", text, re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "scacchi_simulate" in syms and "scacchi_backward" in syms and len(syms) >= 18


def test_library_exports_every_declared_symbol():
    from scacchi_b200 import _lib

    lib = _lib.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_host_key_helpers_match_oracle():
    from oracle import oracle as O
    from scacchi_b200 import random as R

    key = np.array([3, 4], np.uint32)
    assert np.array_equal(R.split(key, 5), O.split(key, 5))
    assert np.array_equal(R.fold_in(key, 77), O.fold_in(key, 77))
    sched = R.key_schedule(key, 6)
    k = key
    for i in range(6):
        s = O.split(k, 4)
        assert np.array_equal(sched[i], s)
        k = s[0]


def test_rejects_bad_arguments_without_launching():
    import ctypes as C
    from scacchi_b200 import _lib

    lib = _lib.lib()
    assert lib.scacchi_simulate(None, None, 1, None, None, None, None, None, None) == _lib.EINVAL
    assert lib.scacchi_prefix_cdf(None, None, None, 1, 82, 10, 8.0, 6.0, 11.0, None, None) == _lib.EINVAL
    t = _lib.ScacchiTree(1, 1, 200, 224, 0)  # 200 actions: above the 128 limit
    assert lib.scacchi_summary(C.byref(t), *([None] * 8)) == _lib.EINVAL
