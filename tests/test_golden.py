"""The oracle still reproduces the committed golden vectors bit for bit."""

import os
import sys

import numpy as np

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import make_golden  # noqa: E402

FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "oracle_vectors.npz")


def test_oracle_reproduces_golden_vectors():
    want = np.load(FIXTURE)
    got = make_golden.generate()
    assert sorted(got) == sorted(want.files)
    for k in want.files:
        assert np.array_equal(np.asarray(got[k]), want[k], equal_nan=True), k
