"""Host-side jax.random key operations (threefry2x32, partitionable layout).

Keys are numpy uint32[2] arrays, bit-compatible with jax.random's raw
threefry keys.  The arithmetic runs in the C library (no device work).
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib


def _k(key) -> tuple[int, int]:
    k = np.asarray(key, dtype=np.uint32).reshape(2)
    return int(k[0]), int(k[1])


def PRNGKey(seed: int) -> np.ndarray:
    """jax.random.PRNGKey with 32-bit seeds (x64 off): [0, seed mod 2^32]."""
    return np.array([0, int(seed) & 0xFFFFFFFF], np.uint32)


def split(key, num: int = 2) -> np.ndarray:
    out = np.zeros((num, 2), np.uint32)
    k0, k1 = _k(key)
    _lib.check(_lib.lib().scacchi_split_host(k0, k1, num, out.ctypes.data_as(C.c_void_p)), "split")
    return out


def fold_in(key, data: int) -> np.ndarray:
    out = np.zeros(2, np.uint32)
    k0, k1 = _k(key)
    _lib.check(_lib.lib().scacchi_fold_in_host(k0, k1, int(data) & 0xFFFFFFFF, out.ctypes.data_as(C.c_void_p)),
               "fold_in")
    return out


def key_schedule(search_key, num_simulations: int) -> np.ndarray:
    """uint32[N, 4, 2]: (next, simulate, expand, backward) keys per simulation."""
    out = np.zeros((max(num_simulations, 0), 4, 2), np.uint32)
    k0, k1 = _k(search_key)
    _lib.check(_lib.lib().scacchi_key_schedule(k0, k1, num_simulations, out.ctypes.data_as(C.c_void_p)),
               "key_schedule")
    return out
