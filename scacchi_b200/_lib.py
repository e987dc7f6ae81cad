"""ctypes binding of libscacchi_b200.so (the C ABI in include/scacchi_b200.h)."""

from __future__ import annotations

import ctypes as C
import functools
import os

from . import _build

OK, EINVAL, ECUDA = 0, 1, 2
ETOOLARGE = 3  # scacchi_search_synthetic_static: batch beyond the library-owned scratch


class ScacchiTree(C.Structure):
    _fields_ = [("batch", C.c_int32), ("num_nodes", C.c_int32), ("num_actions", C.c_int32),
                ("action_stride", C.c_int32), ("emb_bytes", C.c_int32)] + [
        (n, C.c_void_p) for n in (
            "parents", "children_index", "node_to_play", "node_outcome", "node_payload",
            "edge_outcome", "edge_payload", "node_value_prior", "node_value_alpha", "edge_alpha",
            "invalid", "embedding")]


class UpdateParams(C.Structure):
    _fields_ = [("rule", C.c_int32), ("kappa_ge_one", C.c_int32), ("inv_kappa", C.c_float),
                ("kappa", C.c_float), ("samples", C.c_int32), ("half_width", C.c_int32),
                ("tail_scale", C.c_float), ("min_half_range", C.c_float), ("max_half_range", C.c_float),
                ("density_tol", C.c_float)]


class PrefixOut(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "policy", "raw_policy", "raw_mass", "normalization_error", "finite", "grid_half_range",
        "tail_range_clipped", "density_log_integral", "fallback_interval_count")]


class SyntheticParams(C.Structure):
    _fields_ = [("seed_k0", C.c_uint32), ("seed_k1", C.c_uint32), ("num_actions", C.c_int32),
                ("legal_prob", C.c_float), ("terminal_prob", C.c_float),
                ("degenerate_lane_prob", C.c_float), ("degenerate_alpha", C.c_float),
                ("logc_mean", C.c_float), ("logc_std", C.c_float), ("logc_min", C.c_float),
                ("logc_max", C.c_float)]


class Context(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "active", "leaf_active", "leaf_action", "leaf_value", "leaf_to_play", "node_to_play",
        "node_payload", "value_prior", "value_alpha", "edge_alpha", "edge_payload", "edge_outcome",
        "invalid", "child_visited", "child_prior", "child_value", "child_payload", "child_outcome",
        "child_to_play")]


class TowerWeights(C.Structure):
    POINTERS = ("stem_w", "stem_b", "bn_scale", "bn_shift", "conv_w", "conv_b", "head_w", "head_b", "policy_w",
                "policy_b", "value_w1", "value_b1", "value_mean_w", "value_mean_b", "value_conc_w", "value_conc_b",
                "qdir_w1", "qdir_b1", "qdir_w2", "qdir_b2", "qconc_w1", "qconc_b1", "qconc_w2", "qconc_b2")
    _fields_ = [(n, C.c_int32) for n in ("num_blocks", "channels", "height", "width", "in_planes", "num_actions",
                                         "fp16", "terms")] + [
        (n, C.c_void_p) for n in POINTERS]


class LossFrames(C.Structure):
    FIELDS = ("reward", "discount", "terminated", "played_action", "legal", "policy", "search_mask", "q_pair_mask",
              "q_pair_weight", "q_kind", "q_outcome", "q_weight", "q_distance", "v_kind", "v_outcome", "v_weight",
              "v_distance")
    _fields_ = [(n, C.c_void_p) for n in FIELDS]


class LossOut(C.Structure):
    FIELDS = ("value_tgt", "value_mask", "policy_loss_mask", "value_loss_mask", "search_loss_mask", "policy_tgt",
              "q_pair_mask", "q_pair_weight", "q_kind", "q_outcome", "q_weight", "q_distance", "v_kind", "v_outcome",
              "v_weight", "v_distance")
    _fields_ = [(n, C.c_void_p) for n in FIELDS]


P = C.c_void_p
I32 = C.c_int32
F32 = C.c_float
TREE = C.POINTER(ScacchiTree)

SIGNATURES = {
    "scacchi_tree_init": [TREE, P, P, P, P, P, P, I32, P],
    "scacchi_simulate": [TREE, P, I32, P, P, P, P, P, P],
    "scacchi_expand": [TREE, I32, P, P, P, P, P, P, P, P, P, I32, P],
    "scacchi_backward": [TREE, P, P, P, P, P, P, C.POINTER(UpdateParams), P, P],
    "scacchi_root_policy": [TREE, P, P, I32, P, P, P],
    "scacchi_summary": [TREE, P, P, P, P, P, P, P, P],
    "scacchi_prefix_cdf": [P, P, P, I32, I32, I32, F32, F32, F32, C.POINTER(PrefixOut), P],
    "scacchi_posterior_best_policy": [P, P, P, P, I32, I32, I32, P, P],
    "scacchi_thompson_sample": [P, P, P, P, I32, I32, P, P],
    "scacchi_update_posterior": [P, C.POINTER(Context), I32, I32, C.POINTER(UpdateParams), P, P, P, P, P],
    "scacchi_root_readout": [I32, I32, P, P, P, P, P, P, P, I32, F32, I32, F32, F32, F32, P, P, P],
    "scacchi_commitment_policy": [I32, I32, P, P, P, P, P, P, P, I32, I32, I32, F32, F32, F32, P, P],
    "scacchi_commit_action": [I32, P, P, P, I32, I32, F32, P, P],
    "scacchi_synthetic_root": [C.POINTER(SyntheticParams), I32, P, P, P, P, P, P, P, P],
    "scacchi_synthetic_evaluate": [C.POINTER(SyntheticParams), I32, P, P, P, P, P, P, P, P],
    "scacchi_synthetic_recurrent": [C.POINTER(SyntheticParams), I32, P, P, P, P, P, P, P, P, P],
    "scacchi_search_workspace_bytes": [I32, I32, I32],
    "scacchi_search_synthetic": [TREE, C.POINTER(SyntheticParams), P, I32, I32, C.POINTER(UpdateParams), P, P,
                                 P],
    "scacchi_search_synthetic_static": [TREE, C.POINTER(SyntheticParams), P, I32, I32, C.POINTER(UpdateParams),
                                        P, P],
    "scacchi_key_schedule": [C.c_uint32, C.c_uint32, I32, P],
    "scacchi_split_host": [C.c_uint32, C.c_uint32, I32, P],
    "scacchi_fold_in_host": [C.c_uint32, C.c_uint32, C.c_uint32, P],
    "scacchi_hex_init": [I32, I32, P, P, P],
    "scacchi_hex_random_roots": [I32, I32, C.c_uint32, C.c_uint32, I32, I32, P, P],
    "scacchi_hex_step": [I32, P, P, P, P, P, P, P, P, P, P],
    "scacchi_hex_observe": [I32, P, P, P, P, P, P, P, P],
    "scacchi_hex_error": [P],
    "scacchi_hex_launch_count": [],
    "scacchi_tower_rows": [I32],
    "scacchi_tower_workspace_bytes": [I32],
    "scacchi_tower_forward": [C.POINTER(TowerWeights), P, I32, P, P, P, P, P, P, P],
    "scacchi_conv3x3": [P, P, P, I32, I32, I32, P, P, P, P, P, P, P, P, P],
    "scacchi_conv3x3_split": [P, P, P, P, I32, I32, I32, I32, P, P, P, I32, P, P, P, P, P, P],
    "scacchi_tower_error": [P],
    "scacchi_tower_launch_count": [],
    "scacchi_tower_timing": [I32],
    "scacchi_pack_targets": [I32, I32, P, P, P, P, P, I32, I32, P, P, P, P, P, P, P, P, P, P],
    "scacchi_loss_input": [C.POINTER(LossFrames), C.POINTER(LossOut), I32, I32, I32, I32, I32, I32, I32, I32, I32, P],
    "scacchi_target_launch_count": [],
    "scacchi_tower_timing_read": [P, P],
    "scacchi_device_error": [P],
    "scacchi_launch_count": [],
}
RESTYPES = {"scacchi_search_workspace_bytes": C.c_size_t, "scacchi_launch_count": C.c_uint64,
            "scacchi_tower_rows": C.c_uint64, "scacchi_tower_workspace_bytes": C.c_size_t,
            "scacchi_tower_launch_count": C.c_uint64, "scacchi_hex_launch_count": C.c_uint64,
            "scacchi_target_launch_count": C.c_uint64}


class ScacchiError(RuntimeError):
    pass


@functools.lru_cache(maxsize=None)
def lib() -> C.CDLL:
    """Load the in-tree CUDA library, building it first if it is missing.

    There is no fallback: without the library the search cannot run.
    """
    path = os.environ.get("SCACCHI_B200_LIB", _build.LIB)
    if not os.path.exists(path):
        if path != _build.LIB:
            raise FileNotFoundError(f"SCACCHI_B200_LIB={path} does not exist")
        _build.build()
    handle = C.CDLL(path)
    for name, args in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.argtypes = args
        fn.restype = RESTYPES.get(name, C.c_int)
    return handle


def check(rc: int, what: str) -> None:
    if rc == OK:
        return
    if rc == EINVAL:
        raise ValueError(f"{what}: arguments rejected by the CUDA library")
    raise ScacchiError(f"{what}: CUDA launch failed (status {rc})")


def device_error() -> int:
    flags = C.c_uint32(0)
    check(lib().scacchi_device_error(C.byref(flags)), "scacchi_device_error")
    return int(flags.value)


def launch_count() -> int:
    """Kernels this library launched since load (search + network + Hex)."""
    return (int(lib().scacchi_launch_count()) + int(lib().scacchi_tower_launch_count())
            + int(lib().scacchi_hex_launch_count()) + int(lib().scacchi_target_launch_count()))


def tower_error() -> int:
    flags = C.c_uint32(0)
    check(lib().scacchi_tower_error(C.byref(flags)), "scacchi_tower_error")
    return int(flags.value)
