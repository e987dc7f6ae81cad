"""Benchmark: the batched Dirichlet-Thompson search step on B200.

Default workload (one GPU): the full self-play search step on Hex 9x9 --
8192 lanes, 256 simulations (tree capacity 257), the 6 x 128 AZDirichletNet
with the reference's random init evaluating every leaf on the tcgen05 tower
(split bf16 operands, the precision that holds the 2e-2 tolerance), the
guarded prefix-CDF estimator (kappa 1, Q21, Monte Carlo fallback with 8
samples), exact terminal certificates, roots after 0-20 uniform random
legal moves.  One step = one ``search(root_state, key)`` call through
``play_search.make_search``: root evaluation, 256 x (descent, Hex step,
tower, expand, backward), root readout and target packing.

Under torchrun (any number of ranks) the default is the lane-sharded
population step: 8192 lanes per GPU with the 64-sample Thompson-population
estimator, the root targets all-gathered over NCCL at the end of the step
(weak scaling).

Other workloads (also sub-objects of the default line): ``search`` -- the
isolated search kernels on 4096 lanes x 128 simulations with synthetic
network outputs; ``tower`` -- the residual tower alone on 16384 boards.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
       [--workload full|population|search|tower] [--precision NAME]
       [--no-cpu-baseline] [--no-sub] [--profile [--boards B] [--lanes L]]
Prints one JSON line on rank 0 (the line that starts with '{').  With
NCCL_DEBUG=INFO set, NCCL prints its communicator lines into the same
output.  --profile runs warm-up steps and one device-resident step and
prints no line, for ncu captures (--boards / --lanes: smaller cases).
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Hex 9×9 search sims/sec (lanes×sims) at 1/2/4/8 B200; leaf evals/sec"
ACTIONS = 82
KAPPA = 1.0
FALLBACK_SAMPLES = 8
POPULATION_SAMPLES = 64
FULL_LANES = 8192           # per GPU
FULL_SIMS = 256
SEARCH_LANES = 4096         # isolated search kernels
SEARCH_SIMS = 128
TOWER_BOARDS = 16384        # tower alone
ROOT_SEED, SEARCH_SEED = 0, 1
FALLBACK_HBM_GBS = 6650.0
FALLBACK_TFLOPS = 1590.0
FALLBACK_TFLOPS_SUSTAINED = 1400.0

CONV_FLOP_PER_BOARD = 2 * 81 * 128 * 128 * 9          # one 3x3 128->128 conv over a board's 81 cells
TOWER_FLOP_PER_BOARD = 12 * CONV_FLOP_PER_BOARD + 2 * 81 * 4 * 128 * 9 + 2 * (
    81 * 128 * 6 + 162 * 82 + 81 * 128 + 128 * 3 + 162 * 128 + 128 * 164 + 81 * 128 + 128 * 82)

CSRC = os.path.join(ROOT, "scacchi_b200", "csrc")
SEARCH_SOURCES = ("search.cu", "lane_cta.cuh", "smath.h", "threefry.h", "synthetic_env.h")
TOWER_SOURCES = ("tower.cu",)


def source_hash(names) -> str:
    h = hashlib.sha256()
    for n in names:
        with open(os.path.join(CSRC, n), "rb") as f:
            h.update(f.read())
    return h.hexdigest()[:16]


# Figures taken from ncu captures (profiles/), each stamped with the hash of
# the kernel sources it was captured on.  bench.py reports a figure only
# while the sources still hash to its stamp; after a kernel change it prints
# null with "stale" until the figure is captured again.
CAPTURED = {
    # dram__bytes_read.sum + dram__bytes_write.sum of one backward launch
    # (simulation 64 of the isolated-search profile step;
    # profiles/backward_cta_search4096x128.md)
    "backward_traffic_bytes": dict(value=23675648 + 1792, sources=SEARCH_SOURCES, sha="f8154eef933b56af"),
    # smsp__inst_executed.sum of that launch x 128 launches per step (an
    # all-launch capture of an earlier build gave 5 % less: the middle
    # simulation's paths are a little deeper than the step's average)
    "backward_warp_inst_per_step": dict(value=204322290 * 128, sources=SEARCH_SOURCES, sha="f8154eef933b56af"),
    # dram bytes of the 12 conv launches of one 8192-board forward at the
    # default precision, averaged per launch (profiles/conv_tc_split_tower8192.md)
    "conv_traffic_bytes_8192": dict(value=1146349397, sources=TOWER_SOURCES, sha="960603ed2aee9b4f"),
    # smsp__inst_executed.sum over every backward launch of one profile step
    # of the full step (1024 lanes) / that step's backward node updates
    # (profiles/backward_fullstep.md)
    "backward_inst_per_node_prefix": dict(value=26355, sources=SEARCH_SOURCES, sha="f8154eef933b56af"),
    "backward_inst_per_node_population": dict(value=153300, sources=SEARCH_SOURCES, sha="f8154eef933b56af"),
}


def captured(name: str):
    """(value or None, provenance dict) of a stamped ncu figure."""
    c = CAPTURED[name]
    now = source_hash(c["sources"])
    ok = c["value"] is not None and now == c["sha"]
    return (c["value"] if ok else None), {"stamp": c["sha"], "sources_now": now, "stale": not ok}


def read_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            m = json.load(f)
        return {"hbm_gbs": float(m["hbm_gbs"]), "bf16_tflops": float(m["bf16_tflops"]),
                "bf16_tflops_sustained": float(m["bf16_tflops_sustained"]), "source": "measured"}
    except Exception:
        return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_TFLOPS,
                "bf16_tflops_sustained": FALLBACK_TFLOPS_SUSTAINED, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            # nvidia-smi takes a moment to start: begin timing once it samples
            deadline = time.time() + 3.0
            while time.time() < deadline and os.path.getsize(self.path) == 0:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        except Exception:
            pass
        finally:
            if self.path and os.path.exists(self.path):
                os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(float(r[1]) for r in rows), "sm_max_mhz": float(rows[0][2]),
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# ---------------------------------------------------------------------------
# search configurations
# ---------------------------------------------------------------------------

def prefix_cdf_config(sims: int):
    from scacchi_b200.types import (DirichletThompsonSearchConfig, NumericalPosteriorUpdateConfig,
                                    PosteriorUpdateConfig, PosteriorUpdateKind, RootPolicySupport)

    return DirichletThompsonSearchConfig(
        num_simulations=sims, max_depth=sims, root_policy_support=RootPolicySupport.search_evidence,
        policy_target_temperature=1.0,
        posterior_update=PosteriorUpdateConfig(
            kind=PosteriorUpdateKind.numerical,
            numerical=NumericalPosteriorUpdateConfig(kappa=KAPPA, half_width=10, tail_scale=8.0, min_half_range=6.0,
                                                     max_half_range=11.0, fallback_policy_samples=FALLBACK_SAMPLES,
                                                     fallback_policy_sample_chunk_size=32)))


def population_config(sims: int):
    from scacchi_b200.types import (DirichletThompsonSearchConfig, MonteCarloPosteriorUpdateConfig,
                                    PosteriorUpdateConfig, PosteriorUpdateKind, RootPolicySupport)

    return DirichletThompsonSearchConfig(
        num_simulations=sims, max_depth=sims, root_policy_support=RootPolicySupport.search_evidence,
        policy_target_temperature=1.0,
        posterior_update=PosteriorUpdateConfig(
            kind=PosteriorUpdateKind.monte_carlo,
            monte_carlo=MonteCarloPosteriorUpdateConfig(kappa=KAPPA, policy_samples=POPULATION_SAMPLES,
                                                        policy_sample_chunk_size=32)))


def full_workload_config(world: int, population: bool, precision: str) -> dict:
    est = (f"Thompson population, {POPULATION_SAMPLES} samples per node" if population else
           f"prefix_cdf Q21 (kappa 1, Monte Carlo fallback {FALLBACK_SAMPLES} samples)")
    return {
        "workload": (f"full self-play search step: Hex 9x9 (82 actions), {FULL_LANES} lanes/GPU x {FULL_SIMS} "
                     f"simulations, AZDirichletNet 6x128 (reference random init) on the tcgen05 tower ({precision}), "
                     f"{est}, exact terminal certificates, roots after 0-20 uniform random legal moves"),
        "lanes_per_gpu": FULL_LANES, "global_lanes": FULL_LANES * world, "num_simulations": FULL_SIMS,
        "tree_capacity": FULL_SIMS + 1, "num_actions": ACTIONS, "tower_precision": precision, "kappa": KAPPA,
        "l2": "inputs larger than L2: the tree is 3.7 GB per GPU and the tower streams 1.3 GB per evaluation",
        "parallelism": f"dp{world} (lane-sharded)",
    }


# ---------------------------------------------------------------------------
# the full step (configs 4 and 5)
# ---------------------------------------------------------------------------

def default_workload() -> str:
    """The full step (the metric's one-GPU configuration) when run as a
    plain process; the population step (the lane-sharded multi-GPU
    configuration) whenever torchrun launched the process, one rank
    included, so a scaling series run under torchrun measures one
    workload at every N."""
    return "population" if "WORLD_SIZE" in os.environ else "full"


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _all_ranks(x: float, world: int) -> list:
    if world == 1:
        return [x]
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    out = torch.empty((world,), dtype=torch.float64, device="cuda")
    dist.all_gather_into_tensor(out, t)
    return [float(v) for v in out.cpu()]


def _barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def full_step_bench(steps: int, warmup: int, precision: str | None, population: bool, world: int, rank: int,
                    local: int, e2e: bool = True, clocks: bool = True, lanes: int = FULL_LANES) -> dict:
    """The full search step of ``full_workload_config`` on this rank's lanes,
    device-resident, then end to end from pinned host buffers."""
    import ctypes as C

    import torch

    from scacchi_b200 import _lib
    from scacchi_b200 import random as R
    from scacchi_b200.dirichlet_mctx import search as S
    from scacchi_b200.distributed import LaneSharding, gather_targets
    from scacchi_b200.hex import HexGame, HexState
    from scacchi_b200.network import AZDirichletNet, init_params
    from scacchi_b200.play_search import make_evaluator, make_search

    dev = torch.device("cuda", local)
    sharding = LaneSharding(world, rank)
    game = HexGame(9, device=dev)
    net = AZDirichletNet(init_params(0, he_all_layers=False), device=dev, precision=precision)
    cfg = population_config(FULL_SIMS) if population else prefix_cdf_config(FULL_SIMS)
    # work counters of the search kernels (one atomic add per CTA): backward
    # node updates [0], visited children gathered [1], Monte Carlo fallbacks
    # [2]; descent nodes [4], priors gathered [5]
    stats = torch.zeros(6, dtype=torch.int64, device=dev)
    search = make_search(game, make_evaluator(net), cfg, stats=stats)
    state = game.random_roots(lanes, R.fold_in(R.PRNGKey(ROOT_SEED), rank), 0, 20)
    key = sharding.device_key(R.PRNGKey(SEARCH_SEED))
    stream = torch.cuda.current_stream(dev)
    gather_ev = []  # per step: (step start, search done, gather done)

    def step(s):
        s0 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        t = search(s, key)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        out = gather_targets(t, sharding)
        g1.record(stream)
        gather_ev.append((s0, g0, g1))
        return out

    for _ in range(warmup):
        step(state)
    torch.cuda.synchronize()
    _barrier(world)
    torch.cuda.synchronize()
    gather_ev.clear()
    if steps == 0:
        return {"work": [int(v) for v in stats.cpu().tolist()]}
    stats.zero_()
    # live timing of the tower's convolutions and of the loop's phases
    _lib.check(_lib.lib().scacchi_tower_timing(steps * (FULL_SIMS + 1) + 4), "tower_timing")
    timer = S.PhaseTimer()
    S.set_phase_timer(timer)
    launches0 = _lib.launch_count()
    sampler = ClockSampler(local) if clocks else None
    if sampler:
        sampler.__enter__()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step(state)
    e1.record(stream)
    torch.cuda.synchronize()
    if sampler:
        sampler.__exit__(None, None, None)
    S.set_phase_timer(None)
    launches = _lib.launch_count() - launches0
    conv_ms, forwards = C.c_float(0), C.c_int32(0)
    _lib.check(_lib.lib().scacchi_tower_timing_read(C.byref(conv_ms), C.byref(forwards)), "tower_timing_read")
    _lib.check(_lib.lib().scacchi_tower_timing(0), "tower_timing")
    phases = timer.totals_ms()
    _barrier(world)
    my_ms = e0.elapsed_time(e1) / steps
    # this rank's search alone (before the collective) and its all-gather
    # (which includes waiting for the slowest rank's search)
    search_ms = sum(a.elapsed_time(b) for a, b, _ in gather_ev) / steps
    gather_ms = sum(b.elapsed_time(c) for _, b, c in gather_ev) / steps
    rank_ms = _all_ranks(my_ms, world)
    rank_search = _all_ranks(search_ms, world)
    rank_gather = _all_ranks(gather_ms, world)
    ms = max(rank_ms)
    out = {"ms_per_step": ms, "rank_ms": rank_ms, "rank_search_ms": rank_search, "rank_gather_ms": rank_gather,
           "gather_ms": min(rank_gather), "launches_per_step": launches / steps,
           "conv_ms_per_step": conv_ms.value / steps, "forwards": forwards.value,
           "conv_launch_ms": conv_ms.value / max(forwards.value, 1) / 12,
           "phases_ms_per_step": {k: v / steps for k, v in phases.items()}, "precision": net.precision,
           "work_per_step": [v / steps for v in stats.cpu().tolist()],
           "terms": net.terms, "clocks": sampler.summary() if sampler else None}
    if not e2e:
        return out

    # ---- end to end: pinned host roots in, host targets out ----------------
    host = {f: getattr(state, f).cpu().pin_memory() for f in HexState._fields}
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    G = FULL_LANES * world
    sink = dict(policy=torch.empty((G, ACTIONS), dtype=torch.float32).pin_memory(),
                alpha_q=torch.empty((G, ACTIONS, 2), dtype=torch.float32).pin_memory(),
                alpha_v=torch.empty((G, 2), dtype=torch.float32).pin_memory(),
                search_action=torch.empty((G,), dtype=torch.int32).pin_memory())
    d2h = sum(t.numel() * t.element_size() for t in sink.values())

    def e2e_step():
        s = HexState(**{f: t.to(dev, non_blocking=True) for f, t in host.items()})
        t = step(s)
        sink["policy"].copy_(t.prediction.policy, non_blocking=True)
        sink["alpha_q"].copy_(t.prediction.alpha_q, non_blocking=True)
        sink["alpha_v"].copy_(t.prediction.alpha_v, non_blocking=True)
        sink["search_action"].copy_(t.metadata.search_action, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    _barrier(world)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    _barrier(world)
    out["e2e_ms"] = _max_over_ranks(e0.elapsed_time(e1) / steps, world)
    out["h2d_bytes"] = h2d
    out["d2h_bytes"] = d2h
    return out


def backward_issue(f: dict, population: bool, sm_count: int) -> dict:
    """Issue rate of the backward kernel inside the step: warp instructions
    per node update (from an ncu capture of every backward launch of a
    profile step, divided by that step's node updates) x node updates per
    step (live counters) / live backward time, against 4 instructions per
    SM per cycle at the sampled clock."""
    name = "backward_inst_per_node_population" if population else "backward_inst_per_node_prefix"
    per_node, prov = captured(name)
    ms = f["phases_ms_per_step"]["backward"]
    nodes = f["work_per_step"][0]
    mhz = (f["clocks"] or {}).get("sm_mhz") or 1965.0
    peak = sm_count * 4 * mhz / 1e3
    achieved = per_node * nodes / (ms / 1e3) / 1e9 if per_node and ms > 0 else None
    return {"bound": "issue", "kernel": "backward_cta_kernel", "achieved": None if achieved is None else round(achieved, 1),
            "peak": round(peak, 1), "unit": "G warp-inst/s",
            "frac": None if achieved is None else round(achieved / peak, 4),
            "node_updates_per_step": int(nodes), "mc_fallbacks_per_step": int(f["work_per_step"][2]),
            "inst_per_node": per_node, "inst_provenance": prov,
            "peak_source": "4 schedulers x SMs x sampled SM clock"}


def tower_roofline(f: dict, peaks: dict) -> dict:
    """Tensor roofline of the convolutions inside the step: algorithmic
    FLOPs of one conv launch (81 cells x 128 x 128 x 9 x 2 per board, 8192
    boards) over its live average duration, against the measured sustained
    bf16 peak divided by the products per K step of the precision."""
    alg = CONV_FLOP_PER_BOARD * FULL_LANES
    achieved = alg / (f["conv_launch_ms"] / 1e3) / 1e12
    terms = f["terms"]
    peak = peaks["bf16_tflops_sustained"] / terms
    traffic, prov = captured("conv_traffic_bytes_8192")
    issued = achieved * terms * 100 / 81
    return {
        "bound": "tensor", "kernel": "conv_tc_kernel", "achieved": round(achieved, 2), "peak": round(peak, 2),
        "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_provenance": prov,
        "peak_source": (f"{peaks['source']} bf16 sustained ({peaks['bf16_tflops_sustained']} TFLOP/s)"
                        + (f" / {terms}: {f['precision']} issues {terms} bf16-class products per K step"
                           if terms > 1 else "")),
        "avg_launch_ms": round(f["conv_launch_ms"], 5), "launches_timed": 12 * f["forwards"],
        "algorithmic_flop_per_launch": alg,
        "issued_tensor_frac": round(issued / peaks["bf16_tflops_sustained"], 4),
        "note": "algorithmic FLOPs count the 81 cells of each board; the kernel also multiplies the 19 padding "
                "rows of the 100-row padded board (x1.23) and, with split operands, issues one tensor-core product "
                "per operand term; issued_tensor_frac counts both against the bf16 peak",
    }


# ---------------------------------------------------------------------------
# the isolated search kernels (synthetic network outputs, 4096 x 128)
# ---------------------------------------------------------------------------

def search_workload_config(world: int) -> dict:
    return {
        "workload": "isolated search kernels: Hex 9x9 action space (82 actions), synthetic network outputs",
        "lanes_per_gpu": SEARCH_LANES, "global_lanes": SEARCH_LANES * world, "num_simulations": SEARCH_SIMS,
        "tree_capacity": SEARCH_SIMS + 1, "estimator": "prefix_cdf Q21 + MC fallback", "kappa": KAPPA,
        "fallback_policy_samples": FALLBACK_SAMPLES, "root_policy_samples": FALLBACK_SAMPLES,
        "degenerate_lanes": "1% (alpha=1e-3)", "legal_prob": 0.7, "logc": "clip(N(0.5,1),-4,6)",
        "l2": "inputs larger than L2: the tree is 0.9 GB per GPU, rewritten every step",
        "parallelism": f"dp{world} (lane-sharded)",
    }


def search_roofline(ms: dict, sim_stats, bwd_stats, peaks: dict, sm_count: int, sm_mhz: float) -> dict:
    A = ACTIONS
    row = A * (4 + 4 + 8 + 1 + 1)  # children, payload, alpha, outcome, invalid
    bwd_bytes = bwd_stats[0] * (row + 24 + A * 12 + 12) + bwd_stats[1] * 25
    sim_bytes = sim_stats[0] * (row + 5) + sim_stats[1] * 12
    total = sum(ms.values())
    dominant = max(ms, key=ms.get)
    per = {"backward": bwd_bytes, "simulate": sim_bytes}
    bytes_per_launch = per.get(dominant, 0) / SEARCH_SIMS
    avg_s = ms[dominant] / SEARCH_SIMS / 1e3
    achieved = bytes_per_launch / avg_s / 1e9 if avg_s > 0 else 0.0
    issue_peak = sm_count * 4 * sm_mhz / 1e3
    inst, inst_prov = captured("backward_warp_inst_per_step")
    issue = inst / (ms["backward"] / 1e3) / 1e9 if inst and ms.get("backward") else None
    traffic, traffic_prov = captured("backward_traffic_bytes")
    return {
        "bound": "hbm", "kernel": f"{dominant}_kernel", "achieved": round(achieved, 2), "peak": peaks["hbm_gbs"],
        "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 5),
        "traffic": traffic if dominant == "backward" else None, "traffic_provenance": traffic_prov,
        "peak_source": peaks["source"], "algorithmic_bytes_per_launch": int(bytes_per_launch),
        "avg_launch_ms": round(ms[dominant] / SEARCH_SIMS, 5),
        "kernel_share": {k: round(v / total, 4) for k, v in ms.items()},
        "work": {"descent_nodes": sim_stats[0], "descent_prior_gathers": sim_stats[1],
                 "backward_nodes": bwd_stats[0], "backward_child_gathers": bwd_stats[1],
                 "mc_fallback_nodes": bwd_stats[2]},
        "issue": {"bound": "issue", "kernel": "backward_kernel", "achieved": None if issue is None else round(issue, 1),
                  "peak": round(issue_peak, 1), "unit": "G warp-inst/s",
                  "frac": None if issue is None else round(issue / issue_peak, 4), "inst_provenance": inst_prov,
                  "peak_source": "4 schedulers x SMs x sampled SM clock"},
        "note": "search kernels are ALU-bound (in-kernel threefry, Q21 transcendentals); the HBM fraction is "
                "algorithmic bytes over measured copy bandwidth, the issue fraction is warp instructions "
                "over the schedulers' issue rate",
    }


def instrumented_search_step(game, state, key, cfg):
    """One extra (untimed) isolated-search step driven phase by phase from
    Python (the synthetic game otherwise runs its loop inside the library),
    with CUDA events on the launching stream around every kernel and the
    kernels' own work counters, for the per-kernel roofline."""
    import torch

    from scacchi_b200 import random as R
    from scacchi_b200.dirichlet_mctx import RootFnOutput
    from scacchi_b200.dirichlet_mctx import search as S
    from scacchi_b200.dirichlet_mctx.posterior_updates import rule_params
    from scacchi_b200.dirichlet_mctx.tree import _init_tree
    from scacchi_b200.play_search import _make_posterior_update

    dev = state.observation.device
    pred = game.evaluator(state.observation)
    root = RootFnOutput(prior_logits=pred.logits, value=pred.alpha_v, action_values=pred.alpha_q,
                        embedding=state.observation,
                        terminal_outcome=torch.full((SEARCH_LANES,), -1, dtype=torch.int8, device=dev),
                        to_play=state.current_player)
    rparams = rule_params(_make_posterior_update(cfg.posterior_update.active()))
    search_key = R.split(key)[0]
    tree = _init_tree(root, SEARCH_SIMS, ~state.legal_action_mask, full=False)
    sched = torch.from_numpy(R.key_schedule(search_key, SEARCH_SIMS).view("int32")).to(dev)
    bufs = S.SimulationBuffers(SEARCH_LANES, ACTIONS, tree.E, dev)
    sim_stats = torch.zeros(2, dtype=torch.int64, device=dev)
    bwd_stats = torch.zeros(3, dtype=torch.int64, device=dev)
    timer = S.PhaseTimer()
    for i in range(SEARCH_SIMS):
        timer.mark()
        S.simulate(tree, sched[i, 1], SEARCH_SIMS, bufs, sim_stats)
        timer.mark()
        step, child = game((), None, bufs.action, bufs.parent_embedding[:, :tree.E])
        timer.mark()
        v, tp = S.expand(tree, i + 1, bufs, step, child)
        timer.mark()
        S.backward(tree, sched[i, 3], bufs, v, tp, rparams, bwd_stats)
        timer.mark()
    return timer.totals_ms(), sim_stats.cpu().tolist(), bwd_stats.cpu().tolist()


def search_kernels_bench(steps: int, warmup: int, world: int, rank: int, local: int, profile: bool = False) -> dict:
    """The isolated search kernels: device-resident steps, the end-to-end
    call from pinned host buffers, and one instrumented (untimed) step with
    CUDA events around every phase and the kernels' work counters."""
    import torch

    from scacchi_b200 import _lib
    from scacchi_b200 import random as R
    from scacchi_b200.distributed import LaneSharding, gather_targets
    from scacchi_b200.play_search import make_search
    from scacchi_b200.synthetic import SyntheticGame, SyntheticGameConfig, SyntheticState

    dev = torch.device("cuda", local)
    game = SyntheticGame(SyntheticGameConfig(seed=rank, num_actions=ACTIONS), device=dev)
    cfg = prefix_cdf_config(SEARCH_SIMS)
    search = make_search(game, game.evaluator, cfg)
    sharding = LaneSharding(world, rank)
    key = sharding.device_key(R.PRNGKey(0))
    state = game.init(SEARCH_LANES)
    torch.cuda.synchronize()

    def step(s):
        return gather_targets(search(s, key), sharding)

    for _ in range(warmup):
        step(state)
    torch.cuda.synchronize()
    if profile:
        step(state)
        torch.cuda.synchronize()
        return {}
    _barrier(world)
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for _ in range(steps):
            step(state)
        e1.record(stream)
        torch.cuda.synchronize()
    _barrier(world)
    launches = _lib.launch_count() - launches0
    ms = _max_over_ranks(e0.elapsed_time(e1) / steps, world)

    host = dict(observation=state.observation.cpu().pin_memory(),
                legal_action_mask=state.legal_action_mask.cpu().pin_memory(),
                current_player=state.current_player.cpu().pin_memory())
    G = SEARCH_LANES * world
    sink = dict(policy=torch.empty((G, ACTIONS), dtype=torch.float32).pin_memory(),
                alpha_q=torch.empty((G, ACTIONS, 2), dtype=torch.float32).pin_memory(),
                alpha_v=torch.empty((G, 2), dtype=torch.float32).pin_memory(),
                search_action=torch.empty((G,), dtype=torch.int32).pin_memory())
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = sum(t.numel() * t.element_size() for t in sink.values())

    def e2e_step():
        s = SyntheticState(**{f: t.to(dev, non_blocking=True) for f, t in host.items()},
                           rewards=torch.zeros((SEARCH_LANES, 2), device=dev),
                           terminated=torch.zeros((SEARCH_LANES,), dtype=torch.bool, device=dev))
        t = step(s)
        for f in ("policy", "alpha_q", "alpha_v"):
            sink[f].copy_(getattr(t.prediction, f), non_blocking=True)
        sink["search_action"].copy_(t.metadata.search_action, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    _barrier(world)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    _barrier(world)
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1) / steps, world)

    # one instrumented step: per-phase events and work counters
    phase_ms, sim_stats, bwd_stats = instrumented_search_step(game, state, key, cfg)
    peaks = read_peaks()
    sm_count = torch.cuda.get_device_properties(dev).multi_processor_count
    cs = clocks.summary()
    roof = search_roofline(phase_ms, sim_stats, bwd_stats, peaks, sm_count, cs["sm_mhz"] or 1965.0)
    return {
        "metric": METRIC, "value": round(world * SEARCH_LANES * SEARCH_SIMS / (ms / 1e3), 2), "unit": "sims/s",
        "ms_per_step": round(ms, 4), "steps": steps, "warmup": warmup, "dtype": "f32",
        "config": search_workload_config(world),
        "leaf_evals_per_s": round(world * SEARCH_LANES * (SEARCH_SIMS + 1) / (ms / 1e3), 2),
        "e2e": {"value": round(world * SEARCH_LANES * SEARCH_SIMS / (e2e_ms / 1e3), 2), "unit": "sims/s",
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": int(launches), "roofline": roof, "clocks": cs,
    }


# ---------------------------------------------------------------------------
# the residual tower alone (16384 boards)
# ---------------------------------------------------------------------------

def tower_bench(steps: int, warmup: int, precision: str | None = None, boards: int = TOWER_BOARDS) -> dict:
    """Residual tower alone: {0,1} planes (density 0.4), He-normal weights on
    every layer (seed 0), the library's default precision unless named.
    The whole forward, with its 12 convolutions timed inside it by the
    library (the roofline); then each convolution mode timed alone (random
    operands, the forward's launch shape) for the per-mode breakdown; stem +
    heads = the forward minus its convolutions."""
    import ctypes as C

    import torch

    from oracle.network_ref import observations  # input generator only
    from scacchi_b200 import _lib
    from scacchi_b200.dirichlet_mctx.tree import ptr
    from scacchi_b200.network import AZDirichletNet, init_params

    net = AZDirichletNet(init_params(0), precision=precision)
    obs = torch.from_numpy(observations(boards, seed=0)).cuda()
    for _ in range(warmup):
        net(obs)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the library times the 12 conv launches inside each timed forward
    _lib.check(_lib.lib().scacchi_tower_timing(steps), "tower_timing")
    e0.record(stream)
    for _ in range(steps):
        net(obs)
    e1.record(stream)
    torch.cuda.synchronize()
    conv_ms, forwards = C.c_float(0), C.c_int32(0)
    _lib.check(_lib.lib().scacchi_tower_timing_read(C.byref(conv_ms), C.byref(forwards)), "tower_timing_read")
    _lib.check(_lib.lib().scacchi_tower_timing(0), "tower_timing")
    ms = e0.elapsed_time(e1) / steps
    conv_in_forward = conv_ms.value / max(forwards.value, 1)
    rows = int(_lib.lib().scacchi_tower_rows(boards))
    dt = torch.float16 if net.fp16 else torch.bfloat16
    gen = torch.Generator(device="cuda").manual_seed(0)

    def act():
        return torch.relu(torch.randn((rows, 128), device="cuda", generator=gen)).to(dt)

    a_hi, a_lo, res16 = act(), act() * 2 ** -9, act()
    x32 = torch.randn((rows, 128), device="cuda", generator=gen)
    out0, out1 = torch.empty_like(a_hi), torch.empty_like(a_hi)
    head = torch.empty((rows, 8), dtype=torch.float32, device="cuda")
    t = net.weights.tensors
    sh = C.c_void_p(stream.cuda_stream)
    L = _lib.lib()

    def conv(mode):
        w = t["conv_w"][1]
        sc, sf = t["bn_scale"][1], t["bn_shift"][1]
        if net.terms > 1:
            return L.scacchi_conv3x3_split(ptr(a_hi), ptr(a_lo), ptr(w), ptr(t["conv_b"][1]), mode, boards,
                                           int(net.fp16), net.terms, ptr(sc), ptr(sf), ptr(x32), 0, ptr(t["head_w"]),
                                           ptr(t["head_b"]), ptr(out0), ptr(out1), ptr(head), sh)
        return L.scacchi_conv3x3(ptr(a_hi), ptr(w), ptr(t["conv_b"][1]), mode, boards, int(net.fp16), ptr(sc),
                                 ptr(sf), ptr(res16), ptr(t["head_w"]), ptr(t["head_b"]), ptr(out0), ptr(out1),
                                 ptr(head), sh)

    peaks = read_peaks()
    mode_ms = {}
    for mode, name in ((0, "conv1"), (1, "conv2"), (2, "heads_layer")):
        for _ in range(3):
            _lib.check(conv(mode), "conv3x3")
        e0.record(stream)
        for _ in range(10):
            conv(mode)
        e1.record(stream)
        torch.cuda.synchronize()
        mode_ms[name] = e0.elapsed_time(e1) / 10
    assert _lib.tower_error() == 0
    peak = peaks["bf16_tflops"] / net.terms
    # the sustained figure is the rate cuBLAS holds under the power cap; the
    # tower measured right after a long step runs in that regime
    peak_sus = peaks["bf16_tflops_sustained"] / net.terms
    alg = CONV_FLOP_PER_BOARD * boards
    per_mode = {k: {"ms": round(v, 4), "tflops": round(alg / (v / 1e3) / 1e12, 1),
                    "frac": round(alg / (v / 1e3) / 1e12 / peak, 4),
                    "frac_sustained": round(alg / (v / 1e3) / 1e12 / peak_sus, 4)} for k, v in mode_ms.items()}
    # the convolutions as timed inside the forward; the rest of the forward
    # is the stem, the head kernel and the launches between them
    per_mode["stem_and_heads"] = {"ms": round(max(ms - conv_in_forward, 0.0), 4)}
    conv_avg = conv_in_forward / 12
    return {
        "boards": boards, "precision": net.precision, "ms_per_forward": round(ms, 4),
        "evals_per_s": round(boards / (ms / 1e3), 1),
        "tflops": round(TOWER_FLOP_PER_BOARD * boards / (ms / 1e3) / 1e12, 2),
        "forward_frac": round(TOWER_FLOP_PER_BOARD * boards / (ms / 1e3) / 1e12 / peak, 4),
        "per_mode": per_mode,
        "roofline": {"bound": "tensor", "kernel": "conv_tc_kernel (12-layer average, timed inside the forward)",
                     "achieved": round(alg / (conv_avg / 1e3) / 1e12, 2), "peak": round(peak, 2), "unit": "TFLOP/s",
                     "frac": round(alg / (conv_avg / 1e3) / 1e12 / peak, 4), "avg_launch_ms": round(conv_avg, 4),
                     "frac_sustained": round(alg / (conv_avg / 1e3) / 1e12 / peak_sus, 4),
                     "peak_source": f"{peaks['source']} bf16 burst / {net.terms} (products per K step); "
                                    f"frac_sustained against the sustained figure / {net.terms}",
                     "algorithmic_flop_per_launch": alg},
    }


# ---------------------------------------------------------------------------
# CPU: the oracle's full step on a lane sample (cpu_baseline, --impl reference)
# ---------------------------------------------------------------------------

def cpu_fullstep_lanes(lo: int, hi: int, population: bool = False, threads: int = 1, rank: int = 0) -> int:
    """The full step of lanes [lo, hi) of rank ``rank``'s 8192-lane batch on
    the host: the Hex restatement for the environment, the fp32 network
    restatement (random-init weights) for every leaf, the C restatement of
    the search, the root readout and the target packing.  Returns the lanes
    searched."""
    import numpy as np
    import torch

    torch.set_num_threads(threads)
    from oracle import hex_ref as H
    from oracle import network_ref as NR
    from oracle import oracle as O
    from scacchi_b200.network import init_params

    params = init_params(0, he_all_layers=False)
    root_key = O.fold_in(O.PRNGKey(ROOT_SEED), rank)
    boards = [H.random_root(9, root_key, lane, 0, 20) for lane in range(lo, hi)]
    world_key = O.split(O.PRNGKey(SEARCH_SEED), 1)[0]

    def evaluate(obs):
        lg, lav, laq = NR.forward(params, obs.astype(np.float32))
        return lg, np.exp(lav).astype(np.float32), np.exp(laq).astype(np.float32)

    obs = np.stack([b.observation() for b in boards])
    lg, av, aq = evaluate(obs)
    legal = np.stack([b.legal() for b in boards])
    root_term = np.array([(int(b.rewards()[b.current_player()]) + 1) // 2 if b.terminated else -1 for b in boards],
                         np.int8)
    root = dict(prior_logits=lg, value=av, action_values=aq, terminal_outcome=root_term,
                to_play=np.array([b.current_player() for b in boards], np.int32),
                embedding=np.stack([b.record() for b in boards]))

    def recurrent(actions, parent_emb):
        outs = [H.step_outputs(r, a) for r, a in zip(parent_emb, actions)]
        _, v, q = evaluate(np.stack([o["observation"] for o in outs]))
        step = dict(value=v, action_values=q, invalid_actions=np.stack([o["invalid"] for o in outs]),
                    terminal_outcome=np.array([o["terminal"] for o in outs], np.int8),
                    to_play=np.array([o["to_play"] for o in outs], np.int32))
        return step, np.stack([o["record"] for o in outs])

    rule = (O.Rule(prefix_cdf=False, kappa=KAPPA, samples=POPULATION_SAMPLES) if population else
            O.Rule(prefix_cdf=True, kappa=KAPPA, samples=FALLBACK_SAMPLES))
    out = O.dirichlet_thompson_policy(np.asarray(world_key, np.uint32), root=root, recurrent_fn=recurrent,
                                      num_simulations=FULL_SIMS, invalid_actions=~legal, rule=rule,
                                      max_depth=FULL_SIMS, policy_samples=rule.samples, lane_offset=lo,
                                      total_batch=FULL_LANES)
    s = out.search_tree.summary()
    if population:
        policy = out.action_weights
    else:
        policy, _ = O.root_readout(out.action_weights, s, legal, search_evidence=True, temperature=1.0, rule=rule)
    O.pack_targets(s, policy, legal, out.action)
    return hi - lo


def cpu_baseline(population: bool, lanes: int = 16) -> dict:
    t0 = time.perf_counter()
    n = cpu_fullstep_lanes(0, lanes, population, threads=1)
    dt = time.perf_counter() - t0
    return {"value": round(n * FULL_SIMS / dt, 2), "unit": "sims/s", "cores": 1, "kind": "port",
            "sample": f"lanes 0..{lanes - 1} of the {FULL_LANES}-lane x {FULL_SIMS}-simulation workload "
                      f"({n * (FULL_SIMS + 1)} fp32 network evaluations, {dt:.1f} s), one host thread"}


def _reference_worker(args):
    lo, hi, population = args
    return cpu_fullstep_lanes(lo, hi, population, threads=1)


def run_reference(args, world: int, rank: int) -> None:
    """--impl reference: the reference's algorithm on the host cores -- the
    C restatement of the search, the fp32 network restatement and the Hex
    restatement (the JAX reference cannot be installed here) -- on every
    host core, each step a bounded lane sample of this arm's workload."""
    if rank != 0:
        return
    import multiprocessing as mp

    population = (args.workload or default_workload()) == "population"
    cores = os.cpu_count() or 1
    per_process = 2  # lanes per process and step
    chunks = [(i * per_process, (i + 1) * per_process, population) for i in range(cores)]
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        for _ in range(args.warmup):
            pool.map(_reference_worker, chunks)
        times = []
        done = 0
        for _ in range(args.steps):
            t0 = time.perf_counter()
            done = sum(pool.map(_reference_worker, chunks))
            times.append(time.perf_counter() - t0)
    dt = sum(times) / len(times)
    value = done * FULL_SIMS / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "sims/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": full_workload_config(1, population, "fp32 (CPU)"),
        "leaf_evals_per_s": round(done * (FULL_SIMS + 1) / dt, 2),
        "cpu_baseline": {"value": round(value, 2), "unit": "sims/s", "cores": cores, "kind": "port",
                         "sample": f"{done} lanes of the {FULL_LANES}-lane workload per step, {per_process} lanes per "
                                   f"process, {cores} single-threaded processes"},
        "e2e": {"value": round(value, 2), "unit": "sims/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is pure JAX (jax/flax/pgx not installable offline); timed: the C search "
                "restatement with the fp32 network and Hex restatements, all host cores",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------

def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=None, choices=["full", "population", "search", "tower"],
                    help="full: the Hex step with the tower and the prefix-CDF estimator (default on one GPU); "
                         "population: the same with the 64-sample Thompson population (default under torchrun); "
                         "search: the isolated search kernels; tower: the residual tower alone")
    ap.add_argument("--precision", default=None,
                    help="tower precision (scacchi_b200.network.PRECISIONS; default: the library default)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true", help="skip the sub-object workloads of the default line")
    ap.add_argument("--boards", type=int, default=TOWER_BOARDS,
                    help="tower --profile: boards per forward (smaller cases for ncu captures)")
    ap.add_argument("--lanes", type=int, default=FULL_LANES,
                    help="full / population --profile: lanes per GPU (smaller cases for ncu captures)")
    ap.add_argument("--profile", action="store_true",
                    help="profiling mode: warmup steps + one device-resident step, no JSON line "
                         "(for ncu captures of the bench workloads)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    workload = args.workload or default_workload()

    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if workload == "tower":
        if args.profile:
            from oracle.network_ref import observations
            from scacchi_b200.network import AZDirichletNet, init_params

            net = AZDirichletNet(init_params(0), precision=args.precision)
            obs = torch.from_numpy(observations(args.boards, seed=0)).cuda()
            for _ in range(args.warmup + 1):
                net(obs)
            torch.cuda.synchronize()
            return
        if rank == 0:
            with ClockSampler(local) as clocks:
                t = tower_bench(args.steps, args.warmup, args.precision)
            print(json.dumps({"metric": "residual tower leaf evals/s (16384 boards)", "value": t["evals_per_s"],
                              "unit": "evals/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                              "ms_per_step": t["ms_per_forward"], "higher_is_better": True, "scaling": "weak",
                              "vs_baseline": None, "dtype": t["precision"], "data": "synthetic",
                              "config": {"workload": "residual tower alone: 6x128 ResNet, 9x9x4 {0,1} planes "
                                                     "(density 0.4), He-normal weights seed 0",
                                         "boards": TOWER_BOARDS},
                              "tflops": t["tflops"], "per_mode": t["per_mode"], "roofline": t["roofline"],
                              "clocks": clocks.summary()}), flush=True)
        return
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    try:
        if workload == "search":
            r = search_kernels_bench(args.steps, args.warmup, world, rank, local, profile=args.profile)
            if rank == 0 and not args.profile:
                line = {"metric": METRIC, "value": r["value"], "unit": "sims/s", "n_gpus": world, "steps": args.steps,
                        "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
                        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                        "config": r["config"], "leaf_evals_per_s": r["leaf_evals_per_s"], "clocks": r["clocks"],
                        "e2e": r["e2e"], "gpu_launches": r["gpu_launches"], "roofline": r["roofline"]}
                print(json.dumps(line), flush=True)
            return
        population = workload == "population"
        if args.profile:
            w = full_step_bench(0, args.warmup + 1, args.precision, population, world, rank, local, e2e=False,
                                clocks=False, lanes=args.lanes)["work"]
            print(json.dumps({"profile_work": {"backward_nodes": w[0], "child_gathers": w[1], "mc_fallbacks": w[2],
                                               "descent_nodes": w[4], "steps": args.warmup + 1}}), file=sys.stderr)
            return
        f = full_step_bench(args.steps, args.warmup, args.precision, population, world, rank, local)
        peaks = read_peaks()
        lanes = FULL_LANES * world
        ms = f["ms_per_step"]
        sub = {}
        if world == 1 and not args.no_sub:
            sub["search_kernels"] = search_kernels_bench(10, 3, 1, 0, local)
            sub["tower"] = tower_bench(5, 3)
            if not population:
                p = full_step_bench(3, 2, args.precision, True, 1, 0, local, e2e=False, clocks=False)
                sub["population_step"] = {
                    "workload": full_workload_config(1, True, p["precision"])["workload"],
                    "ms_per_step": round(p["ms_per_step"], 2),
                    "sims_per_s": round(FULL_LANES * FULL_SIMS / (p["ms_per_step"] / 1e3), 1), "steps": 3}
        if rank == 0:
            phases = f["phases_ms_per_step"]
            roof = tower_roofline(f, peaks)
            roof["step_share"] = {"tower_convs": round(f["conv_ms_per_step"] / ms, 4),
                                  **{k: round(v / ms, 4) for k, v in phases.items()},
                                  "gather": round(f["gather_ms"] / ms, 4)}
            roof["backward_issue"] = backward_issue(f, population, torch.cuda.get_device_properties(dev).multi_processor_count)
            line = {
                "metric": METRIC, "value": round(lanes * FULL_SIMS / (ms / 1e3), 2), "unit": "sims/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": f["precision"],
                "data": "synthetic", "config": full_workload_config(world, population, f["precision"]),
                "leaf_evals_per_s": round(lanes * (FULL_SIMS + 1) / (ms / 1e3), 2), "clocks": f["clocks"],
                "e2e": {"value": round(lanes * FULL_SIMS / (f["e2e_ms"] / 1e3), 2), "unit": "sims/s",
                        "h2d_bytes_per_step": int(f["h2d_bytes"]), "d2h_bytes_per_step": int(f["d2h_bytes"]),
                        "ms_per_step": round(f["e2e_ms"], 3)},
                "gpu_launches": int(round(f["launches_per_step"] * args.steps)), "roofline": roof,
                "ranks": {"ms_per_step": [round(v, 3) for v in f["rank_ms"]],
                          "search_ms": [round(v, 3) for v in f["rank_search_ms"]],
                          "search_min": round(min(f["rank_search_ms"]), 3),
                          "search_median": round(statistics.median(f["rank_search_ms"]), 3),
                          "search_max": round(max(f["rank_search_ms"]), 3),
                          "gather_ms": [round(v, 4) for v in f["rank_gather_ms"]],
                          "all_gather_ms": round(f["gather_ms"], 4),
                          "note": "search_ms: each rank's search before the collective; gather_ms: its all-gather, "
                                  "which includes waiting for the slowest rank; all_gather_ms: the smallest "
                                  "(the collective itself)"},
                **sub,
            }
            if world == 1 and not args.no_cpu_baseline:
                line["cpu_baseline"] = cpu_baseline(population)
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
