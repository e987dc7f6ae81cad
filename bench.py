"""Benchmark: batched Dirichlet-Thompson search step on B200.

Workload (isolated search kernels): Hex 9x9 action space (82 actions), 4096
lanes per GPU, 128 simulations, tree capacity 129, synthetic network outputs
(scacchi_b200/synthetic.py), guarded prefix-CDF estimator (kappa 1, Q21,
Monte Carlo fallback with 8 samples), root policy with 8 samples and the
search-evidence Q21 root readout.  One step = one ``search(root_state, key)``
call through the public boundary (root evaluation, 128 simulations, root
policy, readout, target packing).

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
Under torchrun (N > 1) every rank searches its own 4096 lanes (weak scaling)
and the root targets are all-gathered over NCCL at the end of the step.
Prints one JSON line on rank 0.
"""

from __future__ import annotations

import argparse
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
LANES = 4096
SIMS = 128
ACTIONS = 82
FALLBACK_SAMPLES = 8
ROOT_SAMPLES = 8
KAPPA = 1.0
FALLBACK_HBM_GBS = 6650.0


def workload_config(world: int) -> dict:
    return {
        "workload": "isolated search kernels: Hex 9x9 (82 actions), synthetic network outputs",
        "lanes_per_gpu": LANES, "global_lanes": LANES * world, "num_simulations": SIMS,
        "tree_capacity": SIMS + 1, "num_actions": ACTIONS, "estimator": "prefix_cdf Q21 + MC fallback",
        "kappa": KAPPA, "fallback_policy_samples": FALLBACK_SAMPLES, "root_policy_samples": ROOT_SAMPLES,
        "degenerate_lanes": "1% (alpha=1e-3)", "legal_prob": 0.7, "logc": "clip(N(0.5,1),-4,6)",
        "l2": "inputs larger than L2: the tree is 0.9 GB per GPU, rewritten every step",
        "parallelism": f"dp{world} (lane-sharded)",
    }


def read_peaks() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


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


def search_config(sims: int = SIMS):
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


def instrumented_step(game, state, key, cfg):
    """One extra (untimed) step driven phase by phase from Python, with CUDA
    events on the launching stream around every kernel and the kernels' own
    work counters, for the per-kernel roofline."""
    import torch

    from scacchi_b200 import random as R
    from scacchi_b200.dirichlet_mctx import search as S
    from scacchi_b200.dirichlet_mctx.tree import _init_tree
    from scacchi_b200.play_search import _make_posterior_update
    from scacchi_b200.dirichlet_mctx.posterior_updates import rule_params

    dev = state.observation.device
    pred = game.evaluator(state.observation)
    from scacchi_b200.dirichlet_mctx import RootFnOutput

    root = RootFnOutput(prior_logits=pred.logits, value=pred.alpha_v, action_values=pred.alpha_q,
                        embedding=state.observation,
                        terminal_outcome=torch.full((LANES,), -1, dtype=torch.int8, device=dev),
                        to_play=state.current_player)
    rparams = rule_params(_make_posterior_update(cfg.posterior_update.active()))
    search_key = R.split(key)[0]
    tree = _init_tree(root, SIMS, ~state.legal_action_mask, full=False)
    sched = torch.from_numpy(R.key_schedule(search_key, SIMS).view("int32")).to(dev)
    bufs = S.SimulationBuffers(LANES, ACTIONS, tree.E, dev)
    sim_stats = torch.zeros(2, dtype=torch.int64, device=dev)
    bwd_stats = torch.zeros(3, dtype=torch.int64, device=dev)
    names = ("simulate", "recurrent", "expand", "backward")
    ev = {n: [] for n in names}
    stream = torch.cuda.current_stream()
    for i in range(SIMS):
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        marks[0].record(stream)
        S.simulate(tree, sched[i, 1], SIMS, bufs, sim_stats)
        marks[1].record(stream)
        step, child = game((), None, bufs.action, bufs.parent_embedding[:, :tree.E])
        marks[2].record(stream)
        v, tp = S.expand(tree, i + 1, bufs, step, child)
        marks[3].record(stream)
        S.backward(tree, sched[i, 3], bufs, v, tp, rparams, bwd_stats)
        marks[4].record(stream)
        for j, n in enumerate(names):
            ev[n].append((marks[j], marks[j + 1]))
    torch.cuda.synchronize()
    ms = {n: sum(a.elapsed_time(b) for a, b in ev[n]) for n in names}
    return ms, sim_stats.cpu().tolist(), bwd_stats.cpu().tolist()


# DRAM bytes (read + write) of one launch from ncu captures of this workload
# (`--metrics`/`--set full`, dram__bytes_read.sum + dram__bytes_write.sum):
# backward launch 65 of the warm-up step, and a conv1-mode tower convolution
# of the 16384-board forward.
BACKWARD_TRAFFIC_BYTES = 23654656 + 3840
# smsp__inst_executed.sum over the 128 backward launches of one step of this
# workload (ncu launch list, profiles/backward_cta_search4096x128.md)
BACKWARD_WARP_INST_PER_STEP = 25875513797
CONV_TRAFFIC_BYTES = 420069888 + 370689536


def roofline(ms: dict, sim_stats, bwd_stats, peak: float, peak_kind: str, sm_count: int, sm_mhz: float) -> dict:
    A = ACTIONS
    row = A * (4 + 4 + 8 + 1 + 1)  # children, payload, alpha, outcome, invalid
    bwd_bytes = bwd_stats[0] * (row + 24 + A * 12 + 12) + bwd_stats[1] * 25
    sim_bytes = sim_stats[0] * (row + 5) + sim_stats[1] * 12
    total = sum(ms.values())
    dominant = max(ms, key=ms.get)
    per = {"backward": bwd_bytes, "simulate": sim_bytes}
    bytes_per_launch = per.get(dominant, 0) / SIMS
    avg_s = ms[dominant] / SIMS / 1e3
    achieved = bytes_per_launch / avg_s / 1e9 if avg_s > 0 else 0.0
    # the resource the backward kernel is actually bound by: instruction
    # issue (one warp instruction per scheduler per cycle, 4 per SM)
    issue_peak = sm_count * 4 * sm_mhz / 1e3
    issue = BACKWARD_WARP_INST_PER_STEP / (ms["backward"] / 1e3) / 1e9 if ms.get("backward") else 0.0
    return {
        "bound": "hbm", "kernel": f"{dominant}_kernel", "achieved": round(achieved, 2), "peak": peak,
        "unit": "GB/s", "frac": round(achieved / peak, 5),
        "traffic": BACKWARD_TRAFFIC_BYTES if dominant == "backward" else None,
        "traffic_source": "ncu capture of one backward launch (simulation 64)", "peak_source": peak_kind,
        "algorithmic_bytes_per_launch": int(bytes_per_launch), "avg_launch_ms": round(ms[dominant] / SIMS, 5),
        "kernel_share": {k: round(v / total, 4) for k, v in ms.items()},
        "work": {"descent_nodes": sim_stats[0], "descent_prior_gathers": sim_stats[1],
                 "backward_nodes": bwd_stats[0], "backward_child_gathers": bwd_stats[1],
                 "mc_fallback_nodes": bwd_stats[2]},
        "issue": {"bound": "issue", "kernel": "backward_kernel", "achieved": round(issue, 1), "peak": round(issue_peak, 1),
                  "unit": "G warp-inst/s", "frac": round(issue / issue_peak, 4) if issue_peak else None,
                  "inst_source": "ncu smsp__inst_executed.sum, backward launches of one step",
                  "peak_source": "4 schedulers x SMs x sampled SM clock"},
        "note": "search kernels are ALU-bound (in-kernel threefry, Q21 transcendentals); the HBM fraction is "
                "algorithmic bytes over measured copy bandwidth, the issue fraction is warp instructions "
                "over the schedulers' issue rate",
    }


TOWER_BOARDS = 16384
CONV_FLOP_PER_BOARD = 2 * 81 * 128 * 128 * 9          # one 3x3 128->128 conv
TOWER_FLOP_PER_BOARD = 12 * CONV_FLOP_PER_BOARD + 2 * 81 * 4 * 128 * 9 + 2 * (
    81 * 128 * 6 + 162 * 82 + 81 * 128 + 128 * 3 + 162 * 128 + 128 * 164 + 81 * 128 + 128 * 82)


def read_tensor_peak() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def tower_bench(steps: int, warmup: int, precision: str | None = None) -> dict:
    """Residual tower alone: 16384 boards of {0,1} planes (density 0.4),
    He-normal weights on every layer (seed 0), 16-bit operands with fp32
    accumulation.  Inputs (12.7 MB of planes) are resident; the activations
    the tower streams (3 x 420 MB) exceed L2."""
    import torch

    from oracle.network_ref import observations  # input generator only
    from scacchi_b200.network import AZDirichletNet, init_params

    net = AZDirichletNet(init_params(0), precision=precision)
    fp16 = net.fp16
    obs = torch.from_numpy(observations(TOWER_BOARDS, seed=0)).cuda()
    for _ in range(warmup):
        net(obs)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        net(obs)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    # the conv kernel alone (one launch of the 12), timed on its stream
    import ctypes as C
    from scacchi_b200 import _lib
    from scacchi_b200.dirichlet_mctx.tree import ptr

    rows = int(_lib.lib().scacchi_tower_rows(TOWER_BOARDS))
    act = torch.zeros((rows, 128), dtype=torch.float16 if fp16 else torch.bfloat16, device="cuda")
    out = torch.empty_like(act)
    w = net.weights.tensors["conv_w"][0]
    b = net.weights.tensors["conv_b"][0]
    sh = C.c_void_p(stream.cuda_stream)
    call = lambda: _lib.lib().scacchi_conv3x3(ptr(act), ptr(w), ptr(b), 0, TOWER_BOARDS, int(fp16), None, None, None,
                                              None, None, ptr(out), None, None, sh)
    for _ in range(3):
        call()
    e0.record(stream)
    for _ in range(10):
        call()
    e1.record(stream)
    torch.cuda.synchronize()
    conv_ms = e0.elapsed_time(e1) / 10
    peak, kind = read_tensor_peak()
    conv_tflops = CONV_FLOP_PER_BOARD * TOWER_BOARDS / (conv_ms / 1e3) / 1e12
    return {
        "boards": TOWER_BOARDS, "dtype": net.precision, "ms_per_forward": round(ms, 4),
        "evals_per_s": round(TOWER_BOARDS / (ms / 1e3), 1),
        "tflops": round(TOWER_FLOP_PER_BOARD * TOWER_BOARDS / (ms / 1e3) / 1e12, 2),
        "roofline": {"bound": "tensor", "kernel": "conv_tc_kernel", "achieved": round(conv_tflops, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(conv_tflops / peak, 4), "traffic": CONV_TRAFFIC_BYTES,
                     "traffic_source": "ncu capture of one conv1-mode launch, 16384 boards", "peak_source": kind,
                     "avg_launch_ms": round(conv_ms, 4),
                     "algorithmic_flop_per_launch": CONV_FLOP_PER_BOARD * TOWER_BOARDS,
                     "note": "algorithmic FLOPs count the 81 board cells; the kernel also multiplies the 19 "
                             "padding rows of each 100-row board (x1.23)"},
    }


FULL_LANES = 8192
FULL_SIMS = 256


POPULATION_SAMPLES = 64


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


def full_step_bench(steps: int, warmup: int, precision: str | None = None, population: bool = False, world: int = 1,
                    rank: int = 0) -> dict:
    """The full self-play search step: Hex 9x9, 8192 lanes per GPU, 256
    simulations (tree capacity 257), the 6x128 AZDirichletNet with the
    reference's random init (zero-initialised heads) evaluating every leaf
    on the tcgen05 tower, exact terminal certificates, roots after 0-20
    uniform random legal moves.  The posterior estimator is the guarded
    prefix-CDF (kappa 1, Monte Carlo fallback with 8 samples), or with
    `population` the Thompson population of 64 samples per node.  One step =
    one make_search(...)(roots, key) call per rank: root evaluation, 256 x
    (descent, Hex step, tower, expand, backward), root readout and target
    packing, then the all-gather of the root targets over NCCL when there
    are several ranks (lanes shard by rank with per-rank keys)."""
    import torch
    import torch.distributed as dist

    from scacchi_b200 import random as R
    from scacchi_b200.distributed import LaneSharding, gather_targets
    from scacchi_b200.hex import HexGame
    from scacchi_b200.network import AZDirichletNet, init_params
    from scacchi_b200.play_search import make_evaluator, make_search

    sharding = LaneSharding(world, rank)
    game = HexGame(9)
    net = AZDirichletNet(init_params(0, he_all_layers=False), precision=precision)
    evaluator = make_evaluator(net)
    tower_ms = []
    stream = torch.cuda.current_stream()

    def timed_evaluator(obs):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        out = evaluator(obs)
        b.record(stream)
        tower_ms.append((a, b))
        return out

    cfg = population_config(FULL_SIMS) if population else search_config(FULL_SIMS)
    search = make_search(game, timed_evaluator, cfg)
    # every rank samples its own roots (fold the rank into the root key)
    state = game.random_roots(FULL_LANES, R.fold_in(R.PRNGKey(0), rank), 0, 20)
    key = sharding.device_key(R.PRNGKey(1))

    def step():
        return gather_targets(search(state, key), sharding)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    tower_ms.clear()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    t_tower = sum(a.elapsed_time(b) for a, b in tower_ms) / steps
    lanes = FULL_LANES * world
    estimator = (f"Thompson population, {POPULATION_SAMPLES} samples, kappa 1" if population else
                 "prefix_cdf kappa 1 (Monte Carlo fallback 8 samples)")
    return {
        "workload": f"full search step: Hex 9x9, {FULL_LANES} lanes/GPU x {FULL_SIMS} simulations, AZDirichletNet "
                    f"6x128 (reference random init) on the tcgen05 tower, {estimator}, roots 0-20 random moves",
        "lanes": lanes, "lanes_per_gpu": FULL_LANES, "num_simulations": FULL_SIMS,
        "dtype": net.precision, "n_gpus": world,
        "ms_per_step": round(ms, 2), "sims_per_s": round(lanes * FULL_SIMS / (ms / 1e3), 1),
        "leaf_evals_per_s": round(lanes * (FULL_SIMS + 1) / (ms / 1e3), 1),
        "tower_share": round(t_tower / ms, 4),
        "tower_tflops": round(TOWER_FLOP_PER_BOARD * FULL_LANES * (FULL_SIMS + 1) / (t_tower / 1e3) / 1e12, 2),
        "steps": steps, "warmup": warmup,
    }


def cpu_baseline(lanes: int = 384) -> dict:
    """The C oracle (a restatement of the reference's JAX path, which cannot
    be installed here) on a bounded sample: lanes [0, lanes) of the same
    4096-lane workload, one host thread."""
    from oracle import oracle as O

    env = O.synth_params(seed=0)
    rule = O.Rule(prefix_cdf=True, kappa=KAPPA, samples=FALLBACK_SAMPLES)
    t0 = time.perf_counter()
    O.search_synthetic(env, LANES, O.PRNGKey(0), SIMS, rule, max_depth=SIMS, policy_samples=ROOT_SAMPLES,
                       lanes=(0, lanes))
    dt = time.perf_counter() - t0
    return {"value": round(lanes * SIMS / dt, 2), "unit": "sims/s", "cores": 1, "kind": "port",
            "sample": f"lanes 0..{lanes - 1} of the {LANES}-lane x {SIMS}-simulation workload ({dt:.1f} s)"}


def _oracle_lane_range(args):
    lo, hi = args
    from oracle import oracle as O

    env = O.synth_params(seed=0)
    rule = O.Rule(prefix_cdf=True, kappa=KAPPA, samples=FALLBACK_SAMPLES)
    O.search_synthetic(env, LANES, O.PRNGKey(0), SIMS, rule, max_depth=SIMS, policy_samples=ROOT_SAMPLES,
                       lanes=(lo, hi))
    return hi - lo


def run_reference(args, world: int, rank: int) -> None:
    """--impl reference: the reference's algorithm on the host cores (the C
    oracle restatement; the JAX reference cannot be installed here), all
    host threads, each step a bounded lane sample of the same workload."""
    if rank != 0:
        return
    import multiprocessing as mp

    cores = os.cpu_count() or 1
    lanes_per_worker = 2
    chunks = [(i * lanes_per_worker, (i + 1) * lanes_per_worker) for i in range(cores)]
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        for _ in range(args.warmup):
            pool.map(_oracle_lane_range, chunks[:1])
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            done = sum(pool.map(_oracle_lane_range, chunks))
            times.append(time.perf_counter() - t0)
    dt = sum(times) / len(times)
    value = done * SIMS / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "sims/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": workload_config(1),
        "cpu_baseline": {"value": round(value, 2), "unit": "sims/s", "cores": cores, "kind": "port",
                         "sample": f"{done} lanes of the {LANES}-lane workload per step, {cores} processes"},
        "e2e": {"value": round(value, 2), "unit": "sims/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference is pure JAX (jax/flax/pgx not installable offline); timed: the C oracle restatement",
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="search", choices=["search", "tower", "full", "population"],
                    help="search: the isolated search kernels (default); tower: the residual tower alone; "
                         "full: the full Hex search step with the tower evaluating leaves (1 GPU); "
                         "population: the full step with the 64-sample Thompson-population estimator, "
                         "lane-sharded over the ranks")
    ap.add_argument("--precision", default=None,
                    help="tower precision (scacchi_b200.network.PRECISIONS; default: the library default)")
    ap.add_argument("--boards", type=int, default=TOWER_BOARDS,
                    help="tower --profile: boards per forward (smaller cases for ncu captures)")
    ap.add_argument("--profile", action="store_true",
                    help="profiling mode: warmup steps + one device-resident step, no JSON line "
                         "(for ncu captures of the bench workload)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, world, rank)
        return

    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.workload == "tower":
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
            t = tower_bench(args.steps, args.warmup, args.precision)
            print(json.dumps({"metric": "residual tower leaf evals/s (16384 boards)", "value": t["evals_per_s"],
                              "unit": "evals/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                              "ms_per_step": t["ms_per_forward"], "higher_is_better": True, "scaling": "weak",
                              "vs_baseline": None, "dtype": t["dtype"], "data": "synthetic",
                              "config": {"workload": "residual tower alone: 6x128 ResNet, 9x9x4 {0,1} planes "
                                                     "(density 0.4), He-normal weights seed 0", "boards": TOWER_BOARDS},
                              "tflops": t["tflops"], "roofline": t["roofline"]}), flush=True)
        return
    if args.workload in ("full", "population"):
        population = args.workload == "population"
        if world > 1 and not population:
            if rank == 0:
                print("--workload full runs on one GPU; use --workload population for several", file=sys.stderr)
            return
        if world > 1:
            dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        with ClockSampler(local) as clocks:
            f = full_step_bench(args.steps, args.warmup, args.precision, population, world, rank)
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": f["sims_per_s"], "unit": "sims/s", "n_gpus": world,
                              "steps": args.steps, "warmup": args.warmup, "ms_per_step": f["ms_per_step"],
                              "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                              "dtype": f["dtype"], "data": "synthetic",
                              "config": {"workload": f["workload"], "lanes": f["lanes"],
                                         "lanes_per_gpu": FULL_LANES, "num_simulations": FULL_SIMS,
                                         "parallelism": f"dp{world} (lane-sharded)"},
                              "leaf_evals_per_s": f["leaf_evals_per_s"], "tower_share": f["tower_share"],
                              "tower_tflops": f["tower_tflops"], "clocks": clocks.summary()}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))

    from scacchi_b200 import _lib
    from scacchi_b200 import random as R
    from scacchi_b200.distributed import LaneSharding, gather_targets
    from scacchi_b200.play_search import make_search
    from scacchi_b200.synthetic import SyntheticGame, SyntheticGameConfig

    game = SyntheticGame(SyntheticGameConfig(seed=rank, num_actions=ACTIONS), device=dev)
    cfg = search_config()
    search = make_search(game, game.evaluator, cfg)
    sharding = LaneSharding(world, rank)
    key = sharding.device_key(R.PRNGKey(0))
    state = game.init(LANES)
    torch.cuda.synchronize()

    def gather(targets):
        # the step's only collective: root targets of every rank, lane order
        return gather_targets(targets, sharding)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timing -------------------------------------------
    for _ in range(args.warmup):
        gather(search(state, key))
    torch.cuda.synchronize()
    if args.profile:
        gather(search(state, key))
        torch.cuda.synchronize()
        if world > 1:
            dist.destroy_process_group()
        return
    barrier()
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    stream = torch.cuda.current_stream()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            gather(search(state, key))
        stop.record(stream)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches = _lib.launch_count() - launches0
    ms_step = max_over_ranks(start.elapsed_time(stop) / args.steps)
    value = world * LANES * SIMS / (ms_step / 1e3)
    evals = world * LANES * (SIMS + 1) / (ms_step / 1e3)

    # ---- end to end: host buffers through the public call ------------------
    host_obs = state.observation.cpu().pin_memory()
    host_legal = state.legal_action_mask.cpu().pin_memory()
    host_player = state.current_player.cpu().pin_memory()
    out_policy = torch.empty((LANES, ACTIONS), dtype=torch.float32).pin_memory()
    out_alpha_q = torch.empty((LANES, ACTIONS, 2), dtype=torch.float32).pin_memory()
    out_alpha_v = torch.empty((LANES, 2), dtype=torch.float32).pin_memory()
    out_action = torch.empty((LANES,), dtype=torch.int32).pin_memory()
    h2d = host_obs.numel() + host_legal.numel() + host_player.numel() * 4
    d2h = (out_policy.numel() + out_alpha_q.numel() + out_alpha_v.numel() + out_action.numel()) * 4

    def e2e_step():
        from scacchi_b200.synthetic import SyntheticState

        s = SyntheticState(observation=host_obs.to(dev, non_blocking=True),
                           legal_action_mask=host_legal.to(dev, non_blocking=True),
                           current_player=host_player.to(dev, non_blocking=True),
                           rewards=torch.zeros((LANES, 2), device=dev),
                           terminated=torch.zeros((LANES,), dtype=torch.bool, device=dev))
        t = search(s, key)
        gather(t)
        out_policy.copy_(t.prediction.policy, non_blocking=True)
        out_alpha_q.copy_(t.prediction.alpha_q, non_blocking=True)
        out_alpha_v.copy_(t.prediction.alpha_v, non_blocking=True)
        out_action.copy_(t.metadata.search_action, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    e2e_value = world * LANES * SIMS / (e2e_ms / 1e3)

    # ---- per-kernel roofline (one instrumented, untimed step) --------------
    peak, peak_kind = read_peaks()
    ms, sim_stats, bwd_stats = instrumented_step(game, state, key, cfg)
    sm_count = torch.cuda.get_device_properties(dev).multi_processor_count
    clock_summary = clocks.summary()
    roof = roofline(ms, sim_stats, bwd_stats, peak, peak_kind, sm_count, clock_summary["sm_mhz"] or 1965.0)
    barrier()

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "sims/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": workload_config(world),
            "leaf_evals_per_s": round(evals, 2), "clocks": clock_summary,
            "e2e": {"value": round(e2e_value, 2), "unit": "sims/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "ms_per_step": round(e2e_ms, 4)},
            "gpu_launches": int(launches), "roofline": roof,
        }
        if world == 1:
            line["tower"] = tower_bench(5, 3)
            line["full_step"] = full_step_bench(3, 3)
            line["population_step"] = full_step_bench(3, 3, population=True)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
