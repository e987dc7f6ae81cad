"""bench.py's bookkeeping on the CPU: stamped ncu figures go stale when
their kernel sources change, and the roofline arithmetic of the full-step
line."""

import bench


def test_stamped_figures_report_staleness(monkeypatch):
    name = "conv_traffic_bytes_8192"
    entry = dict(bench.CAPTURED[name])
    now = bench.source_hash(entry["sources"])
    monkeypatch.setitem(bench.CAPTURED, name, dict(entry, value=123, sha=now))
    value, prov = bench.captured(name)
    assert value == 123 and not prov["stale"]
    monkeypatch.setitem(bench.CAPTURED, name, dict(entry, value=123, sha="0" * 16))
    value, prov = bench.captured(name)
    assert value is None and prov["stale"]


def test_tower_roofline_arithmetic():
    peaks = {"hbm_gbs": 6000.0, "bf16_tflops": 1700.0, "bf16_tflops_sustained": 1400.0, "source": "test"}
    f = {"conv_launch_ms": 0.5, "terms": 3, "precision": "bf16x3", "forwards": 10}
    r = bench.tower_roofline(f, peaks)
    alg = bench.CONV_FLOP_PER_BOARD * bench.FULL_LANES
    assert r["algorithmic_flop_per_launch"] == alg
    assert abs(r["achieved"] - alg / 0.5e-3 / 1e12) < 0.01
    assert abs(r["peak"] - 1400.0 / 3) < 0.01
    assert abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-3
    assert r["launches_timed"] == 120


def test_backward_issue_arithmetic(monkeypatch):
    name = "backward_inst_per_node_prefix"
    entry = dict(bench.CAPTURED[name])
    monkeypatch.setitem(bench.CAPTURED, name, dict(entry, value=30000, sha=bench.source_hash(entry["sources"])))
    f = {"phases_ms_per_step": {"backward": 100.0}, "work_per_step": [20000.0, 0, 5.0, 0, 0, 0],
         "clocks": {"sm_mhz": 1800.0}}
    r = bench.backward_issue(f, False, 148)
    assert abs(r["achieved"] - 30000 * 20000 / 0.1 / 1e9) < 0.1
    assert abs(r["peak"] - 148 * 4 * 1800 / 1e3) < 0.1
    assert r["node_updates_per_step"] == 20000 and r["mc_fallbacks_per_step"] == 5


def test_default_workload_follows_the_launcher(monkeypatch):
    """A plain process times the metric's one-GPU workload (the full step);
    any torchrun launch, one rank included, times the population step, so a
    scaling series measures one workload at every N."""
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    assert bench.default_workload() == "full"
    for world in ("1", "2", "8"):
        monkeypatch.setenv("WORLD_SIZE", world)
        assert bench.default_workload() == "population"


def test_stamped_figures_match_the_current_sources():
    """Every stamped ncu figure was captured on the kernel sources as they
    are now (a kernel change without a new capture shows up here)."""
    for name in bench.CAPTURED:
        value, prov = bench.captured(name)
        assert value is not None and not prov["stale"], (name, prov)
