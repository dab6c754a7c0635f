"""CPU tests of bench.py's reference arm, the line the driver compares the
GPU arm against: it runs on host cores only, prints one JSON line with the
GPU arm's metric, unit and workload, carries cpu_baseline and an e2e with no
host-device bytes, and under torchrun only rank 0 prints."""
import json
import os
import subprocess
import sys

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402


def _run(args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                       timeout=600, env=e, cwd=ROOT)
    assert p.returncode == 0, p.stderr[-2000:]
    return p.stdout


def test_reference_arm_line():
    out = _run(["--impl", "reference", "--steps", "1", "--warmup", "0"])
    d = json.loads(out.strip().splitlines()[-1])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.metric_of("C4") == bench.METRIC
    assert d["unit"] == "TOPS" and d["higher_is_better"] is True
    assert d["warmup"] >= 3 and d["steps"] == 1 and d["n_gpus"] == 1
    assert d["config"]["workload"] == bench.WORKLOADS["C4"]["desc"]
    assert d["value"] > 0 and d["ms_per_step"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing():
    out = _run(["--impl", "reference", "--steps", "1"], env={"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"})
    assert out.strip() == ""


def test_metrics_are_one_per_workload():
    names = sorted(bench.WORKLOADS)
    assert len({bench.metric_of(n) for n in names}) == len(names)
    assert all("TOPS" in bench.metric_of(n) for n in names)


def test_c4_is_head_sharded_strong_scaling():
    # the fixed global C4 job; its 32 (batch, kv head) units split over the ranks
    for world in (1, 2, 4, 8):
        B, H, G, sharded = bench.shard_of("C4", world)
        assert sharded and B == 4 and H * world == 32 and G * world == 8
        cfg = bench.config_of("C4", world)
        assert cfg["global_batch"] == 4 and f"hs{world}" in cfg["parallelism"]
    assert bench.shard_of("C3", 4)[3] is False and bench.config_of("C3", 4)["global_batch"] == 8


def test_reference_arm_config_matches_ours_at_two_ranks():
    out = _run(["--impl", "reference", "--steps", "1", "--warmup", "0"], env={"WORLD_SIZE": "2", "RANK": "0",
                                                                              "LOCAL_RANK": "0"})
    d = json.loads(out.strip().splitlines()[-1])
    assert d["config"] == bench.config_of("C4", 2)
    assert d["scaling"] == "strong" and d["n_gpus"] == 2
