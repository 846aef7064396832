"""The bench's reference arm (the reference's own CPU path for the same
workload) runs without a GPU and prints the JSON line the driver parses."""
import json
import subprocess
import sys
from pathlib import Path


def test_reference_arm_prints_one_json_line():
    root = Path(__file__).resolve().parents[1]
    r = subprocess.run([sys.executable, str(root / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1"],
                       capture_output=True, text=True, timeout=600, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip().startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    if "unavailable" in d:
        return
    assert d["metric"] == "MoE-layer tokens/sec" and d["value"] > 0 and d["higher_is_better"]
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_weight_copies_keep_reuse_distance_past_l2():
    """Between two uses of one layer copy's weights the steps read at least
    twice the L2: one copy at the headline workload, several where a step
    touches little (config 0, one expert on a rank)."""
    import importlib.util
    root = Path(__file__).resolve().parents[1]
    spec = importlib.util.spec_from_file_location("bench_mod", root / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    bench.load_pkg()
    import moe_b200.synth as synth
    c0, c1 = synth.CONFIGS[0], synth.CONFIGS[1]
    assert bench.weight_copies(32 * bench.expert_bytes(c1)) == 1       # 423 MB routed per step
    assert bench.weight_copies(8 * bench.expert_bytes(c0)) == 7        # config 0: 37 MB
    assert bench.weight_copies(bench.expert_bytes(c1)) == bench.MAX_COPIES
    for touched in (1e6, 3e7, 1.3e8, 2.6e8, 5e8):
        n = bench.weight_copies(touched)
        assert 1 <= n <= bench.MAX_COPIES
        assert n * touched >= 2 * bench.L2_BYTES or n == bench.MAX_COPIES


def test_replica_placement_invariants():
    """The bench's expert placement for multi-GPU runs: every expert on 1 to
    world distinct ranks, hot experts split by their load, every rank used
    when there are enough replicas, and no rank above the mean load by more
    than one replica's share (greedy largest-first placement)."""
    import importlib.util
    import numpy as np
    root = Path(__file__).resolve().parents[1]
    spec = importlib.util.spec_from_file_location("bench_mod2", root / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    rng = np.random.default_rng(3)
    for trial in range(60):
        E = int(rng.choice([8, 32, 128, 256]))
        world = int(rng.choice([1, 2, 4, 8]))
        if trial % 2:
            counts = (1.0 / np.arange(1, E + 1) ** 1.1) * 4096  # Zipf(1.1) loads
            rng.shuffle(counts)
        else:
            counts = rng.integers(0, 200, E).astype(np.float64)
        placement, imbalance = bench.place_replicas(counts, world)
        assert len(placement) == E
        share = counts.sum() / world
        load = np.zeros(world)
        for e, ranks in enumerate(placement):
            assert 1 <= len(ranks) <= world and len(set(ranks)) == len(ranks)
            assert all(0 <= q < world for q in ranks)
            assert len(ranks) == min(world, max(1, int(np.ceil(counts[e] / max(share, 1.0)))))
            for q in ranks:
                load[q] += counts[e] / len(ranks)
        if sum(len(r) for r in placement) >= world and counts.sum() > 0:
            assert all(any(q in r for r in placement) for q in range(world))
        biggest = max(counts[e] / len(r) for e, r in enumerate(placement))
        assert load.max() <= load.mean() + biggest + 1e-9
        assert abs(imbalance - load.max() / max(load.mean(), 1e-9)) < 1e-9


def test_tensor_roofline_arithmetic():
    """The headline roofline: gate/up algorithmic FLOPs (4 H I per permuted
    row, P = T (k + shared)) over the launch time, against the 9 PF MXFP4
    peak; the issued view doubles the FLOPs (hi + lo terms) against the
    4.5 PF FP8 rate, or keeps them against 9 PF in the fast mode; the
    reference arm's config dict equals the GPU arm's."""
    import importlib.util
    import argparse
    root = Path(__file__).resolve().parents[1]
    spec = importlib.util.spec_from_file_location("bench_mod3", root / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    bench.load_pkg()
    import moe_b200.synth as synth
    c4 = synth.CONFIGS[4]
    T = 16384
    r = bench.tensor_roofline(c4, T, 8.0, 4.0, None)
    flops = T * 9 * 4.0 * 7168 * 2048
    assert abs(r["algorithmic_flops_per_launch"] - flops) < 1
    assert abs(r["achieved"] - flops / 8e-3 / 1e12) < 1e-6
    assert r["peak"] == 9000.0 and abs(r["frac"] - r["achieved"] / 9000.0) < 1e-12
    assert abs(r["issued"]["frac"] - 2 * r["achieved"] / 4500.0) < 1e-12 and r["bound"] == "tensor"
    f = bench.tensor_roofline(c4, T, 8.0, 4.0, None, fp4=True)
    assert abs(f["issued"]["frac"] - f["achieved"] / 9000.0) < 1e-12
    args = argparse.Namespace(config=4, tokens=T, gpus=1)
    assert bench.config_dict(c4, args) == bench.config_dict(c4, args)
    assert "weight_copies_cycled" not in bench.config_dict(c4, args)
