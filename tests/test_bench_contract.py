"""bench.py's JSON-line contract, checked on CPU through the reference arm
(the CPU restatement timed on this host): one line on stdout with the keys
the driver reads, the metric string of BASELINE.json, and the algorithmic
work per launch that the roofline divides by."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "2",
                        "--warmup", "1", "--ref-budget", "1"], cwd=ROOT, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    with open(os.path.join(ROOT, "BASELINE.json")) as f:
        assert d["metric"] == json.load(f)["metric"]
    for k in ("impl", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
              "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["steps"] == 2
    assert d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["kind"] == "port"
    assert "workload" in d["config"]


def test_algorithmic_work_per_launch():
    import bench

    W = bench.WORKLOADS
    assert W["softmax"][3] == 2 * 4 * 4096 * 16384
    assert W["vadd"][3] == 3 * 4 * (1 << 28)
    assert W["gemm"][3] == 2 * 8192 ** 3
    assert W["bgemm"][3] == 32 * 2 * 2048 ** 3
    assert W["fmha"][3] == 4 * 8 * 32 * 8192 * 8192 * 128
    assert W["fmha_causal"][3] * 2 == W["fmha"][3]
    assert W["moe"][3] == 2 * 16384 * 2 * 14336 * 4096
    assert set(bench.SUITE_ORDER) == set(W)


def test_strong_scaling_shards_cover_each_job_once():
    """--scaling strong splits one BASELINE job: for 1, 2, 4 and 8 ranks the
    rank shards of every workload are disjoint, cover all its units and keep
    the alignment the kernels' fast paths want."""
    import bench
    from cutile_b200.shard import shard_range

    for name, (total, align) in bench.Case.UNITS.items():
        assert name in bench.WORKLOADS
        for world in (1, 2, 4, 8):
            got = [shard_range(total, r, world, align) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == total
            for (lo, hi), (lo2, _) in zip(got, got[1:]):
                assert hi == lo2 and lo <= hi
            assert all(lo % align == 0 for lo, _ in got)
            assert all(hi - lo > 0 for lo, hi in got), (name, world)
