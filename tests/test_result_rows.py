"""bench.py's `RESULT` rows (the bench/examples.jl:51 protocol) and the
CUTILE_BACKEND=b200 patch of the reference's bench driver."""
import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
PATCH = os.path.join(ROOT, "cutile-triton_b200", "julia", "examples_b200.patch")

# name, impl, min ms, mean ms, rate: the reference's row layout
ROW = re.compile(r"^RESULT\t(\S+)\t([^\t]+)\t([0-9.]+)\t([0-9.]+)\t([0-9.]+) (GB/s|TFLOPS)$")


def test_rows_follow_examples_jl_format_and_rate():
    import bench

    for name in bench.SUITE_ORDER:
        _, unit, _, work = bench.WORKLOADS[name]
        row = bench.result_row(name, 0.123456, 0.2)
        m = ROW.match(row)
        assert m, row
        ex, impl = bench.RESULT_NAMES[name]
        assert m.group(1) == ex and m.group(2) == impl and impl.startswith("b200")
        assert float(m.group(3)) == round(0.123456, 4) and float(m.group(4)) == 0.2
        # rate from the MIN time: integer GB/s, TFLOPS to one decimal (examples.jl:45-48)
        if unit == "GB/s":
            assert m.group(6) == "GB/s" and m.group(5) == str(round(work / 0.123456e-3 / 1e9))
        else:
            assert m.group(6) == "TFLOPS"
            assert float(m.group(5)) == round(work / 0.123456e-3 / 1e12, 1)


def test_rows_use_the_shard_work_when_given():
    import bench

    row = bench.result_row("softmax", 0.05, 0.06, work=2 * 4 * 512 * 16384)
    assert row.endswith(f"{round(2 * 4 * 512 * 16384 / 0.05e-3 / 1e9)} GB/s")


def test_examples_patch_is_a_unified_diff_adding_the_b200_backend():
    text = open(PATCH).read()
    assert text.startswith("--- a/bench/examples.jl\n+++ b/bench/examples.jl\n")
    added = [l[1:] for l in text.splitlines() if l.startswith("+") and not l.startswith("+++")]
    assert any('BACKEND == "b200"' in l for l in added)
    assert any("use_b200!()" in l for l in added)
    assert any("install_shim!()" in l for l in added)


def _reference_root():
    for cand in (os.environ.get("CTB_REFERENCE_ROOT"), os.path.join(os.path.dirname(ROOT),
                                                                    "reference")):
        if cand and os.path.isfile(os.path.join(cand, "bench", "examples.jl")):
            return cand
    return None


@pytest.mark.skipif(_reference_root() is None, reason="reference tree not present")
def test_examples_patch_applies_to_the_reference_driver(tmp_path):
    ref = _reference_root()
    (tmp_path / "bench").mkdir()
    (tmp_path / "bench" / "examples.jl").write_text(
        open(os.path.join(ref, "bench", "examples.jl")).read())
    r = subprocess.run(["patch", "-p1", "--dry-run", "-i", PATCH], cwd=tmp_path,
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
