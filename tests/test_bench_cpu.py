"""The benchmark's CPU-side contract: the reference arm (`bench.py --impl reference`, timed
beside ours) prints one JSON line with the fields it promises, and the helpers the GPU arm
uses (workload shapes, sharding, the recorded traffic figure) behave. Nothing here needs a
GPU."""
import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                         timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_arm_prints_the_contract_line():
    rec = _run("--impl", "reference", "--steps", "1", "--warmup", "0", "--cpu-sample-lines", "4")
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in rec, key
    assert rec["impl"] == "reference" and rec["unit"] == "timesteps/s" and rec["value"] > 0
    assert rec["e2e"]["h2d_bytes_per_step"] == 0 and rec["e2e"]["d2h_bytes_per_step"] == 0
    assert rec["cpu_baseline"]["kind"] == "port" and rec["cpu_baseline"]["cores"] >= 1
    assert "workload" in rec["config"]


def test_reference_arm_for_the_fp32_head():
    """The FP32 head's CPU arm times matmul_transposed_b's blocked kernel restated."""
    rec = _run("--impl", "reference", "--weights", "f32", "--steps", "1", "--warmup", "0",
               "--cpu-sample-lines", "4")
    assert rec["impl"] == "reference" and rec["value"] > 0 and rec["metric"].startswith("FP32")
    assert rec["cpu_baseline"]["kind"] == "port"


def test_bench_helpers():
    sys.path.insert(0, ROOT)
    import bench

    off, rows, global_rows, desc, scaling = bench.workload_for("cfg2", 4, 1)
    assert rows == 122880 and global_rows == 4 * 122880 and scaling == "weak"
    off, rows, global_rows, desc, scaling = bench.workload_for("cfg3", 2, 0)
    assert scaling == "strong" and 0 < rows < global_rows and off[0] == 0 and off[-1] == rows
    assert bench.head_dims("tiny") == (80, 6906) and bench.head_dims("cfg2") == (120, 18710)
    w, b = bench.head_weights("tiny")
    assert w.shape == (6906, 80) and b.shape == (6906,)
    t, src = bench.profiled_traffic("cfg2", "int8")
    # DRAM bytes of one cfg2 launch, recorded for the current kernel sources (else None + why)
    assert (t is None and src) or t > 60_000_000
    assert len(bench.kernel_source_sha16()) == 16
    assert bench.profiled_traffic("nonexistent", "int8")[0] is None
    # preprocessing: DRAM bytes of one step's two launches, recorded for the current sources
    t, src = bench.recpre_traffic()
    assert (t is None and src) or t > 600_000_000
    assert len(bench.source_sha16(bench.RECPRE_SOURCES)) == 16
    assert np.all(np.diff(off) >= 0)


def test_gather_shards_on_one_rank_unpacks_in_place():
    """With one rank (no process group) the strong-scaling record's gather only unpacks its own
    pack: idx from the front, probabilities from the bits after the padding."""
    import torch

    sys.path.insert(0, ROOT)
    import bench

    n, max_rows = 5, 7
    idx = np.arange(n, dtype=np.int32) * 3
    prob = np.linspace(0.25, 1.0, n, dtype=np.float32)
    pack = torch.full((2 * max_rows,), -9, dtype=torch.int32)
    pack[:n] = torch.from_numpy(idx)
    pack[max_rows:max_rows + n] = torch.from_numpy(prob.view(np.int32))
    idx_all, prob_all = np.zeros(n, np.int32), np.zeros(n, np.float32)
    bench.gather_shards(pack, max_rows, [0], [n], 0, None, None, idx_all, prob_all)
    np.testing.assert_array_equal(idx_all, idx)
    np.testing.assert_array_equal(prob_all, prob)


def test_reference_arm_for_preprocessing():
    rec = _run("--impl", "reference", "--workload", "recpre", "--steps", "1", "--warmup", "0",
               "--cpu-sample-lines", "8")
    assert rec["impl"] == "reference" and rec["unit"] == "lines/s" and rec["value"] > 0
    assert rec["cpu_baseline"]["kind"] == "port" and rec["e2e"]["h2d_bytes_per_step"] == 0


def test_preprocessing_workload():
    sys.path.insert(0, ROOT)
    import bench

    blob, offsets, widths, heights = bench.recpre_workload(0, n_lines=16)
    assert np.all(widths == 20 * heights) and np.all((heights >= 24) & (heights <= 64))
    assert offsets[0] == 0 and int(offsets[-1]) + int(widths[-1]) * int(heights[-1]) * 3 == blob.size
