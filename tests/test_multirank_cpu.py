"""The N>1 path on CPU: two and four gloo ranks shard a ragged line batch the way bench.py does under
torchrun, and their gathered outputs equal the single-process decode (no GPU needed)."""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_shard_lines_and_agree_with_one_process(tmp_path, oracle, world):
    sys.path.insert(0, os.path.dirname(HERE))
    from rust_ppocrv6_b200 import workloads

    port, out = _free_port(), str(tmp_path / "r0.json")
    env = dict(os.environ, MASTER_ADDR="127.0.0.1")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "multirank_worker.py"), str(r), str(world),
                               str(port), out], env=env) for r in range(world)]
    for p in procs:
        assert p.wait(timeout=240) == 0
    res = json.load(open(out))
    assert res["max_time"] == float(world)  # MAX over ranks of 1.0, 2.0, ...
    parts = sorted(res["gathered"])
    assert parts[0][1] == 0  # contiguous, disjoint line ranges
    assert all(parts[i][2] == parts[i + 1][1] for i in range(world - 1))
    idx = np.concatenate([np.array(p[3], np.int32) for p in parts])
    prob = np.concatenate([np.array(p[4], np.float32) for p in parts])

    rng = np.random.default_rng(workloads.SEED + 3)
    off_all = workloads.ragged_offsets(rng, 40)
    assert parts[-1][2] == off_all.size - 1
    wrng = np.random.default_rng(5)
    n, k = 512, 120
    w = (0.05 * wrng.standard_normal((n, k))).astype(np.float32)
    bias = (0.01 * wrng.standard_normal(n)).astype(np.float32)
    x_all = wrng.standard_normal((int(off_all[-1]), k), dtype=np.float32)
    q, s = oracle.pack(w)
    ref = oracle.head_decode(x_all, off_all, q, s, bias, threads=2)
    np.testing.assert_array_equal(idx, ref["idx"])
    np.testing.assert_array_equal(prob, ref["prob"])
    # the benchmark's host gather rebuilt the whole batch in rank 0's arrays, bit for bit, from
    # shards of unequal size (padding never read back)
    assert len(set(res["shard_rows"])) > 1
    np.testing.assert_array_equal(np.array(res["idx_all"], np.int32), ref["idx"])
    np.testing.assert_array_equal(np.array(res["prob_all_bits"], np.uint32),
                                  ref["prob"].astype(np.float32).view(np.uint32))
