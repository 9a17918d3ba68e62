"""One rank of the CPU (gloo) test of the sharded multi-rank path; launched twice by
tests/test_multirank_cpu.py as plain subprocesses.

Each rank takes its share of a ragged line batch exactly as bench.py does under torchrun
(`bench.workload_for`, i.e. `workloads.shard_lines`), decodes it with the CPU oracle (the
checker, no GPU here), and the ranks then combine results the way the benchmark does: the
strong-scaling record's host gather (`bench.gather_shards`) into rank 0's global idx/prob
arrays and a MAX all-reduce of per-rank times.
"""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    rank, world, port, out = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]), sys.argv[4]
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    import bench
    from oracle import oracle
    from rust_ppocrv6_b200 import workloads

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    rng = np.random.default_rng(workloads.SEED + 3)
    off_all = workloads.ragged_offsets(rng, 40)
    l0, l1 = workloads.shard_lines(off_all, world, rank)
    off, rows, global_rows, _, scaling = bench.workload_for("cfg3", world, rank)
    # the benchmark's own sharding of its 8192-line batch must agree with shard_lines
    big = workloads.ragged_offsets(np.random.default_rng(workloads.SEED + 3), 8192)
    b0, b1 = workloads.shard_lines(big, world, rank)
    assert np.array_equal(off, big[b0:b1 + 1] - big[b0]) and scaling == "strong"

    wrng = np.random.default_rng(5)
    n, k = 512, 120
    w = (0.05 * wrng.standard_normal((n, k))).astype(np.float32)
    bias = (0.01 * wrng.standard_normal(n)).astype(np.float32)
    x_all = wrng.standard_normal((int(off_all[-1]), k), dtype=np.float32)
    q, s = oracle.pack(w)
    lo, hi = int(off_all[l0]), int(off_all[l1])
    mine = oracle.head_decode(x_all[lo:hi], off_all[l0:l1 + 1] - off_all[l0], q, s, bias, threads=2)
    gathered = [None] * world
    dist.all_gather_object(gathered, (rank, l0, l1, mine["idx"].tolist(), mine["prob"].tolist()))

    # the benchmark's host gather of the strong-scaling record: idx then prob bits, padded to
    # the largest shard, gathered into rank 0's global arrays
    cuts = [workloads.shard_lines(off_all, world, r) for r in range(world)]
    shard_rows = [int(off_all[b] - off_all[a]) for a, b in cuts]
    starts = [int(off_all[a]) for a, _ in cuts]
    max_rows = max(shard_rows)
    pack = torch.full((2 * max_rows,), -7, dtype=torch.int32)  # padding must never be read back
    n = shard_rows[rank]
    pack[:n] = torch.from_numpy(mine["idx"].astype(np.int32))
    pack[max_rows:max_rows + n] = torch.from_numpy(mine["prob"].astype(np.float32).view(np.int32))
    recv = [torch.empty(2 * max_rows, dtype=torch.int32) for _ in range(world)] if rank == 0 else None
    idx_all = np.full(int(off_all[-1]), -1, np.int32)
    prob_all = np.full(int(off_all[-1]), np.nan, np.float32)
    bench.gather_shards(pack, max_rows, starts, shard_rows, rank, dist.group.WORLD, recv, idx_all, prob_all)

    t = torch.tensor([1.0 + rank], dtype=torch.float64)  # per-rank "device time"
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        with open(out, "w") as f:
            json.dump({"gathered": gathered, "max_time": float(t.item()), "global_rows": int(global_rows),
                       "shard_rows": shard_rows, "idx_all": idx_all.tolist(),
                       "prob_all_bits": prob_all.view(np.uint32).tolist()}, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
