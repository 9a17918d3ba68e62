"""The no-allocation entry point, rh_head_decode_device_noalloc, called through the C ABI.

It serves callers that cannot allocate device memory while they run (a host that reserves
all GPU memory for its own allocator, or a latency-critical loop that must not call
cudaMalloc/cudaFree, which synchronise the device): its scratch is a fixed 4 MiB array in the
library's device image. Its results must match the allocating entry point,
rh_head_decode_device, within the parity tolerances the other GPU tests use, on two calls
in a row (the array keeps the previous call's contents, which must not leak into the next).

This file is named to be collected last, so a run that stops at the first failure has run
every other test before it; it creates its own context and passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PROB_REL_TOL = 1e-5        # as tests/test_gpu_parity.py
NOALLOC_MAX_ROWS = 262144  # the limit documented in include/rechead.h


def _compare_twice(rh, lib, ctx, qw, x, rows, stream, label):
    """Runs rh_head_decode_device once and the no-allocation entry point twice on the same
    rows; returns the launches the no-allocation call made."""
    import torch

    vp = ctypes.c_void_p
    ref_idx = torch.empty(rows, dtype=torch.int32, device="cuda")
    ref_prob = torch.empty(rows, dtype=torch.float32, device="cuda")
    rh.head_decode_device(qw, x.data_ptr(), rows, ref_idx.data_ptr(), ref_prob.data_ptr(), stream)
    torch.cuda.synchronize()
    ctx.sync()
    ref_i, ref_p = ref_idx.cpu().numpy(), ref_prob.cpu().numpy()
    launches = None
    for call in range(2):
        idx = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
        prob = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
        before = ctx.launch_count(0)
        rc = lib.rh_head_decode_device_noalloc(ctx.handle, qw.handle, 0, vp(x.data_ptr()), rows,
                                               vp(idx.data_ptr()), vp(prob.data_ptr()), vp(stream))
        assert rc == rh.RH_OK, lib.rh_last_error().decode()
        torch.cuda.synchronize()
        ctx.sync()
        launches = ctx.launch_count(0) - before
        got_i, got_p = idx.cpu().numpy(), prob.cpu().numpy()
        # the maximum and its first index are exact in any summation grouping
        assert np.array_equal(got_i, ref_i), f"[{label}] rows={rows} call={call}"
        rel = np.abs(got_p.astype(np.float64) - ref_p) / ref_p
        assert rel.max() <= PROB_REL_TOL, f"[{label}] rows={rows} call={call}: prob rel err {rel.max():.3g}"
    return launches


def test_no_alloc_entry_point_matches_allocating_entry_point_twice():
    import torch

    import rust_ppocrv6_b200 as rh
    from rust_ppocrv6_b200 import workloads

    lib = rh.load()
    vp = ctypes.c_void_p
    rng = np.random.default_rng(77)
    w_t, bias = workloads.head_weights(rng)
    with rh.Context(devices=[0]) as ctx:
        qw = rh.QuantizedWeight.from_f32_transposed(w_t, ctx=ctx, bias=bias)
        stream = torch.cuda.current_stream().cuda_stream
        # 1000 rows: 8 row blocks, each split into 17 class ranges. From one wave of row blocks
        # on, full waves of whole row blocks, then the rest split: 122,880 rows (cfg2) 72
        # blocks in 2 ranges, 100,000 rows 42 blocks in 7, 140,000 rows 58 blocks in 5, and
        # 262,144 rows (the limit) 124 blocks in 7, whose partials (111,104 entries) fill most
        # of the static array. Every one writes partials and launches the head and a merge.
        for rows in (1000, 122880, 100000, 140000, NOALLOC_MAX_ROWS):
            x = torch.from_numpy(rng.standard_normal((rows, workloads.K), dtype=np.float32)).cuda()
            launches = _compare_twice(rh, lib, ctx, qw, x, rows, stream, "int8")
            assert launches == 2, f"rows={rows}: {launches} launches per call (head and merge expected)"
        # beyond the static limit: a clear error and nothing launched
        before = ctx.launch_count(0)
        x = torch.zeros((8, workloads.K), dtype=torch.float32, device="cuda")
        out_i = torch.empty(8, dtype=torch.int32, device="cuda")
        out_p = torch.empty(8, dtype=torch.float32, device="cuda")
        rc = lib.rh_head_decode_device_noalloc(ctx.handle, qw.handle, 0, vp(x.data_ptr()), NOALLOC_MAX_ROWS + 1,
                                               vp(out_i.data_ptr()), vp(out_p.data_ptr()), vp(stream))
        assert rc == rh.RH_ERR_INVALID_ARG
        assert "262144" in lib.rh_last_error().decode()
        assert ctx.launch_count(0) == before
        qw.free()


def test_no_alloc_entry_point_runs_the_fp32_head():
    """The engine's default FP32 head (rh_weight_pack_f32) through the same entry point: its
    weight tiles are the 64 KB hi/lo pairs, which the launch must know about."""
    import torch

    import rust_ppocrv6_b200 as rh
    from rust_ppocrv6_b200 import workloads

    lib = rh.load()
    rng = np.random.default_rng(78)
    w_t, bias = workloads.head_weights(rng)
    with rh.Context(devices=[0]) as ctx:
        fw = rh.Fp32Weight.from_f32_transposed(w_t, ctx=ctx, bias=bias)
        stream = torch.cuda.current_stream().cuda_stream
        for rows in (1000, 100000):
            x = torch.from_numpy(rng.standard_normal((rows, workloads.K), dtype=np.float32)).cuda()
            _compare_twice(rh, lib, ctx, fw, x, rows, stream, "f32")
        fw.free()
