"""Benchmark: decoded timesteps/s of the fused W8A32 recognition head on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg2|cfg3|tiny|recpre]

One step = one pass of the hot path (MatMul.12 + Add.204 -> Softmax.2 -> per-timestep
argmax) over one batch. Default workload cfg2: 1024 text lines x T=120 timesteps per GPU
(M = 122,880 rows, K = 120, N = 18,710), weak scaling over N GPUs (one process per GPU
under torchrun; lines are independent, so no collective is in the data path; a MAX
all-reduce of the per-rank device times is the only communication). --workload cfg3
instead shards one global 8192-line ragged batch over the ranks (strong scaling).

`value`  device-resident throughput: inputs already in HBM (rotating over enough copies to
         exceed 2x the 126 MB L2), CUDA events on the launching stream, max over ranks.
`e2e`    the same metric through the public host API (rh_head_decode on pinned host
         memory): H2D of the features and D2H of idx/prob inside the timed region.
--impl reference  times the reference algorithm's CPU implementation (the C restatement in
         oracle/, all host threads, lines spread over workers like src/pipeline.rs:417-427)
         on bounded samples of the same workload.
--workload recpre  the producer side instead: batched recognition preprocessing
         (RecPreprocess::process of 1024 text-line crops per GPU, each resized to 48 x 960,
         packed into [1024, 3, 48, 960]) in lines/s, HBM roofline.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

K_DIM = 120        # SVTR features per timestep (the small model's head; --workload tiny: 80)
N_CLASSES = 18710  # CTC classes (--workload tiny: 6906)


def head_dims(workload: str):
    """(K, N) of the head the workload runs."""
    from rust_ppocrv6_b200 import workloads

    return (workloads.K_TINY, workloads.N_TINY) if workload == "tiny" else (K_DIM, N_CLASSES)
L2_BYTES = 126 * 1024 * 1024
METRIC = "W8A32 rec-head decoded timesteps/s (MatMul.12+Add.204 -> Softmax.2 -> argmax)"
METRIC_F32 = "FP32 rec-head decoded timesteps/s (MatMul.12+Add.204 -> Softmax.2 -> argmax)"
UNIT = "timesteps/s"
RECPRE_METRIC = ("rec preprocessing lines/s (RecPreprocess::process: triangle resize to 48 rows + normalise, "
                 "packed [N,3,48,Wmax])")
RECPRE_UNIT = "lines/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["cfg2", "cfg3", "tiny", "recpre"], default="cfg2")
    ap.add_argument("--weights", choices=["int8", "compact", "f32"], default="int8",
                    help="int8: the quantised head with the fp16 operand image in HBM (the metric's path); "
                         "compact: the quantised head with int8 tiles in HBM (rh_weight_pack_compact); "
                         "f32: the engine's default FP32 head")
    ap.add_argument("--cpu-sample-lines", type=int, default=512)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-strong", action="store_true", help="skip the cfg3 strong-scaling sub-record")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def workload_for(name: str, world: int, rank: int):
    """(line_offsets of this rank's lines rebased to 0, rows, global rows, description)."""
    from rust_ppocrv6_b200 import workloads

    if name == "cfg2":
        off = workloads.uniform_offsets(1024, 120)
        desc = f"cfg2: 1024 lines x T=120 per GPU (M=122880/GPU), K=120, N=18710; global batch {1024 * world} lines"
        return off, int(off[-1]), int(off[-1]) * world, desc, "weak"
    if name == "tiny":
        off = workloads.uniform_offsets(1024, 120)
        desc = (f"cfg5 (tiny model head): 1024 lines x T=120 per GPU (M=122880/GPU), K=80, N=6906; "
                f"global batch {1024 * world} lines")
        return off, int(off[-1]), int(off[-1]) * world, desc, "weak"
    rng = np.random.default_rng(workloads.SEED + 3)
    off_all = workloads.ragged_offsets(rng, 8192)
    l0, l1 = workloads.shard_lines(off_all, world, rank)
    off = off_all[l0:l1 + 1] - off_all[l0]
    desc = f"cfg3: 8192 ragged lines T~U{{10..120}} (M={int(off_all[-1])}) sharded over {world} GPU(s)"
    return off, int(off[-1]), int(off_all[-1]), desc, "strong"


def synth(rows: int, seed: int, k: int = K_DIM):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((rows, k), dtype=np.float32)


def head_weights(workload: str = "cfg2"):
    from rust_ppocrv6_b200 import workloads

    k, n = head_dims(workload)
    rng = np.random.default_rng(workloads.SEED + 2)
    return workloads.head_weights(rng, n=n, k=k)


class ClockSampler:
    """Samples the SM clock and throttle reasons through NVML from a background thread that is
    started before the warm-up (so NVML is warm and sampling is steady when timing begins);
    `window(t0, t1)` keeps the samples taken inside the timed region (host perf_counter)."""

    NAMES = {
        "hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
        "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index: int):
        self.samples = []  # (perf_counter, sm MHz, throttle-reason bits)
        self.max_mhz = None
        self._stop = threading.Event()
        self._ok = False
        self._t0 = self._t1 = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
        except Exception:
            self._ok = False

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                bits = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                self.samples.append((time.perf_counter(), mhz, bits))
            except Exception:
                pass
            time.sleep(0.001)

    def start(self):
        if self._ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def stop(self):
        if self._ok:
            self._stop.set()
            self._t.join()

    def window(self, t0: float, t1: float):
        self._t0, self._t1 = t0, t1

    def summary(self):
        if not self._ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        inside = [x for x in self.samples if self._t0 is None or self._t0 <= x[0] <= self._t1]
        reasons = sorted({k for _, _, bits in inside for k, bit in self.NAMES.items() if bits & bit})
        return {"sm_mhz": statistics.median([m for _, m, _ in inside]) if inside else None,
                "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(inside)}


def measured_peak_tflops():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured bf16 dense (MEASURED_PEAKS.json, burst)"
    except Exception:
        return 1590.0, "fallback 1.59 PFLOP/s bf16 dense"


def output_checksum(*tensors):
    """CRC32 of the raw bytes of the last step's device outputs (same work, same bytes: equal
    across runs and across the kernel's versions, whatever the timing)."""
    import zlib

    crc = 0
    for t in tensors:
        crc = zlib.crc32(t.detach().cpu().contiguous().numpy().tobytes(), crc)
    return f"crc32:{crc:08x}"


def measured_hbm_gbs():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured HBM copy (MEASURED_PEAKS.json)"
    except Exception:
        return 6650.0, "fallback 6.65 TB/s"


KERNEL_SOURCES = ("rust_ppocrv6_b200/csrc/rechead_kernels.cu", "rust_ppocrv6_b200/csrc/sm100_ptx.cuh",
                  "rust_ppocrv6_b200/csrc/head_params.h")
TRAFFIC_RECORD = os.path.join(ROOT, "profiles", "head_kernel_traffic.json")
RECPRE_SOURCES = ("rust_ppocrv6_b200/csrc/recpre_kernels.cu", "rust_ppocrv6_b200/csrc/recpre_params.h")
RECPRE_TRAFFIC_RECORD = os.path.join(ROOT, "profiles", "recpre_kernel_traffic.json")


def source_sha16(sources) -> str:
    """First 16 hex digits of the SHA-256 over the given source files: a DRAM-traffic figure
    captured by ncu applies only to the kernels built from the same sources."""
    import hashlib

    h = hashlib.sha256()
    for rel in sources:
        with open(os.path.join(ROOT, rel), "rb") as f:
            h.update(f.read())
    return h.hexdigest()[:16]


def kernel_source_sha16() -> str:
    """Source hash of the head kernel (rechead_kernels.cu, sm100_ptx.cuh, head_params.h)."""
    return source_sha16(KERNEL_SOURCES)


def recpre_traffic():
    """(DRAM bytes read + written per preprocessing step, i.e. one tap-table and one resize
    launch over the bench's 1,024 crops, description) from the ncu capture recorded for the
    current preprocessing sources, or (None, reason)."""
    try:
        with open(RECPRE_TRAFFIC_RECORD) as f:
            r = json.load(f)
    except (OSError, ValueError):
        return None, "no ncu capture recorded"
    sha = source_sha16(RECPRE_SOURCES)
    if r.get("source_sha16") != sha:
        return None, f"the ncu capture is of preprocessing sources {r.get('source_sha16')}, not {sha}"
    return int(r["dram_bytes_per_step"]), ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one rec_weights "
                                           "and one rec_resize launch (1,024 crops)")


def profiled_traffic(workload: str = "cfg2", weights: str = "int8"):
    """(DRAM bytes read + written per head-kernel launch, description) from the ncu capture
    recorded for this workload and these kernel sources, or (None, reason) when the kernel
    changed since the capture or none was recorded."""
    try:
        with open(TRAFFIC_RECORD) as f:
            records = json.load(f)["records"]
    except (OSError, ValueError, KeyError):
        return None, "no ncu capture recorded"
    sha = kernel_source_sha16()
    for r in records:
        if r.get("workload") == workload and r.get("weights") == weights:
            if r.get("kernel_source_sha16") != sha:
                return None, f"the ncu capture is of kernel sources {r.get('kernel_source_sha16')}, not {sha}"
            return int(r["dram_bytes_per_launch"]), (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                                     f"{r.get('kernel', 'head_kernel')} launch on {workload}")
    return None, f"no ncu capture recorded for {workload}/{weights}"


def cpu_reference(lines_off: np.ndarray, x: np.ndarray, w_t, bias, sample_lines: int, target_s: float = 10.0):
    """Times the oracle port (the reference's AVX2 path, restated) on `sample_lines` lines
    of the workload with every host thread, repeating the sample until about `target_s`
    seconds of CPU work have run. Returns (timesteps/s, threads, rows per pass, passes, seconds)."""
    from oracle import oracle

    q, s = oracle.pack(w_t)
    nl = min(sample_lines, lines_off.size - 1)
    off = lines_off[:nl + 1]
    rows = int(off[-1])
    xs = np.ascontiguousarray(x[:rows])
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    t0 = time.perf_counter()
    oracle.head_decode(xs, off, q, s, bias, threads=threads)  # warm caches, size the repeat count
    reps = max(1, int(np.ceil(target_s / max(time.perf_counter() - t0, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(reps):
        oracle.head_decode(xs, off, q, s, bias, threads=threads)
    dt = time.perf_counter() - t0
    return rows * reps / dt, threads, rows, reps, dt


def recpre_workload(rank: int, n_lines: int = 1024):
    """Seeded text-line crops: heights U{24..64}, width 20 x height (every line resizes to
    48 x 960, the input of one cfg2 line), random bytes. Returns (blob, offsets, widths, heights)."""
    from rust_ppocrv6_b200 import workloads

    rng = np.random.default_rng(workloads.SEED + 5 + rank)
    heights = rng.integers(24, 65, n_lines).astype(np.uint32)
    widths = (20 * heights).astype(np.uint32)
    sizes = widths.astype(np.int64) * heights * 3
    offsets = np.zeros(n_lines, np.int64)
    offsets[1:] = np.cumsum(sizes)[:-1]
    blob = rng.integers(0, 256, int(sizes.sum()), dtype=np.uint8)
    return blob, offsets, widths, heights


RECPRE_DESC = ("recpre: 1024 RGB8 text-line crops per GPU, h~U{24..64}, w=20h (mean 44 x 880), each resized "
               "to 48 x 960 and packed into [1024,3,48,960] f32")


def cpu_recpre(blob, offsets, widths, heights, sample_lines: int, target_s: float = 10.0, steps: int | None = None,
               warmup: int = 1):
    """Times the oracle's preprocessing (RecPreprocess::process + build_batch restated) on the
    first `sample_lines` crops with every host thread. Returns (lines/s, threads, lines, reps, s)."""
    from oracle import oracle

    n = min(sample_lines, len(widths))
    crops = [blob[offsets[i]:offsets[i] + int(widths[i]) * int(heights[i]) * 3].reshape(int(heights[i]),
                                                                                            int(widths[i]), 3)
             for i in range(n)]
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    t0 = time.perf_counter()
    for _ in range(max(warmup, 1)):
        oracle.rec_preprocess_batch(crops, threads=threads)
    one = (time.perf_counter() - t0) / max(warmup, 1)
    reps = steps if steps is not None else max(1, int(np.ceil(target_s / max(one, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(reps):
        oracle.rec_preprocess_batch(crops, threads=threads)
    dt = time.perf_counter() - t0
    return n * reps / dt, threads, n, reps, dt


def run_reference_arm(args, world, rank):
    if rank != 0:
        return
    if args.workload == "recpre":
        blob, offsets, widths, heights = recpre_workload(0)
        v, threads, n, reps, dt = cpu_recpre(blob, offsets, widths, heights, min(args.cpu_sample_lines, 256),
                                             steps=args.steps, warmup=args.warmup)
        sample = f"{n} crops of the workload per step"
        print(json.dumps({
            "impl": "reference", "metric": RECPRE_METRIC, "value": v, "unit": RECPRE_UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / reps, "higher_is_better": True,
            "scaling": "none (host CPU)", "vs_baseline": None, "dtype": "u8->f32",
            "data": "synthetic (seeded random RGB8 crops)", "config": {"workload": RECPRE_DESC, "sample": sample},
            "cpu_baseline": {"value": v, "unit": RECPRE_UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": RECPRE_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return
    off, rows, _, desc, _ = workload_for(args.workload, 1, 0)
    w_t, bias = head_weights(args.workload)
    x = synth(min(rows, int(off[min(args.cpu_sample_lines, off.size - 1)])), 1234, w_t.shape[1])
    from oracle import oracle

    nl = min(args.cpu_sample_lines, off.size - 1)
    soff = off[:nl + 1]
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    if args.weights == "f32":  # matmul_transposed_b's register-blocked AVX2 kernel restated
        def one():
            oracle.head_decode_f32(x, soff, w_t, bias, threads=threads)
    else:
        q, s = oracle.pack(w_t)

        def one():
            oracle.head_decode(x, soff, q, s, bias, threads=threads)
    for _ in range(max(args.warmup, 0)):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    dt = time.perf_counter() - t0
    srows = int(soff[-1])
    value = srows * args.steps / dt
    sample = f"{nl} lines x T=120 ({srows} timesteps) of {desc.split(';')[0]} per step"
    print(json.dumps({
        "impl": "reference", "metric": METRIC_F32 if args.weights == "f32" else METRIC, "value": value,
        "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "none (host CPU)", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) features, N(0,0.05^2) weights, N(0,0.01^2) bias)",
        "config": {"workload": desc, "sample": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_recpre(args, world, rank, local, torch, rh, barrier, max_over_ranks):
    """Batched recognition preprocessing: device-resident throughput (rh_rec_preprocess_device,
    crops already in HBM), end to end through rh_rec_preprocess (pinned host crops in, pinned
    host tensor out), HBM roofline of the step, CPU baseline."""
    import ctypes

    blob, offsets, widths, heights = recpre_workload(rank)
    n = len(widths)
    out_w, out_h, wmax = rh.batch_shape(widths, heights)
    out_len = n * 3 * out_h * wmax
    ctx = rh.Context(devices=[local])
    d_blobs = [torch.from_numpy(blob).cuda()]
    d_blobs.append(d_blobs[0].roll(1).contiguous())  # two copies: 2 x 119 MB > L2
    d_out = torch.empty(out_len, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream

    def step(i):
        rh.rec_preprocess_device(ctx, d_blobs[i % 2].data_ptr(), blob.size, offsets, widths, heights,
                                 d_out.data_ptr(), out_len, stream=sptr)

    clocks = ClockSampler(local).start()
    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    ctx.sync()
    l0 = ctx.launch_count(0)
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    t_start = time.perf_counter()
    ev0.record(stream)
    for i in range(args.steps):
        step(i)
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks.window(t_start, time.perf_counter())
    clocks.stop()
    barrier()
    ctx.sync()
    launches = ctx.launch_count(0) - l0
    dev_ms = ev0.elapsed_time(ev1)
    dev_ms_max = max_over_ranks(dev_ms)
    value = n * world * args.steps / (dev_ms_max / 1e3)

    # end to end through the host API
    lib = rh.load()
    pin_in = torch.from_numpy(blob).pin_memory()
    pin_out = torch.empty(out_len, dtype=torch.float32).pin_memory()
    got_w = np.zeros(n, np.uint32)
    got_max = ctypes.c_uint32(0)
    vp = ctypes.c_void_p

    def e2e_step():
        rh._lib.check(lib.rh_rec_preprocess(ctx.handle, vp(pin_in.data_ptr()), blob.size,
                                            offsets.ctypes.data_as(vp), widths.ctypes.data_as(vp),
                                            heights.ctypes.data_as(vp), n, 48, 960, vp(pin_out.data_ptr()), out_len,
                                            got_w.ctypes.data_as(vp), ctypes.byref(got_max)))

    for _ in range(max(3, args.warmup)):
        e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()

    # roofline: algorithmic bytes = every crop byte read once + every output float written once
    alg_bytes = int(blob.size) + out_len * 4
    traffic, traffic_src = recpre_traffic()
    achieved = alg_bytes / (dev_ms / args.steps / 1e3) / 1e9
    peak, peak_src = measured_hbm_gbs()
    out = {
        "metric": RECPRE_METRIC, "value": value, "unit": RECPRE_UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8->f32",
        "data": "synthetic (seeded random RGB8 crops; no public dataset)",
        "config": {"workload": RECPRE_DESC, "lines_per_step": n * world, "parallelism": f"crops sharded x{world}",
                   "l2": f"crops rotate over 2 device copies ({2 * blob.size / 2**20:.0f} MiB), output "
                         f"{out_len * 4 / 2**20:.0f} MiB per step (> L2)"},
        "e2e": {"value": n * world * args.steps / e2e_s, "unit": RECPRE_UNIT, "h2d_bytes_per_step": int(blob.size),
                "d2h_bytes_per_step": int(out_len * 4), "ms_per_step": e2e_s * 1e3 / args.steps},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_src, "traffic": traffic, "traffic_source": traffic_src,
                     "note": "achieved = (crop bytes + output bytes) per step / device time per step (tap-table "
                             "kernel + resize kernel + descriptor copy)"},
        "clocks": clocks.summary(),
        "checksum": output_checksum(d_out),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, threads, ns, reps, dt = cpu_recpre(blob, offsets, widths, heights, min(args.cpu_sample_lines, 256))
        out["cpu_baseline"] = {"value": v, "unit": RECPRE_UNIT, "cores": threads, "kind": "port",
                               "sample": f"{ns} crops of the workload x {reps} passes, {dt:.1f} s wall"}
    ctx.close()
    if rank == 0:
        print(json.dumps(out), flush=True)


def main():
    args = parse()
    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference_arm(args, world, rank)
        return

    import torch

    import rust_ppocrv6_b200 as rh

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        # the host-side gather of the strong-scaling record's idx/prob (host arrays, as the
        # reference's per-line fan-out returns them)
        host_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=120))

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if world == 1:
        host_group = None
    if args.workload == "recpre":
        run_recpre(args, world, rank, local, torch, rh, barrier, max_over_ranks)
        if dist is not None:
            dist.destroy_process_group()
        return

    off, rows, global_rows, desc, scaling = workload_for(args.workload, world, rank)
    w_t, bias = head_weights(args.workload)
    k_dim, n_classes = w_t.shape[1], w_t.shape[0]
    ctx = rh.Context(devices=[local])
    if args.weights == "f32":
        qw = rh.Fp32Weight.from_f32_transposed(w_t, ctx=ctx, bias=bias)
    else:
        qw = rh.QuantizedWeight.from_f32_transposed(w_t, ctx=ctx, bias=bias, compact=args.weights == "compact")

    x_host = synth(rows, 1000 + rank, k_dim)
    x_bytes = x_host.nbytes
    n_copies = max(2, int(np.ceil(2 * L2_BYTES / max(x_bytes, 1))) + 1)
    n_copies = min(n_copies, 64)
    xs = [torch.from_numpy(x_host).cuda()]
    for i in range(1, n_copies):
        xs.append(xs[0].roll(i, dims=0).contiguous())  # distinct buffers, same statistics
    idx = torch.empty(rows, dtype=torch.int32, device="cuda")
    prob = torch.empty(rows, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream

    def step(i):
        rh.head_decode_device(qw, xs[i % n_copies].data_ptr(), rows, idx.data_ptr(), prob.data_ptr(), sptr)

    clocks = ClockSampler(local).start()
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    ctx.sync()
    l0 = ctx.launch_count(0)
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    t_start = time.perf_counter()
    ev0.record(stream)
    for i in range(args.steps):
        step(args.warmup + i)
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks.window(t_start, time.perf_counter())
    clocks.stop()
    barrier()
    ctx.sync()
    launches = ctx.launch_count(0) - l0
    dev_ms = ev0.elapsed_time(ev1)
    dev_ms_max = max_over_ranks(dev_ms)
    value = global_rows * args.steps / (dev_ms_max / 1e3)
    ms_per_step = dev_ms_max / args.steps

    # end to end through the public host API (pinned host buffers, H2D + D2H inside)
    x_pin = torch.from_numpy(x_host).pin_memory()
    idx_h = torch.empty(rows, dtype=torch.int32).pin_memory()
    prob_h = torch.empty(rows, dtype=torch.float32).pin_memory()
    import ctypes

    lib = rh.load()

    def e2e_step():
        rh._lib.check(lib.rh_head_decode(ctx.handle, qw.handle, ctypes.c_void_p(x_pin.data_ptr()), rows, k_dim,
                                         ctypes.c_void_p(idx_h.data_ptr()), ctypes.c_void_p(prob_h.data_ptr())))

    for _ in range(max(3, args.warmup)):
        e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()
    e2e_value = global_rows * args.steps / e2e_s
    # the link the e2e leg crosses: a bare pinned H2D copy of one step's features
    h2d_gbs = h2d_bandwidth(torch, x_pin, xs[0], stream)

    # roofline of the dominant kernel (the fused head; the split merge is <1 % of a step)
    peak, peak_src = measured_peak_tflops()
    achieved = 2 * k_dim * n_classes * rows / (dev_ms / args.steps / 1e3) / 1e12  # 2*K*N per timestep
    traffic, traffic_src = profiled_traffic(args.workload, args.weights)
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_source": peak_src,
                "traffic": traffic, "traffic_source": traffic_src,
                "tf32_equiv_frac": achieved / (peak / 2),
                "note": "achieved = 2*K*N*rows per step / device time per step (head + merge kernels)"}

    strong = None
    if args.workload == "cfg2" and not args.no_strong:
        strong = strong_record(args, world, rank, local, torch, rh, ctx, qw, barrier, max_over_ranks, host_group)

    out = {
        "metric": METRIC_F32 if args.weights == "f32" else METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) features, N(0,0.05^2) weights, N(0,0.01^2) bias; no public dataset)",
        "config": {"workload": desc, "timesteps_per_step": global_rows, "parallelism": f"lines sharded x{world}",
                   "l2": f"inputs rotate over {n_copies} device copies ({n_copies * x_bytes / 2**20:.0f} MiB > 2x L2)"},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(x_bytes),
                "d2h_bytes_per_step": int(rows * 8), "ms_per_step": e2e_s * 1e3 / args.steps,
                "h2d_gbs_measured": h2d_gbs,
                "link_bound_value": global_rows / (x_bytes / (h2d_gbs * 1e9)) if h2d_gbs else None,
                "note": "rh_head_decode from pinned host memory; link_bound_value = the rate if every step took "
                        "only its features' H2D at the measured bare-copy bandwidth"},
        "gpu_launches": int(launches),
        "roofline": roofline,
        "clocks": clocks.summary(),
        "checksum": output_checksum(idx, prob),
    }
    if strong is not None:
        out["strong"] = strong
    out["config"]["weights"] = {
        "int8": "int8 head, fp16 operand image in HBM (rh_weight_pack), %d device bytes" % qw.device_bytes,
        "compact": "int8 head, int8 tiles in HBM expanded in shared memory (rh_weight_pack_compact), %d device bytes"
                   % qw.device_bytes,
        "f32": "f32 (hi/lo fp16 images, 23 MMA K-steps per tile), %d device bytes" % qw.device_bytes}[args.weights]
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.weights != "f32":
        v, threads, srows, reps, dt = cpu_reference(off, x_host, w_t, bias, args.cpu_sample_lines)
        out["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                               "sample": f"{srows} timesteps ({args.cpu_sample_lines} lines of the workload) "
                                         f"x {reps} passes, {dt:.1f} s wall"}
    qw.free()
    ctx.close()
    if rank == 0:
        print(json.dumps(out), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def h2d_bandwidth(torch, src_pinned, dst, stream, reps: int = 5):
    """GB/s of a bare pinned host -> device copy of `src_pinned` (best of `reps`, CUDA events)."""
    best = None
    for _ in range(reps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dst.copy_(src_pinned, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    return src_pinned.numel() * src_pinned.element_size() / (best / 1e3) / 1e9 if best else None


def gather_shards(pack, max_rows, starts, shard_rows, rank, group, gathered, idx_all, prob_all):
    """Collects every rank's decoded shard into rank 0's host arrays idx_all/prob_all.

    `pack` (int32, 2 * max_rows) holds this rank's class indices in [0, n) and the bit patterns
    of its probabilities in [max_rows, max_rows + n), n = shard_rows[rank]; rank r's shard
    starts at global row starts[r]. With `group` None (one rank) the pack is unpacked in place;
    otherwise one gather over `group` (gloo, host tensors) brings every pack to rank 0, whose
    `gathered` holds one receive buffer per rank."""
    if group is None:
        gathered = [pack]
    else:
        import torch.distributed as dist

        dist.gather(pack, gathered if rank == 0 else None, dst=0, group=group)
    if rank != 0:
        return
    for r, (g0, n) in enumerate(zip(starts, shard_rows)):
        idx_all[g0:g0 + n] = gathered[r][:n].numpy()
        prob_all[g0:g0 + n] = gathered[r][max_rows:max_rows + n].numpy().view(np.float32)


def strong_record(args, world, rank, local, torch, rh, ctx, qw, barrier, max_over_ranks, host_group):
    """cfg3 (one 8192-line ragged batch, ~528k timesteps) sharded over the N ranks by balanced
    timestep counts: device-resident time (max over ranks) and end to end through
    rh_head_decode_lines from pinned host memory with every rank's idx/prob gathered to rank 0's
    host memory (gloo) inside the timed region."""
    import ctypes

    from rust_ppocrv6_b200 import workloads

    off_all = workloads.ragged_offsets(np.random.default_rng(workloads.SEED + 3), 8192)
    total = int(off_all[-1])
    cuts = [workloads.shard_lines(off_all, world, r) for r in range(world)]
    shard_rows = [int(off_all[l1] - off_all[l0]) for l0, l1 in cuts]
    l0, l1 = cuts[rank]
    r0, rows = int(off_all[l0]), shard_rows[rank]
    off = np.ascontiguousarray(off_all[l0:l1 + 1] - off_all[l0])
    x_all = synth(total, 3000, K_DIM)  # the same global batch on every rank
    x = np.ascontiguousarray(x_all[r0:r0 + rows])
    k_dim = x.shape[1]
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    n_copies = max(2, int(np.ceil(2 * L2_BYTES / max(x.nbytes, 1))) + 1) if rows else 1
    xs = [torch.from_numpy(x).cuda()]
    for i in range(1, min(n_copies, 64)):
        xs.append(xs[0].roll(i, dims=0).contiguous())
    n_copies = len(xs)
    d_idx = torch.empty(max(rows, 1), dtype=torch.int32, device="cuda")
    d_prob = torch.empty(max(rows, 1), dtype=torch.float32, device="cuda")

    def dev_step(i):
        if rows:
            rh.head_decode_device(qw, xs[i % n_copies].data_ptr(), rows, d_idx.data_ptr(), d_prob.data_ptr(), sptr)

    clocks = ClockSampler(local).start()
    for i in range(max(3, args.warmup)):
        dev_step(i)
    torch.cuda.synchronize()
    ctx.sync()
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    t_start = time.perf_counter()
    ev0.record(stream)
    for i in range(args.steps):
        dev_step(i)
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks.window(t_start, time.perf_counter())
    clocks.stop()
    ctx.sync()
    dev_ms = max_over_ranks(ev0.elapsed_time(ev1))
    barrier()

    # end to end: host features in, every rank's results in rank 0's host arrays out
    lib = rh.load()
    vp = ctypes.c_void_p
    x_pin = torch.from_numpy(x).pin_memory()
    max_rows = max(shard_rows)
    pack = torch.zeros(2 * max_rows, dtype=torch.int32).pin_memory()  # idx then prob bits
    gathered = [torch.empty(2 * max_rows, dtype=torch.int32) for _ in range(world)] if rank == 0 else None
    idx_all = np.empty(total, np.int32)
    prob_all = np.empty(total, np.float32)
    starts = [int(off_all[a]) for a, _ in cuts]

    def e2e_step():
        if rows:
            rh._lib.check(lib.rh_head_decode_lines(ctx.handle, qw.handle, vp(x_pin.data_ptr()),
                                                   off.ctypes.data_as(vp), off.size - 1, k_dim,
                                                   vp(pack.data_ptr()), vp(pack.data_ptr() + 4 * max_rows)))
        gather_shards(pack, max_rows, starts, shard_rows, rank, host_group, gathered, idx_all, prob_all)

    for _ in range(max(3, args.warmup)):
        e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()
    import zlib

    return {
        "workload": f"cfg3: 8192 ragged lines T~U{{10..120}} (M={total}), K=120, N=18710, sharded by balanced "
                    f"timestep counts over {world} GPU(s)",
        "scaling": "strong", "timesteps_per_step": total, "rows_per_rank": shard_rows,
        "value": total * args.steps / (dev_ms / 1e3), "unit": UNIT, "ms_per_step": dev_ms / args.steps,
        "l2": f"inputs rotate over {n_copies} device copies per rank", "clocks": clocks.summary(),
        "e2e": {"value": total * args.steps / e2e_s, "unit": UNIT, "ms_per_step": e2e_s * 1e3 / args.steps,
                "h2d_bytes_per_step": int(total * k_dim * 4), "d2h_bytes_per_step": int(total * 8),
                "gather": "each rank: rh_head_decode_lines on its shard (pinned host memory); then idx/prob "
                          "of every rank gathered into rank 0's host arrays (gloo)" if world > 1 else
                          "rh_head_decode_lines on the whole batch (pinned host memory)"},
        "idx_crc32": f"{zlib.crc32(idx_all.tobytes()):08x}" if rank == 0 else None,
    }


if __name__ == "__main__":
    main()
