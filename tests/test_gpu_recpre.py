"""GPU parity of the batched recognition preprocessing (rh_rec_preprocess*, the sm_100a
kernels of recpre_kernels.cu) against the CPU oracle's restatement of RecPreprocess::process
+ build_batch, on identical seeded crops. The resized pixels are bytes before normalisation,
so the bar is bit-exact: every output float equal."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MIXED = [(100, 30), (40, 40), (900, 20), (10, 60), (0, 5), (7, 0), (1, 1), (300, 48), (65_000, 1), (20, 3000),
         (8000, 20), (5000, 700), (33, 47), (2, 200), (1500, 64)]


@pytest.fixture(scope="module")
def rh():
    import rust_ppocrv6_b200 as rh

    rh.load()
    return rh


@pytest.fixture(scope="module")
def ctx(rh):
    c = rh.Context()
    yield c
    c.close()


def crops_of(dims, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 256, (h, w, 3), dtype=np.uint8) for w, h in dims]


def assert_same(got, ref, label):
    assert got.shape == ref.shape, (label, got.shape, ref.shape)
    bad = got != ref
    assert not bad.any(), f"[{label}] {bad.sum()} of {bad.size} floats differ; first at {np.argwhere(bad)[0]}"


def test_mixed_batch_bit_exact(rh, ctx, oracle):
    crops = crops_of(MIXED, 11)
    got, widths = rh.RecPreprocess(ctx=ctx).process_batch(crops)
    ref, ref_w = oracle.rec_preprocess_batch(crops, threads=4)
    assert np.array_equal(widths, ref_w)
    assert_same(got, ref, "mixed")
    assert ctx.launch_count() > 0


@pytest.mark.parametrize("target_h,max_w", [(48, 960), (32, 320), (0, 960), (64, 8), (1, 100)])
def test_other_heights_and_widths(rh, ctx, oracle, target_h, max_w):
    crops = crops_of(MIXED[:8] + [(123, 45), (640, 32)], 12 + target_h)
    got, _ = rh.RecPreprocess(target_h, max_w, ctx=ctx).process_batch(crops)
    ref, _ = oracle.rec_preprocess_batch(crops, target_h, max_w, threads=4)
    assert_same(got, ref, f"H={target_h} max_w={max_w}")


def test_reference_rec_unit_cases(rh, ctx, oracle):
    """The cases of src/preprocess/rec.rs:108-182, through the GPU path."""
    def solid(w, h, rgb=(128, 64, 32)):
        a = np.zeros((h, w, 3), np.uint8)
        a[:, :] = rgb
        return a

    cases = [(solid(100, 10), 48, 8, (1, 3, 48, 32)), (solid(64, 64), 0, 960, (1, 3, 1, 32)),
             (solid(1000, 10), 48, 200, (1, 3, 48, 200)), (solid(65_000, 1), 48, 960, (1, 3, 48, 960)),
             (solid(50, 100), 48, 960, (1, 3, 48, 32)), (solid(400, 40, (0, 0, 0)), 48, 960, (1, 3, 48, 480))]
    for img, th, mw, shape in cases:
        got = rh.RecPreprocess.with_max_w(th, mw)
        got.ctx = ctx
        t = got.process(img)
        assert t.shape == shape
        assert_same(t, oracle.rec_preprocess(img, th, mw), f"{img.shape} H={th} max_w={mw}")
    t = rh.RecPreprocess(ctx=ctx).process(solid(400, 40, (0, 0, 0)))
    assert np.all(t == -1.0)


def test_text_line_batch_bit_exact(rh, ctx, oracle):
    """The bench's workload shape (every line resized to 48 x 960), 96 lines."""
    rng = np.random.default_rng(13)
    hs = rng.integers(24, 65, 96)
    crops = [rng.integers(0, 256, (int(h), int(20 * h), 3), dtype=np.uint8) for h in hs]
    got, widths = rh.RecPreprocess(ctx=ctx).process_batch(crops)
    assert np.all(widths == 960)
    ref, _ = oracle.rec_preprocess_batch(crops, threads=8)
    assert_same(got, ref, "text lines")


def test_empty_batch_and_empty_crops(rh, ctx, oracle):
    out, widths = rh.RecPreprocess(ctx=ctx).process_batch([])
    assert out.shape == (0, 3, 48, 0) and widths.size == 0
    crops = [np.zeros((0, 10, 3), np.uint8), np.zeros((5, 0, 3), np.uint8)]
    got, _ = rh.RecPreprocess(ctx=ctx).process_batch(crops)
    ref, _ = oracle.rec_preprocess_batch(crops)
    assert_same(got, ref, "empty crops")
    assert np.all(got[0] == -1.0)


def test_device_entry_point(rh, ctx, oracle):
    import torch

    from rust_ppocrv6_b200.preprocess import _pack_crops

    crops = crops_of(MIXED, 14)
    blob, offsets, widths, heights = _pack_crops(crops)
    out_w, h, wmax = rh.batch_shape(widths, heights)
    d_rgb = torch.from_numpy(blob).to("cuda:0")
    d_out = torch.full((len(crops) * 3 * h * wmax,), float("nan"), device="cuda:0")
    stream = torch.cuda.current_stream(0)
    got_w, got_max = rh.rec_preprocess_device(ctx, d_rgb.data_ptr(), blob.size, offsets, widths, heights,
                                              d_out.data_ptr(), d_out.numel(), stream=stream.cuda_stream)
    assert got_max == wmax and np.array_equal(got_w, out_w)
    stream.synchronize()
    ctx.sync()
    ref, _ = oracle.rec_preprocess_batch(crops, threads=4)
    assert_same(d_out.cpu().numpy().reshape(ref.shape), ref, "device entry point")


def test_argument_errors_are_reported_before_any_launch(rh, ctx):
    import ctypes

    from rust_ppocrv6_b200._lib import load
    from rust_ppocrv6_b200.preprocess import _p, _pack_crops

    crops = crops_of([(100, 30), (40, 40)], 15)
    blob, offsets, widths, heights = _pack_crops(crops)
    lib = load()
    _, h, wmax = rh.batch_shape(widths, heights)
    out = np.empty(2 * 3 * h * wmax, np.float32)
    got_w = np.zeros(2, np.uint32)
    got_max = ctypes.c_uint32(0)
    before = ctx.launch_count()
    # short output
    rc = lib.rh_rec_preprocess(ctx.handle, _p(blob), blob.size, _p(offsets), _p(widths), _p(heights), 2, 48, 960,
                               _p(out), out.size - 1, _p(got_w), ctypes.byref(got_max))
    assert rc == rh.RH_ERR_INVALID_ARG and b"needs" in lib.rh_last_error()
    # a crop that runs past the end of the pixel buffer
    rc = lib.rh_rec_preprocess(ctx.handle, _p(blob), blob.size - 1, _p(offsets), _p(widths), _p(heights), 2, 48,
                               960, _p(out), out.size, _p(got_w), ctypes.byref(got_max))
    assert rc == rh.RH_ERR_INVALID_ARG and b"outside the pixel buffer" in lib.rh_last_error()
    assert ctx.launch_count() == before


def test_sharded_over_every_device(rh, oracle, monkeypatch):
    import torch

    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("one device")
    crops = crops_of(MIXED * 3, 16)
    ref, _ = oracle.rec_preprocess_batch(crops, threads=8)
    with rh.Context(list(range(n))) as c:
        got, _ = rh.RecPreprocess(ctx=c).process_batch(crops)
        assert_same(got, ref, f"{n} devices")
        # a shard whose device fails (injected on the host) is redone on a healthy device
        monkeypatch.setenv("RH_FAULT_DEVICE", "1")
        got2, _ = rh.RecPreprocess(ctx=c).process_batch(crops)
        assert_same(got2, ref, f"{n} devices, slot 1 failed")


def test_crops_out_of_order_shared_and_in_a_larger_buffer(rh, ctx, oracle):
    """Offsets need not follow line order: crops stored backwards, one crop used twice, and
    unrelated bytes around them in the pixel buffer."""
    import ctypes

    from rust_ppocrv6_b200._lib import load
    from rust_ppocrv6_b200.preprocess import _p

    dims = [(120, 33), (64, 50), (9, 2), (300, 60)]
    crops = crops_of(dims, 17)
    rng = np.random.default_rng(18)
    parts, offs = [rng.integers(0, 256, 37, dtype=np.uint8)], {}
    pos = 37
    for i in reversed(range(len(crops))):
        offs[i] = pos
        parts.append(crops[i].reshape(-1))
        pos += crops[i].size
        parts.append(rng.integers(0, 256, 11, dtype=np.uint8))
        pos += 11
    blob = np.concatenate(parts)
    order = [0, 1, 2, 3, 1]  # line 4 reuses crop 1's bytes
    offsets = np.array([offs[i] for i in order], np.int64)
    widths = np.array([dims[i][0] for i in order], np.uint32)
    heights = np.array([dims[i][1] for i in order], np.uint32)
    _, h, wmax = rh.batch_shape(widths, heights)
    out = np.empty((len(order), 3, h, wmax), np.float32)
    got_w = np.zeros(len(order), np.uint32)
    got_max = ctypes.c_uint32(0)
    rc = load().rh_rec_preprocess(ctx.handle, _p(blob), blob.size, _p(offsets), _p(widths), _p(heights), len(order),
                                  48, 960, _p(out), out.size, _p(got_w), ctypes.byref(got_max))
    assert rc == 0, load().rh_last_error()
    ref, _ = oracle.rec_preprocess_batch([crops[i] for i in order])
    assert_same(out, ref, "out of order")


def test_many_lines_run_in_pieces(rh, ctx, oracle):
    """600 lines: the host path cuts the batch into pieces of ~32 MB of output (58 lines at
    48 x 960) whose copies overlap the resize; every piece must land in its place."""
    rng = np.random.default_rng(19)
    hs = rng.integers(8, 90, 600)
    ws = rng.integers(1, 1400, 600)
    crops = [rng.integers(0, 256, (int(h), int(w), 3), dtype=np.uint8) for w, h in zip(ws, hs)]
    got, widths = rh.RecPreprocess(ctx=ctx).process_batch(crops)
    ref, ref_w = oracle.rec_preprocess_batch(crops, threads=8)
    assert np.array_equal(widths, ref_w)
    assert_same(got, ref, "600 lines")


def test_concurrent_callers_share_a_context(rh, ctx, oracle):
    """The engine calls preprocessing from several worker threads; calls on one context are
    serialised per device and each gets its own result."""
    from concurrent.futures import ThreadPoolExecutor

    batches = [crops_of(MIXED[:6] + [(200 + 10 * i, 40)], 20 + i) for i in range(6)]
    pre = rh.RecPreprocess(ctx=ctx)
    with ThreadPoolExecutor(6) as ex:
        results = list(ex.map(pre.process_batch, batches))
    for i, (got, _) in enumerate(results):
        ref, _ = oracle.rec_preprocess_batch(batches[i])
        assert_same(got, ref, f"thread {i}")


def test_wide_lines_staged_in_several_chunks(rh, ctx, oracle):
    """max_w = 4000: lines wider than one 2,048-column stage are resized in chunks of output
    columns, through the horizontal pass that reads its windows from the tables (kx = 2 and
    3); a narrow line in the same batch still stages its windows once per block."""
    dims = [(3000, 30), (1500, 20), (2900, 64), (100, 40), (4000, 10)]
    crops = crops_of(dims, 23)
    got, widths = rh.RecPreprocess(48, 4000, ctx=ctx).process_batch(crops)
    assert list(widths) == [4000, 3600, 2175, 120, 4000]
    ref, _ = oracle.rec_preprocess_batch(crops, 48, 4000, threads=4)
    assert_same(got, ref, "wide lines")


def _random_batches(seed=31, n_batches=24):
    """Seeded batches of crops of every shape class: text lines, tall/narrow, wide/flat, tiny
    or empty; random target heights and width caps."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n_batches):
        n = int(rng.integers(1, 9))
        th = int(rng.choice([1, 16, 32, 48, 64]))
        mw = int(rng.choice([8, 100, 320, 960, 2000, 4000]))
        dims = []
        for _ in range(n):
            kind = rng.integers(0, 4)
            if kind == 0:
                h = int(rng.integers(8, 100))
                w = int(h * rng.uniform(2, 30))
            elif kind == 1:
                w, h = int(rng.integers(1, 40)), int(rng.integers(40, 600))
            elif kind == 2:
                h, w = int(rng.integers(1, 12)), int(rng.integers(100, 9000))
            else:
                w, h = int(rng.integers(0, 6)), int(rng.integers(0, 6))
            dims.append((w, h))
        out.append((dims, th, mw))
    return out


def test_randomized_batches_bit_exact(rh, ctx, oracle):
    for i, (dims, th, mw) in enumerate(_random_batches()):
        crops = crops_of(dims, 100 + i)
        got, widths = rh.RecPreprocess(th, mw, ctx=ctx).process_batch(crops)
        ref, ref_w = oracle.rec_preprocess_batch(crops, th, mw, threads=8)
        assert np.array_equal(widths, ref_w), (i, dims, th, mw)
        assert_same(got, ref, f"batch {i}: {dims} H={th} max_w={mw}")


def test_every_staged_tap_count_bit_exact(rh, ctx, oracle):
    """One line per horizontal tap bound of the staged path: kx = ceil(2 s) is 2 (a line that
    grows), 3 and 4 (shrinking by up to 1.5x and 2x: the fourth weight comes from its own
    shared-memory array), and a line shrinking by more than 2x (the general path). With a
    48-row target the horizontal ratio is about h / 48."""
    dims = [(400, 40), (1200, 60), (1700, 85), (1900, 95), (2000, 100), (500, 30), (1300, 70)]
    ratios = [w / min(max(int(np.ceil(48 * w / h)), 32), 2000) for w, h in dims]
    kx = [int(np.ceil(2 * max(r, 1.0))) if max(r, 1.0) <= 2.0 else 0 for r in ratios]
    assert {2, 3, 4, 0} <= set(kx), kx
    for rep in range(3):
        crops = crops_of(dims, 300 + rep)
        got, widths = rh.RecPreprocess(48, 2000, ctx=ctx).process_batch(crops)
        ref, ref_w = oracle.rec_preprocess_batch(crops, 48, 2000, threads=4)
        assert np.array_equal(widths, ref_w)
        assert_same(got, ref, f"tap bounds {kx}, seed {300 + rep}")
