"""Pins the CPU oracle to the reference: the reference's own unit tests for this path,
re-run against oracle/ref_w8a32.c with the same input generators and tolerances, plus the
pack of real PP-OCRv6 head weights checked bit-exact against an independent numpy
restatement (tests/golden/real_head_slice.npz).

Each test names the reference test it restates (file:line inside rust-ppocrv6).
"""
import math
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "real_head_slice.npz")


def sinpat(count, mul, amp=1.0, cos=False):
    i = np.arange(count, dtype=np.float32) * np.float32(mul)
    return ((np.cos(i) if cos else np.sin(i)) * np.float32(amp)).astype(np.float32)


# ---------------------------------------------------------------- pack


def test_pack_real_weights_bit_exact_vs_numpy_restatement(oracle):
    g = np.load(GOLDEN)
    q, s = oracle.pack(g["w_t"])
    assert np.array_equal(q, g["q"])
    assert np.array_equal(s.view(np.uint32), g["scales"].view(np.uint32))
    # the real head matches the distribution quoted for it (std 0.042, mean -0.033)
    assert abs(float(g["stats"][0]) + 0.0327) < 1e-3 and abs(float(g["stats"][1]) - 0.0424) < 1e-3


def test_pack_edge_rows(oracle):
    # zero row -> scale 1, q 0; tiny row (max <= 1e-8) -> scale 1; half-way rounding is
    # away from zero (f32::round); NaN is ignored by f32::max and casts to 0.
    w = np.zeros((5, 8), np.float32)
    w[1, :] = 5e-9
    w[2, :] = [127.0, 63.5, -63.5, 0.5, -0.5, 1.5, -1.5, 0.0]
    w[3, :] = [1.0, np.nan, -2.0, 0, 0, 0, 0, 0]
    w[4, :] = [3e38, -3e38, 1e-30, 0, 0, 0, 0, 0]
    q, s = oracle.pack(w)
    assert s[0] == 1.0 and not q[0].any()
    assert s[1] == 1.0 and not q[1].any()
    assert s[2] == np.float32(1.0)
    assert q[2].tolist() == [127, 64, -64, 1, -1, 2, -2, 0]
    assert q[3].tolist()[:3] == [64, 0, -127]
    assert q[4].tolist()[:3] == [127, -127, 0]


# ------------------------------------------------------- projection


def test_quantized_matmul_handles_leading_batch_dims(oracle):
    """src/ops/matmul.rs:1673-1697."""
    batch, k, n = 3, 8, 1024
    bt = sinpat(n * k, 0.07).reshape(n, k)
    q, s = oracle.pack(bt)
    a = sinpat(batch * k, 0.11, cos=True).reshape(batch, 1, k)
    got = oracle.matmul_quantized_b(a, q, s, None)
    assert got.shape == (batch, 1, n)
    fp32 = oracle.matmul_transposed_b(a, bt)
    assert np.all(np.abs(got - fp32) <= 0.05 + 0.05 * np.abs(fp32))


def test_a_wrong_length_bias_is_an_error(oracle):
    """src/ops/matmul.rs:1700-1721 (FP32 sibling); the INT8 check is :1288-1295."""
    a = np.arange(8, dtype=np.float32).reshape(1, 8)
    q, s = oracle.pack(np.ones((16, 8), np.float32))
    for n_bias in (0, 1, 15, 17):
        with pytest.raises(ValueError):
            oracle.matmul_quantized_b(a, q, s, np.full(n_bias, 0.25, np.float32))
    oracle.matmul_quantized_b(a, q, s, np.full(16, 0.25, np.float32))


def test_matmul_quantized_b_tracks_fp32_within_quantization_error(oracle):
    """src/ops/matmul.rs:1812-1840."""
    k, n = 64, 48
    a = (sinpat(k, 0.19) * np.float32(2.0)).reshape(1, k)
    i = np.arange(n * k)
    w = (np.cos(i.astype(np.float32) * np.float32(0.07)) * np.float32(0.5)
         + (i % 11).astype(np.float32) * np.float32(0.01)).astype(np.float32).reshape(n, k)
    q, s = oracle.pack(w)
    fp32 = oracle.matmul_transposed_b(a, w)
    int8 = oracle.matmul_quantized_b(a, q, s, None)
    max_abs = np.max(np.abs(fp32))
    tol = 1e-4 + 0.02 * np.abs(fp32) + 0.02 * max_abs
    assert np.all(np.abs(int8 - fp32) <= tol)


@pytest.mark.skipif("not __import__('oracle.oracle', fromlist=['x']).has_avx2()")
def test_matmul_quantized_b_avx2_matches_scalar(oracle):
    """src/ops/matmul.rs:1879-1904 (K and N tails: K=123, N=533)."""
    m, k, n = 1, 123, 533
    a = sinpat(m * k, 0.083).reshape(m, k)
    w = (sinpat(n * k, 0.037, cos=True) * np.float32(1.3)).reshape(n, k)
    q, s = oracle.pack(w)
    scalar = oracle.matmul_quantized_b(a, q, s, None, use_avx2=False)
    avx2 = oracle.matmul_quantized_b(a, q, s, None, use_avx2=True)
    assert np.all(np.abs(avx2 - scalar) <= 1e-4 + 1e-4 * np.abs(scalar))


def test_matmul_rejects_incompatible_inner_dimensions(oracle):
    """src/ops/matmul.rs:1842-1848."""
    q, s = oracle.pack(np.zeros((2, 4), np.float32))
    with pytest.raises(ValueError):
        oracle.matmul_quantized_b(np.zeros((2, 3), np.float32), q, s, None)


def test_colsplit_schedule_close_to_serial(oracle):
    """The column-split schedule (:1297-1328) only moves columns between the 4-wide and the
    tail kernels, so it agrees with the serial one to rounding."""
    rng = np.random.default_rng(1)
    a = rng.standard_normal((3, 120), dtype=np.float32)
    w = (rng.standard_normal((1000, 120)) * 0.05).astype(np.float32)
    q, s = oracle.pack(w)
    b = (rng.standard_normal(1000) * 0.01).astype(np.float32)
    ser = oracle.matmul_quantized_b(a, q, s, b)
    for th in (1, 3, 7):
        cs = oracle.matmul_quantized_b_colsplit(a, q, s, b, threads=th)
        assert np.max(np.abs(cs - ser)) <= 1e-5


# ---------------------------------------------- FP32 projection (matmul_transposed_b)


def _ref_transposed_b(a, b_t):
    """reference_transposed_b of src/ops/matmul.rs:1539-1550: the f64 product per row."""
    return a.astype(np.float64) @ b_t.astype(np.float64).T


def test_fp32_matmul_handles_leading_batch_dims(oracle):
    """src/ops/matmul.rs:1559-1588 ([3, 1, K] input)."""
    batch, k, n = 3, 8, 1024
    bt = sinpat(n * k, 0.07).reshape(n, k)
    a = sinpat(batch * k, 0.11, cos=True).reshape(batch, 1, k)
    got = oracle.matmul_transposed_b(a, bt)
    assert got.shape == (batch, 1, n)
    assert np.all(np.abs(got.reshape(batch, n) - _ref_transposed_b(a.reshape(batch, k), bt)) < 1e-4)


@pytest.mark.skipif("not __import__('oracle.oracle', fromlist=['x']).has_avx2()")
@pytest.mark.parametrize("shape", [(3, 1, 8), (2, 3, 8), (4, 1, 16)])
def test_fp32_matmul_identical_on_both_paths(oracle, shape):
    """src/ops/matmul.rs:1590-1636: scalar and AVX2 paths agree and both match f64."""
    batch, m, k = shape
    n = 1024
    bt = sinpat(n * k, 0.03, cos=True).reshape(n, k)
    a = sinpat(batch * m * k, 0.05).reshape(shape)
    scalar = oracle.matmul_transposed_b(a, bt, use_avx2=False)
    wide = oracle.matmul_transposed_b(a, bt, use_avx2=True)
    assert np.all(np.abs(wide - scalar) <= 1e-4 + 1e-4 * np.abs(scalar))
    ref = _ref_transposed_b(a.reshape(-1, k), bt)
    assert np.all(np.abs(scalar.reshape(-1, n) - ref) < 1e-4)


def test_fp32_blocked_kernel_ragged_edges(oracle):
    """src/ops/matmul.rs:1638-1671: rows 1..TILE_ROWS+2, column tails 0..3, with and without
    a bias (which pins the column offset the tile reads it at)."""
    k = 8
    for n_tail in range(4):
        n = 4 * 6 + n_tail
        bt = sinpat(n * k, 0.031, cos=True).reshape(n, k)
        for rows in range(1, 3 + 3):
            a = sinpat(rows * k, 0.07).reshape(rows, k)
            for bias in (None, np.full(n, 0.5, np.float32)):
                got = oracle.matmul_transposed_b(a, bt, bias)
                want = _ref_transposed_b(a, bt) + (0.5 if bias is not None else 0.0)
                assert got.shape == (rows, n)
                assert np.all(np.abs(got - want) < 1e-4), (n, rows, bias is not None)


def test_fp32_matmul_argument_errors(oracle):
    """src/ops/matmul.rs:1700-1721 and the inner-dimension check :531-536."""
    a = np.arange(8, dtype=np.float32).reshape(1, 8)
    bt = np.ones((16, 8), np.float32)
    for n_bias in (0, 1, 15, 17):
        with pytest.raises(ValueError):
            oracle.matmul_transposed_b(a, bt, np.full(n_bias, 0.25, np.float32))
    with pytest.raises(ValueError):
        oracle.matmul_transposed_b(np.zeros((2, 7), np.float32), bt)


@pytest.mark.skipif("not __import__('oracle.oracle', fromlist=['x']).has_avx2()")
def test_fp32_head_shape_rows_and_fused_decode(oracle):
    """The recognition head's shape (n = 18710: a tail of 2 columns through avx2_dot_product,
    the rest through the blocked tile): within 1e-4 of the f64 product, each row's bits
    independent of the row group of 3 it falls in, and the per-line fused decode equal to
    projection -> softmax -> find_argmax."""
    rng = np.random.default_rng(5)
    n, k, m = 18710, 120, 7
    bt = (0.05 * rng.standard_normal((n, k))).astype(np.float32)
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = (0.01 * rng.standard_normal(n)).astype(np.float32)
    got = oracle.matmul_transposed_b(a, bt, b)
    ref = _ref_transposed_b(a, bt) + b
    assert np.max(np.abs(got - ref)) < 1e-4
    # rows are independent of their grouping: one row at a time gives the same bits
    for r in range(m):
        one = oracle.matmul_transposed_b(a[r:r + 1], bt, b)
        assert np.array_equal(one.view(np.uint32), got[r:r + 1].view(np.uint32))
    # per-line fused head over the FP32 projection = projection -> softmax -> argmax
    off = np.array([0, 3, 7], np.int64)
    h = oracle.head_decode_f32(a, off, bt, b, threads=2, want_logits=True, want_gap=True)
    assert np.array_equal(h["logits"].view(np.uint32), got.view(np.uint32))
    p = oracle.softmax_lastaxis(got)
    for r in range(m):
        i, v = oracle.find_argmax(p[r])
        assert h["idx"][r] == i and h["prob"][r] == np.float32(v)


# ------------------------------------------------------------- softmax


def softmax_f64(x, axis):
    x = x.astype(np.float64)
    e = np.exp(x - x.max(axis=axis, keepdims=True))
    return e / e.sum(axis=axis, keepdims=True)


def test_softmax_matches_f64_reference_on_last_axis(oracle):
    """src/ops/softmax.rs:483-508."""
    data = np.array([1.0, 2.0, 3.0, 4.0, 5.0, -1.0, 0.0, 0.0, 0.5, 100.0, 0.25, -0.25, 0.75, -0.75, 0.0],
                    np.float32).reshape(3, 5)
    out = oracle.softmax_lastaxis(data)
    assert out.shape == (3, 5)
    assert np.all(np.abs(out - softmax_f64(data, 1)) <= 1e-6)
    assert np.all(np.abs(out.sum(axis=1) - 1.0) < 1e-5)


def test_softmax_matches_f64_reference_on_middle_axis(oracle):
    """src/ops/softmax.rs:510-523 (general inner_size > 1 path)."""
    data = (sinpat(24, 0.37) * np.float32(3.0)).reshape(2, 4, 3)
    out = oracle.softmax_general(data, 1)
    assert np.all(np.abs(out - softmax_f64(data, 1)) <= 1e-6)


def test_softmax_is_stable_on_large_magnitudes(oracle):
    """src/ops/softmax.rs:525-542."""
    data = np.array([1000.0, 1001.0, 999.0, 1000.5, -1000.0, -999.0, -1001.0, -1000.5], np.float32).reshape(2, 4)
    out = oracle.softmax_lastaxis(data)
    assert np.all(np.isfinite(out))
    assert np.all(np.abs(out.sum(axis=1) - 1.0) < 1e-5)


@pytest.mark.parametrize("shape", [(0,), (3, 0), (2, 5, 0), (1, 1, 0, 4)])
def test_softmax_empty_input_returns_empty(oracle, shape):
    """src/ops/softmax.rs:553-570."""
    out = oracle.softmax_lastaxis(np.full(shape, 0.5, np.float32))
    assert out.shape == shape and out.size == 0


def test_single_row_softmax_still_works(oracle):
    """src/ops/softmax.rs:572-579."""
    out = oracle.softmax_lastaxis(np.array([1.0, 2.0, 3.0], np.float32))
    assert abs(float(out.sum()) - 1.0) < 1e-6 and out[2] > out[1]


@pytest.mark.skipif("not __import__('oracle.oracle', fromlist=['x']).has_avx2()")
def test_softmax_avx2_row_matches_scalar(oracle):
    """src/ops/softmax.rs:581-599."""
    i = np.arange(1600)
    data = (np.sin(i.astype(np.float32) * np.float32(0.113)) * np.float32(6.0)
            + (i % 7).astype(np.float32) * np.float32(0.5)).astype(np.float32).reshape(1, 1, 40, 40)
    scalar = oracle.softmax_lastaxis(data, use_avx2=False)
    avx2 = oracle.softmax_lastaxis(data, use_avx2=True)
    assert np.all(np.abs(avx2 - scalar) <= 1e-6 + 1e-5 * np.abs(scalar))


def test_exp_polynomial_properties(oracle):
    """avx2_exp_ps (src/ops/softmax.rs:5-47): exp(0) is exactly 1, so the max probability of a
    row is exactly 1/sum; the polynomial tracks exp to ~1e-7 relative on the softmax range."""
    assert oracle.exp_poly(0.0) == 1.0
    for x in np.linspace(-30.0, 0.0, 301):
        e = oracle.exp_poly(float(x))
        assert abs(e - math.exp(float(np.float32(x)))) <= 2e-7 * math.exp(float(x)) + 1e-30
        assert e <= 1.0


# ----------------------------------------------------------------- CTC


def test_find_argmax_avx2_matches_scalar(oracle):
    """src/postprocess/ctc.rs:309-328."""
    data = np.full(18710, 0.01, np.float32)
    data[42] = 0.95
    data[1000] = 0.88
    assert oracle.find_argmax(data) == oracle.find_argmax_scalar(data)
    assert oracle.find_argmax(data)[0] == 42
    data2 = np.full(35, -1.0, np.float32)
    data2[34] = 10.0
    assert oracle.find_argmax(data2) == oracle.find_argmax_scalar(data2) == (34, 10.0)


def test_find_argmax_first_index_on_ties(oracle):
    for n in (5, 16, 35, 18710):
        for pos in sorted({p for p in (0, 1, 7, 8, n // 2, n - 1) if p < n}):
            d = np.zeros(n, np.float32)
            d[pos] = 1.0
            d[n - 1] = 1.0
            assert oracle.find_argmax(d)[0] == pos
            assert oracle.find_argmax_scalar(d)[0] == pos


def one_hot(seq_len, vocab, picks):
    d = np.zeros((seq_len, vocab), np.float32)
    for t, c in picks:
        d[t, c] = 1.0
    return d


def test_decode_collapses_repeats_and_blank(oracle):
    """src/postprocess/ctc.rs:272-284: frames a, a, blank, b -> "ab", score 1."""
    probs = one_hot(4, 4, [(0, 1), (1, 1), (2, 0), (3, 2)])
    idx = np.array([oracle.find_argmax(r)[0] for r in probs], np.int32)
    val = np.array([oracle.find_argmax(r)[1] for r in probs], np.float32)
    toks, scores = oracle.ctc_collapse(idx, val, np.array([0, 4]))
    assert toks[0].tolist() == [1, 2] and abs(scores[0] - 1.0) < 1e-6


def test_decode_batch_decodes_multiple_lines(oracle):
    """src/postprocess/ctc.rs:338-363: batch lines (a, b) and (b, blank) -> "ab", "b"."""
    probs = np.zeros((2, 2, 4), np.float32)
    probs[0, 0, 1] = probs[0, 1, 2] = probs[1, 0, 2] = probs[1, 1, 0] = 1.0
    flat = probs.reshape(4, 4)
    idx = np.array([oracle.find_argmax(r)[0] for r in flat], np.int32)
    val = np.array([oracle.find_argmax(r)[1] for r in flat], np.float32)
    toks, _ = oracle.ctc_collapse(idx, val, np.array([0, 2, 4]))
    assert [t.tolist() for t in toks] == [[1, 2], [2]]


def test_collapse_empty_and_blank_lines(oracle):
    toks, scores = oracle.ctc_collapse(np.zeros(0, np.int32), np.zeros(0, np.float32), np.array([0]))
    assert toks == [] and scores.size == 0
    toks, scores = oracle.ctc_collapse(np.zeros(3, np.int32), np.ones(3, np.float32), np.array([0, 0, 3]))
    assert [t.tolist() for t in toks] == [[], []] and scores.tolist() == [0.0, 0.0]


# ------------------------------------------------------- whole head


def test_head_decode_matches_composition(oracle):
    """MatMul.12 (+ folded Add.204) -> Softmax.2 -> find_argmax, as src/engine/model.rs:1245-1302
    and src/postprocess/ctc.rs:144-149 chain them; independent of the thread count."""
    rng = np.random.default_rng(7)
    n, k = 777, 120
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    b = (rng.standard_normal(n) * 0.01).astype(np.float32)
    q, s = oracle.pack(w)
    a = rng.standard_normal((50, k), dtype=np.float32)
    off = np.array([0, 7, 7, 30, 50])
    ref_logits = oracle.matmul_quantized_b(a, q, s, b)
    ref_p = oracle.softmax_lastaxis(ref_logits)
    exp_idx = np.array([oracle.find_argmax(r)[0] for r in ref_p])
    exp_val = np.array([oracle.find_argmax(r)[1] for r in ref_p], np.float32)
    for th in (1, 3):
        h = oracle.head_decode(a, off, q, s, b, threads=th, want_logits=True, want_gap=True)
        assert np.array_equal(h["logits"].view(np.uint32), ref_logits.view(np.uint32))
        assert np.array_equal(h["idx"], exp_idx)
        assert np.array_equal(h["prob"].view(np.uint32), exp_val.view(np.uint32))
        assert np.all(h["gap"] >= 0)


def test_int8_head_footprint_at_least_3p5x_smaller():
    """src/engine/model.rs:2836-2941: the INT8 head (i8 payload + f32 scales) is at least 3.5x
    smaller than the FP32 transposed copy it replaces."""
    n, k = 18710, 120
    head_fp32 = n * k * 4
    head_int8 = n * k + n * 4
    assert head_int8 * 7 < head_fp32 * 2
