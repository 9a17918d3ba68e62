"""Full-size parity: every benchmark config decoded on the GPU through the C ABI
(rh_head_decode_lines) and checked row by row against the CPU oracle on all host threads.

The oracle runs ~1e5 timesteps/s on 16 host cores, so even cfg3's ~530k rows take seconds:
no config is sampled. Per config the summary at the end of the run reports the rows checked,
the argmax disagreements (each must sit at an oracle top-2 logit gap below 1e-5, a near-tie)
and the largest relative probability error where the argmax agrees.

Probability bar, per row: 1e-5 relative, plus two units in the last place of the row's largest
logit (f32). The reference's logits are f32 values, so a row whose largest logit is L carries
rounding of ~ulp(L) in every logit difference, and its probability moves by that much
relative: on cfg4, whose constructed near-tie rows reach L ~ 100-200, the reference's own
result is up to 8e-6 away from the exact (f64) probability. Where a row needs that allowance,
the summary also gives both sides' distance from the exact probability.

A row beyond that bar passes only through the logits it came from: its GPU logits (the
MatMul.12 drop-in on the same row) must meet the logits bar against the oracle's, and its fused
probability must equal the exact softmax of those same GPU logits within the probability bar.
The difference then lies in the logits, within their tolerance, not in the fused softmax.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TIE_GAP = 1e-5
PROB_REL_TOL = 1e-5
THREADS = os.cpu_count() or 1


@pytest.fixture(scope="module")
def rh():
    import rust_ppocrv6_b200 as rh

    rh.load()
    return rh


@pytest.fixture(scope="module")
def ctx(rh):
    c = rh.Context(devices=[0])
    yield c
    c.close()


def exact_prob_int8(x, q, s, bias):
    """1 / sum exp(l - max l) with the logits of the quantised head in f64 (no rounding but
    the final one): the probability both f32 implementations approximate."""
    lg = (x.astype(np.float64) @ q.astype(np.float64).T) * s.astype(np.float64) + bias.astype(np.float64)
    return 1.0 / np.exp(lg - lg.max(axis=1, keepdims=True)).sum(axis=1)


def exact_prob_f32(x, w_t, bias):
    lg = x.astype(np.float64) @ w_t.astype(np.float64).T + bias.astype(np.float64)
    return 1.0 / np.exp(lg - lg.max(axis=1, keepdims=True)).sum(axis=1)


def softmax_max_prob_f64(lg):
    lg = lg.astype(np.float64)
    return 1.0 / np.exp(lg - lg.max(axis=1, keepdims=True)).sum(axis=1)


def check_rows(label, idx, prob, ref, parity_log, tie_rows=None, exact=None, logits=None):
    """Asserts the parity bars on every row and records the statistics. `exact(rows)` gives the
    f64 probability of those rows (reported for the rows beyond 1e-5); `logits(rows)` gives
    (GPU logits, oracle logits, logits tolerance) of those rows, for the rows beyond the
    probability bar."""
    rows = idx.size
    assert ref["idx"].size == rows
    mism = idx != ref["idx"]
    gaps = ref["gap"][mism]
    assert np.all(gaps < TIE_GAP), f"[{label}] argmax differs where the top-2 gap is {gaps.max():.3g}"
    ok = ~mism
    rel_all = np.abs(prob.astype(np.float64) - ref["prob"]) / ref["prob"]
    tol = PROB_REL_TOL + 2.0 * np.spacing(np.abs(ref["lmax"]).astype(np.float32)).astype(np.float64)
    rel = rel_all[ok]
    worst = float(rel.max()) if rel.size else 0.0
    bad = np.flatnonzero(ok & (rel_all > tol))
    via_logits = ""
    if bad.size:
        assert logits is not None and bad.size <= 1000, (
            f"[{label}] {bad.size} rows beyond 1e-5 + 2 ulp(max logit); worst rel err {rel_all[bad].max():.3g}")
        got_l, ref_l, l_tol = logits(bad)
        l_err = np.abs(got_l.astype(np.float64) - ref_l)
        assert np.all(l_err <= l_tol), f"[{label}] logits beyond their bar on {int((l_err > l_tol).any(axis=1).sum())} rows"
        own = softmax_max_prob_f64(got_l)
        rel_own = np.abs(prob[bad].astype(np.float64) - own) / own
        assert np.all(rel_own <= tol[bad]), f"[{label}] fused prob vs its own logits: {rel_own.max():.3g}"
        via_logits = (f"; {bad.size} rows beyond 1e-5 + 2 ulp(max logit) (worst {rel_all[bad].max():.3g}) pass through"
                      f" their logits: GPU logits within the logits bar (max |diff| {l_err.max():.3g}), fused prob"
                      f" within {rel_own.max():.3g} of the exact softmax of those GPU logits")
    if mism.any():  # at a near-tie both classes carry (almost) the same probability
        assert rel_all[mism].max() <= 1e-3
    beyond = np.flatnonzero(ok & (rel_all > PROB_REL_TOL))
    line = (f"{label}: {rows} rows checked, {int(mism.sum())} near-tie argmax disagreements"
            f"{' (gaps < %.1g)' % TIE_GAP if mism.any() else ''}, max prob rel err {worst:.3g}")
    if beyond.size:
        line += (f" ({beyond.size} rows above 1e-5, largest logit there up to {np.abs(ref['lmax'][beyond]).max():.4g}")
        if exact is not None:
            worst_rows = np.argsort(rel_all)[-min(32, rows):]
            pe = exact(worst_rows)
            ours = np.abs(prob[worst_rows] - pe) / pe
            theirs = np.abs(ref["prob"][worst_rows] - pe) / pe
            line += (f"; on the {worst_rows.size} worst rows the distance from the exact f64 probability is "
                     f"<= {ours.max():.3g} here and <= {theirs.max():.3g} for the reference")
        line += ")"
    line += via_logits
    if tie_rows is not None:
        line += (f", {tie_rows.size} constructed near-tie rows ({int(mism[tie_rows].sum())} of them"
                 f" decoded to the other class of the pair)")
    parity_log.append(line)
    return int(mism.sum())


@pytest.mark.parametrize("cfg,compact", [(0, False), (1, False), (2, False), (3, False), (4, False), (5, False),
                                         (2, True), (4, True)])
def test_every_row_of_every_config_int8(rh, ctx, oracle, parity_log, cfg, compact):
    """cfg0 one line, cfg1 64 ragged lines, cfg2 1024 x 120, cfg3 8192 ragged lines (~530k
    rows), cfg4 256 x 240 with Student-t weights and 5 % constructed near-ties, cfg5 the tiny
    model's head (K=80, N=6906): the quantised head, every row (cfg2 and cfg4 also with the
    compact int8 weight form)."""
    from rust_ppocrv6_b200 import workloads

    wl = workloads.make(cfg)
    qw = rh.QuantizedWeight.from_f32_transposed(wl.w_t, ctx=ctx, bias=wl.bias, compact=compact)
    q, s = oracle.pack(wl.w_t)
    assert np.array_equal(qw.data, q) and np.array_equal(qw.scales.view(np.uint32), s.view(np.uint32))
    idx, prob = rh.head_decode(wl.x, qw, line_offsets=wl.line_offsets)
    ref = oracle.head_decode(wl.x, wl.line_offsets, q, s, wl.bias, threads=THREADS, want_gap=True)

    def logits(r):
        got = rh.matmul_quantized_b(wl.x[r], qw, wl.bias)
        want = oracle.matmul_quantized_b(wl.x[r], q, s, wl.bias).astype(np.float64)
        return got, want, 1e-4 + 2e-6 * np.abs(want)

    check_rows(f"cfg{cfg} int8{' compact' if compact else ''}", idx, prob, ref, parity_log,
               wl.tie_rows if cfg == 4 else None, exact=lambda r: exact_prob_int8(wl.x[r], q, s, wl.bias),
               logits=logits)
    if cfg == 4:
        assert np.all(ref["gap"][wl.tie_rows] < 1.2e-4)  # the construction did build near-ties
    qw.free()


@pytest.mark.parametrize("cfg", [2, 4])
def test_every_row_fp32_head(rh, ctx, oracle, parity_log, cfg):
    """The engine's default FP32 head (quantize_rec_head = false) on cfg2 and the cfg4 stress
    set, against the reference's register-blocked matmul_transposed_b restated."""
    from rust_ppocrv6_b200 import workloads

    wl = workloads.make(cfg)
    fw = rh.Fp32Weight.from_f32_transposed(wl.w_t, ctx=ctx, bias=wl.bias)
    idx, prob = rh.head_decode(wl.x, fw, line_offsets=wl.line_offsets)
    ref = oracle.head_decode_f32(wl.x, wl.line_offsets, wl.w_t, wl.bias, threads=THREADS, want_gap=True)

    def logits(r):
        # the FP32 logits bar: 1e-4 plus 2e-6 of the sum of |terms| (the error any f32 dot
        # product carries, the reference's FP32 kernel included)
        got = rh.matmul_transposed_b(wl.x[r], fw, wl.bias)
        want = oracle.matmul_transposed_b(wl.x[r], wl.w_t, wl.bias).astype(np.float64)
        terms = np.abs(wl.x[r]).astype(np.float64) @ np.abs(wl.w_t).astype(np.float64).T
        return got, want, 1e-4 + 2e-6 * terms

    check_rows(f"cfg{cfg} fp32", idx, prob, ref, parity_log, exact=lambda r: exact_prob_f32(wl.x[r], wl.w_t, wl.bias),
               logits=logits)
    fw.free()


def test_every_row_of_cfg2_through_the_device_entry_point_and_the_svtr_layout(rh, ctx, oracle, parity_log):
    """cfg2 through rh_head_decode_device (features already in HBM, the bench's timed call) and
    through rh_head_decode_kt (the SVTR tail's [B, K, T] layout): every row against the oracle."""
    import torch

    from rust_ppocrv6_b200 import workloads

    wl = workloads.make(2)
    qw = rh.QuantizedWeight.from_f32_transposed(wl.w_t, ctx=ctx, bias=wl.bias)
    q, s = oracle.pack(wl.w_t)
    ref = oracle.head_decode(wl.x, wl.line_offsets, q, s, wl.bias, threads=THREADS, want_gap=True)
    m = wl.rows
    dx = torch.from_numpy(wl.x).cuda()
    di = torch.empty(m, dtype=torch.int32, device="cuda")
    dp = torch.empty(m, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    rh.head_decode_device(qw, dx.data_ptr(), m, di.data_ptr(), dp.data_ptr())
    ctx.sync()
    check_rows("cfg2 int8 device entry point", di.cpu().numpy(), dp.cpu().numpy(), ref, parity_log)
    xt = np.ascontiguousarray(wl.x.reshape(1024, 120, workloads.K).transpose(0, 2, 1))
    idx, prob = rh.head_decode_kt(xt, qw)
    check_rows("cfg2 int8 [B,K,T] layout", idx.reshape(-1), prob.reshape(-1), ref, parity_log)
    qw.free()
