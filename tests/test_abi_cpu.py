"""CPU-only checks of the boundary: the C-ABI library builds, loads and exports every symbol
include/rechead.h declares; the host-only parts (CTC collapse, CtcDecoder mirror, line
sharding) behave like the reference; and with no GPU the compute path fails loudly
instead of falling back to the CPU."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def rh():
    import rust_ppocrv6_b200 as rh

    rh.load()
    return rh


def test_library_exports_every_declared_symbol(rh):
    lib_path = os.path.join(ROOT, "rust_ppocrv6_b200", "librechead.so")
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    declared = rh.header_symbols()
    assert len(declared) >= 20
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    lib = rh.load()
    for s in declared:
        assert hasattr(lib, s)


def test_no_device_fails_loudly(rh):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(rh.RecHeadError) as e:
        rh.Context()
    assert e.value.code == rh.RH_ERR_NO_DEVICE
    with pytest.raises(rh.RecHeadError):
        rh.QuantizedWeight.from_f32_transposed(np.zeros((4, 8), np.float32))


def test_host_collapse_matches_oracle(rh, oracle):
    rng = np.random.default_rng(2)
    off = np.concatenate([[0], np.cumsum(rng.integers(0, 40, size=50))]).astype(np.int64)
    m = int(off[-1])
    idx = rng.integers(0, 6, size=m).astype(np.int32)  # many blanks and repeats
    prob = rng.random(m).astype(np.float32)
    dec = rh.CtcDecoder.from_vocab(["blank", "a", "b", "c", "d", " "])
    toks, scores = dec.collapse(idx, prob, off)
    rtoks, rscores = oracle.ctc_collapse(idx, prob, off)
    assert [t.tolist() for t in toks] == [t.tolist() for t in rtoks]
    assert np.array_equal(scores.view(np.uint32), rscores.view(np.uint32))


def test_decoder_mirrors_reference_ctc_tests(rh, oracle, tmp_path):
    """src/postprocess/ctc.rs:272-363 on the (idx, prob) interface."""
    dec = rh.CtcDecoder.from_vocab(["blank", "a", "b", " "])
    # a, a, blank, b -> "ab", score 1
    probs = np.zeros((4, 4), np.float32)
    for t, c in [(0, 1), (1, 1), (2, 0), (3, 2)]:
        probs[t, c] = 1.0
    idx = np.array([oracle.find_argmax(r)[0] for r in probs], np.int32)
    val = np.array([oracle.find_argmax(r)[1] for r in probs], np.float32)
    text, score = dec.decode(idx, val, n_classes=4)
    assert text == "ab" and abs(score - 1.0) < 1e-6
    # dictionary mismatch is an error, not silent truncation
    with pytest.raises(rh.RecHeadError) as e:
        rh.CtcDecoder.from_vocab(["blank", "a", " "]).decode(idx, val, n_classes=4)
    assert "mismatch" in str(e.value)
    # empty batch decodes to ("", 0.0)
    assert dec.decode(np.zeros(0, np.int32), np.zeros(0, np.float32), n_classes=4) == ("", 0.0)
    # batch of two lines -> "ab", "b"
    res = dec.decode_indices(np.array([1, 2, 2, 0], np.int32), np.ones(4, np.float32), np.array([0, 2, 4]))
    assert [r[0] for r in res] == ["ab", "b"]
    # from_file: blank + lines + trailing space
    p = tmp_path / "keys.txt"
    p.write_text("x\ny\r\nz\n", encoding="utf-8")
    d2 = rh.CtcDecoder.from_file(str(p))
    assert d2.vocab == ["blank", "x", "y", "z", " "] and d2.vocab_size == 5


def test_collapse_rejects_bad_offsets(rh):
    dec = rh.CtcDecoder.from_vocab(["blank", "a", " "])
    with pytest.raises(rh.RecHeadError):
        dec.collapse(np.zeros(4, np.int32), np.zeros(4, np.float32), np.array([0, 3, 2]))
    with pytest.raises(rh.RecHeadError):
        dec.collapse(np.zeros(4, np.int32), np.zeros(4, np.float32), np.array([0, 5]))


def test_shard_lines_partition(rh):
    from rust_ppocrv6_b200 import workloads

    rng = np.random.default_rng(9)
    off = workloads.ragged_offsets(rng, 8192)
    for world in (1, 2, 3, 4, 8):
        ranges = [workloads.shard_lines(off, world, r) for r in range(world)]
        assert ranges[0][0] == 0 and ranges[-1][1] == 8192
        for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
            assert a1 == b0 and a0 <= a1
        rows = [off[b] - off[a] for a, b in ranges]
        assert max(rows) - min(rows) <= 2 * 120 + 1


def test_workload_generators(rh):
    from rust_ppocrv6_b200 import workloads

    wl = workloads.make(0)
    assert wl.x.shape == (120, 120) and wl.w_t.shape == (18710, 120) and wl.bias.shape == (18710,)
    assert abs(float(wl.w_t.std()) - 0.05) < 1e-3
    wl1 = workloads.make(1)
    t = np.diff(wl1.line_offsets)
    assert t.size == 64 and t.min() >= 10 and t.max() <= 120
    wl4 = workloads.make(4, scale=4 / 256)
    assert wl4.x.shape == (960, 120) and wl4.tie_rows.size == 48
