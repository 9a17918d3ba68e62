"""Recognition preprocessing on the CPU: the oracle's restatement pinned to the reference's
own unit tests (src/preprocess/rec.rs:108-182) and to an independent pure-Python
restatement of the resampler, plus the host-only parts of the C ABI (width rule, batch
shape, argument checks). No GPU needed."""
import numpy as np
import pytest

INV = np.float32(1.0) / np.float32(127.5)


def solid(w, h, rgb=(128, 64, 32)):
    a = np.zeros((h, w, 3), np.uint8)
    a[:, :] = rgb
    return a


# --------------------------------------------- the reference's rec.rs unit tests, on the oracle

def test_max_w_below_lower_bound_does_not_panic(oracle):
    assert oracle.rec_preprocess(solid(100, 10), 48, 8).shape == (1, 3, 48, 32)


def test_zero_target_h_is_clamped_to_one(oracle):
    assert oracle.rec_preprocess(solid(64, 64), 0, 960).shape == (1, 3, 1, 32)


def test_wide_image_respects_max_w(oracle):
    assert oracle.rec_preprocess(solid(1000, 10), 48, 200).shape[3] == 200


def test_extreme_aspect_ratio_saturates_instead_of_overflowing(oracle):
    assert oracle.rec_preprocess(solid(65_000, 1), 48, 960).shape == (1, 3, 48, 960)


def test_floor_is_32_not_the_reference_320(oracle):
    assert oracle.rec_preprocess(solid(50, 100), 48, 960).shape == (1, 3, 48, 32)


def test_output_is_a_tight_crop_with_no_padding(oracle):
    t = oracle.rec_preprocess(solid(400, 40, (0, 0, 0)), 48, 960)
    assert t.shape == (1, 3, 48, 480)
    assert np.all(np.abs(t[0, 2, 0, :] - (-1.0)) < 1e-6)


# ----------------------------------------------------------- properties of the restatement

def _py_window(n_in, n_out, o):
    f = np.float32
    ratio = f(n_in) / f(n_out)
    s = f(1.0) if ratio < f(1.0) else ratio
    centre = (f(o) + f(0.5)) * ratio
    lo = min(max(int(np.floor(centre - s)), 0), n_in - 1)
    hi = min(max(int(np.ceil(centre + s)), lo + 1), n_in)
    c0 = centre - f(0.5)
    ws = []
    for i in range(lo, hi):
        x = abs((f(i) - c0) / s)
        ws.append(f(1.0) - x if x < f(1.0) else f(0.0))
    total = f(0.0)
    for w in ws:
        total = total + w
    return lo, [w / total for w in ws]


def _py_resize(img, nw, nh):
    """Independent restatement (pure Python, float32 scalars): vertical pass, then horizontal."""
    h, w = img.shape[:2]
    if w == 0 or h == 0:
        return np.zeros((nh, nw, 3), np.uint8)
    tmp = np.zeros((nh, w, 3), np.float32)
    for oy in range(nh):
        top, ws = _py_window(h, nh, oy)
        for x in range(w):
            for c in range(3):
                t = np.float32(0.0)
                for j, wj in enumerate(ws):
                    t = t + np.float32(img[top + j, x, c]) * wj
                tmp[oy, x, c] = t
    out = np.zeros((nh, nw, 3), np.uint8)
    for ox in range(nw):
        left, ws = _py_window(w, nw, ox)
        for y in range(nh):
            for c in range(3):
                t = np.float32(0.0)
                for j, wj in enumerate(ws):
                    t = t + tmp[y, left + j, c] * wj
                t = min(max(t, np.float32(0.0)), np.float32(255.0))
                out[y, ox, c] = int(np.floor(np.float64(t) + 0.5))  # half away from zero (t >= 0; exact in f64)
    return out


@pytest.mark.parametrize("src,dst", [((7, 5), (11, 9)), ((13, 4), (5, 3)), ((9, 9), (9, 4)), ((1, 6), (32, 48)),
                                     ((40, 2), (3, 7)), ((6, 1), (2, 48))])
def test_resampler_matches_independent_restatement(oracle, src, dst):
    rng = np.random.default_rng(hash(src + dst) & 0xFFFF)
    (w, h), (nw, nh) = src, dst
    img = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
    assert np.array_equal(oracle.resize_triangle_rgb8(img, nw, nh), _py_resize(img, nw, nh))


def test_resize_to_the_same_size_is_the_identity(oracle):
    rng = np.random.default_rng(3)
    for w, h in [(1, 1), (32, 48), (300, 48), (7, 13)]:
        img = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
        assert np.array_equal(oracle.resize_triangle_rgb8(img, w, h), img)
    # through process(): a 48-row crop whose width is already in [32, max_w] is only normalised
    img = rng.integers(0, 256, (48, 300, 3), dtype=np.uint8)
    got = oracle.rec_preprocess(img)[0]
    assert np.array_equal(got, img.transpose(2, 0, 1).astype(np.float32) * INV - np.float32(1.0))


def test_solid_colours_stay_solid(oracle):
    rng = np.random.default_rng(4)
    for _ in range(12):
        w, h = int(rng.integers(1, 400)), int(rng.integers(1, 80))
        rgb = tuple(int(v) for v in rng.integers(0, 256, 3))
        t = oracle.rec_preprocess(solid(w, h, rgb))[0]
        for c in range(3):
            assert np.all(t[c] == np.float32(rgb[c]) * INV - np.float32(1.0)), (w, h, rgb, c)


def test_empty_crop_is_black(oracle):
    # height 0 counts as 1 for the aspect ratio (rec.rs:62): 10 / 1 * 48 = 480 columns, all black
    t = oracle.rec_preprocess(np.zeros((0, 10, 3), np.uint8))
    assert t.shape == (1, 3, 48, 480) and np.all(t == -1.0)
    t = oracle.rec_preprocess(np.zeros((7, 0, 3), np.uint8))
    assert t.shape == (1, 3, 48, 32) and np.all(t == -1.0)


def test_batch_pads_with_white_and_matches_single_crops(oracle):
    rng = np.random.default_rng(5)
    crops = [rng.integers(0, 256, (int(h), int(w), 3), dtype=np.uint8)
             for w, h in [(100, 30), (40, 40), (900, 20), (10, 60), (0, 5)]]
    out, widths = oracle.rec_preprocess_batch(crops, threads=3)
    assert out.shape == (5, 3, 48, int(widths.max()))
    for i, c in enumerate(crops):
        one = oracle.rec_preprocess(c)[0]
        assert np.array_equal(out[i, :, :, : widths[i]], one)
        assert np.all(out[i, :, :, widths[i]:] == 1.0)


# ------------------------------------------------------------------- host side of the C ABI

@pytest.fixture(scope="module")
def rh():
    import rust_ppocrv6_b200 as rh

    rh.load()
    return rh


def test_width_rule_matches_oracle(rh, oracle):
    rng = np.random.default_rng(6)
    for _ in range(5000):
        w, h = int(rng.integers(0, 100_000)), int(rng.integers(0, 500))
        th, mw = int(rng.integers(0, 200)), int(rng.integers(0, 3000))
        assert rh.resized_width(w, h, th, mw) == oracle.rec_resized_width(w, h, th, mw), (w, h, th, mw)
    big = 2**32 - 1
    assert rh.resized_width(big, 1, big, big) == oracle.rec_resized_width(big, 1, big, big)


def test_batch_shape(rh):
    widths, h, wmax = rh.batch_shape([100, 64, 1000, 65_000, 50, 400, 0], [10, 64, 10, 1, 100, 40, 0])
    assert list(widths) == [480, 48, 960, 960, 32, 480, 32] and h == 48 and wmax == 960
    assert rh.batch_shape([], [])[1:] == (48, 0)


def test_batch_shape_rejects_unsupported_sizes(rh):
    with pytest.raises(rh.RecHeadError) as e:
        rh.batch_shape([10], [10], target_h=(1 << 20) + 1)
    assert e.value.code == rh.RH_ERR_UNSUPPORTED
    with pytest.raises(rh.RecHeadError) as e:
        rh.batch_shape([(1 << 30) + 1], [10])
    assert e.value.code == rh.RH_ERR_UNSUPPORTED
    # a crop that shrinks by more than the kernel's staged span allows (width 32 from 600,000)
    with pytest.raises(rh.RecHeadError) as e:
        rh.batch_shape([600_000], [900_000])
    assert e.value.code == rh.RH_ERR_UNSUPPORTED


# --------------------------------------------- the kernel's rounding step, checked exhaustively

_ROUNDING_C = r"""
#include <fenv.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#pragma STDC FENV_ACCESS ON
/* For every float t in [+0, 255]: fma(24929, 336.5, t) rounded toward -inf, minus 2^23,
   against roundf(t) (half away from zero). argv[1] = "down" or "nearest"; argv[2], argv[3] =
   the bit patterns of the first and the last t. */
int main(int argc, char** argv) {
    volatile float a = 24929.0f, b = 336.5f, bias = 8388608.0f;
    unsigned long long n = 0, bad = 0;
    if (fesetround(strcmp(argv[1], "down") == 0 ? FE_DOWNWARD : FE_TONEAREST) != 0) return 2;
    const uint32_t first = (uint32_t)strtoul(argv[2], NULL, 16), last = (uint32_t)strtoul(argv[3], NULL, 16);
    for (uint32_t u = first; u <= last; ++u) {
        float t;
        memcpy(&t, &u, 4);
        if (fmaf(a, b, t) - bias != roundf(t)) ++bad;
        ++n;
    }
    printf("%llu %llu\n", n, bad);
    return 0;
}
"""


def test_kernel_rounding_step_is_round_half_away_for_every_float(tmp_path):
    """The resize kernel rounds the clamped horizontal sum t (0 <= t <= 255) as
    fma(24929, 336.5, t) with rounding toward -inf, minus 2^23: 24929 * 336.5 = 2^23 + 1/2, the
    exact value lands among the integers of [2^23, 2^24), and rounding it down is
    floor(t + 1/2). This checks the identity against roundf for all 1,132,396,545 floats of
    [+0, 255], with the C library's correctly rounded fmaf standing for the GPU's fma.rm; in
    round-to-nearest the same formula is wrong (t = 0.25 gives 1), which shows the check can fail."""
    import shutil
    import subprocess

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not found")
    src, exe = tmp_path / "rounding.c", tmp_path / "rounding"
    src.write_text(_ROUNDING_C)
    subprocess.run([gcc, "-O2", "-frounding-math", "-o", str(exe), str(src), "-lm"], check=True)
    n, bad = map(int, subprocess.run([str(exe), "down", "0", "437F0000"], check=True, capture_output=True,
                                     text=True).stdout.split())
    assert (n, bad) == (0x437F0000 + 1, 0)
    n, bad = map(int, subprocess.run([str(exe), "nearest", "3E800000", "3E8000FF"], check=True,
                                     capture_output=True, text=True).stdout.split())  # 256 floats from 0.25
    assert n == 256 and bad > 0
