"""Generate the committed golden fixtures for the recognition-head parity tests.

Run once in a checkout that has the rust-ppocrv6 model files (pass the project root):

    python tests/golden/make_golden.py /path/to/rust-ppocrv6

It reads the real PP-OCRv6 small-rec head, ``linear_8.w_0`` (graph layout [K=120, N=18710])
and ``linear_8.b_0`` [18710], from ``models/PP-OCRv6_small_rec.safetensors`` and writes
``real_head_slice.npz`` with:

* ``w_t``      f32 [R, 120]: rows of the load-time transposed weight (the [N, K] tensor that
               src/engine/model.rs:565-605 builds), every 16th class;
* ``rows``     int64 [R]: which classes those are;
* ``bias``     f32 [R]: the matching bias entries;
* ``q``, ``scales``: the INT8 packing of ``w_t`` computed by an independent numpy restatement
               of QuantizedWeight::from_f32_transposed (src/ops/matmul.rs:1173-1202), written
               here without reference to the C oracle, so the two restatements pin each other;
* ``stats``    f32 [4]: mean/std of the whole weight and of the whole bias (for the synthetic
               generators' sanity checks).

The tests and the GPU box only read the .npz; nothing reads the model file at run time.
"""
from __future__ import annotations

import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def read_safetensors(path: str, names):
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(hlen))
        base = 8 + hlen
        out = {}
        for name in names:
            meta = header[name]
            assert meta["dtype"] == "F32", meta
            s, e = meta["data_offsets"]
            f.seek(base + s)
            out[name] = np.frombuffer(f.read(e - s), dtype="<f4").reshape(meta["shape"]).copy()
    return out


def numpy_pack(w_t: np.ndarray):
    """Independent restatement of QuantizedWeight::from_f32_transposed.

    max|w| per row; scale = max/127 in f32 (or 1 when max <= 1e-8); q = round-half-away(w *
    (1/scale)) clamped to [-127, 127]. The product is formed in f32 (as the reference does),
    the rounding in f64 so that |x| + 0.5 is exact.
    """
    w_t = w_t.astype(np.float32)
    max_abs = np.max(np.abs(w_t), axis=1).astype(np.float32)
    scale = np.where(max_abs > np.float32(1e-8), max_abs / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    prod = (w_t * inv[:, None]).astype(np.float32).astype(np.float64)
    rounded = np.sign(prod) * np.floor(np.abs(prod) + 0.5)
    q = np.clip(rounded, -127, 127).astype(np.int8)
    return q, scale


def main(root: str) -> None:
    path = os.path.join(root, "models", "PP-OCRv6_small_rec.safetensors")
    t = read_safetensors(path, ["linear_8.w_0", "linear_8.b_0"])
    w = t["linear_8.w_0"]  # [120, 18710]
    b = t["linear_8.b_0"]  # [18710]
    assert w.shape == (120, 18710) and b.shape == (18710,), (w.shape, b.shape)
    w_t = np.ascontiguousarray(w.T)  # [18710, 120]
    rows = np.arange(0, w_t.shape[0], 16, dtype=np.int64)
    w_slice = np.ascontiguousarray(w_t[rows])
    q, s = numpy_pack(w_slice)
    stats = np.array([w.mean(), w.std(), b.mean(), b.std()], dtype=np.float32)
    out = os.path.join(HERE, "real_head_slice.npz")
    np.savez_compressed(out, w_t=w_slice, rows=rows, bias=b[rows].astype(np.float32), q=q, scales=s, stats=stats)
    print(f"wrote {out}: {w_slice.shape[0]} rows, stats={stats}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <rust-ppocrv6 project root>")
    main(sys.argv[1])
