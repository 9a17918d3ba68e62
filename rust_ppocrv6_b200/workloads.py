"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configs.

No public dataset is involved: the head's inputs are SVTR features (K=120 per timestep) and
the reference publishes no feature corpus, so every config draws them from N(0, 1) with a
fixed seed. Weights follow N(0, 0.05^2) (real head: std 0.042) or, for the precision stress
config, 0.05 * Student-t(3); biases N(0, 0.01^2) (real head: std 0.015).

  cfg0  one line, T=120                        M = 120
  cfg1  64 ragged lines, T ~ U{10..120}         M ~ 4.2k
  cfg2  1024 lines x T=120                      M = 122,880   (bench headline)
  cfg3  8192 ragged lines, T ~ U{10..120}       M ~ 532k      (multi-GPU sharding)
  cfg4  256 lines x T=240, Student-t weights,   M = 61,440
        5 % of timesteps built as near-ties (top-2 logits within 1e-4)
  cfg5  the tiny recognition model's head (linear_1.w_0, K=80 -> N=6906),
        1024 lines x T=120                      M = 122,880
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

K = 120
N = 18710
K_TINY = 80
N_TINY = 6906
SEED = 0x5EED


@dataclass
class Workload:
    name: str
    w_t: np.ndarray          # f32 [N, K] transposed head weight
    bias: np.ndarray         # f32 [N]
    x: np.ndarray            # f32 [M, K] timestep rows, lines packed densely
    line_offsets: np.ndarray  # int64 [lines + 1]
    tie_rows: np.ndarray     # rows built as near-ties (cfg4), else empty

    @property
    def rows(self) -> int:
        return int(self.x.shape[0])


def head_weights(rng: np.random.Generator, n: int = N, k: int = K, student_t: bool = False):
    if student_t:
        w = (0.05 * rng.standard_t(3.0, size=(n, k))).astype(np.float32)
    else:
        w = (0.05 * rng.standard_normal((n, k))).astype(np.float32)
    b = (0.01 * rng.standard_normal(n)).astype(np.float32)
    return w, b


def ragged_offsets(rng: np.random.Generator, lines: int, lo: int = 10, hi: int = 120) -> np.ndarray:
    t = rng.integers(lo, hi + 1, size=lines)
    return np.concatenate([[0], np.cumsum(t)]).astype(np.int64)


def uniform_offsets(lines: int, t: int) -> np.ndarray:
    return (np.arange(lines + 1, dtype=np.int64) * t)


def dequantized(w_t: np.ndarray):
    """f64 dequantised weight per QuantizedWeight::from_f32_transposed (for input design only)."""
    w = w_t.astype(np.float32)
    max_abs = np.max(np.abs(w), axis=1).astype(np.float32)
    scale = np.where(max_abs > np.float32(1e-8), max_abs / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    prod = (w * inv[:, None]).astype(np.float32).astype(np.float64)
    q = np.clip(np.sign(prod) * np.floor(np.abs(prod) + 0.5), -127, 127)
    return q * scale.astype(np.float64)[:, None]


def make_near_ties(rng, x: np.ndarray, rows: np.ndarray, w_deq: np.ndarray, bias: np.ndarray) -> None:
    """Rewrites x[rows] so that two chosen classes are the top-2 logits with a gap in
    [1e-6, 1e-4) (on the quantised weights, in f64 before the f32 rounding of x).

    The two classes come from the highest-norm tenth of the vocabulary; x is the least-norm
    solution of w1.x = L - b1, w2.x = L - b2 - gap plus a little noise orthogonal to both,
    and the construction is verified (top-2 are the chosen classes, third logit at least
    0.5 below), else retried with another pair and a larger L."""
    n, k = w_deq.shape
    b = bias.astype(np.float64)
    norms = np.linalg.norm(w_deq, axis=1)
    strong = np.argsort(norms)[-max(2, n // 10):]
    for r in rows:
        target = 4.0
        for attempt in range(64):
            c1, c2 = rng.choice(strong, size=2, replace=False)
            W = np.stack([w_deq[c1], w_deq[c2]])
            gap = rng.uniform(1e-6, 1e-4)
            rhs = np.array([target - b[c1], target - gap - b[c2]])
            gram = W @ W.T
            if abs(np.linalg.det(gram)) < 1e-12:
                continue
            xr = W.T @ np.linalg.solve(gram, rhs)
            noise = 0.2 * rng.standard_normal(k)
            noise -= W.T @ np.linalg.solve(gram, W @ noise)  # keep both target logits exact
            xr = xr + noise
            logits = w_deq @ xr + b
            order = np.argsort(logits)[::-1]
            if {order[0], order[1]} == {c1, c2} and logits[order[2]] < logits[order[1]] - 0.5:
                x[r] = xr.astype(np.float32)
                break
            target *= 1.15
        else:
            raise RuntimeError("could not build a near-tie row")


def make(cfg: int, scale: float = 1.0, seed: int = SEED) -> Workload:
    """Config `cfg` (0-5). `scale` < 1 shrinks the number of lines (test-sized variants)."""
    rng = np.random.default_rng(seed + cfg)
    student = cfg == 4
    n, k = (N_TINY, K_TINY) if cfg == 5 else (N, K)
    w_t, bias = head_weights(rng, n=n, k=k, student_t=student)
    if cfg == 0:
        off = uniform_offsets(1, 120)
    elif cfg == 1:
        off = ragged_offsets(rng, max(1, int(round(64 * scale))))
    elif cfg == 2:
        off = uniform_offsets(max(1, int(round(1024 * scale))), 120)
    elif cfg == 3:
        off = ragged_offsets(rng, max(1, int(round(8192 * scale))))
    elif cfg == 4:
        off = uniform_offsets(max(1, int(round(256 * scale))), 240)
    elif cfg == 5:
        off = uniform_offsets(max(1, int(round(1024 * scale))), 120)
    else:
        raise ValueError(f"unknown config {cfg}")
    m = int(off[-1])
    x = rng.standard_normal((m, k), dtype=np.float32)
    tie_rows = np.zeros(0, np.int64)
    if cfg == 4:
        tie_rows = np.sort(rng.choice(m, size=max(1, m // 20), replace=False))
        make_near_ties(rng, x, tie_rows, dequantized(w_t), bias)
    return Workload(f"cfg{cfg}", w_t, bias, x, off, tie_rows)


def shard_lines(line_offsets: np.ndarray, world: int, rank: int):
    """Contiguous line range [l0, l1) of `rank` with balanced timestep counts (rows), the
    partition every rank computes identically; no data moves between ranks."""
    off = np.asarray(line_offsets, dtype=np.int64)
    n_lines = off.size - 1
    total = int(off[-1] - off[0])

    def cut(d):
        if d <= 0:
            return 0
        if d >= world:
            return n_lines
        target = off[0] + (total * d) // world
        return int(np.searchsorted(off[:-1], target, side="left"))

    return cut(rank), cut(rank + 1)
