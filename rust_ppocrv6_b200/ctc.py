"""CtcDecoder mirror (src/postprocess/ctc.rs) that consumes the fused head's per-timestep
(argmax index, max probability) instead of the [batch, time, vocab] probability tensor.

The collapse itself runs in librechead.so: rh_ctc_collapse on the host (no device needed), or
rh_ctc_collapse_device / rh_head_decode_ctc on the GPU.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import RH_ERR_INVALID_ARG, RecHeadError, load


class CtcDecoder:
    """Vocabulary = blank + dictionary lines + trailing space (src/postprocess/ctc.rs:12-30)."""

    def __init__(self, vocab):
        self.vocab = list(vocab)

    @classmethod
    def from_file(cls, dict_path) -> "CtcDecoder":
        try:
            with open(dict_path, "r", encoding="utf-8", newline="") as f:
                lines = f.read().split("\n")
        except OSError as e:
            raise RecHeadError(RH_ERR_INVALID_ARG, f"Failed to open dict file: {e}") from e
        if lines and lines[-1] == "":
            lines.pop()  # BufRead::lines() yields no entry after a final newline
        return cls(["blank"] + [ln.rstrip("\r\n") for ln in lines] + [" "])

    @classmethod
    def from_vocab(cls, vocab) -> "CtcDecoder":
        return cls(vocab)

    @property
    def vocab_size(self) -> int:
        return len(self.vocab)

    def check_classes(self, n_classes: int) -> None:
        """The dictionary/model mismatch check of decode/decode_batch (src/postprocess/ctc.rs:61-79)."""
        if n_classes != len(self.vocab):
            raise RecHeadError(
                RH_ERR_INVALID_ARG,
                f"dictionary/model mismatch: model outputs {n_classes} classes but the dictionary has "
                f"{len(self.vocab)} entries (expected blank + {max(len(self.vocab) - 2, 0)} characters + trailing space)")

    def collapse(self, idx, prob, line_offsets):
        """(token index arrays per line, f32 mean scores) via rh_ctc_collapse."""
        idx = np.ascontiguousarray(idx, dtype=np.int32).reshape(-1)
        prob = np.ascontiguousarray(prob, dtype=np.float32).reshape(-1)
        off = np.ascontiguousarray(line_offsets, dtype=np.int64)
        n_lines = off.size - 1
        if n_lines < 0 or (n_lines > 0 and (off[0] < 0 or off[-1] > idx.size or prob.size != idx.size)):
            raise RecHeadError(RH_ERR_INVALID_ARG, "line offsets do not match the timestep arrays")
        tokens = np.empty(max(idx.size, 1), np.int32)
        toff = np.empty(n_lines + 1, np.int64)
        scores = np.empty(max(n_lines, 1), np.float32)
        vp = ctypes.c_void_p
        got = load().rh_ctc_collapse(idx.ctypes.data_as(vp), prob.ctypes.data_as(vp), off.ctypes.data_as(vp),
                                     n_lines, tokens.ctypes.data_as(vp), toff.ctypes.data_as(vp),
                                     scores.ctypes.data_as(vp))
        if got < 0:
            raise RecHeadError(RH_ERR_INVALID_ARG, load().rh_last_error().decode())
        return [tokens[toff[l]:toff[l + 1]].copy() for l in range(n_lines)], scores[:n_lines].copy()

    def decode_indices(self, idx, prob, line_offsets, n_classes: int | None = None):
        """decode_batch (src/postprocess/ctc.rs:103-175) on (idx, prob): [(text, score)] per line."""
        if n_classes is not None:
            self.check_classes(n_classes)
        toks, scores = self.collapse(idx, prob, line_offsets)
        out = []
        for t, s in zip(toks, scores):
            if t.size and (t.max() >= len(self.vocab) or t.min() < 0):
                raise RecHeadError(RH_ERR_INVALID_ARG, "class index outside the dictionary")
            out.append(("".join(self.vocab[i] for i in t), float(s)))
        return out

    def decode_lines(self, a, qw, line_offsets):
        """The whole head of a line batch with the collapse on the GPU (rh_head_decode_ctc):
        decode_batch's [(text, score)] per line straight from the SVTR features."""
        from .head import head_decode_ctc

        self.check_classes(qw.rows)
        tokens, toff, scores = head_decode_ctc(a, qw, line_offsets)
        out = []
        for l in range(toff.size - 1):
            t = tokens[toff[l]:toff[l + 1]]
            if t.size and (t.max() >= len(self.vocab) or t.min() < 0):
                raise RecHeadError(RH_ERR_INVALID_ARG, "class index outside the dictionary")
            out.append(("".join(self.vocab[i] for i in t), float(scores[l])))
        return out

    def decode(self, idx, prob, n_classes: int | None = None):
        """decode (src/postprocess/ctc.rs:40-100) for one line; ("", 0.0) when it is empty."""
        idx = np.asarray(idx)
        if idx.size == 0:
            if n_classes is not None:
                self.check_classes(n_classes)
            return "", 0.0
        return self.decode_indices(idx, prob, np.array([0, idx.size]), n_classes)[0]
