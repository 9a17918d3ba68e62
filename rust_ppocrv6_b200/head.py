"""Host-side mirror of rust-ppocrv6's recognition-head operator surface, backed by the
sm_100a kernels in librechead.so.

Reference items mirrored (paths inside rust-ppocrv6):
  QuantizedWeight.from_f32_transposed  src/ops/matmul.rs:1165-1202
  matmul_quantized_b                   src/ops/matmul.rs:1204-1336 (MatMul.12 drop-in)
  head_decode                          matmul_quantized_b -> softmax_inplace
                                       (src/ops/softmax.rs:199-285) -> find_argmax
                                       (src/postprocess/ctc.rs:178-258), fused
  Model.quantize_matmul_weights        src/engine/model.rs:628-638 (graph [K,N] weight)
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import RH_ERR_INVALID_ARG, RecHeadError, check, load


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


def _p(x: np.ndarray):
    return x.ctypes.data_as(ctypes.c_void_p)


class Context:
    """An rh_ctx over one or more CUDA devices (default: device 0)."""

    def __init__(self, devices=None, timeout_ms: int | None = None):
        lib = load()
        h = ctypes.c_void_p()
        if devices is None:
            check(lib.rh_ctx_create(None, 0, ctypes.byref(h)))
        else:
            arr = (ctypes.c_int * len(devices))(*devices)
            check(lib.rh_ctx_create(arr, len(devices), ctypes.byref(h)))
        self._h = h
        if timeout_ms is not None:
            check(lib.rh_ctx_set_timeout_ms(h, int(timeout_ms)))

    @property
    def handle(self):
        if self._h is None:
            raise RecHeadError(RH_ERR_INVALID_ARG, "context is closed")
        return self._h

    @property
    def num_devices(self) -> int:
        return load().rh_ctx_num_devices(self.handle)

    def set_timeout_ms(self, ms: int) -> None:
        check(load().rh_ctx_set_timeout_ms(self.handle, int(ms)))

    def sync(self, slot: int = -1) -> None:
        check(load().rh_sync(self.handle, slot))

    def launch_count(self, slot: int = 0) -> int:
        return int(load().rh_launch_count(self.handle, slot))

    def close(self) -> None:
        if self._h is not None:
            load().rh_ctx_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_default_ctx: Context | None = None


def default_context() -> Context:
    global _default_ctx
    if _default_ctx is None:
        _default_ctx = Context()
    return _default_ctx


class QuantizedWeight:
    """QuantizedWeight (src/ops/matmul.rs:1165-1171), resident on the context's GPUs.

    `data` / `scales` copy the canonical int8 [rows][cols] payload and f32 per-row scales
    back from the device; they are bit-exact with the reference's packing."""

    def __init__(self, ctx: Context, handle, rows: int, cols: int, bias):
        self._ctx = ctx
        self._h = handle
        self.rows = rows
        self.cols = cols
        self._bias = None if bias is None else _f32(bias).copy()

    @classmethod
    def from_f32_transposed(cls, w_t, ctx: Context | None = None, bias=None,
                            compact: bool = False) -> "QuantizedWeight":
        """Pack the transposed weight w_t [N, K] (QuantizedWeight::from_f32_transposed), with
        an optional bias folded in (the Add.204 fold, src/engine/model.rs:141-155).

        compact=False keeps the fp16 image of the tensor-core operand in HBM (rh_weight_pack,
        the faster head); compact=True keeps int8 tiles, expanded in shared memory
        (rh_weight_pack_compact: the reference's >= 3.5x footprint cut, same results)."""
        ctx = ctx or default_context()
        w_t = _f32(w_t)
        if w_t.ndim != 2:
            raise RecHeadError(RH_ERR_INVALID_ARG, f"expected [N, K] weight, got shape {w_t.shape}")
        n, k = w_t.shape
        b = None if bias is None else _f32(bias).reshape(-1)
        h = ctypes.c_void_p()
        fn = load().rh_weight_pack_compact if compact else load().rh_weight_pack
        check(fn(ctx.handle, _p(w_t), n, k, None if b is None else _p(b), 0 if b is None else b.size,
                 ctypes.byref(h)))
        return cls(ctx, h, n, k, b)

    @classmethod
    def from_graph_weight(cls, w_kn, ctx: Context | None = None, bias=None) -> "QuantizedWeight":
        """Pack a graph-layout MatMul weight [K, N] the way the model loader does: transpose to
        [N, K] (src/engine/model.rs:565-605), then quantise (:628-638)."""
        return cls.from_f32_transposed(np.ascontiguousarray(_f32(w_kn).T), ctx=ctx, bias=bias)

    @property
    def handle(self):
        if self._h is None:
            raise RecHeadError(RH_ERR_INVALID_ARG, "weight is freed")
        return self._h

    @property
    def data(self) -> np.ndarray:
        q = np.empty((self.rows, self.cols), np.int8)
        check(load().rh_weight_export(self._ctx.handle, self.handle, _p(q), None))
        return q

    @property
    def scales(self) -> np.ndarray:
        s = np.empty(self.rows, np.float32)
        check(load().rh_weight_export(self._ctx.handle, self.handle, None, _p(s)))
        return s

    def device_image(self):
        """(tiles uint8 [n_chunks, tile bytes], table f32 [n_chunks, 2, 128]) as held on the
        device: the tiles (fp16 operand image, or compact int8 q + 128 in the kernel's expansion
        order; layouts in include/rechead.h) and, per tile, the classes' scales then biases."""
        n_chunks = (self.rows + 127) // 128
        tiles = np.empty((n_chunks, int(load().rh_weight_tile_bytes(self.handle))), np.uint8)
        table = np.empty((n_chunks, 2, 128), np.float32)
        check(load().rh_weight_export_image(self._ctx.handle, self.handle, _p(tiles), _p(table)))
        return tiles, table

    @property
    def device_bytes(self) -> int:
        return int(load().rh_weight_device_bytes(self.handle))

    @property
    def bias(self):
        return self._bias

    def set_bias(self, bias) -> None:
        b = None if bias is None else _f32(bias).reshape(-1)
        check(load().rh_weight_set_bias(self._ctx.handle, self.handle, None if b is None else _p(b),
                                        0 if b is None else b.size))
        self._bias = None if b is None else b.copy()

    def free(self) -> None:
        if self._h is not None:
            load().rh_weight_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Fp32Weight(QuantizedWeight):
    """The FP32 head weight (the engine's default, quantize_rec_head = false): the transposed
    [N, K] f32 weight used by matmul_transposed_b (src/ops/matmul.rs:514-897), packed on the
    GPU as power-of-two-scaled fp16 hi/lo images (rh_weight_pack_f32). No int8 payload."""

    @classmethod
    def from_f32_transposed(cls, w_t, ctx: Context | None = None, bias=None) -> "Fp32Weight":
        ctx = ctx or default_context()
        w_t = _f32(w_t)
        if w_t.ndim != 2:
            raise RecHeadError(RH_ERR_INVALID_ARG, f"expected [N, K] weight, got shape {w_t.shape}")
        n, k = w_t.shape
        b = None if bias is None else _f32(bias).reshape(-1)
        h = ctypes.c_void_p()
        check(load().rh_weight_pack_f32(ctx.handle, _p(w_t), n, k, None if b is None else _p(b),
                                        0 if b is None else b.size, ctypes.byref(h)))
        return cls(ctx, h, n, k, b)

    @property
    def data(self):
        raise RecHeadError(RH_ERR_INVALID_ARG, "an FP32 weight has no int8 data")

    @property
    def scales(self):
        raise RecHeadError(RH_ERR_INVALID_ARG, "an FP32 weight has no int8 scales")


def _use_bias(qw: QuantizedWeight, bias) -> None:
    if bias is None:
        if qw.bias is not None:
            qw.set_bias(None)
        return
    b = _f32(bias).reshape(-1)
    if b.size != qw.rows:
        raise RecHeadError(RH_ERR_INVALID_ARG, f"bias has {b.size} elements but n is {qw.rows}")
    if qw.bias is None or qw.bias.size != b.size or not np.array_equal(qw.bias.view(np.uint32), b.view(np.uint32)):
        qw.set_bias(b)


def _rows(a: np.ndarray, k: int):
    if a.ndim < 1:
        raise RecHeadError(RH_ERR_INVALID_ARG, "Operand must have valid dimensions")
    if a.shape[-1] != k:
        raise RecHeadError(RH_ERR_INVALID_ARG, f"Inner dimensions must match: {a.shape[-1]} != {k}")
    lead = a.shape[:-1]
    rows = int(np.prod(lead)) if lead else 1
    return lead, rows


def matmul_quantized_b(a, qw: QuantizedWeight, bias=None) -> np.ndarray:
    """out[..., m, n] = (sum_k a[..., m, k] * q[n, k]) * scale[n] + bias[n] on the GPU.

    Same argument meaning and errors as the reference (K mismatch, bias length != n)."""
    a = _f32(a)
    lead, rows = _rows(a, qw.cols)
    _use_bias(qw, bias)
    out = np.empty(lead + (qw.rows,), np.float32)
    if rows:
        check(load().rh_matmul_quantized_b(qw._ctx.handle, qw.handle, _p(a), rows, qw.cols, _p(out)))
    return out


def matmul_transposed_b(a, w: Fp32Weight, bias=None) -> np.ndarray:
    """The FP32 MatMul.12 drop-in (ops::matmul_transposed_b with an Fp32Weight): logits [..., N]."""
    a = _f32(a)
    lead, rows = _rows(a, w.cols)
    _use_bias(w, bias)
    out = np.empty(lead + (w.rows,), np.float32)
    if rows:
        check(load().rh_matmul_transposed_b(w._ctx.handle, w.handle, _p(a), rows, w.cols, _p(out)))
    return out


def head_decode(a, qw: QuantizedWeight, bias=None, line_offsets=None):
    """Fused MatMul.12 + Softmax.2 + per-timestep argmax: returns (idx int32 [rows],
    prob f32 [rows]) for a [..., k]. With line_offsets, lines are sharded over the context's
    devices (rh_head_decode_lines)."""
    a = _f32(a)
    lead, rows = _rows(a, qw.cols)
    if bias is not None:
        _use_bias(qw, bias)
    idx = np.empty(rows, np.int32)
    prob = np.empty(rows, np.float32)
    if rows == 0:
        return idx.reshape(lead), prob.reshape(lead)
    lib = load()
    if line_offsets is None:
        check(lib.rh_head_decode(qw._ctx.handle, qw.handle, _p(a), rows, qw.cols, _p(idx), _p(prob)))
    else:
        off = np.ascontiguousarray(line_offsets, dtype=np.int64)
        if off.size < 1 or off[0] != 0 or off[-1] != rows:
            raise RecHeadError(RH_ERR_INVALID_ARG, "line_offsets must run from 0 to the row count")
        check(lib.rh_head_decode_lines(qw._ctx.handle, qw.handle, _p(a), _p(off), off.size - 1, qw.cols,
                                       _p(idx), _p(prob)))
    return idx.reshape(lead), prob.reshape(lead)


def head_decode_kt(x, qw: QuantizedWeight, bias=None):
    """head_decode on the SVTR tail's [batch, k, T] output (before Transpose.8), the transpose
    folded into the kernel: returns (idx int32 [batch, T], prob f32 [batch, T])."""
    x = _f32(x)
    if x.ndim != 3 or x.shape[1] != qw.cols:
        raise RecHeadError(RH_ERR_INVALID_ARG, f"expected [batch, {qw.cols}, T] features, got {x.shape}")
    if bias is not None:
        _use_bias(qw, bias)
    b, k, t = x.shape
    idx = np.empty((b, t), np.int32)
    prob = np.empty((b, t), np.float32)
    if b * t:
        check(load().rh_head_decode_kt(qw._ctx.handle, qw.handle, _p(x), b, k, t, _p(idx), _p(prob)))
    return idx, prob


def head_decode_kt_ctc(x, qw: QuantizedWeight, valid_t, bias=None):
    """A padded batch end to end (rh_head_decode_kt_ctc): the SVTR tail's [batch, k, T] output,
    line b valid for its first valid_t[b] timesteps; the head on the GPU, then the CTC collapse
    over each line's valid timesteps. Returns (tokens, token_offsets, scores) as
    rh_ctc_collapse."""
    x = _f32(x)
    if x.ndim != 3 or x.shape[1] != qw.cols:
        raise RecHeadError(RH_ERR_INVALID_ARG, f"expected [batch, {qw.cols}, T] features, got {x.shape}")
    if bias is not None:
        _use_bias(qw, bias)
    b, k, t = x.shape
    vt = np.ascontiguousarray(valid_t, dtype=np.int64)
    if vt.shape != (b,):
        raise RecHeadError(RH_ERR_INVALID_ARG, f"valid_t must hold one length per line ({b}), got {vt.shape}")
    tokens = np.empty(max(int(vt.sum()) if b else 0, 1), np.int32)
    toff = np.zeros(b + 1, np.int64)
    scores = np.empty(max(b, 1), np.float32)
    check(load().rh_head_decode_kt_ctc(qw._ctx.handle, qw.handle, _p(x), b, k, t, _p(vt) if b else None, _p(tokens),
                                       _p(toff), _p(scores)))
    return tokens[:toff[-1]].copy(), toff, scores[:b].copy()


def head_decode_ctc(a, qw: QuantizedWeight, line_offsets, bias=None):
    """The head of a line batch with the CTC collapse on the GPU (rh_head_decode_ctc):
    returns (tokens int32 [total], token_offsets int64 [n_lines + 1], scores f32 [n_lines]),
    the outputs of rh_ctc_collapse, with only those leaving the GPUs."""
    a = _f32(a)
    lead, rows = _rows(a, qw.cols)
    if bias is not None:
        _use_bias(qw, bias)
    off = np.ascontiguousarray(line_offsets, dtype=np.int64)
    if off.size < 1 or off[0] != 0 or off[-1] != rows:
        raise RecHeadError(RH_ERR_INVALID_ARG, "line_offsets must run from 0 to the row count")
    n_lines = off.size - 1
    tokens = np.empty(max(rows, 1), np.int32)
    toff = np.empty(n_lines + 1, np.int64)
    scores = np.empty(max(n_lines, 1), np.float32)
    check(load().rh_head_decode_ctc(qw._ctx.handle, qw.handle, _p(a), _p(off), n_lines, qw.cols, _p(tokens),
                                    _p(toff), _p(scores)))
    return tokens[:toff[-1]].copy(), toff, scores[:n_lines].copy()


def ctc_collapse_device(ctx: Context, idx_ptr: int, prob_ptr: int, offsets_ptr: int, n_lines: int, tokens_ptr: int,
                        token_offsets_ptr: int, scores_ptr: int, stream: int = 0, slot: int = 0) -> None:
    """rh_ctc_collapse_device on raw CUDA pointers (e.g. torch tensors' data_ptr())."""
    vp = ctypes.c_void_p
    check(load().rh_ctc_collapse_device(ctx.handle, slot, vp(idx_ptr), vp(prob_ptr), vp(offsets_ptr), n_lines,
                                        vp(tokens_ptr), vp(token_offsets_ptr), vp(scores_ptr), vp(stream or None)))


def head_decode_device(qw: QuantizedWeight, a_ptr: int, rows: int, idx_ptr: int, prob_ptr: int, stream: int = 0,
                       slot: int = 0) -> None:
    """Device-memory fused head (raw CUDA pointers, e.g. torch tensors' data_ptr()) on `stream`."""
    check(load().rh_head_decode_device(qw._ctx.handle, qw.handle, slot, ctypes.c_void_p(a_ptr), rows,
                                       ctypes.c_void_p(idx_ptr), ctypes.c_void_p(prob_ptr),
                                       ctypes.c_void_p(stream or None)))


def matmul_quantized_b_device(qw: QuantizedWeight, a_ptr: int, rows: int, out_ptr: int, stream: int = 0,
                              slot: int = 0) -> None:
    check(load().rh_matmul_quantized_b_device(qw._ctx.handle, qw.handle, slot, ctypes.c_void_p(a_ptr), rows,
                                              ctypes.c_void_p(out_ptr), ctypes.c_void_p(stream or None)))
