"""CPU ORACLE wrapper — test infrastructure only.

ctypes bindings for ``oracle/ref_w8a32.c``, the C restatement of rust-ppocrv6's quantised
recognition-head path (pack -> W8A32 projection -> softmax -> argmax -> CTC collapse).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` /
``--impl reference`` legs import this module, and only as the checker or as the timed CPU
baseline. The product package ``rust_ppocrv6_b200`` never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int


def build() -> str:
    """Compile the oracle with its Makefile (gcc, seconds) and return the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    srcs = [os.path.join(_HERE, f) for f in ("ref_w8a32.c", "ref_rec_pre.c", "Makefile")]
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < max(os.path.getmtime(f) for f in srcs):
        build()
    L = ctypes.CDLL(_LIB_PATH)
    L.oracle_cpu_has_avx2_fma.restype = _int
    L.oracle_pack.argtypes = [_f32p, _i64, _i64, _i8p, _f32p]
    L.oracle_matmul_quantized_b.argtypes = [_f32p, _i64, _i64, _i8p, _f32p, _i64, _i64, _vp, _i64, _f32p, _int]
    L.oracle_matmul_quantized_b.restype = _int
    L.oracle_matmul_quantized_b_colsplit.argtypes = [_f32p, _i64, _i64, _i8p, _f32p, _i64, _vp, _f32p, _int, _int]
    L.oracle_softmax_rows_inplace.argtypes = [_f32p, _i64, _i64, _int]
    L.oracle_softmax_general.argtypes = [_f32p, _f32p, _i64, _i64, _i64]
    L.oracle_find_argmax.argtypes = [_f32p, _i64, _int, ctypes.POINTER(_i64), ctypes.POINTER(ctypes.c_float)]
    L.oracle_find_argmax_scalar.argtypes = [_f32p, _i64, ctypes.POINTER(_i64), ctypes.POINTER(ctypes.c_float)]
    L.oracle_ctc_collapse.argtypes = [_i32p, _f32p, _i64p, _i64, _i32p, _i64p, _f32p]
    L.oracle_ctc_collapse.restype = _i64
    L.oracle_head_decode.argtypes = [_f32p, _i64p, _i64, _i64, _i8p, _f32p, _i64, _vp, _i32p, _f32p, _vp, _vp,
                                     _vp, _int, _int]
    L.oracle_head_decode_one_line.argtypes = [_f32p, _i64, _i64, _i8p, _f32p, _i64, _vp, _i32p, _f32p, _f32p,
                                              _int, _int]
    L.oracle_matmul_f32_transposed_b.argtypes = [_f32p, _i64, _i64, _f32p, _i64, _vp, _f32p]
    L.oracle_matmul_transposed_b.argtypes = [_f32p, _i64, _i64, _f32p, _i64, _vp, _f32p, _int]
    L.oracle_head_decode_f32.argtypes = [_f32p, _i64p, _i64, _i64, _f32p, _i64, _vp, _i32p, _f32p, _vp, _vp, _vp,
                                         _int, _int]
    L.oracle_exp_poly.argtypes = [ctypes.c_float]
    L.oracle_exp_poly.restype = ctypes.c_float
    _u32 = ctypes.c_uint32
    _u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
    _u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
    L.oracle_rec_resized_width.argtypes = [_u32, _u32, _u32, _u32]
    L.oracle_rec_resized_width.restype = _u32
    L.oracle_resize_triangle_rgb8.argtypes = [_u8p, _u32, _u32, _u32, _u32, _u8p]
    L.oracle_resize_triangle_rgb8.restype = _int
    L.oracle_rec_preprocess.argtypes = [_u8p, _u32, _u32, _u32, _u32, _f32p, ctypes.POINTER(_u32)]
    L.oracle_rec_preprocess.restype = _int
    L.oracle_rec_preprocess_batch.argtypes = [_u8p, _i64p, _u32p, _u32p, _i64, _u32, _u32, _f32p, _u32p,
                                              ctypes.POINTER(_u32), _int]
    L.oracle_rec_preprocess_batch.restype = _int
    _lib = L
    return L


def _c(x, dt):
    return np.ascontiguousarray(x, dtype=dt)


def _ptr(x):
    return None if x is None else x.ctypes.data_as(ctypes.c_void_p)


def has_avx2() -> bool:
    return bool(lib().oracle_cpu_has_avx2_fma())


def pack(w_t: np.ndarray):
    """QuantizedWeight::from_f32_transposed (src/ops/matmul.rs:1173-1202): w_t [n,k] -> (q int8 [n,k], scales f32 [n])."""
    w_t = _c(w_t, np.float32)
    n, k = w_t.shape
    q = np.empty((n, k), np.int8)
    s = np.empty(n, np.float32)
    lib().oracle_pack(w_t, n, k, q, s)
    return q, s


def matmul_quantized_b(a: np.ndarray, q: np.ndarray, scales: np.ndarray, bias=None, use_avx2: bool = True):
    """matmul_quantized_b (src/ops/matmul.rs:1204-1336), serial per-row schedule.

    a is [..., k]; returns [..., n]. Raises ValueError where the reference returns
    OcrError::OperatorError (K mismatch :1227-1232, bias length :1288-1295).
    """
    a = _c(a, np.float32)
    n, k = q.shape
    if a.ndim < 1:
        raise ValueError("MatMulQuantizedB: Operand must have valid dimensions")
    lead = a.shape[:-1]
    rows = int(np.prod(lead)) if lead else 1
    b = None if bias is None else _c(bias, np.float32).reshape(-1)
    out = np.empty(lead + (n,), np.float32)
    rc = lib().oracle_matmul_quantized_b(a.reshape(rows, a.shape[-1]), rows, a.shape[-1], _c(q, np.int8),
                                         _c(scales, np.float32), n, k, _ptr(b), 0 if b is None else b.size,
                                         out.reshape(rows, n), int(use_avx2))
    if rc != 0:
        raise ValueError("MatMulQuantizedB: inner dimension or bias length mismatch")
    return out


def matmul_quantized_b_colsplit(a, q, scales, bias=None, threads=1, use_avx2=True):
    a = _c(a, np.float32)
    n, k = q.shape
    rows = a.shape[0]
    b = None if bias is None else _c(bias, np.float32)
    out = np.empty((rows, n), np.float32)
    lib().oracle_matmul_quantized_b_colsplit(a, rows, k, _c(q, np.int8), _c(scales, np.float32), n, _ptr(b), out,
                                             int(threads), int(use_avx2))
    return out


def softmax_lastaxis(x: np.ndarray, use_avx2: bool = True) -> np.ndarray:
    """softmax_inplace over the last axis (src/ops/softmax.rs:199-285), on a copy."""
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    if y.size == 0:
        return y
    n = y.shape[-1]
    lib().oracle_softmax_rows_inplace(y.reshape(-1, n), y.size // n, n, int(use_avx2))
    return y


def softmax_general(x: np.ndarray, axis: int) -> np.ndarray:
    """The inner_size > 1 path of softmax (src/ops/softmax.rs:143-196)."""
    x = _c(x, np.float32)
    axis = axis % x.ndim
    outer = int(np.prod(x.shape[:axis])) if axis else 1
    inner = int(np.prod(x.shape[axis + 1:])) if axis + 1 < x.ndim else 1
    out = np.empty_like(x)
    lib().oracle_softmax_general(x.reshape(-1), out.reshape(-1), outer, x.shape[axis], inner)
    return out


def find_argmax(x: np.ndarray, use_avx2: bool = True):
    x = _c(x, np.float32)
    i, v = _i64(), ctypes.c_float()
    lib().oracle_find_argmax(x, x.size, int(use_avx2), ctypes.byref(i), ctypes.byref(v))
    return int(i.value), float(v.value)


def find_argmax_scalar(x: np.ndarray):
    x = _c(x, np.float32)
    i, v = _i64(), ctypes.c_float()
    lib().oracle_find_argmax_scalar(x, x.size, ctypes.byref(i), ctypes.byref(v))
    return int(i.value), float(v.value)


def ctc_collapse(idx: np.ndarray, prob: np.ndarray, line_offsets: np.ndarray):
    """Collapse + score of CtcDecoder::decode_batch (src/postprocess/ctc.rs:144-169).

    Returns (list of int32 token arrays, f32 scores [n_lines])."""
    idx = _c(idx, np.int32)
    prob = _c(prob, np.float32)
    off = _c(line_offsets, np.int64)
    n_lines = off.size - 1
    tokens = np.empty(max(idx.size, 1), np.int32)
    toff = np.empty(n_lines + 1, np.int64)
    scores = np.empty(max(n_lines, 0), np.float32)
    lib().oracle_ctc_collapse(idx, prob, off, n_lines, tokens, toff, scores)
    return [tokens[toff[l]:toff[l + 1]].copy() for l in range(n_lines)], scores


def head_decode(a, line_offsets, q, scales, bias, threads=1, use_avx2=True, want_logits=False, want_gap=False):
    """The whole head per timestep row: MatMul.12 (+ folded bias) -> Softmax.2 -> argmax.

    a [M,k] with lines at line_offsets; returns dict(idx int32[M], prob f32[M], logits?, and
    with want_gap: gap = top-2 logit gap and lmax = largest logit, f32[M] each).
    """
    a = _c(a, np.float32)
    off = _c(line_offsets, np.int64)
    n, k = q.shape
    m = a.shape[0]
    idx = np.empty(m, np.int32)
    prob = np.empty(m, np.float32)
    logits = np.empty((m, n), np.float32) if want_logits else None
    gap = np.empty(m, np.float32) if want_gap else None
    lmax = np.empty(m, np.float32) if want_gap else None
    b = None if bias is None else _c(bias, np.float32)
    lib().oracle_head_decode(a, off, off.size - 1, k, _c(q, np.int8), _c(scales, np.float32), n, _ptr(b), idx,
                             prob, _ptr(logits), _ptr(gap), _ptr(lmax), int(threads), int(use_avx2))
    out = {"idx": idx, "prob": prob}
    if want_logits:
        out["logits"] = logits
    if want_gap:
        out["gap"] = gap
        out["lmax"] = lmax
    return out


def head_decode_one_line(a, q, scales, bias, scratch, threads=1, use_avx2=True):
    a = _c(a, np.float32)
    n, k = q.shape
    m = a.shape[0]
    idx = np.empty(m, np.int32)
    prob = np.empty(m, np.float32)
    b = None if bias is None else _c(bias, np.float32)
    lib().oracle_head_decode_one_line(a, m, k, _c(q, np.int8), _c(scales, np.float32), n, _ptr(b), idx, prob,
                                      scratch, int(threads), int(use_avx2))
    return idx, prob


def matmul_f32_transposed_b(a, b_t, bias=None):
    a = _c(a, np.float32)
    b_t = _c(b_t, np.float32)
    rows, k = a.reshape(-1, a.shape[-1]).shape
    n = b_t.shape[0]
    out = np.empty(a.shape[:-1] + (n,), np.float32)
    b = None if bias is None else _c(bias, np.float32)
    lib().oracle_matmul_f32_transposed_b(a.reshape(rows, k), rows, k, b_t, n, _ptr(b), out.reshape(rows, n))
    return out


def matmul_transposed_b(a, b_t, bias=None, use_avx2: bool = True):
    """matmul_transposed_b (src/ops/matmul.rs:514-897) as a recognition worker runs it
    (ScopedDisableParallel: register-blocked tiles of 3 rows x 4 columns, the n % 4 tail
    columns through avx2_dot_product). a [..., k] -> [..., n]; raises ValueError where the
    reference returns OperatorError (inner dimension :531-536, bias length :585-593)."""
    a = _c(a, np.float32)
    b_t = _c(b_t, np.float32)
    n, k = b_t.shape
    if a.shape[-1] != k:
        raise ValueError(f"MatMulTransposedB: Inner dimensions must match: {a.shape[-1]} != {k}")
    b = None if bias is None else _c(bias, np.float32).reshape(-1)
    if b is not None and b.size != n:
        raise ValueError(f"MatMulTransposedB: bias has {b.size} elements but n is {n}")
    rows = int(np.prod(a.shape[:-1])) if a.ndim > 1 else 1
    out = np.empty(a.shape[:-1] + (n,), np.float32)
    lib().oracle_matmul_transposed_b(a.reshape(rows, k), rows, k, b_t, n, _ptr(b), out.reshape(rows, n),
                                     int(use_avx2))
    return out


def head_decode_f32(a, line_offsets, w_t, bias, threads=1, use_avx2=True, want_logits=False, want_gap=False):
    """The FP32 head per timestep row: MatMul.12 through matmul_transposed_b (+ folded bias)
    -> Softmax.2 -> argmax; the same dict as head_decode."""
    a = _c(a, np.float32)
    off = _c(line_offsets, np.int64)
    w_t = _c(w_t, np.float32)
    n, k = w_t.shape
    m = a.shape[0]
    idx = np.empty(m, np.int32)
    prob = np.empty(m, np.float32)
    logits = np.empty((m, n), np.float32) if want_logits else None
    gap = np.empty(m, np.float32) if want_gap else None
    lmax = np.empty(m, np.float32) if want_gap else None
    b = None if bias is None else _c(bias, np.float32)
    lib().oracle_head_decode_f32(a, off, off.size - 1, k, w_t, n, _ptr(b), idx, prob, _ptr(logits), _ptr(gap),
                                 _ptr(lmax), int(threads), int(use_avx2))
    out = {"idx": idx, "prob": prob}
    if want_logits:
        out["logits"] = logits
    if want_gap:
        out["gap"] = gap
        out["lmax"] = lmax
    return out


def exp_poly(x: float) -> float:
    return float(lib().oracle_exp_poly(float(x)))


# ------------------------------------------------------------ rec preprocessing

def rec_resized_width(w: int, h: int, target_h: int = 48, max_w: int = 960) -> int:
    """RecPreprocess::process's width rule (src/preprocess/rec.rs:62-75)."""
    return int(lib().oracle_rec_resized_width(w, h, target_h, max_w))


def resize_triangle_rgb8(img: np.ndarray, new_w: int, new_h: int) -> np.ndarray:
    """image 0.25 resize_exact(new_w, new_h, FilterType::Triangle) of an RGB8 [h,w,3] array."""
    img = _c(img, np.uint8)
    h, w = img.shape[:2]
    out = np.zeros((new_h, new_w, 3), np.uint8)
    if img.size == 0:
        img = np.zeros(1, np.uint8)
    rc = lib().oracle_resize_triangle_rgb8(img.reshape(-1), w, h, new_w, new_h, out.reshape(-1))
    if rc:
        raise RuntimeError("oracle resize failed")
    return out


def rec_preprocess(img: np.ndarray, target_h: int = 48, max_w: int = 960) -> np.ndarray:
    """RecPreprocess::process (src/preprocess/rec.rs:60-105): RGB8 [h,w,3] -> f32 [1,3,H,W]."""
    img = _c(img, np.uint8)
    h, w = img.shape[:2]
    th = max(target_h, 1)
    tw = rec_resized_width(w, h, target_h, max_w)
    out = np.empty((1, 3, th, tw), np.float32)
    got = ctypes.c_uint32(0)
    flat = img.reshape(-1) if img.size else np.zeros(1, np.uint8)
    rc = lib().oracle_rec_preprocess(flat, w, h, target_h, max_w, out.reshape(-1), ctypes.byref(got))
    if rc:
        raise RuntimeError("oracle rec_preprocess failed")
    return out


def rec_preprocess_batch(crops, target_h: int = 48, max_w: int = 960, threads: int = 1):
    """Batched RecPreprocess::process + build_batch (tools/profiling/batch_poc.rs:14-32):
    list of RGB8 [h_i,w_i,3] arrays -> (f32 [N,3,H,Wmax] padded with +1.0, widths u32 [N])."""
    widths = np.array([c.shape[1] for c in crops], np.uint32)
    heights = np.array([c.shape[0] for c in crops], np.uint32)
    sizes = np.array([c.size for c in crops], np.int64)
    offsets = np.zeros(len(crops), np.int64)
    if len(crops):
        offsets[1:] = np.cumsum(sizes)[:-1]
    blob = np.concatenate([_c(c, np.uint8).reshape(-1) for c in crops]) if len(crops) else np.zeros(0, np.uint8)
    if blob.size == 0:
        blob = np.zeros(1, np.uint8)
    th = max(target_h, 1)
    wmax = max([rec_resized_width(int(w), int(h), target_h, max_w) for w, h in zip(widths, heights)], default=0)
    out = np.empty((len(crops), 3, th, wmax), np.float32)
    out_w = np.zeros(len(crops), np.uint32)
    got = ctypes.c_uint32(0)
    flat = out.reshape(-1) if out.size else np.zeros(1, np.float32)
    rc = lib().oracle_rec_preprocess_batch(blob, offsets, widths, heights, len(crops), target_h, max_w, flat, out_w,
                                           ctypes.byref(got), threads)
    if rc:
        raise RuntimeError("oracle rec_preprocess_batch failed")
    return out, out_w
