"""Batched recognition preprocessing on the GPU, mirroring rust-ppocrv6's RecPreprocess.

Reference items mirrored (paths inside rust-ppocrv6):
  RecPreprocess (target_h, max_w, new, with_max_w)  src/preprocess/rec.rs:5-30
  RecPreprocess.process                             src/preprocess/rec.rs:60-105
  build_batch ([N,3,H,Wmax], +1.0 padding)          tools/profiling/batch_poc.rs:14-32

Crops are RGB8 arrays [h, w, 3] (the output of get_rotate_crop_image, src/postprocess/warp.rs).
Every call runs the sm_100a kernels of librechead.so (rh_rec_preprocess); there is no CPU path.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import check, load
from .head import Context, default_context


def _p(x: np.ndarray):
    return x.ctypes.data_as(ctypes.c_void_p)


def _pack_crops(crops):
    crops = [np.ascontiguousarray(c, dtype=np.uint8) for c in crops]
    for c in crops:
        if c.ndim != 3 or c.shape[2] != 3:
            raise ValueError(f"a crop must be an RGB8 array [h, w, 3], got shape {c.shape}")
    widths = np.array([c.shape[1] for c in crops], np.uint32)
    heights = np.array([c.shape[0] for c in crops], np.uint32)
    sizes = np.array([c.size for c in crops], np.int64)
    offsets = np.zeros(len(crops), np.int64)
    if len(crops) > 1:
        offsets[1:] = np.cumsum(sizes)[:-1]
    blob = np.concatenate([c.reshape(-1) for c in crops]) if crops else np.zeros(0, np.uint8)
    return blob, offsets, widths, heights


def resized_width(orig_w: int, orig_h: int, target_h: int = 48, max_w: int = 960) -> int:
    """The output width RecPreprocess::process gives a crop (src/preprocess/rec.rs:62-75)."""
    return int(load().rh_rec_resized_width(orig_w, orig_h, target_h, max_w))


def batch_shape(widths, heights, target_h: int = 48, max_w: int = 960):
    """(per-line widths, H, wmax) of a batch of crops with the given sizes."""
    widths = np.ascontiguousarray(widths, dtype=np.uint32)
    heights = np.ascontiguousarray(heights, dtype=np.uint32)
    out_w = np.zeros(len(widths), np.uint32)
    h, wmax = ctypes.c_uint32(0), ctypes.c_uint32(0)
    check(load().rh_rec_batch_shape(_p(widths), _p(heights), len(widths), target_h, max_w, _p(out_w),
                                    ctypes.byref(h), ctypes.byref(wmax)))
    return out_w, int(h.value), int(wmax.value)


class RecPreprocess:
    """RecPreprocess of src/preprocess/rec.rs: resize a text-line crop to `target_h` rows with
    the triangle filter (aspect kept, width clamped to [32, max_w]) and normalise to [-1, 1]."""

    def __init__(self, target_h: int = 48, max_w: int = 960, ctx: Context | None = None):
        self.target_h = int(target_h)
        self.max_w = int(max_w)
        self.ctx = ctx

    @classmethod
    def new(cls, target_h: int) -> "RecPreprocess":
        return cls(target_h)

    @classmethod
    def with_max_w(cls, target_h: int, max_w: int) -> "RecPreprocess":
        return cls(target_h, max_w)

    def process(self, img) -> np.ndarray:
        """One crop -> f32 [1, 3, H, W] (no padding), as RecPreprocess::process."""
        out, widths = self.process_batch([img])
        return np.ascontiguousarray(out[:, :, :, : int(widths[0])])

    def process_batch(self, crops):
        """A batch of crops -> (f32 [N, 3, H, Wmax] with +1.0 past each line's width, widths u32 [N])."""
        ctx = self.ctx or default_context()
        blob, offsets, widths, heights = _pack_crops(crops)
        out_w, h, wmax = batch_shape(widths, heights, self.target_h, self.max_w)
        out = np.empty((len(crops), 3, h, wmax), np.float32)
        if len(crops) == 0:
            return out, out_w
        got_w = np.zeros(len(crops), np.uint32)
        got_max = ctypes.c_uint32(0)
        check(load().rh_rec_preprocess(ctx.handle, _p(blob) if blob.size else None, blob.size, _p(offsets),
                                       _p(widths), _p(heights), len(crops), self.target_h, self.max_w,
                                       _p(out) if out.size else None, out.size, _p(got_w), ctypes.byref(got_max)))
        return out, got_w


def rec_preprocess_device(ctx: Context, d_rgb: int, rgb_len: int, offsets, widths, heights, d_out: int,
                          out_len: int, target_h: int = 48, max_w: int = 960, slot: int = 0, stream: int = 0):
    """Device-memory variant (rh_rec_preprocess_device): crops at device address d_rgb, output
    [N, 3, H, wmax] f32 at d_out, enqueued on `stream`. Returns (widths, wmax)."""
    offsets = np.ascontiguousarray(offsets, dtype=np.int64)
    widths = np.ascontiguousarray(widths, dtype=np.uint32)
    heights = np.ascontiguousarray(heights, dtype=np.uint32)
    got_w = np.zeros(len(widths), np.uint32)
    got_max = ctypes.c_uint32(0)
    check(load().rh_rec_preprocess_device(ctx.handle, slot, ctypes.c_void_p(d_rgb), rgb_len, _p(offsets),
                                          _p(widths), _p(heights), len(widths), target_h, max_w,
                                          ctypes.c_void_p(d_out), out_len, _p(got_w), ctypes.byref(got_max),
                                          ctypes.c_void_p(stream)))
    return got_w, int(got_max.value)
