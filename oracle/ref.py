"""ctypes access to oracle/_ref/libref.so — the reference's own CPU position
functions (mrope.cpp, pos_embed_interp.cpp) compiled in place by
oracle/Makefile.  TEST INFRASTRUCTURE ONLY; absent on machines without the
reference checkout (``available()`` is then False)."""

import ctypes
import os

import numpy as np

_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libref.so")
_lib = None


def available():
    return os.path.exists(_PATH)


def _L():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(_PATH)
        P = ctypes.c_void_p
        i32, i64, f32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_float
        _lib.ref_pos_embed_interp.argtypes = [P, i32, i32, i32, P, i64, P]
        _lib.ref_get_rope_index.argtypes = [P, i64, i64, P, i64, i64, i64, i64, P]
        _lib.ref_mrope_compute.argtypes = [P, i64, i64, i32, f32, i32, i32, i32, P, P]
        _lib.ref_vision_rope.argtypes = [P, i64, i32, i32, P, P]
        _lib.ref_vision_rope.restype = i64
    return _lib


def pos_embed_interp(table_fp16, grid_thw, num_grid=48, merge_size=2):
    t = np.ascontiguousarray(table_fp16, np.float16)
    g = np.ascontiguousarray(grid_thw, np.int64)
    rows = int(sum(a * b * c for a, b, c in g))
    out = np.zeros((rows, t.shape[1]), np.float16)
    _L().ref_pos_embed_interp(t.ctypes.data, t.shape[1], num_grid, merge_size, g.ctypes.data, len(g), out.ctypes.data)
    return out


def get_rope_index(input_ids, image_grid_thw, image_token_id=151655, vision_start_token_id=151652, merge_size=2):
    ids = np.ascontiguousarray(input_ids, np.int64)
    B, S = ids.shape
    g = np.ascontiguousarray(np.zeros((0, 3)) if image_grid_thw is None else image_grid_thw, np.int64)
    out = np.zeros((3, B, S), np.int64)
    _L().ref_get_rope_index(ids.ctypes.data, B, S, g.ctypes.data if len(g) else None, len(g), image_token_id,
                            vision_start_token_id, merge_size, out.ctypes.data)
    return out


def mrope_cos_sin(position_ids, head_dim=128, theta=5e6, sections=(24, 20, 20)):
    pid = np.ascontiguousarray(position_ids, np.int64)
    _, B, S = pid.shape
    c = np.zeros((B * S, head_dim), np.float32)
    s = np.zeros_like(c)
    _L().ref_mrope_compute(pid.ctypes.data, B, S, head_dim, theta, *sections, c.ctypes.data, s.ctypes.data)
    return c, s


def vision_rope_cos_sin(grid_thw, head_dim=64, merge_size=2):
    g = np.ascontiguousarray(grid_thw, np.int64)
    rows = int(sum(a * b * c for a, b, c in g))
    c = np.zeros((rows, head_dim), np.float32)
    s = np.zeros_like(c)
    n = _L().ref_vision_rope(g.ctypes.data, len(g), head_dim // 2, merge_size, c.ctypes.data, s.ctypes.data)
    assert n == rows
    return c, s
