"""Qwen3-VL image preprocessing (test infrastructure: the checker of the
CUDA preprocess kernels).

Restates the reference's CPU chain, ``PreprocessImage``
(atb_cpp_llm/src/adapters/qwen3vl_embedding/qwen3vl_preprocess.cpp:245-366):

1. ``SmartResize`` (:219-243) — banker's rounding of size/factor in float32,
   then the max/min-pixel rescale in double.
2. Pillow's 8-bit antialiased BICUBIC resample, which the reference ports bit
   for bit (``ResampleCore8bpc``, :152-191; coefficients
   ``PrecomputeCoeffs8bpc``, :52-99; passes :102-150): per axis, the bicubic
   kernel (a = -0.5) stretched by the downscale factor, coefficients
   normalised then quantised to 22 fractional bits with +/-0.5 bias and int
   truncation; a horizontal pass then a vertical pass, each accumulating
   ``2^21 + sum(u8 * coeff)`` in int32 and clipping ``>> 22`` to [0, 255]; a
   pass whose axis keeps its size is skipped.
3. ``(u8 / 255 - mean) / std`` in float32 per channel (:281-291).
4. Patchify in the merge-block order of the Python processor's
   reshape(grid_t, tp, C, gh/ms, ms, ps, gw/ms, ms, ps).permute(0,3,6,4,7,2,1,5,8)
   (:299-359), the single frame duplicated over the temporal patch, then
   float16 (round to nearest even).

The reference's C++ file needs the Ascend ATB SDK headers to compile, so it
is not built here; this restatement is pinned instead to real PIL
(``Image.resize(BICUBIC)`` per channel — the ground truth the reference's own
golden generator uses, gen_cpu_reference.py:400-470) through the fixtures in
``tests/golden/preprocess.npz``.
"""

import math

import numpy as np

PRECISION_BITS = 22


def bankers_round_f32(x):
    """Python round() of a float32 value (half to even), as BankersRound (:209-217)."""
    x = np.float32(x)
    f = np.float32(math.floor(x))
    frac = np.float32(x - f)
    if frac < 0.5:
        return int(f)
    if frac > 0.5:
        return int(f) + 1
    lo = int(f)
    return lo if lo % 2 == 0 else lo + 1


def smart_resize(height, width, factor=32, min_pixels=4096, max_pixels=1800 * 32 * 32):
    """(new_h, new_w), restating SmartResize (:219-243)."""
    h_bar = bankers_round_f32(np.float32(height) / np.float32(factor)) * factor
    w_bar = bankers_round_f32(np.float32(width) / np.float32(factor)) * factor
    if h_bar * w_bar > max_pixels:
        beta = math.sqrt(float(height * width) / max_pixels)
        h_bar = max(factor, int(math.floor(height / beta / factor)) * factor)
        w_bar = max(factor, int(math.floor(width / beta / factor)) * factor)
    elif h_bar * w_bar < min_pixels:
        beta = math.sqrt(float(min_pixels) / (height * width))
        h_bar = int(math.ceil(height * beta / factor)) * factor
        w_bar = int(math.ceil(width * beta / factor)) * factor
    return h_bar, w_bar


def _bicubic(x):
    a = -0.5
    x = abs(x)
    if x < 1.0:
        return ((a + 2.0) * x - (a + 3.0)) * x * x + 1.0
    if x < 2.0:
        return (((x - 5.0) * x + 8.0) * x - 4.0) * a
    return 0.0


def coeffs_8bpc(in_size, out_size):
    """(ksize, bounds [out, 2] = (first tap, taps), int32 coeffs [out, ksize])."""
    scale = in_size / out_size
    filterscale = max(scale, 1.0)
    support = 2.0 * filterscale
    ksize = int(math.ceil(support)) * 2 + 1
    bounds = np.zeros((out_size, 2), np.int32)
    kk = np.zeros((out_size, ksize), np.float64)
    for xx in range(out_size):
        center = (xx + 0.5) * scale
        rss = 1.0 / filterscale
        xmin = max(int(center - support + 0.5), 0)  # int() truncates toward zero, as the C cast
        xmax = min(int(center + support + 0.5), in_size) - xmin
        w = [_bicubic((x + xmin - center + 0.5) * rss) for x in range(xmax)]
        ww = 0.0
        for v in w:
            ww += v
        for x in range(xmax):
            kk[xx, x] = w[x] / ww if ww != 0.0 else w[x]
        bounds[xx] = (xmin, xmax)
    one = float(1 << PRECISION_BITS)
    ki = np.where(kk < 0, (-0.5 + kk * one), (0.5 + kk * one))
    ki = np.trunc(ki).astype(np.int64).astype(np.int32)
    return ksize, bounds, ki


def _clip8(acc):
    return np.clip(acc >> PRECISION_BITS, 0, 255).astype(np.uint8)


def resample_u8(img, out_h, out_w):
    """img [C, H, W] uint8 -> [C, out_h, out_w] uint8 (ResampleCore8bpc)."""
    img = np.asarray(img, np.uint8)
    C, H, W = img.shape
    cur = img
    if out_w != W:
        _, b, k = coeffs_8bpc(W, out_w)
        acc = np.full((C, H, out_w), 1 << (PRECISION_BITS - 1), np.int64)
        src = cur.astype(np.int64)
        for xx in range(out_w):
            x0, n = b[xx]
            acc[:, :, xx] += (src[:, :, x0:x0 + n] * k[xx, :n].astype(np.int64)).sum(-1)
        cur = _clip8(acc.astype(np.int32))
    if out_h != H:
        _, b, k = coeffs_8bpc(H, out_h)
        Wc = cur.shape[2]
        acc = np.full((C, out_h, Wc), 1 << (PRECISION_BITS - 1), np.int64)
        src = cur.astype(np.int64)
        for yy in range(out_h):
            y0, n = b[yy]
            acc[:, yy, :] += (src[:, y0:y0 + n, :] * k[yy, :n].astype(np.int64)[None, :, None]).sum(1)
        cur = _clip8(acc.astype(np.int32))
    return cur.copy()


def patchify(norm, patch=16, tp=2, merge=2):
    """[C, h, w] float32 -> [N, C*tp*patch*patch] in merge-block order, frame duplicated."""
    C, h, w = norm.shape
    gh, gw = h // patch, w // patch
    frames = np.stack([norm] * tp, 0)
    p = frames.reshape(1, tp, C, gh // merge, merge, patch, gw // merge, merge, patch)
    p = np.transpose(p, (0, 3, 6, 4, 7, 2, 1, 5, 8))
    return np.ascontiguousarray(p.reshape(gh * gw, C * tp * patch * patch))


def preprocess_image(img, patch=16, tp=2, merge=2, min_pixels=4096, max_pixels=1800 * 32 * 32,
                     mean=(0.5, 0.5, 0.5), std=(0.5, 0.5, 0.5)):
    """img [C, H, W] uint8 -> (pixel_values [N, C*tp*ps*ps] float16, grid_thw (1, gh, gw))."""
    C, H, W = img.shape
    nh, nw = smart_resize(H, W, patch * merge, min_pixels, max_pixels)
    r = resample_u8(img, nh, nw)
    m = np.asarray(mean, np.float32).reshape(-1, 1, 1)[:C]
    s = np.asarray(std, np.float32).reshape(-1, 1, 1)[:C]
    norm = ((r.astype(np.float32) / np.float32(255.0)) - m) / s
    return patchify(norm.astype(np.float32), patch, tp, merge).astype(np.float16), (1, nh // patch, nw // patch)
