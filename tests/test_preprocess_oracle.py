"""The image preprocessing oracle (oracle.preprocess) against the golden data
the reference generator made with real PIL (tests/golden/preprocess.npz):
SmartResize sizes, the 8-bit antialiased bicubic resample (bit-exact uint8,
including the production-size images whose inputs are regenerated from the
generator's seed and whose outputs are pinned by sha256), and the whole
PreprocessImage chain (bit-exact float16 pixel values and grid)."""

import hashlib
import os

import numpy as np
import pytest

from oracle import preprocess as P

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "preprocess.npz"))
PROD = [(416, 672), (720, 1280), (1080, 1920), (1440, 2560)]


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def prod_inputs():
    """The generator's production-size inputs: seed 2026, drawn in this order."""
    rs = np.random.RandomState(2026)
    for h, w in PROD:
        img = (rs.rand(3, h, w) * 255.0).astype(np.float32)
        yield (h, w), np.clip(np.round(img), 0.0, 255.0).astype(np.uint8)


def test_smart_resize_cases():
    for h, w, nh, nw in GOLD["smart_resize"]:
        assert P.smart_resize(int(h), int(w), 32, 4096, 1843200) == (nh, nw), (h, w)


@pytest.mark.parametrize("name", ["2x2_to_4x4", "4x4_to_2x2", "random_8x8_to_16x16_3ch"])
def test_bicubic_small_cases_bit_exact(name):
    x, y = GOLD[f"bicubic_{name}__input"], GOLD[f"bicubic_{name}__pil"]
    np.testing.assert_array_equal(P.resample_u8(x, y.shape[1], y.shape[2]), y)


def test_bicubic_production_sizes_bit_exact():
    for (h, w), x in prod_inputs():
        key = f"bicubic_prod_{h}x{w}"
        assert _sha(x) == str(GOLD[f"{key}__in_sha256"])
        oh, ow = (int(v) for v in GOLD[f"{key}__out_shape"][1:])
        assert _sha(P.resample_u8(x, oh, ow)) == str(GOLD[f"{key}__out_sha256"]), key


@pytest.mark.parametrize("name", ["gradient_64x64", "random_96x96", "down_144x272"])
def test_preprocess_chain_bit_exact(name):
    x = GOLD[f"preprocess_{name}__input"]
    pv, grid = P.preprocess_image(x)
    np.testing.assert_array_equal(np.array([grid]), GOLD[f"preprocess_{name}__grid"])
    np.testing.assert_array_equal(pv.view(np.uint16), GOLD[f"preprocess_{name}__pil"].view(np.uint16))


def test_coefficients_sum_and_bounds():
    # every output sample's taps lie inside the input and its quantised weights sum to ~2^22
    for n_in, n_out in [(4, 2), (2, 4), (1440, 992), (672, 672 * 3 // 2), (13, 7)]:
        ks, b, k = P.coeffs_8bpc(n_in, n_out)
        assert np.all(b[:, 0] >= 0) and np.all(b[:, 0] + b[:, 1] <= n_in) and np.all(b[:, 1] <= ks)
        s = k.astype(np.int64).sum(1)
        assert np.all(np.abs(s - (1 << 22)) <= ks), (n_in, n_out)


def test_library_smart_resize_matches_oracle():
    # host function of the shipped library (no GPU involved)
    import ctypes

    from atb_llm_study_b200 import capi

    L = capi.lib()
    rng = np.random.default_rng(0)
    cases = [tuple(int(v) for v in r[:2]) for r in GOLD["smart_resize"]]
    cases += [(int(h), int(w)) for h, w in rng.integers(1, 5000, (300, 2))]
    cases += [(48, 80), (16, 16), (4000, 30), (30, 4000), (1, 1)]
    for h, w in cases:
        nh, nw = ctypes.c_int(), ctypes.c_int()
        assert L.b200_smart_resize(h, w, 32, 4096, 1843200, ctypes.byref(nh), ctypes.byref(nw)) == 0
        assert (nh.value, nw.value) == P.smart_resize(h, w, 32, 4096, 1843200), (h, w)
