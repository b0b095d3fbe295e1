"""Pin the numpy oracle against the reference's own compiled CPU functions
(oracle/_ref, built from atb_cpp_llm/src/components/common/mrope.cpp and
atb_cpp_llm/src/components/vision/pos_embed_interp.cpp by oracle/Makefile).
Skipped where the reference checkout or oracle/_ref is absent."""

import numpy as np
import pytest

import oracle
from oracle import ref

pytestmark = pytest.mark.skipif(not ref.available(), reason="oracle/_ref not built (no reference checkout)")

VS, IMG = 151652, 151655


def _random_prompt(rng, n_images):
    ids, grids = [], []
    for _ in range(n_images):
        ids += list(rng.integers(0, 1000, int(rng.integers(0, 6))))
        h, w = (int(v) * 2 for v in rng.integers(1, 5, 2))
        grids.append([1, h, w])
        ids += [VS] + [IMG] * (h * w // 4)
    ids += list(rng.integers(0, 1000, int(rng.integers(0, 6))))
    return np.array([ids], np.int64), np.array(grids, np.int64)


@pytest.mark.parametrize("seed", range(20))
def test_get_rope_index_matches_reference_cpp(seed):
    rng = np.random.default_rng(seed)
    ids, grids = _random_prompt(rng, int(rng.integers(0, 4)))
    mine = oracle.get_rope_index(ids, grids if len(grids) else None, None, None)
    theirs = ref.get_rope_index(ids, grids if len(grids) else None)
    np.testing.assert_array_equal(mine, theirs)


def test_mrope_matches_reference_cpp():
    rng = np.random.default_rng(0)
    pid = rng.integers(0, 4096, (3, 1, 300))
    c, s = oracle.mrope_cos_sin(pid, 128, 5e6, (24, 20, 20))
    rc, rs = ref.mrope_cos_sin(pid, 128, 5e6, (24, 20, 20))
    # inv_freq: numpy float32 power vs the reference's std::pow(float) — up to
    # one ulp apart; at positions < 4096 the angle differs by < 2.5e-4 rad
    np.testing.assert_allclose(c[0], rc, atol=5e-4, rtol=0)
    np.testing.assert_allclose(s[0], rs, atol=5e-4, rtol=0)


@pytest.mark.parametrize("grid", [[[1, 4, 6]], [[1, 28, 28]], [[2, 4, 4], [1, 6, 8]]])
def test_vision_rope_matches_reference_cpp(grid):
    c, s = oracle.vision_rope_cos_sin(grid, 64, 2)
    rc, rs = ref.vision_rope_cos_sin(grid, 64, 2)
    np.testing.assert_allclose(c, rc, atol=2e-5, rtol=0)
    np.testing.assert_allclose(s, rs, atol=2e-5, rtol=0)


@pytest.mark.parametrize("grid", [[[1, 28, 28]], [[1, 8, 12]], [[1, 2, 2]], [[2, 4, 4], [1, 6, 8]], [[1, 46, 92]]])
def test_pos_embed_interp_matches_reference_cpp(grid):
    """Bilinear 48x48 -> h x w interpolation, merge order, repeat over t."""
    rng = np.random.default_rng(7)
    table = (rng.standard_normal((48 * 48, 64)) * 0.02).astype(np.float16)
    mine = oracle.pos_embed_interp(table.astype(np.float32), grid, 48, 2).astype(np.float16)
    theirs = ref.pos_embed_interp(table, grid, 48, 2)
    assert mine.shape == theirs.shape
    # same fp32 expression order; allow one fp16 ulp for libm/compiler rounding
    diff = np.abs(mine.astype(np.float32) - theirs.astype(np.float32))
    ulp = np.abs(theirs.astype(np.float32)) * 2.0 ** -10 + 2.0 ** -24
    assert np.all(diff <= ulp), float(diff.max())
    assert np.mean(mine == theirs) > 0.99
