"""The engine's host-side position ids (b200_get_rope_index, a C-ABI host
function that runs without a GPU) against the reference's golden position
ids (gen_cpu_reference.py mrope_pid cases, bit-exact), the oracle on random
prompts with and without an attention mask, and the reference's own compiled
GetRopeIndex where oracle/_ref is built."""

import ctypes
import json
import os

import numpy as np
import pytest

import oracle
from atb_llm_study_b200 import capi
from conftest import load_fixture

pytestmark = pytest.mark.skipif(not os.path.exists(capi.LIB_PATH), reason="library not built")

VS, IMG = 151652, 151655


def rope_index(ids, grids=None, mask=None, image=IMG, vs=VS, merge=2):
    ids = np.ascontiguousarray(ids, np.int64)
    B, S = ids.shape
    out = np.full((3, B, S), -7, np.int64)
    g = None if grids is None else np.ascontiguousarray(grids, np.int64)
    m = None if mask is None else np.ascontiguousarray(mask, np.int64)
    rc = capi.lib().b200_get_rope_index(ids.ctypes.data, B, S, None if m is None else m.ctypes.data,
                                        None if g is None else g.ctypes.data, 0 if g is None else len(g), image, vs,
                                        merge, out.ctypes.data)
    assert rc == 0, rc
    return out


@pytest.mark.parametrize("case", ["simple", "no_img", "image_text", "multi_img", "chat_template", "boundary"])
def test_rope_index_golden_bit_exact(case):
    fx = load_fixture("mrope")
    pre = f"rope_index_{case}__"
    kw = json.loads(str(fx[pre + "kw"]))
    out = rope_index(fx[pre + "input_ids"], fx.get(pre + "image_grid_thw"), fx.get(pre + "attention_mask"),
                     kw["image_token_id"], kw["vision_start_token_id"], kw["spatial_merge_size"])
    np.testing.assert_array_equal(out, fx[pre + "position_ids"])


def _prompt(rng, n_images, t_max=1):
    ids, grids = [], []
    for _ in range(n_images):
        ids += list(rng.integers(0, 1000, int(rng.integers(0, 6))))
        h, w = (int(v) * 2 for v in rng.integers(1, 5, 2))
        t = int(rng.integers(1, t_max + 1))
        grids.append([t, h, w])
        ids += [VS] + [IMG] * (t * h * w // 4)
    ids += list(rng.integers(0, 1000, int(rng.integers(1, 6))))
    return ids, grids


@pytest.mark.parametrize("seed", range(12))
def test_rope_index_matches_oracle(seed):
    rng = np.random.default_rng(seed)
    ids, grids = _prompt(rng, int(rng.integers(0, 4)), t_max=2)
    a = np.array([ids], np.int64)
    g = np.array(grids, np.int64) if grids else None
    np.testing.assert_array_equal(rope_index(a, g), oracle.get_rope_index(a, g))


@pytest.mark.parametrize("seed", range(6))
def test_rope_index_masked_batch_matches_oracle(seed):
    """Two rows padded to one length (left or right), images consumed in order across rows."""
    rng = np.random.default_rng(100 + seed)
    rows = [_prompt(rng, int(rng.integers(0, 3))) for _ in range(2)]
    S = max(len(r[0]) for r in rows) + 2
    ids = np.zeros((2, S), np.int64)
    mask = np.zeros((2, S), np.int64)
    grids = []
    for b, (toks, gr) in enumerate(rows):
        off = (S - len(toks)) if (seed + b) % 2 else 0
        ids[b, off:off + len(toks)] = toks
        mask[b, off:off + len(toks)] = 1
        grids += gr
    g = np.array(grids, np.int64) if grids else None
    np.testing.assert_array_equal(rope_index(ids, g, mask), oracle.get_rope_index(ids, g, None, mask))


def test_rope_index_matches_reference_cpp():
    from oracle import ref

    if not ref.available():
        pytest.skip("oracle/_ref not built (no reference checkout)")
    for seed in range(20):
        rng = np.random.default_rng(200 + seed)
        ids, grids = _prompt(rng, int(rng.integers(0, 4)))
        a = np.array([ids], np.int64)
        g = np.array(grids, np.int64) if grids else None
        np.testing.assert_array_equal(rope_index(a, g), ref.get_rope_index(a, g))


def test_rope_index_rejects_bad_arguments():
    L = capi.lib()
    ids = np.zeros((1, 4), np.int64)
    out = np.zeros((3, 1, 4), np.int64)
    assert L.b200_get_rope_index(None, 1, 4, None, None, 0, IMG, VS, 2, out.ctypes.data) == -1
    assert L.b200_get_rope_index(ids.ctypes.data, 1, 0, None, None, 0, IMG, VS, 2, out.ctypes.data) == -1
    assert L.b200_get_rope_index(ids.ctypes.data, 1, 4, None, None, 2, IMG, VS, 2, out.ctypes.data) == -1
    bad = np.array([[1, 0, 4]], np.int64)
    assert L.b200_get_rope_index(ids.ctypes.data, 1, 4, None, bad.ctypes.data, 1, IMG, VS, 2,
                                 out.ctypes.data) == -1
    assert ctypes.c_int(L.b200_get_rope_index(ids.ctypes.data, 1, 4, None, None, 0, IMG, VS, 2,
                                              out.ctypes.data)).value == 0
    np.testing.assert_array_equal(out[:, 0], np.tile(np.arange(4), (3, 1)))
