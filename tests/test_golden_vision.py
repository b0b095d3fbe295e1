"""Pin the vision-tower oracle against the reference's golden vectors
(gen_cpu_reference.py stages vision_attention / vision_mlp / vision_block /
patch_embed / vision_merger).  The goldens round intermediates to fp16 the way
the NPU stores them; the oracle stays fp32, so the bar is cosine >= 0.9999 and
max |err| within 1 % of max |ref|."""

import numpy as np
import pytest

import oracle
from oracle import vision
from conftest import checked_inputs, cosine, load_fixture

F = np.float32


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / np.max(np.abs(b)))


@pytest.mark.parametrize("real", [False, True])
def test_vision_attention_golden(real):
    fx = load_fixture("vision_attn")
    N, nh, hd = (int(v) for v in fx["meta"])
    sfx = "_real" if real else ""
    out = vision.vision_attention(*(fx[k].astype(F) for k in ("x", "qkv_w", "qkv_b", "proj_w", "proj_b")),
                                  fx["cos" + sfx].astype(F), fx["sin" + sfx].astype(F), nh, hd)
    ref = fx["ref" + sfx].astype(F)
    assert cosine(out, ref) > 0.9999 and _rel(out, ref) < 0.01
    if real:  # the golden's cos/sin are the vision rope of grid [1,4,4]
        c, s = oracle.vision_rope_cos_sin([[1, 4, 4]], hd, 2)
        np.testing.assert_allclose(oracle.fp16_round(c), fx["cos_real"].astype(F), atol=1e-3)
        np.testing.assert_allclose(oracle.fp16_round(s), fx["sin_real"].astype(F), atol=1e-3)


@pytest.mark.parametrize("case", ["", "nobias_", "typical_"])
def test_vision_mlp_golden(case):
    import regen

    fx = load_fixture("vision_mlp")
    N, hidden, inter = (int(v) for v in fx[case + "meta"])
    if case == "typical_":
        inp = regen.vision_mlp_inputs(N, hidden, inter, 5202)
        checked_inputs("vision_mlp", case, inp)
    else:
        inp = {k: fx[case + k] for k in ("x", "fc1_w", "fc1_b", "fc2_w", "fc2_b")}
    out = vision.vision_mlp(*(inp[k].astype(F) for k in ("x", "fc1_w", "fc1_b", "fc2_w", "fc2_b")))
    ref = fx[case + "ref"].astype(F)
    assert cosine(out, ref) > 0.9999 and _rel(out, ref) < 0.01


BLOCK_CASES = {"": (5301, None), "real_small_": (5302, [[1, 4, 4]]), "real_typical_": (5303, [[1, 16, 16]])}


@pytest.mark.parametrize("case", list(BLOCK_CASES))
def test_vision_block_golden(case):
    import regen

    fx = load_fixture("vision_block")
    N, nh, hd, inter = (int(v) for v in fx[case + "meta"])
    seed, grid = BLOCK_CASES[case]
    inp = regen.vision_block_inputs(N, nh, hd, inter, seed)
    checked_inputs("vision_block", case, inp)
    w = {k: v.astype(F) for k, v in inp.items() if k != "x"}
    cos, sin = fx[case + "cos"].astype(F), fx[case + "sin"].astype(F)
    if grid is not None:
        c, s = oracle.vision_rope_cos_sin(grid, hd, 2)
        np.testing.assert_allclose(oracle.fp16_round(c), cos, atol=1e-3)
    out = vision.vision_block(inp["x"].astype(F), w, cos, sin, nh, hd)
    ref = fx[case + "ref"].astype(F)
    assert cosine(out, ref) > 0.9999 and _rel(out, ref) < 0.01


@pytest.mark.parametrize("case", ["", "tiny_", "typical_"])
def test_patch_embed_golden(case):
    import regen

    fx = load_fixture("patch_embed")
    N, C, tp, p, E = (int(v) for v in fx[case + "meta"])
    if case == "typical_":
        inp = regen.patch_embed_inputs(N, C * tp * p * p, E, 5402)
        checked_inputs("patch_embed", case, {"pixels": inp["pixels"].reshape(-1), "w": inp["w"], "b": inp["b"]})
    else:
        inp = {"pixels": fx[case + "pixels"].reshape(N, -1), "w": fx[case + "w"], "b": fx[case + "b"]}
    out = vision.patch_embed(inp["pixels"].astype(F), inp["w"].astype(F), inp["b"].astype(F))
    ref = fx[case + "ref"].astype(F)
    assert cosine(out, ref) > 0.9999 and _rel(out, ref) < 0.01


@pytest.mark.parametrize("name", ["main", "deepstack"])
def test_vision_merger_golden(name):
    fx = load_fixture("vision_merger")
    N, hidden, merge, out_h, ds = (int(v) for v in fx[name + "_meta"])
    args = [fx[f"{name}_{k}"].astype(F) for k in ("x", "n_w", "n_b", "f1_w", "f1_b", "f2_w", "f2_b")]
    out = vision.vision_merger(*args, merge=merge, deepstack=bool(ds))
    ref = fx[name + "_ref"].astype(F)
    assert out.shape == ref.shape == (N // (merge * merge), out_h)
    assert cosine(out, ref) > 0.9999 and _rel(out, ref) < 0.01
