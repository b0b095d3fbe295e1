"""Pin the CPU oracle against the reference's own golden vectors.

The fixtures were produced by running the reference generator
(atb_cpp_llm/tests/python_reference/gen_cpu_reference.py) — see
tests/golden/make_golden.py.  Tolerances follow the reference's policy
(py/tests/THRESHOLDS.md:7-14 and the level-1/level-2 C++ tests): integers
exact; fp32 restatements of fp32 goldens to ~1e-5; restatements of fp16
goldens within one fp16 rounding.
"""

import json

import numpy as np
import pytest

import oracle
from conftest import DEC_CASES, cosine, decoder_case, load_fixture, manifest


@pytest.mark.parametrize("name", list(DEC_CASES))
def test_decoder_layer_golden(name):
    c = decoder_case(name)
    w = {k: c["inputs"][k].astype(np.float32) for k in
         ("q_w", "k_w", "v_w", "o_w", "qn_w", "kn_w", "gate_w", "up_w", "down_w", "iln_w", "pln_w")}
    x = c["inputs"]["x"].astype(np.float32)
    cos = c["inputs"]["cos"].astype(np.float32)
    sin = c["inputs"]["sin"].astype(np.float32)
    mask = None if c["mask"] is None else c["mask"].astype(np.float32)
    out = oracle.decoder_layer(x, w, cos, sin, c["nh"], c["kvh"], c["hd"], 1e-6, mask=mask)
    ref = c["out_ref"].astype(np.float32)
    # the golden is fp16-rounded; the oracle's own fp16 rounding must agree
    # to within one fp16 ulp on nearly every element
    diff = np.abs(oracle.fp16_round(out) - ref)
    ulp = np.abs(ref) * 2.0 ** -10 + 2.0 ** -24
    assert np.mean(diff <= 1.01 * ulp) > 0.999
    assert cosine(out, ref) > 0.99999


@pytest.mark.parametrize("name", list(DEC_CASES))
def test_decoder_layer_causal_flag_equals_mask(name):
    """The in-kernel causal rule (j > i masked) equals the reference's additive
    -65504 fp16 mask (text_runner.cpp:74-85) for every masked case."""
    c = decoder_case(name)
    if c["mask"] is None:
        pytest.skip("no-mask case")
    np.testing.assert_array_equal(c["mask"], oracle.causal_mask_fp16(c["S"]))
    w = {k: c["inputs"][k].astype(np.float32) for k in c["inputs"] if k.endswith("_w")}
    args = (c["inputs"]["x"].astype(np.float32), w, c["inputs"]["cos"].astype(np.float32),
            c["inputs"]["sin"].astype(np.float32), c["nh"], c["kvh"], c["hd"], 1e-6)
    a = oracle.decoder_layer(*args, mask=c["mask"].astype(np.float32))
    b = oracle.decoder_layer(*args, causal=True)
    np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-6)


def test_rms_norm_golden():
    fx = load_fixture("rms_norm")
    for name in ("typical", "small", "medium"):
        out = oracle.rms_norm(fx[f"{name}_input"], fx[f"{name}_weight"], 1e-6)
        np.testing.assert_allclose(out, fx[f"{name}_output"], rtol=2e-5, atol=2e-6)
    for name in ("typical", "small"):
        x, r, w = (fx[f"prenorm_{name}_{k}"] for k in ("input", "residual", "weight"))
        np.testing.assert_allclose(x + r, fx[f"prenorm_{name}_res_out"], rtol=0, atol=0)
        np.testing.assert_allclose(oracle.rms_norm(x + r, w, 1e-5), fx[f"prenorm_{name}_output"],
                                   rtol=2e-5, atol=2e-6)
        x, r, w = (fx[f"postnorm_{name}_{k}"] for k in ("input", "residual", "weight"))
        np.testing.assert_allclose(oracle.rms_norm(x + r, w, 1e-5), fx[f"postnorm_{name}_output"],
                                   rtol=2e-5, atol=2e-6)


def test_linear_golden():
    import regen

    fx = load_fixture("linear")
    man = manifest()
    inp = regen.linear_inputs(16, 2048, 2048)
    np.testing.assert_array_equal(inp["input"], fx["typical_input"])
    assert regen.sha256(inp["weight"]) == man["linear/typical_weight"]["sha256"]
    np.testing.assert_allclose(oracle.linear(inp["input"], inp["weight"]), fx["typical_output"],
                               rtol=1e-4, atol=2e-5)
    out = oracle.linear(fx["small_bias_input"], fx["small_bias_weight"], fx["small_bias_bias"])
    np.testing.assert_allclose(out, fx["small_bias_output"], rtol=1e-5, atol=1e-6)


def test_rope_golden():
    fx = load_fixture("rope")
    for name in ("basic", "gqa"):
        S, nh, kvh, hd = (int(v) for v in fx[f"{name}_meta"])
        q = fx[f"{name}_q"].astype(np.float32).reshape(S, nh, hd)
        k = fx[f"{name}_k"].astype(np.float32).reshape(S, kvh, hd)
        cos = fx[f"{name}_cos"].astype(np.float32)
        sin = fx[f"{name}_sin"].astype(np.float32)
        rq = oracle.fp16_round(oracle.rope_half(q, cos, sin)).reshape(S, -1)
        rk = oracle.fp16_round(oracle.rope_half(k, cos, sin)).reshape(S, -1)
        np.testing.assert_allclose(rq, fx[f"{name}_rq_ref"].astype(np.float32), rtol=1e-3, atol=1e-4)
        np.testing.assert_allclose(rk, fx[f"{name}_rk_ref"].astype(np.float32), rtol=1e-3, atol=1e-4)


def test_self_attention_golden():
    fx = load_fixture("self_attention")
    names = sorted({k[: -len("_meta")] for k in fx if k.endswith("_meta")})
    assert len(names) == 10
    for name in names:
        S, nh, kvh, hd, has_mask = (int(v) for v in fx[f"{name}_meta"])
        q, k, v = (fx[f"{name}_{t}"].astype(np.float32) for t in "qkv")
        mask = fx[f"{name}_mask"].astype(np.float32) if has_mask else None
        out = oracle.sdpa_gqa(q, k, v, nh, kvh, mask=mask)
        ref = fx[f"{name}_out_ref"].astype(np.float32)
        np.testing.assert_allclose(oracle.fp16_round(out), ref, rtol=2e-3, atol=2e-5)
        if has_mask:
            causal = oracle.sdpa_gqa(q, k, v, nh, kvh, causal=True)
            np.testing.assert_allclose(causal, out, rtol=1e-5, atol=1e-6)


def test_swiglu_golden():
    import regen

    fx = load_fixture("swiglu")
    man = manifest()
    out = oracle.swiglu_mlp(*(fx[f"small_{k}"].astype(np.float32) for k in ("x", "gate_w", "up_w", "down_w")))
    np.testing.assert_allclose(oracle.fp16_round(out), fx["small_out_ref"].astype(np.float32), rtol=2e-3, atol=1e-5)
    inp = regen.swiglu_inputs(16, 2048, 6144, 5002)
    np.testing.assert_array_equal(inp["x"], fx["typical_x"])
    for k in ("gate_w", "up_w", "down_w"):
        assert regen.sha256(inp[k]) == man[f"swiglu/typical_{k}"]["sha256"]
    out = oracle.swiglu_mlp(*(inp[k].astype(np.float32) for k in ("x", "gate_w", "up_w", "down_w")))
    ref = fx["typical_out_ref"].astype(np.float32)
    assert cosine(out, ref) > 0.99999
    np.testing.assert_allclose(oracle.fp16_round(out), ref, rtol=2e-3, atol=2e-5)


def test_activation_golden():
    fx = load_fixture("activation")
    for size in ("typical", "small"):
        np.testing.assert_allclose(oracle.silu(fx[f"silu_{size}_input"]), fx[f"silu_{size}_output"],
                                   rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(oracle.gelu_tanh(fx[f"gelu_{size}_input"]), fx[f"gelu_{size}_output"],
                                   rtol=1e-5, atol=1e-6)


def test_mrope_cos_sin_golden():
    fx = load_fixture("mrope")
    cos, sin = oracle.mrope_cos_sin(fx["pid"], 128, 5e6, (24, 20, 20))
    # test_mrope_cpu.cpp:396 gates cosine > 0.9999; the fp32 restatement is far tighter
    np.testing.assert_allclose(cos, fx["cos"], rtol=0, atol=2e-6)
    np.testing.assert_allclose(sin, fx["sin"], rtol=0, atol=2e-6)


ROPE_INDEX_CASES = ["simple", "no_img", "image_text", "multi_img", "chat_template", "boundary"]


@pytest.mark.parametrize("case", ROPE_INDEX_CASES)
def test_get_rope_index_bit_exact(case):
    fx = load_fixture("mrope")
    pre = f"rope_index_{case}__"
    kw = json.loads(str(fx[pre + "kw"]))
    out = oracle.get_rope_index(fx[pre + "input_ids"], fx.get(pre + "image_grid_thw"), None,
                                fx.get(pre + "attention_mask"), **kw)
    assert out.dtype == np.int64
    np.testing.assert_array_equal(out, fx[pre + "position_ids"])
    np.testing.assert_array_equal(out, fx["pid_" + case])


def test_vision_rope_golden():
    fx = load_fixture("vision_rope")
    cos, sin = oracle.vision_rope_cos_sin([[1, 4, 6]], 64, 2)
    # test_vision_rope_cpu.cpp:311 gates max-abs <= 1e-6
    np.testing.assert_allclose(cos, fx["rope_cos"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(sin, fx["rope_sin"], rtol=0, atol=1e-6)
    cos, sin = oracle.vision_rope_cos_sin([[1, 4, 4], [1, 6, 6]], 64, 2)
    np.testing.assert_allclose(cos, fx["rope_multi_cos"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(sin, fx["rope_multi_sin"], rtol=0, atol=1e-6)


def test_paged_decode_equals_dense_last_row():
    """Unpinned-by-reference path: paged decode over a shuffled block table must
    equal the last row of dense causal attention over the same K/V."""
    rng = np.random.default_rng(0)
    nh, kvh, d, bs = 8, 2, 32, 16
    L = 53
    q = rng.standard_normal((L, nh, d)).astype(np.float32)
    k = rng.standard_normal((L, kvh, d)).astype(np.float32)
    v = rng.standard_normal((L, kvh, d)).astype(np.float32)
    nblk = (L + bs - 1) // bs
    table = rng.permutation(10)[:nblk]
    kc = np.zeros((10, kvh, bs, d), np.float32)
    vc = np.zeros_like(kc)
    slots = oracle.slot_mapping(table, np.arange(L), bs)
    assert len(set(slots.tolist())) == L
    oracle.kv_cache_write(kc, k, slots)
    oracle.kv_cache_write(vc, v, slots)
    out = oracle.paged_decode_attention(q[-1:], kc, vc, table[None], [L])
    dense = oracle.sdpa_gqa(q, k, v, nh, kvh, causal=True)[-1:]
    np.testing.assert_allclose(out, dense, rtol=1e-5, atol=1e-5)


def test_manifest_is_consistent():
    man = manifest()
    assert all(len(e["sha256"]) == 64 for e in man.values())
