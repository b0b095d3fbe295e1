"""Self-consistency of the MLA restatement (the reference has no MLA
implementation or goldens, so its parity is unpinned): the absorbed form —
W_UK folded into the query projection, W_UV into the output projection,
attention over the 576-wide latent cache — equals the decompressed form for
the last token of a prefix; YaRN frequencies reduce to plain rope inside the
original context band."""

import numpy as np

from oracle import mla

CFG = dict(heads=4, qk_nope=128, qk_rope=64, v_head=128, kv_lora=512, eps=1e-6, theta=10000.0,
           yarn=dict(factor=40.0, orig_max_pos=4096, beta_fast=32, beta_slow=1, mscale=0.707, mscale_all_dim=0.707))


def weights(rng, H=128, cfg=CFG):
    nh, dn, dr, dv, R = cfg["heads"], cfg["qk_nope"], cfg["qk_rope"], cfg["v_head"], cfg["kv_lora"]
    f = np.float32
    return {"q_w": rng.standard_normal((nh * (dn + dr), H)).astype(f) * 0.1,
            "kva_w": rng.standard_normal((R + dr, H)).astype(f) * 0.1,
            "kv_norm": (1 + 0.1 * rng.standard_normal(R)).astype(f),
            "kvb_w": rng.standard_normal((nh * (dn + dv), R)).astype(f) * 0.05,
            "o_w": rng.standard_normal((H, nh * dv)).astype(f) * 0.05}


def test_absorbed_equals_decompressed():
    rng = np.random.default_rng(0)
    w = weights(rng)
    T = 9
    x = rng.standard_normal((T, 128)).astype(np.float32)
    pos = np.arange(T)
    full = mla.mla_attention(x, w, pos, CFG)
    cos, sin = mla.rope_cfg_tables(pos, CFG)
    _, _, c, k_pe = mla.mla_project(x, w, cos, sin, CFG)
    last = mla.mla_decode_absorbed(x[-1:], w, pos[-1:], CFG, [c[:-1]], [k_pe[:-1]])
    np.testing.assert_allclose(last[0], full[-1], rtol=2e-4, atol=2e-5)


def test_yarn_frequencies():
    inv = mla.yarn_inv_freq(64, 10000.0, 40.0, 4096, 32, 1)
    plain = 1.0 / np.power(10000.0, np.arange(0, 64, 2) / 64.0)
    # high-frequency pairs keep the original frequency, low-frequency ones are divided by the factor
    np.testing.assert_allclose(inv[:5], plain[:5], rtol=1e-6)
    np.testing.assert_allclose(inv[-3:], plain[-3:] / 40.0, rtol=1e-6)
    assert mla.yarn_get_mscale(40.0, 0.707) > 1.2
