"""Decoder-layer parity on the GPU against the reference's golden layer outputs
(gen_cpu_reference.py:1500-1629, the data behind
test_text_decoder_layer_precision.cpp) and the oracle.

The layer is composed from the C-ABI kernels exactly as the engine composes it:
RMSNorm -> fused QKV GEMM -> QK-norm + rope -> causal flash attention ->
O GEMM (+residual epilogue) -> fused residual RMSNorm -> gate/up GEMM with the
SwiGLU epilogue -> down GEMM (+residual epilogue).

Bar: cosine >= 0.999 per layer output; max |err| / max |ref| < 2 %.
"""

import numpy as np
import pytest
import torch

import oracle
from conftest import DEC_CASES, decoder_case

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gpu_util as G


def interleave_gate_up(gate, up):
    """Rows 2j / 2j+1 = gate[j] / up[j] — the layout the SwiGLU epilogue reads."""
    gu = np.empty((2 * gate.shape[0], gate.shape[1]), np.float32)
    gu[0::2] = gate
    gu[1::2] = up
    return gu


def run_layer(x, w, cos, sin, nh, kvh, hd, eps=1e-6, causal=True):
    S, H = x.shape
    Wqkv = (nh + 2 * kvh) * hd
    L, st = G.L(), G.stream()
    xd = G.bf16(x)
    wqkv = G.bf16(np.concatenate([w["q_w"], w["k_w"], w["v_w"]], 0))
    wo = G.bf16(w["o_w"])
    wgu = G.bf16(interleave_gate_up(w["gate_w"], w["up_w"]))
    wd = G.bf16(w["down_w"])
    iln, pln = G.bf16(w["iln_w"]), G.bf16(w["pln_w"])
    qn, kn = G.bf16(w["qn_w"]), G.bf16(w["kn_w"])
    I = w["gate_w"].shape[0]
    normed = torch.empty_like(xd)
    G.check(L.b200_rmsnorm(xd.data_ptr(), None, iln.data_ptr(), normed.data_ptr(), None, S, H, H, eps, st))
    qkv = G.gemm(normed, wqkv)
    G.check(L.b200_qk_norm_rope(qkv.data_ptr(), S, nh, kvh, hd, Wqkv, qn.data_ptr(), kn.data_ptr(), eps,
                                G.f32(cos).data_ptr(), G.f32(sin).data_ptr(), None, None, None, 0, 0, st))
    attn = torch.empty(S, nh * hd, dtype=torch.bfloat16, device=G.DEV)
    cu = G.i32([0, S])
    G.check(L.b200_flash_prefill(qkv.data_ptr(), Wqkv, qkv.data_ptr() + nh * hd * 2,
                                 qkv.data_ptr() + (nh + kvh) * hd * 2, Wqkv, attn.data_ptr(), nh * hd, cu.data_ptr(),
                                 1, S, nh, kvh, hd, 1.0 / np.sqrt(hd), int(causal), st))
    h1 = xd.clone()
    G.gemm(attn, wo, epi=2, R=h1, out=h1)  # h1 = x + O(attn)
    n2 = torch.empty_like(xd)
    G.check(L.b200_rmsnorm(h1.data_ptr(), None, pln.data_ptr(), n2.data_ptr(), None, S, H, H, eps, st))
    act = G.gemm(n2, wgu, epi=3)  # [S, I]
    assert act.shape == (S, I)
    out = h1.clone()
    G.gemm(act, wd, epi=2, R=out, out=out)
    torch.cuda.synchronize()
    return G.host(out)


@pytest.mark.parametrize("name", list(DEC_CASES))
def test_decoder_layer_golden(name):
    c = decoder_case(name)
    inp = {k: v.astype(np.float32) for k, v in c["inputs"].items()}
    w = {k: inp[k] for k in inp if k.endswith("_w")}
    causal = c["mask"] is not None
    out = run_layer(inp["x"], w, inp["cos"], inp["sin"], c["nh"], c["kvh"], c["hd"], causal=causal)
    ref = c["out_ref"].astype(np.float32)
    cos_ref = G.cosine(out, ref)
    # the oracle on the same bf16-rounded inputs
    wr = {k: G.rounded(v) for k, v in w.items()}
    orc = oracle.decoder_layer(G.rounded(inp["x"]), wr, inp["cos"], inp["sin"], c["nh"], c["kvh"], c["hd"], 1e-6,
                               causal=causal)
    assert cos_ref >= 0.999, cos_ref
    assert G.cosine(out, orc) >= 0.999
    assert G.max_rel_err(out, orc) < 0.02
    assert G.device_errors() == 0


def test_qwen3vl_layer_config():
    """The Qwen3-VL-2B text layer config (hidden 2048, 16q/8kv x 128, I 6144,
    eps 1e-6, QK-norm, interleaved mrope [24,20,20] theta 5e6, ids
    t=h=w=arange(256), S=256, weights N(0,0.02), x N(0,1)) vs the oracle."""
    S, H, nh, kvh, hd, I = 256, 2048, 16, 8, 128, 6144
    rw = np.random.default_rng(0)
    w = {
        "q_w": rw.standard_normal((nh * hd, H), np.float32) * 0.02,
        "k_w": rw.standard_normal((kvh * hd, H), np.float32) * 0.02,
        "v_w": rw.standard_normal((kvh * hd, H), np.float32) * 0.02,
        "o_w": rw.standard_normal((H, nh * hd), np.float32) * 0.02,
        "qn_w": 1 + rw.standard_normal(hd, np.float32) * 0.02,
        "kn_w": 1 + rw.standard_normal(hd, np.float32) * 0.02,
        "gate_w": rw.standard_normal((I, H), np.float32) * 0.02,
        "up_w": rw.standard_normal((I, H), np.float32) * 0.02,
        "down_w": rw.standard_normal((H, I), np.float32) * 0.02,
        "iln_w": 1 + rw.standard_normal(H, np.float32) * 0.02,
        "pln_w": 1 + rw.standard_normal(H, np.float32) * 0.02,
    }
    x = np.random.default_rng(1).standard_normal((S, H), np.float32)
    pos = np.arange(S)
    cos, sin = oracle.mrope_cos_sin(np.stack([pos, pos, pos])[:, None, :], hd, 5e6, (24, 20, 20))
    out = run_layer(x, w, cos[0], sin[0], nh, kvh, hd)
    wr = {k: G.rounded(v) for k, v in w.items()}
    ref = oracle.decoder_layer(G.rounded(x), wr, cos[0], sin[0], nh, kvh, hd, 1e-6, causal=True)
    assert G.cosine(out, ref) >= 0.999
    assert G.max_rel_err(out, ref) < 0.02
