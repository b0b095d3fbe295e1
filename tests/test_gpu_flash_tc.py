"""tcgen05 prefill attention (b200_flash_prefill_packed: 64- and 128-wide heads,
and latent attention's decompressed 192-wide query/key with 128-wide value
heads) against the numpy oracle and a torch fp32 reference.

Cases: packed variable-length sequences around the 128-row tile edges, causal
and bidirectional, 16-, 32-, 64- and 128-wide heads (the narrow ones through
zero-filled 64-wide tiles), GQA, the packed q|k|v layout of the
engine; the Qwen3-8B
prefill shape (8 x 2048, 32 query / 8 kv heads) against torch fp32 SDPA; and
scores that keep growing along the keys so the running max moves (the rescale
of the TMEM output rows) many times.

Bar: cosine > 0.9999 and max relative error < 0.02 against fp32 (bf16
inputs, bf16 P, fp32 accumulation); the device error word stays clear.
"""

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gpu_util as G


def _run(d, W, nq, nkv, hd, cu, lens, causal, T, out=None):
    out = torch.empty(T, nq * hd, dtype=torch.bfloat16, device=G.DEV) if out is None else out
    G.check(G.L().b200_flash_prefill_packed(d.data_ptr(), W, hd, d.data_ptr() + nq * hd * 2, W, hd,
                                            d.data_ptr() + (nq + nkv) * hd * 2, W, hd, out.data_ptr(), nq * hd, hd,
                                            G.i32(cu).data_ptr(), len(lens), max(lens), T, nq, nkv, hd, hd,
                                            1.0 / np.sqrt(hd), causal, G.stream()), "flash_prefill_packed")
    return out


@pytest.mark.parametrize("causal,hd", [(1, 128), (0, 128), (1, 64), (0, 64), (1, 32), (0, 32), (1, 16), (0, 16)])
def test_varlen_tile_edges(causal, hd):
    rng = np.random.default_rng(7 + causal + hd)
    lens = [1, 63, 127, 128, 129, 300, 17, 1000]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T, nq, nkv = int(cu[-1]), 8, 2
    W = (nq + 2 * nkv) * hd
    qkv = rng.standard_normal((T, W)).astype(np.float32)
    d = G.bf16(qkv)
    x = G.rounded(qkv)
    got = G.host(_run(d, W, nq, nkv, hd, cu, lens, causal, T)).reshape(T, nq, hd)
    q = x[:, : nq * hd].reshape(T, nq, hd)
    k = x[:, nq * hd: (nq + nkv) * hd].reshape(T, nkv, hd)
    v = x[:, (nq + nkv) * hd:].reshape(T, nkv, hd)
    if causal:
        ref = oracle.varlen_causal_attention(q, k, v, cu, nq, nkv)
    else:
        ref = np.concatenate([oracle.sdpa_gqa(q[a:b], k[a:b], v[a:b], nq, nkv) for a, b in zip(cu[:-1], cu[1:])])
    assert G.cosine(got, ref) > 0.9999
    assert G.max_rel_err(got, ref) < 0.02
    # the legacy-MMA kernel on the same inputs
    old = torch.empty(T, nq * hd, dtype=torch.bfloat16, device=G.DEV)
    G.check(G.L().b200_flash_prefill(d.data_ptr(), W, d.data_ptr() + nq * hd * 2, d.data_ptr() + (nq + nkv) * hd * 2,
                                     W, old.data_ptr(), nq * hd, G.i32(cu).data_ptr(), len(lens), max(lens), nq, nkv,
                                     hd, 1.0 / np.sqrt(hd), causal, G.stream()), "flash_prefill")
    assert G.cosine(got, G.host(old).reshape(T, nq, hd)) > 0.9999
    assert G.device_errors() == 0


def _torch_ref(q, k, v, cu, nq, nkv, causal):
    outs = []
    g = nq // nkv
    for a, b in zip(cu[:-1].tolist(), cu[1:].tolist()):
        qs = q[a:b].float().transpose(0, 1)
        ks = k[a:b].float().repeat_interleave(g, dim=1).transpose(0, 1)
        vs = v[a:b].float().repeat_interleave(g, dim=1).transpose(0, 1)
        o = torch.nn.functional.scaled_dot_product_attention(qs, ks, vs, is_causal=bool(causal))
        outs.append(o.transpose(0, 1))
    return torch.cat(outs)


def test_qwen3_8b_prefill_shape():
    torch.manual_seed(0)
    S, B, nq, nkv, hd = 2048, 8, 32, 8, 128
    T = S * B
    W = (nq + 2 * nkv) * hd
    d = torch.randn(T, W, device=G.DEV).to(torch.bfloat16)
    cu = np.arange(0, T + 1, S, dtype=np.int32)
    got = _run(d, W, nq, nkv, hd, cu, [S] * B, 1, T).float().reshape(T, nq, hd)
    q = d[:, : nq * hd].reshape(T, nq, hd)
    k = d[:, nq * hd: (nq + nkv) * hd].reshape(T, nkv, hd)
    v = d[:, (nq + nkv) * hd:].reshape(T, nkv, hd)
    ref = _torch_ref(q, k, v, cu, nq, nkv, 1)
    cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
    rel = ((got - ref).abs().max() / ref.abs().max()).item()
    assert cos > 0.9999, cos
    assert rel < 0.02, rel
    assert G.device_errors() == 0


def test_growing_scores_rescale_output_rows():
    # key t scaled by (1 + t/40): scores rise along the keys, the running max moves tile after tile
    torch.manual_seed(1)
    S, nq, nkv, hd = 1100, 4, 4, 128
    W = (nq + 2 * nkv) * hd
    d = torch.randn(S, W, device=G.DEV)
    d[:, : nq * hd] = d[:, : nq * hd].abs() * 0.5
    grow = (1 + torch.arange(S, device=G.DEV, dtype=torch.float32) / 40.0)[:, None]
    d[:, nq * hd: (nq + nkv) * hd] = d[:, nq * hd: (nq + nkv) * hd].abs() * grow
    d = d.to(torch.bfloat16)
    cu = np.array([0, S], np.int32)
    for causal in (0, 1):
        got = _run(d, W, nq, nkv, hd, cu, [S], causal, S).float().reshape(S, nq, hd)
        q = d[:, : nq * hd].reshape(S, nq, hd)
        k = d[:, nq * hd: (nq + nkv) * hd].reshape(S, nkv, hd)
        v = d[:, (nq + nkv) * hd:].reshape(S, nkv, hd)
        ref = _torch_ref(q, k, v, cu, nq, nkv, causal)
        cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
        rel = ((got - ref).abs().max() / ref.abs().max()).item()
        assert cos > 0.9999, (causal, cos)
        assert rel < 0.02, (causal, rel)
    assert G.device_errors() == 0


@pytest.mark.parametrize("causal", [1, 0])
def test_mla_heads_192_qk_128_v(causal):
    """DeepSeek-V2's decompressed heads in the engine's layout: q from the fused
    projection (row stride 16 x 192 + 576, head stride 192), k packed [T, 16 x
    192], v the value half of kv_b's output (row stride 16 x 256, head stride
    256, offset 128); the YaRN softmax scale; tile edges around 128 rows."""
    rng = np.random.default_rng(192 + causal)
    lens = [1, 127, 128, 129, 640, 33]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T, nh = int(cu[-1]), 16
    NQP, KVB = nh * 192 + 576, nh * 256
    qf = rng.standard_normal((T, NQP)).astype(np.float32)
    kf = rng.standard_normal((T, nh * 192)).astype(np.float32)
    vf = rng.standard_normal((T, KVB)).astype(np.float32)
    qd, kd, vd = G.bf16(qf), G.bf16(kf), G.bf16(vf)
    scale = 0.1355
    out = torch.empty(T, nh * 128, dtype=torch.bfloat16, device=G.DEV)
    G.check(G.L().b200_flash_prefill_packed(qd.data_ptr(), NQP, 192, kd.data_ptr(), nh * 192, 192,
                                            vd.data_ptr() + 128 * 2, KVB, 256, out.data_ptr(), nh * 128, 128,
                                            G.i32(cu).data_ptr(), len(lens), max(lens), T, nh, nh, 192, 128, scale,
                                            causal, G.stream()), "flash_prefill_packed 192/128")
    got = G.host(out).reshape(T, nh, 128)
    q = G.rounded(qf)[:, :nh * 192].reshape(T, nh, 192)
    k = G.rounded(kf).reshape(T, nh, 192)
    v = G.rounded(vf).reshape(T, nh, 256)[:, :, 128:]
    ref = np.zeros((T, nh, 128), np.float32)
    for a, b in zip(cu[:-1], cu[1:]):
        s = np.einsum("qhd,khd->hqk", q[a:b], k[a:b]) * np.float32(scale)
        if causal:
            s = np.where(np.triu(np.ones((b - a, b - a), bool), 1)[None], -np.inf, s)
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        ref[a:b] = np.einsum("hqk,khd->qhd", p, v[a:b])
    assert G.cosine(got, ref) > 0.9999
    assert G.max_rel_err(got, ref) < 0.02
    # the legacy-MMA kernel behind b200_flash_prefill_ex on the same inputs
    old = torch.empty_like(out)
    G.check(G.L().b200_flash_prefill_ex(qd.data_ptr(), NQP, 192, kd.data_ptr(), nh * 192, 192,
                                        vd.data_ptr() + 128 * 2, KVB, 256, old.data_ptr(), nh * 128, 128,
                                        G.i32(cu).data_ptr(), len(lens), max(lens), nh, nh, 192, 128, scale, causal,
                                        G.stream()), "flash_prefill_ex 192/128")
    assert G.cosine(got, G.host(old).reshape(T, nh, 128)) > 0.9999
    assert G.device_errors() == 0
