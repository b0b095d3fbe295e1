"""tcgen05 prefill attention (b200_flash_prefill_packed, 64- and 128-wide heads)
against the numpy oracle and a torch fp32 reference.

Cases: packed variable-length sequences around the 128-row tile edges, causal
and bidirectional, 64- and 128-wide heads, GQA, the packed q|k|v layout of the
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


@pytest.mark.parametrize("causal,hd", [(1, 128), (0, 128), (1, 64), (0, 64)])
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
