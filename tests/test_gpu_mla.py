"""GPU parity of the multi-head latent attention kernels through the C ABI
against oracle.mla: YaRN rope tables, the per-token latent preparation
(RMSNorm of the compressed KV, de-interleaved rope, latent cache write, query
rope in place), the absorbed-latent paged decode (split and unsplit, ragged
contexts, shuffled block tables) and the decompressed 192/128 prefill
attention.

Bars: rope tables within 5e-5; prepared rows cosine >= 0.9999 and within 1 %
of max |ref| (bf16 storage); attention outputs cosine >= 0.999, max |err| <=
2 % of max |ref|.
"""

import numpy as np
import pytest
import torch

from oracle import mla

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gpu_util as G

F = np.float32
CFG = dict(heads=16, qk_nope=128, qk_rope=64, v_head=128, kv_lora=512, eps=1e-6, theta=10000.0,
           yarn=dict(factor=40.0, orig_max_pos=4096, beta_fast=32, beta_slow=1, mscale=0.707, mscale_all_dim=0.707))


def rope_tables(pos, cfg=CFG):
    y = cfg["yarn"]
    inv = mla.yarn_inv_freq(64, cfg["theta"], y["factor"], y["orig_max_pos"], y["beta_fast"], y["beta_slow"])
    ms = mla.yarn_get_mscale(y["factor"], y["mscale"]) / mla.yarn_get_mscale(y["factor"], y["mscale_all_dim"])
    T = len(pos)
    c = torch.empty(T, 64, device=G.DEV)
    s = torch.empty_like(c)
    inv = np.ascontiguousarray(inv, F)
    G.check(G.L().b200_rope_table_freqs(G.i64(pos).data_ptr(), T, 64, inv.ctypes.data, ms, c.data_ptr(), s.data_ptr(),
                                        G.stream()))
    return c, s


def close(got, ref, cos=0.999, tol=0.02):
    assert G.cosine(got, ref) >= cos, G.cosine(got, ref)
    assert G.max_rel_err(got, ref) <= tol, G.max_rel_err(got, ref)


def test_rope_table_freqs():
    pos = np.array([0, 1, 7, 100, 2047, 4095], np.int64)
    c, s = rope_tables(pos)
    rc, rs = mla.rope_cfg_tables(pos, CFG)
    np.testing.assert_allclose(G.host(c), rc, atol=5e-5, rtol=0)
    np.testing.assert_allclose(G.host(s), rs, atol=5e-5, rtol=0)


@pytest.mark.parametrize("q_hs,q_off", [(192, 128), (576, 512)], ids=["prefill-layout", "decode-layout"])
def test_mla_prep(q_hs, q_off):
    rng = np.random.default_rng(q_hs)
    T, nh = 37, 16
    q = G.rounded(rng.standard_normal((T, nh * q_hs)).astype(F))
    kva = G.rounded(rng.standard_normal((T, 576)).astype(F))
    nw = G.rounded(1 + 0.1 * rng.standard_normal(512).astype(F))
    pos = rng.integers(0, 4000, T).astype(np.int64)
    c, s = rope_tables(pos)
    qd = G.bf16(q)
    slots = rng.permutation(64)[:T].astype(np.int64)
    slots[3] = -1  # not cached
    cache = torch.zeros(64, 576, dtype=torch.bfloat16, device=G.DEV)
    ckv = torch.empty(T, 512, dtype=torch.bfloat16, device=G.DEV)
    kpe = torch.empty(T, 64, dtype=torch.bfloat16, device=G.DEV)
    G.check(G.L().b200_mla_prep(qd.data_ptr(), nh * q_hs, q_hs, nh, q_off, G.bf16(kva).data_ptr(), 576,
                                G.bf16(nw).data_ptr(), 1e-6, c.data_ptr(), s.data_ptr(), G.i64(slots).data_ptr(),
                                cache.data_ptr(), 64, ckv.data_ptr(), kpe.data_ptr(), T, G.stream()), "mla_prep")
    torch.cuda.synchronize()
    rc, rs = mla.rope_cfg_tables(pos, CFG)
    ref_c = kva[:, :512] / np.sqrt((kva[:, :512].astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6) * nw
    ref_k = mla.rope_deinterleave(kva[:, 512:], rc, rs)
    close(G.host(ckv), ref_c, 0.9999, 0.01)
    close(G.host(kpe), ref_k, 0.9999, 0.01)
    ch = G.host(cache)
    for t in range(T):
        if slots[t] >= 0:
            np.testing.assert_array_equal(ch[slots[t], :512], G.host(ckv)[t])
            np.testing.assert_array_equal(ch[slots[t], 512:], G.host(kpe)[t])
    qh = q.reshape(T, nh, q_hs).copy()
    qh[:, :, q_off:q_off + 64] = mla.rope_deinterleave(qh[:, :, q_off:q_off + 64], rc[:, None], rs[:, None])
    close(G.host(qd), qh.reshape(T, -1), 0.9999, 0.01)
    assert G.device_errors() == 0


@pytest.mark.parametrize("nh,ctx,block,split,ramp", [
    (16, [1, 63, 64, 65, 1000, 4096], 64, True, False),
    (16, [1, 63, 64, 65, 1000, 4096], 128, False, False),
    (32, [1300, 17], 128, True, False),
    # 192-token blocks: a 128-token tile spans two cache blocks
    (16, [129, 191, 193, 2000], 192, True, False),
    # scores that grow along the context: the running max moves tile after tile
    (16, [3000, 700, 128], 64, False, True),
    (16, [3000, 700, 128], 128, True, True),
    # more (sequence, head group) pairs than SMs: several waves of split CTAs
    (16, [(37 * i) % 400 + 1 for i in range(150)], 64, True, False),
])
def test_mla_decode(nh, ctx, block, split, ramp):
    rng = np.random.default_rng(nh + block)
    B = len(ctx)
    max_ctx = max(ctx)
    mb = (max_ctx + block - 1) // block
    nblocks = B * mb + 3
    cache = rng.standard_normal((nblocks * block, 576)).astype(F)
    tables = rng.permutation(nblocks)[:B * mb].reshape(B, mb).astype(np.int32)
    q = G.rounded(rng.standard_normal((B, nh * 576)).astype(F) * (0.5 if ramp else 0.05))
    if ramp:
        # row j of block table entry k of sequence b holds token k*block + j:
        # scale it by 1 + 3 * position / max_ctx (the same direction per token)
        q[:, :] = np.abs(q)
        for b in range(B):
            for k in range(mb):
                pos = k * block + np.arange(block)
                rows = slice(tables[b, k] * block, (tables[b, k] + 1) * block)
                cache[rows] = np.abs(cache[rows]) * (1.0 + 3.0 * pos / max_ctx)[:, None]
    cache = G.rounded(cache)
    scale = mla.softmax_scale(CFG)
    out = torch.empty(B, nh * 512, dtype=torch.bfloat16, device=G.DEV)
    L = G.L()
    wsb = L.b200_mla_decode_workspace_bytes(B, nh, max_ctx) if split else 0
    ws = torch.zeros(max(wsb, 16), dtype=torch.uint8, device=G.DEV)
    if split:
        assert wsb > 0
    G.check(L.b200_mla_decode(G.bf16(q).data_ptr(), nh * 576, G.bf16(cache).data_ptr(), G.i32(tables).data_ptr(), mb,
                              G.i32(np.array(ctx, np.int32)).data_ptr(), B, nh, block, nblocks, scale, out.data_ptr(),
                              nh * 512, ws.data_ptr() if split else None, wsb, max_ctx, G.stream()), "mla_decode")
    torch.cuda.synchronize()
    rows = [cache[np.concatenate([np.arange(tables[b, j] * block, (tables[b, j] + 1) * block) for j in range(mb)])]
            for b in range(B)]
    ref = mla.latent_decode(q, rows, ctx, nh, scale)
    close(G.host(out), ref)
    assert G.device_errors() == 0


def test_flash_prefill_mla_heads():
    """Decompressed MLA heads: Q/K 192 wide (K assembled from k_nope + shared
    k_pe), V 128 wide read in place from the kv_b output (head stride 256)."""
    rng = np.random.default_rng(5)
    nh = 16
    cu = [0, 70, 200]
    T = cu[-1]
    q = G.rounded(rng.standard_normal((T, nh * 192)).astype(F))
    k = G.rounded(rng.standard_normal((T, nh * 192)).astype(F))
    kvb = G.rounded(rng.standard_normal((T, nh * 256)).astype(F))
    out = torch.empty(T, nh * 128, dtype=torch.bfloat16, device=G.DEV)
    scale = mla.softmax_scale(CFG)
    kvd = G.bf16(kvb)
    G.check(G.L().b200_flash_prefill_ex(G.bf16(q).data_ptr(), nh * 192, 192, G.bf16(k).data_ptr(), nh * 192, 192,
                                        kvd.data_ptr() + 128 * 2, nh * 256, 256, out.data_ptr(), nh * 128, 128,
                                        G.i32(np.array(cu, np.int32)).data_ptr(), 2, 130, nh, nh, 192, 128, scale, 1,
                                        G.stream()), "flash_prefill_ex")
    torch.cuda.synchronize()
    ref = np.zeros((T, nh, 128), F)
    qh, kh, vh = q.reshape(T, nh, 192), k.reshape(T, nh, 192), kvb.reshape(T, nh, 256)[:, :, 128:]
    for a, b in zip(cu[:-1], cu[1:]):
        n = b - a
        s = np.einsum("qhd,khd->hqk", qh[a:b], kh[a:b]) * scale
        s = np.where(np.triu(np.ones((n, n), bool), 1)[None], -np.inf, s)
        p = np.exp(s - s.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        ref[a:b] = np.einsum("hqk,khd->qhd", p, vh[a:b])
    close(G.host(out), ref.reshape(T, -1))
