"""GPU parity of each kernel against the CPU oracle (and the reference's
golden vectors), all calls through the C ABI.

Tolerances (floating point): the kernels read bf16 inputs and write bf16
outputs, so the oracle is evaluated on the same bf16-rounded inputs and the
comparison allows bf16 output rounding (2^-8 relative) plus fp32 accumulation
order differences: cosine >= 0.9999 per op and max |err| <= 1-2 % of max |ref|.
Integer work (slot mapping, argmax) is compared bit-exactly.
"""

import numpy as np
import pytest
import torch

import oracle
from conftest import load_fixture

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gpu_util as G


def test_rmsnorm_golden_and_fused_residual():
    fx = load_fixture("rms_norm")
    for name in ("typical", "small", "medium"):
        x, w = fx[f"{name}_input"], fx[f"{name}_weight"]
        xd, wd = G.bf16(x), G.bf16(w)
        out = torch.empty_like(xd)
        G.check(G.L().b200_rmsnorm(xd.data_ptr(), None, wd.data_ptr(), out.data_ptr(), None, x.shape[0], x.shape[1],
                                   x.shape[1], 1e-6, G.stream()))
        ref = oracle.rms_norm(G.rounded(x), G.rounded(w), 1e-6)
        assert G.cosine(G.host(out), ref) > 0.9999
        assert G.max_rel_err(G.host(out), ref) < 0.01
        # against the reference's own golden (fp32 inputs): bf16 input rounding only
        assert G.cosine(G.host(out), fx[f"{name}_output"]) > 0.9999
    for name in ("typical", "small"):
        x, r, w = (fx[f"prenorm_{name}_{k}"] for k in ("input", "residual", "weight"))
        xd, rd, wd = G.bf16(x), G.bf16(r), G.bf16(w)
        out, rout = torch.empty_like(xd), torch.empty_like(xd)
        G.check(G.L().b200_rmsnorm(xd.data_ptr(), rd.data_ptr(), wd.data_ptr(), out.data_ptr(), rout.data_ptr(),
                                   x.shape[0], x.shape[1], x.shape[1], 1e-5, G.stream()))
        h = G.rounded(x) + G.rounded(r)
        assert G.max_rel_err(G.host(rout), h) < 0.005
        assert G.cosine(G.host(out), fx[f"prenorm_{name}_output"]) > 0.9999
        assert G.cosine(G.host(out), oracle.rms_norm(h, G.rounded(w), 1e-5)) > 0.9999


def test_layernorm():
    rng = np.random.default_rng(3)
    for rows, dim in ((4, 64), (784, 1024), (196, 4096)):
        x = rng.standard_normal((rows, dim)).astype(np.float32)
        g = (rng.random(dim).astype(np.float32) - 0.5) * 0.4 + 1
        b = (rng.random(dim).astype(np.float32) - 0.5) * 0.2
        xd, gd, bd = G.bf16(x), G.bf16(g), G.bf16(b)
        out = torch.empty_like(xd)
        G.check(G.L().b200_layernorm(xd.data_ptr(), gd.data_ptr(), bd.data_ptr(), out.data_ptr(), rows, dim, 1e-6,
                                     G.stream()))
        ref = oracle.layer_norm(G.rounded(x), G.rounded(g), G.rounded(b), 1e-6)
        assert G.cosine(G.host(out), ref) > 0.9999
        assert G.max_rel_err(G.host(out), ref) < 0.01


GEMM_SHAPES = [
    # (M, N, K) — prefill-like (normal orientation) and decode-like (swapped)
    (256, 512, 256), (300, 520, 264), (1024, 768, 1024), (129, 136, 72), (2048, 6144, 512),
    (16, 2048, 2048), (1, 64, 128), (64, 4096, 4096), (100, 264, 8), (128, 1024, 640),
]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_shapes(M, N, K):
    torch.manual_seed(M * 7 + N * 3 + K)
    A = (torch.randn(M, K, device=G.DEV) * 0.5).to(torch.bfloat16)
    B = (torch.randn(N, K, device=G.DEV) * 0.5).to(torch.bfloat16)
    ref = (A.float() @ B.float().T).cpu().numpy()
    for ws in (True, False):
        out = G.gemm(A, B, ws=ws)
        torch.cuda.synchronize()
        got = G.host(out)
        assert np.isfinite(got).all()
        assert G.cosine(got, ref) > 0.9999, (M, N, K, ws)
        assert G.max_rel_err(got, ref) < 0.01, (M, N, K, ws)
    assert G.device_errors() == 0


def test_gemm_splitk_workspace_reuse():
    """One workspace, zeroed once, serves a sequence of split-K calls of
    different shapes and epilogues: each call must leave its tile counters at
    zero for the next (a stale counter would make a wrong split finish a tile)."""
    torch.manual_seed(0)
    shapes = [(64, 4096, 4096, 0), (64, 2048, 4096, 3), (7, 4096, 1024, 2), (64, 1024, 8192, 0)]
    L = G.L()
    wsb = max(L.b200_gemm_workspace_bytes(M, N, K, e) for M, N, K, e in shapes)
    assert wsb > 0
    ws = torch.zeros(wsb, dtype=torch.uint8, device=G.DEV)
    for rep in range(2):
        for M, N, K, epi in shapes:
            A = (torch.randn(M, K, device=G.DEV) * 0.5).to(torch.bfloat16)
            B = (torch.randn(N, K, device=G.DEV) * 0.1).to(torch.bfloat16)
            R = torch.randn(M, N, device=G.DEV).to(torch.bfloat16)
            acc = A.float() @ B.float().T
            ref = {0: acc, 2: acc + R.float(), 3: torch.nn.functional.silu(acc[:, 0::2]) * acc[:, 1::2]}[epi]
            got = G.host(G.gemm(A, B, epi=epi, R=R, ws=ws))
            assert G.cosine(got, ref.cpu().numpy()) > 0.9999, (rep, M, N, K, epi)
            assert G.max_rel_err(got, ref.cpu().numpy()) < 0.01, (rep, M, N, K, epi)
    assert G.device_errors() == 0


@pytest.mark.parametrize("M", [8, 96, 640])
def test_gemm_epilogues(M):
    torch.manual_seed(M)
    N, K = 384, 512
    A = (torch.randn(M, K, device=G.DEV) * 0.5).to(torch.bfloat16)
    B = (torch.randn(N, K, device=G.DEV) * 0.1).to(torch.bfloat16)
    bias = (torch.randn(N, device=G.DEV)).to(torch.bfloat16)
    R = (torch.randn(M, N, device=G.DEV)).to(torch.bfloat16)
    acc = A.float() @ B.float().T
    cases = {
        1: acc + bias.float(),
        2: acc + R.float(),
        4: torch.nn.functional.gelu(acc + bias.float(), approximate="tanh"),
        5: acc + bias.float() + R.float(),
        3: torch.nn.functional.silu(acc[:, 0::2]) * acc[:, 1::2],
    }
    for epi, ref in cases.items():
        for ws in (True, False):
            out = G.gemm(A, B, epi=epi, bias=bias, R=R, ws=ws)
            got = G.host(out)
            ref_np = ref.cpu().numpy()
            assert G.cosine(got, ref_np) > 0.9999, (epi, ws)
            assert G.max_rel_err(got, ref_np) < 0.01, (epi, ws)
    # residual epilogue in place (R aliases C): h += x W^T
    h = R.clone()
    G.gemm(A, B, epi=2, R=h, out=h)
    assert G.max_rel_err(G.host(h), (acc + R.float()).cpu().numpy()) < 0.01


def test_gemm_linear_golden():
    import regen

    fx = load_fixture("linear")
    inp = regen.linear_inputs(16, 2048, 2048)
    out = G.gemm(G.bf16(inp["input"]), G.bf16(inp["weight"]))
    assert G.cosine(G.host(out), fx["typical_output"]) > 0.9999
    x, w, b = fx["small_bias_input"], fx["small_bias_weight"], fx["small_bias_bias"]
    out = G.gemm(G.bf16(x), G.bf16(w), epi=1, bias=G.bf16(b))
    assert G.cosine(G.host(out), fx["small_bias_output"]) > 0.9999


def test_rope_tables_mrope_golden_and_1d():
    fx = load_fixture("mrope")
    pid = fx["pid"][:, 0, :]  # [3, S]
    T = pid.shape[1]
    c = torch.empty(T, 128, device=G.DEV)
    s = torch.empty_like(c)
    G.check(G.L().b200_rope_table_mrope(G.i64(pid).data_ptr(), T, 128, 5e6, 24, 20, 20, c.data_ptr(), s.data_ptr(),
                                        G.stream()))
    np.testing.assert_allclose(G.host(c), fx["cos"][0], atol=2e-6, rtol=0)
    np.testing.assert_allclose(G.host(s), fx["sin"][0], atol=2e-6, rtol=0)
    # text-only ids t=h=w=arange(256): interleaved mrope equals 1-D rope
    pos = np.arange(256)
    pid3 = np.stack([pos, pos, pos])
    cm, sm = torch.empty(256, 128, device=G.DEV), torch.empty(256, 128, device=G.DEV)
    G.check(G.L().b200_rope_table_mrope(G.i64(pid3).data_ptr(), 256, 128, 5e6, 24, 20, 20, cm.data_ptr(),
                                        sm.data_ptr(), G.stream()))
    rc, rs = oracle.mrope_cos_sin(pid3[:, None, :], 128, 5e6, (24, 20, 20))
    # inv_freq from the host's powf and numpy's float32 power may differ by one
    # ulp (6e-8 relative); times positions up to 255 that moves the angle by up
    # to ~1.5e-5 rad.  The reference gates this table at cosine > 0.9999
    # (test_mrope_cpu.cpp:396).
    np.testing.assert_allclose(G.host(cm), rc[0], atol=3e-5, rtol=0)
    np.testing.assert_allclose(G.host(sm), rs[0], atol=3e-5, rtol=0)
    assert G.cosine(G.host(cm), rc[0]) > 0.9999999
    pos = np.arange(0, 4096, 3)
    c1, s1 = torch.empty(len(pos), 128, device=G.DEV), torch.empty(len(pos), 128, device=G.DEV)
    G.check(G.L().b200_rope_table_1d(G.i64(pos).data_ptr(), len(pos), 128, 1e6, c1.data_ptr(), s1.data_ptr(),
                                     G.stream()))
    rc, rs = oracle.rope1d_cos_sin(pos, 128, 1e6)
    # same one-ulp inv_freq difference as above; at positions up to 4095 the
    # angle can move by 4095 x 2^-24 = 2.4e-4 rad
    np.testing.assert_allclose(G.host(c1), rc, atol=5e-4, rtol=0)
    np.testing.assert_allclose(G.host(s1), rs, atol=5e-4, rtol=0)
    assert G.cosine(G.host(c1), rc) > 0.999999 and G.cosine(G.host(s1), rs) > 0.999999


def test_qk_norm_rope_golden_no_norm():
    fx = load_fixture("rope")
    for name in ("basic", "gqa"):
        S, nh, kvh, hd = (int(v) for v in fx[f"{name}_meta"])
        q = fx[f"{name}_q"].astype(np.float32)
        k = fx[f"{name}_k"].astype(np.float32)
        qkv = np.concatenate([q, k, np.zeros_like(k)], 1)
        d = G.bf16(qkv)
        cos = G.f32(fx[f"{name}_cos"].astype(np.float32))
        sin = G.f32(fx[f"{name}_sin"].astype(np.float32))
        G.check(G.L().b200_qk_norm_rope(d.data_ptr(), S, nh, kvh, hd, qkv.shape[1], None, None, 1e-6, cos.data_ptr(),
                                        sin.data_ptr(), None, None, None, 0, 0, G.stream()))
        got = G.host(d)
        assert G.cosine(got[:, : nh * hd], fx[f"{name}_rq_ref"].astype(np.float32)) > 0.9999
        assert G.cosine(got[:, nh * hd: (nh + kvh) * hd], fx[f"{name}_rk_ref"].astype(np.float32)) > 0.9999


@pytest.mark.parametrize("hd", [64, 128])
def test_qk_norm_rope_with_norm_and_cache_write(hd):
    rng = np.random.default_rng(hd)
    T, nq, nkv, bs, nblk = 37, 8, 2, 16, 9
    W = (nq + 2 * nkv) * hd
    qkv = rng.standard_normal((T, W)).astype(np.float32)
    qn = rng.standard_normal(hd).astype(np.float32) * 0.1 + 1
    kn = rng.standard_normal(hd).astype(np.float32) * 0.1 + 1
    pos = rng.integers(0, 3000, T)
    cos, sin = oracle.rope1d_cos_sin(pos, hd, 1e6)
    table = rng.permutation(nblk)[:3]
    slots = oracle.slot_mapping(table, np.arange(T), bs)
    slots[5] = -1  # skipped token
    d = G.bf16(qkv)
    kc = torch.zeros(nblk, nkv, bs, hd, dtype=torch.bfloat16, device=G.DEV)
    vc = torch.zeros_like(kc)
    G.check(G.L().b200_qk_norm_rope(d.data_ptr(), T, nq, nkv, hd, W, G.bf16(qn).data_ptr(), G.bf16(kn).data_ptr(),
                                    1e-6, G.f32(cos).data_ptr(), G.f32(sin).data_ptr(), G.i64(slots).data_ptr(),
                                    kc.data_ptr(), vc.data_ptr(), nblk, bs, G.stream()))
    x = G.rounded(qkv)
    q = oracle.rope_half(oracle.rms_norm(x[:, : nq * hd].reshape(T, nq, hd), G.rounded(qn), 1e-6), cos, sin)
    k = oracle.rope_half(oracle.rms_norm(x[:, nq * hd: (nq + nkv) * hd].reshape(T, nkv, hd), G.rounded(kn), 1e-6),
                         cos, sin)
    got = G.host(d)
    assert G.cosine(got[:, : nq * hd], q.reshape(T, -1)) > 0.9999
    assert G.max_rel_err(got[:, : nq * hd], q.reshape(T, -1)) < 0.01
    assert G.cosine(got[:, nq * hd: (nq + nkv) * hd], k.reshape(T, -1)) > 0.9999
    # v untouched; cache holds exactly the bf16 k / v of each written token
    np.testing.assert_array_equal(got[:, (nq + nkv) * hd:], x[:, (nq + nkv) * hd:])
    kch, vch = G.host(kc), G.host(vc)
    for t in range(T):
        s = slots[t]
        if s < 0:
            continue
        np.testing.assert_array_equal(kch[s // bs, :, s % bs].reshape(-1), got[t, nq * hd: (nq + nkv) * hd])
        np.testing.assert_array_equal(vch[s // bs, :, s % bs].reshape(-1), got[t, (nq + nkv) * hd:])
    assert G.device_errors() == 0


def test_slot_mapping_bit_exact():
    rng = np.random.default_rng(1)
    B, maxb, bs = 5, 7, 128
    bt = rng.integers(0, 1000, (B, maxb)).astype(np.int32)
    seq = rng.integers(0, B, 999).astype(np.int32)
    pos = rng.integers(0, maxb * bs, 999)
    out = torch.empty(999, dtype=torch.int64, device=G.DEV)
    G.check(G.L().b200_slot_mapping(G.i32(bt).data_ptr(), maxb, G.i32(seq).data_ptr(), G.i64(pos).data_ptr(), 999, bs,
                                    out.data_ptr(), G.stream()))
    ref = np.array([oracle.slot_mapping(bt[s], p, bs) for s, p in zip(seq, pos)])
    np.testing.assert_array_equal(out.cpu().numpy(), ref)
    assert G.device_errors() == 0


def test_prefill_attention_goldens():
    fx = load_fixture("self_attention")
    names = sorted({k[: -len("_meta")] for k in fx if k.endswith("_meta")})
    for name in names:
        S, nh, kvh, hd, has_mask = (int(v) for v in fx[f"{name}_meta"])
        q = G.rounded(fx[f"{name}_q"].astype(np.float32).reshape(S, -1))
        k = G.rounded(fx[f"{name}_k"].astype(np.float32).reshape(S, -1))
        v = G.rounded(fx[f"{name}_v"].astype(np.float32).reshape(S, -1))
        out = torch.empty(S, nh * hd, dtype=torch.bfloat16, device=G.DEV)
        cu = G.i32([0, S])
        G.check(G.L().b200_flash_prefill(G.bf16(q).data_ptr(), nh * hd, G.bf16(k).data_ptr(), G.bf16(v).data_ptr(),
                                         kvh * hd, out.data_ptr(), nh * hd, cu.data_ptr(), 1, S, nh, kvh, hd,
                                         1.0 / np.sqrt(hd), has_mask, G.stream()))
        ref = oracle.sdpa_gqa(q.reshape(S, nh, hd), k.reshape(S, kvh, hd), v.reshape(S, kvh, hd), nh, kvh,
                              causal=bool(has_mask)).reshape(S, -1)
        got = G.host(out)
        assert G.cosine(got, ref) > 0.9999, name
        assert G.max_rel_err(got, ref) < 0.02, name
        assert G.cosine(got, fx[f"{name}_out_ref"].astype(np.float32).reshape(S, -1)) > 0.999, name


@pytest.mark.parametrize("hd", [64, 128])
def test_prefill_attention_varlen(hd):
    rng = np.random.default_rng(hd + 1)
    lens = [1, 63, 64, 65, 200, 17]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T, nq, nkv = int(cu[-1]), 8, 2
    qkv = rng.standard_normal((T, (nq + 2 * nkv) * hd)).astype(np.float32)
    d = G.bf16(qkv)
    x = G.rounded(qkv)
    out = torch.empty(T, nq * hd, dtype=torch.bfloat16, device=G.DEV)
    W = (nq + 2 * nkv) * hd
    for causal in (1, 0):
        G.check(G.L().b200_flash_prefill(d.data_ptr(), W, d.data_ptr() + nq * hd * 2, d.data_ptr() + (nq + nkv) * hd * 2,
                                         W, out.data_ptr(), nq * hd, G.i32(cu).data_ptr(), len(lens), max(lens), nq,
                                         nkv, hd, 1.0 / np.sqrt(hd), causal, G.stream()))
        q = x[:, : nq * hd].reshape(T, nq, hd)
        k = x[:, nq * hd: (nq + nkv) * hd].reshape(T, nkv, hd)
        v = x[:, (nq + nkv) * hd:].reshape(T, nkv, hd)
        if causal:
            ref = oracle.varlen_causal_attention(q, k, v, cu, nq, nkv)
        else:
            ref = np.concatenate([oracle.sdpa_gqa(q[a:b], k[a:b], v[a:b], nq, nkv) for a, b in zip(cu[:-1], cu[1:])])
        got = G.host(out).reshape(T, nq, hd)
        assert G.cosine(got, ref) > 0.9999
        assert G.max_rel_err(got, ref) < 0.02


@pytest.mark.parametrize("bs", [128, 64])
def test_paged_decode(bs):
    rng = np.random.default_rng(bs)
    B, nq, nkv, hd = 6, 32, 8, 128
    ctx = np.array([1, 63, 64, 65, 700, 2048])
    maxb = int((ctx.max() + bs - 1) // bs)
    nblk = B * maxb + 3
    kc = rng.standard_normal((nblk, nkv, bs, hd)).astype(np.float32)
    vc = rng.standard_normal((nblk, nkv, bs, hd)).astype(np.float32)
    tables = rng.permutation(nblk)[: B * maxb].reshape(B, maxb).astype(np.int32)
    q = rng.standard_normal((B, nq * hd)).astype(np.float32)
    kcd, vcd, qd = G.bf16(kc), G.bf16(vc), G.bf16(q)
    ref = oracle.paged_decode_attention(G.rounded(q).reshape(B, nq, hd), G.rounded(kc), G.rounded(vc), tables, ctx)
    for use_ws in (True, False):
        out = torch.empty(B, nq * hd, dtype=torch.bfloat16, device=G.DEV)
        wsb = G.L().b200_paged_decode_workspace_bytes(B, nq, hd, int(ctx.max())) if use_ws else 0
        ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=G.DEV)
        G.check(G.L().b200_paged_decode(qd.data_ptr(), nq * hd, kcd.data_ptr(), vcd.data_ptr(), G.i32(tables).data_ptr(),
                                        maxb, G.i32(ctx).data_ptr(), B, nq, nkv, hd, bs, nblk, 1.0 / np.sqrt(hd),
                                        out.data_ptr(), nq * hd, ws.data_ptr() if wsb else None, wsb, int(ctx.max()),
                                        G.stream()))
        got = G.host(out).reshape(B, nq, hd)
        for b in range(B):
            assert G.cosine(got[b], ref[b]) > 0.9999, (b, use_ws)
            assert G.max_rel_err(got[b], ref[b]) < 0.02, (b, use_ws)
    assert G.device_errors() == 0


def test_embedding_argmax_scatter():
    rng = np.random.default_rng(5)
    V, H = 1000, 64
    table = rng.standard_normal((V, H)).astype(np.float32)
    ids = np.array([0, 5, 999, 1000, -1, 17])
    out = torch.empty(len(ids), H, dtype=torch.bfloat16, device=G.DEV)
    G.check(G.L().b200_embedding(G.i64(ids).data_ptr(), len(ids), G.bf16(table).data_ptr(), V, H, out.data_ptr(),
                                 G.stream()))
    got = G.host(out)
    tr = G.rounded(table)
    for i, t in enumerate(ids):
        np.testing.assert_array_equal(got[i], tr[t] if 0 <= t < V else np.zeros(H, np.float32))
    logits = rng.standard_normal((7, 5000)).astype(np.float32)
    logits[3, 10] = logits[3, 4000] = 50.0  # tie -> lowest index
    am = torch.empty(7, dtype=torch.int64, device=G.DEV)
    G.check(G.L().b200_argmax(G.bf16(logits).data_ptr(), 7, 5000, 5000, am.data_ptr(), G.stream()))
    np.testing.assert_array_equal(am.cpu().numpy(), np.argmax(G.rounded(logits), 1))
    hid = rng.standard_normal((20, H)).astype(np.float32)
    feat = rng.standard_normal((4, H)).astype(np.float32)
    idx = np.array([3, 0, 19, 7], np.int32)
    hd = G.bf16(hid)
    G.check(G.L().b200_scatter_add_rows(hd.data_ptr(), 20, H, G.i32(idx).data_ptr(), G.bf16(feat).data_ptr(), 4, 1.0,
                                        G.stream()))
    ref = G.rounded(hid).copy()
    ref[idx] += G.rounded(feat)
    assert G.max_rel_err(G.host(hd), ref) < 0.01
    assert G.device_errors() == 0
