"""GPU parity of the MoE path through the C ABI against oracle.moe and
per-group fp32 matmuls: router top-k (expert ids bit-exact, ties to the lower
index), the expert permutation (bit-exact), the grouped tcgen05 GEMM (both the
few-tokens-per-expert and the many-tokens-per-expert tilings, empty experts,
ragged feature tails), the weighted combine with fused residual + RMSNorm, and
the whole routed + shared expert MLP composed from them.

Bars: integers exact; GEMM outputs cosine >= 0.9999 and max |err| <= 1 % of
max |ref| (bf16 output rounding); routing weights within 1e-5; composed MLP
cosine >= 0.999, max |err| <= 2 %.
"""

import numpy as np
import pytest
import torch

from oracle import moe
from oracle.layers import silu

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gpu_util as G

F = np.float32


def topk(logits, k, renorm=1, scale=1.0):
    T, E = logits.shape
    lg = G.f32(logits)
    ids = torch.empty(T, k, dtype=torch.int32, device=G.DEV)
    w = torch.empty(T, k, dtype=torch.float32, device=G.DEV)
    G.check(G.L().b200_moe_topk(lg.data_ptr(), T, E, k, renorm, scale, ids.data_ptr(), w.data_ptr(), G.stream()))
    return ids.cpu().numpy(), G.host(w)


@pytest.mark.parametrize("E,k,renorm", [(8, 2, 1), (64, 6, 0), (128, 8, 1), (5, 5, 1)])
def test_topk_bit_exact_with_ties(E, k, renorm):
    rng = np.random.default_rng(E)
    T = 777
    lg = (rng.integers(-4, 5, (T, E)) * 0.5).astype(F)  # many exact ties
    lg[::7] = rng.standard_normal((len(lg[::7]), E)).astype(F)
    ids, w = topk(lg, k, renorm, 1.0 if renorm else 1.5)
    rid, rw = moe.route_topk(lg, k, bool(renorm), 1.0 if renorm else 1.5)
    np.testing.assert_array_equal(ids, rid)
    np.testing.assert_allclose(w, rw, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("E,k,H", [(8, 2, 4096), (64, 6, 2048)])
def test_route_gate_gemv(E, k, H):
    rng = np.random.default_rng(3)
    T = 300
    x = G.rounded(rng.standard_normal((T, H)).astype(F))
    wg = G.rounded(rng.standard_normal((E, H)).astype(F) * 0.02)
    ids = torch.empty(T, k, dtype=torch.int32, device=G.DEV)
    w = torch.empty(T, k, dtype=torch.float32, device=G.DEV)
    lg = torch.empty(T, E, dtype=torch.float32, device=G.DEV)
    G.check(G.L().b200_moe_route(G.bf16(x).data_ptr(), H, G.bf16(wg).data_ptr(), T, H, E, k, 1, 1.0, ids.data_ptr(),
                                 w.data_ptr(), lg.data_ptr(), G.stream()))
    ref = x.astype(np.float64) @ wg.astype(np.float64).T
    np.testing.assert_allclose(G.host(lg), ref, rtol=0, atol=1e-4 * np.abs(ref).max())
    # the selection is exact on the kernel's own logits; against the fp64 logits
    # it may only differ where the k-th and (k+1)-th logits are within noise
    rid, rw = moe.route_topk(G.host(lg), k)
    np.testing.assert_array_equal(ids.cpu().numpy(), rid)
    np.testing.assert_allclose(G.host(w), rw, rtol=1e-5, atol=1e-6)
    srt = np.sort(ref, 1)[:, ::-1]
    clear = (srt[:, k - 1] - srt[:, k]) > 1e-3
    fid, _ = moe.route_topk(ref.astype(F), k)
    np.testing.assert_array_equal(ids.cpu().numpy()[clear], fid[clear])


def permute(ids, E, x=None):
    T, k = ids.shape
    L = G.L()
    wsb = L.b200_moe_permute_workspace_bytes(T, k, E)
    ws = torch.zeros(max(wsb, 16), dtype=torch.uint8, device=G.DEV)
    idd = G.i32(ids)
    off = torch.full((E + 1,), -5, dtype=torch.int32, device=G.DEV)
    pos = torch.full((T * k,), -5, dtype=torch.int32, device=G.DEV)
    src = torch.full((T * k,), -5, dtype=torch.int32, device=G.DEV)
    H = 0 if x is None else x.shape[1]
    xp = None if x is None else torch.zeros(T * k, H, dtype=torch.bfloat16, device=G.DEV)
    xd = None if x is None else G.bf16(x)
    G.check(L.b200_moe_permute(idd.data_ptr(), T, k, E, G.ptr(xd), H, H, G.ptr(xp), off.data_ptr(), pos.data_ptr(),
                               src.data_ptr(), ws.data_ptr(), wsb, G.stream()), "moe_permute")
    torch.cuda.synchronize()
    return off.cpu().numpy(), pos.cpu().numpy(), src.cpu().numpy(), xp


@pytest.mark.parametrize("T,k,E", [(1, 2, 8), (300, 2, 8), (4096, 6, 64), (1000, 1, 3)])
def test_permute_bit_exact(T, k, E):
    rng = np.random.default_rng(T)
    ids = rng.integers(0, E, (T, k)).astype(np.int32)
    if E == 64:
        ids[:, 0] = 5  # a hot expert spanning many blocks
    x = rng.standard_normal((T, 64)).astype(F)
    off, pos, src, xp = permute(ids, E, x)
    roff, rpos, rsrc = moe.permute(ids, E)
    np.testing.assert_array_equal(off, roff)
    np.testing.assert_array_equal(pos, rpos)
    np.testing.assert_array_equal(src, rsrc)
    np.testing.assert_array_equal(G.host(xp), G.rounded(x)[rsrc])


def grouped(A, B, sizes, N, epi, rows_extra=0):
    """Run the grouped GEMM on bf16-rounded A [rows, K] and B [G*N, K]."""
    Gn = len(sizes)
    off = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    rows = int(off[-1]) + rows_extra
    K = A.shape[1]
    outN = N // 2 if epi == 3 else N
    C = torch.full((rows, outN), 7.0, dtype=torch.bfloat16, device=G.DEV)
    G.check(G.L().b200_grouped_gemm_bf16(G.bf16(A).data_ptr(), K, G.bf16(B).data_ptr(), K, C.data_ptr(), outN,
                                         G.i32(off).data_ptr(), Gn, rows, N, K, epi, G.stream()), "grouped_gemm")
    torch.cuda.synchronize()
    return G.host(C), off


def grouped_ref(A, B, off, N, epi):
    out = []
    for g in range(len(off) - 1):
        acc = A[off[g]:off[g + 1]].astype(np.float64) @ B[g * N:(g + 1) * N].astype(np.float64).T
        if epi == 3:
            acc = silu(acc[:, 0::2].astype(F)) * acc[:, 1::2]
        out.append(acc)
    return np.concatenate(out).astype(F)


@pytest.mark.parametrize("sizes,N,K,epi", [
    ([3, 0, 17, 64, 1, 0, 100, 7], 256, 512, 3),     # few tokens per expert (weights on the MMA M side)
    ([3, 0, 17, 64, 1, 0, 100, 7], 200, 512, 0),     # ragged feature tail
    ([300, 0, 513, 129], 512, 256, 3),               # many tokens per expert (tokens on the MMA M side)
    ([300, 0, 513, 129], 136, 256, 0),
    ([0, 0, 0, 40], 128, 128, 0),
], ids=["swap-swiglu", "swap-ragged", "tok-swiglu", "tok-ragged", "leading-empty"])
def test_grouped_gemm(sizes, N, K, epi):
    rng = np.random.default_rng(sum(sizes) + N)
    rows = int(sum(sizes))
    A = G.rounded(rng.standard_normal((rows, K)).astype(F))
    B = G.rounded(rng.standard_normal((len(sizes) * N, K)).astype(F) * 0.05)
    C, off = grouped(A, B, sizes, N, epi, rows_extra=5)
    ref = grouped_ref(A, B, off, N, epi)
    got = C[:rows]
    assert G.cosine(got, ref) >= 0.9999
    assert G.max_rel_err(got, ref) <= 0.01
    assert (C[rows:] == 7.0).all()  # rows past the last group are not written
    assert G.device_errors() == 0


def test_grouped_gemm_64_experts_decode_shape():
    rng = np.random.default_rng(64)
    sizes = rng.integers(0, 7, 64)
    N, K = 2 * 1408, 2048
    rows = int(sizes.sum())
    A = G.rounded(rng.standard_normal((rows, K)).astype(F))
    B = G.rounded(rng.standard_normal((64 * N, K)).astype(F) * 0.03)
    C, off = grouped(A, B, sizes, N, 3)
    ref = grouped_ref(A, B, off, N, 3)
    assert G.cosine(C, ref) >= 0.9999 and G.max_rel_err(C, ref) <= 0.01


def test_combine_with_residual_and_norm():
    rng = np.random.default_rng(8)
    T, k, H = 50, 2, 1024
    ids = rng.integers(0, 8, (T, k)).astype(np.int32)
    _, pos, _ = moe.permute(ids, 8)
    y = G.rounded(rng.standard_normal((T * k, H)).astype(F))
    w = rng.uniform(0, 1, (T, k)).astype(F)
    res = G.rounded(rng.standard_normal((T, H)).astype(F))
    sh = G.rounded(rng.standard_normal((T, H)).astype(F))
    nw = G.rounded(1 + 0.1 * rng.standard_normal(H).astype(F))
    hid = G.bf16(res)
    normed = torch.empty(T, H, dtype=torch.bfloat16, device=G.DEV)
    G.check(G.L().b200_moe_combine(G.bf16(y).data_ptr(), G.i32(pos).data_ptr(), G.f32(w).data_ptr(), T, k, H,
                                   hid.data_ptr(), G.bf16(sh).data_ptr(), hid.data_ptr(), G.bf16(nw).data_ptr(),
                                   normed.data_ptr(), 1e-6, G.stream()))
    ref = res + sh + (w[:, :, None] * y[pos.reshape(T, k)]).sum(1)
    got = G.host(hid)
    assert G.max_rel_err(got, ref) <= 0.005
    rn = got / np.sqrt((got.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6) * nw
    assert G.max_rel_err(G.host(normed), rn) <= 0.01


def run_moe_ffn(x, gate_w, experts, k, renorm, scale, shared=None):
    """route -> permute -> grouped gate/up (SwiGLU) -> grouped down -> combine (+ shared, + residual 0)."""
    L = G.L()
    T, H = x.shape
    E = len(experts)
    I = experts[0]["gate_w"].shape[0]
    xd = G.bf16(x)
    ids = torch.empty(T, k, dtype=torch.int32, device=G.DEV)
    w = torch.empty(T, k, dtype=torch.float32, device=G.DEV)
    G.check(L.b200_moe_route(xd.data_ptr(), H, G.bf16(gate_w).data_ptr(), T, H, E, k, renorm, scale, ids.data_ptr(),
                             w.data_ptr(), None, G.stream()))
    wsb = L.b200_moe_permute_workspace_bytes(T, k, E)
    ws = torch.zeros(max(wsb, 16), dtype=torch.uint8, device=G.DEV)
    off = torch.empty(E + 1, dtype=torch.int32, device=G.DEV)
    pos = torch.empty(T * k, dtype=torch.int32, device=G.DEV)
    src = torch.empty(T * k, dtype=torch.int32, device=G.DEV)
    xp = torch.empty(T * k, H, dtype=torch.bfloat16, device=G.DEV)
    G.check(L.b200_moe_permute(ids.data_ptr(), T, k, E, xd.data_ptr(), H, H, xp.data_ptr(), off.data_ptr(),
                               pos.data_ptr(), src.data_ptr(), ws.data_ptr(), wsb, G.stream()))
    gu = np.empty((E * 2 * I, H), F)
    for e, ew in enumerate(experts):
        gu[e * 2 * I:(e + 1) * 2 * I:2] = ew["gate_w"]
        gu[e * 2 * I + 1:(e + 1) * 2 * I:2] = ew["up_w"]
    dn = np.concatenate([ew["down_w"] for ew in experts])
    act = torch.empty(T * k, I, dtype=torch.bfloat16, device=G.DEV)
    G.check(L.b200_grouped_gemm_bf16(xp.data_ptr(), H, G.bf16(gu).data_ptr(), H, act.data_ptr(), I, off.data_ptr(),
                                     E, T * k, 2 * I, H, 3, G.stream()))
    y = torch.empty(T * k, H, dtype=torch.bfloat16, device=G.DEV)
    G.check(L.b200_grouped_gemm_bf16(act.data_ptr(), I, G.bf16(dn).data_ptr(), I, y.data_ptr(), H, off.data_ptr(), E,
                                     T * k, H, I, 0, G.stream()))
    shd = None
    if shared is not None:
        gus = np.empty((2 * shared["gate_w"].shape[0], H), F)
        gus[0::2], gus[1::2] = shared["gate_w"], shared["up_w"]
        sa = G.gemm(xd, G.bf16(gus), epi=3)
        shd = G.gemm(sa, G.bf16(shared["down_w"]))
    out = torch.empty(T, H, dtype=torch.bfloat16, device=G.DEV)
    G.check(L.b200_moe_combine(y.data_ptr(), pos.data_ptr(), w.data_ptr(), T, k, H, None, G.ptr(shd), out.data_ptr(),
                               None, None, 1e-6, G.stream()))
    torch.cuda.synchronize()
    return G.host(out), ids.cpu().numpy()


def _experts(rng, E, I, H, std):
    return [{"gate_w": G.rounded(rng.standard_normal((I, H)).astype(F) * std),
             "up_w": G.rounded(rng.standard_normal((I, H)).astype(F) * std),
             "down_w": G.rounded(rng.standard_normal((H, I)).astype(F) * std)} for _ in range(E)]


@pytest.mark.parametrize("T", [8, 700])
def test_moe_ffn_mixtral_like(T):
    rng = np.random.default_rng(T)
    H, I, E = 512, 1024, 8
    x = G.rounded(rng.standard_normal((T, H)).astype(F))
    gate = G.rounded(rng.standard_normal((E, H)).astype(F) * 0.05)
    ex = _experts(rng, E, I, H, 0.04)
    got, ids = run_moe_ffn(x, gate, ex, 2, 1, 1.0)
    ref, rid, _ = moe.moe_ffn(x, gate, ex, 2)
    same = (ids == rid).all(1)
    assert same.mean() > 0.97  # routing may differ only on near-ties of the fp32 logits
    assert G.cosine(got[same], ref[same]) >= 0.999
    assert G.max_rel_err(got[same], ref[same]) <= 0.02


def test_moe_ffn_deepseek_like_with_shared():
    rng = np.random.default_rng(11)
    T, H, I, E, k = 96, 256, 128, 64, 6
    x = G.rounded(rng.standard_normal((T, H)).astype(F))
    gate = G.rounded(rng.standard_normal((E, H)).astype(F) * 0.05)
    ex = _experts(rng, E, I, H, 0.06)
    sh = _experts(rng, 1, 2 * I, H, 0.06)[0]
    got, ids = run_moe_ffn(x, gate, ex, k, 0, 1.0, shared=sh)
    ref, rid, _ = moe.moe_ffn(x, gate, ex, k, renormalize=False, scale=1.0, shared=sh)
    same = (np.sort(ids, 1) == np.sort(rid, 1)).all(1)
    assert same.mean() > 0.9
    assert G.cosine(got[same], ref[same]) >= 0.999
    assert G.max_rel_err(got[same], ref[same]) <= 0.02
