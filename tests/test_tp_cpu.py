"""Tensor-parallel partitioning on CPU (2 gloo ranks, no GPU): each rank keeps
the engine's shard of a decoder layer — query/key/value heads and gate/up rows
(column-parallel), the matching o / down columns (row-parallel) and a block of
vocabulary rows — sums its partial outputs with an all-reduce, and picks the
greedy token from the exchanged per-shard maxima.  The result must equal the
unsharded oracle layer and argmax."""

import multiprocessing as mp
import os
import socket
import traceback

import numpy as np

import oracle


def _layer_weights(rng, H=64, nq=4, nkv=2, hd=32, I=96):
    def n(*s):
        return (rng.standard_normal(s) * 0.1).astype(np.float32)

    return {"q_w": n(nq * hd, H), "k_w": n(nkv * hd, H), "v_w": n(nkv * hd, H), "o_w": n(H, nq * hd),
            "qn_w": 1 + n(hd), "kn_w": 1 + n(hd), "gate_w": n(I, H), "up_w": n(I, H), "down_w": n(H, I),
            "iln_w": 1 + n(H), "pln_w": 1 + n(H)}, dict(nq=nq, nkv=nkv, hd=hd, I=I)


def shard(w, d, P, r):
    """The engine's per-rank slices (q/k/v rows by head block, o/down columns, gate/up rows)."""
    nq, nkv, hd, I = d["nq"] // P, d["nkv"] // P, d["hd"], d["I"] // P
    s = dict(w)
    s["q_w"] = w["q_w"][r * nq * hd:(r + 1) * nq * hd]
    s["k_w"] = w["k_w"][r * nkv * hd:(r + 1) * nkv * hd]
    s["v_w"] = w["v_w"][r * nkv * hd:(r + 1) * nkv * hd]
    s["o_w"] = w["o_w"][:, r * nq * hd:(r + 1) * nq * hd]
    s["gate_w"] = w["gate_w"][r * I:(r + 1) * I]
    s["up_w"] = w["up_w"][r * I:(r + 1) * I]
    s["down_w"] = w["down_w"][:, r * I:(r + 1) * I]
    return s, nq, nkv


def partial_layer(x, s, nq, nkv, hd, cos, sin, allreduce):
    """Column-parallel attention + MLP of one rank; partial o / down outputs are all-reduced."""
    S = x.shape[0]
    n = oracle.rms_norm(x, s["iln_w"], 1e-6)
    q = oracle.rms_norm(oracle.linear(n, s["q_w"]).reshape(S, nq, hd), s["qn_w"], 1e-6)
    k = oracle.rms_norm(oracle.linear(n, s["k_w"]).reshape(S, nkv, hd), s["kn_w"], 1e-6)
    v = oracle.linear(n, s["v_w"]).reshape(S, nkv, hd)
    a = oracle.sdpa_gqa(oracle.rope_half(q, cos, sin), oracle.rope_half(k, cos, sin), v, nq, nkv, causal=True)
    h = x + allreduce(oracle.linear(a.reshape(S, nq * hd), s["o_w"]))
    n2 = oracle.rms_norm(h, s["pln_w"], 1e-6)
    act = oracle.silu(oracle.linear(n2, s["gate_w"])) * oracle.linear(n2, s["up_w"])
    return h + allreduce(oracle.linear(act, s["down_w"]))


def _rank(r, P, port, q):
    try:
        import torch
        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=r, world_size=P)

        def allreduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
            dist.all_reduce(t)
            return t.numpy()

        rng = np.random.default_rng(0)
        w, d = _layer_weights(rng)
        x = rng.standard_normal((9, 64)).astype(np.float32)
        lm = (rng.standard_normal((40, 64)) * 0.3).astype(np.float32)
        cos, sin = oracle.rope1d_cos_sin(np.arange(9), d["hd"], 1e6)
        s, nq, nkv = shard(w, d, P, r)
        y = partial_layer(x, s, nq, nkv, d["hd"], cos, sin, allreduce)
        # vocabulary-parallel greedy token: per-shard (max, global id), exchanged, max then lowest id
        Vl = lm.shape[0] // P
        lg = oracle.linear(y, lm[r * Vl:(r + 1) * Vl])
        pairs = torch.from_numpy(np.stack([lg.max(1), lg.argmax(1) + r * Vl], 1).astype(np.float64))
        allp = [torch.zeros_like(pairs) for _ in range(P)]
        dist.all_gather(allp, pairs)
        allp = np.stack([p.numpy() for p in allp])  # [P, rows, 2]
        best = []
        for row in range(allp.shape[1]):
            cand = sorted(((-allp[k, row, 0], allp[k, row, 1]) for k in range(P)))
            best.append(int(cand[0][1]))
        dist.destroy_process_group()
        q.put((r, y, np.array(best)))
    except Exception:
        q.put((r, traceback.format_exc(), None))


def test_tp2_partitioning_matches_unsharded_layer():
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict((r, (y, b)) for r, y, b in (q.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(out[r][0], str), out[r][0]
    rng = np.random.default_rng(0)
    w, d = _layer_weights(rng)
    x = rng.standard_normal((9, 64)).astype(np.float32)
    lm = (rng.standard_normal((40, 64)) * 0.3).astype(np.float32)
    cos, sin = oracle.rope1d_cos_sin(np.arange(9), d["hd"], 1e6)
    ref = oracle.decoder_layer(x, w, cos, sin, d["nq"], d["nkv"], d["hd"], causal=True)
    for r in range(2):
        np.testing.assert_allclose(out[r][0], ref, rtol=1e-4, atol=1e-5)
        np.testing.assert_array_equal(out[r][1], oracle.linear(ref, lm).argmax(1))


def _moe_weights(rng, H=64, E=6, Im=48, Is=32):
    def n(*s):
        return (rng.standard_normal(s) * 0.1).astype(np.float32)

    ex = [{"gate_w": n(Im, H), "up_w": n(Im, H), "down_w": n(H, Im)} for _ in range(E)]
    sh = {"gate_w": n(Is, H), "up_w": n(Is, H), "down_w": n(H, Is)}
    return n(E, H) * 5, ex, sh


def _slice_mlp(m, P, r):
    """The engine's expert split: gate/up rows r*I/P.., down columns r*I/P.."""
    I = m["gate_w"].shape[0] // P
    return {"gate_w": m["gate_w"][r * I:(r + 1) * I], "up_w": m["up_w"][r * I:(r + 1) * I],
            "down_w": m["down_w"][:, r * I:(r + 1) * I]}


def _moe_rank(r, P, port, q):
    try:
        import torch
        import torch.distributed as dist

        from oracle.moe import moe_ffn

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=r, world_size=P)
        rng = np.random.default_rng(5)
        router, ex, sh = _moe_weights(rng)
        x = rng.standard_normal((11, 64)).astype(np.float32)
        # replicated router (same selection on every rank), this rank's slice of every expert
        part, ids, _ = moe_ffn(x, router, [_slice_mlp(e, P, r) for e in ex], 2, shared=_slice_mlp(sh, P, r))
        t = torch.from_numpy(np.ascontiguousarray(part))
        dist.all_reduce(t)
        dist.destroy_process_group()
        q.put((r, t.numpy(), ids))
    except Exception:
        q.put((r, traceback.format_exc(), None))


def test_tp2_expert_split_matches_whole_moe():
    from oracle.moe import moe_ffn

    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_moe_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict((r, (y, ids)) for r, y, ids in (q.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(out[r][0], str), out[r][0]
    rng = np.random.default_rng(5)
    router, ex, sh = _moe_weights(rng)
    x = rng.standard_normal((11, 64)).astype(np.float32)
    ref, ids, _ = moe_ffn(x, router, ex, 2, shared=sh)
    for r in range(2):
        np.testing.assert_array_equal(out[r][1], ids)
        np.testing.assert_allclose(out[r][0], ref, rtol=1e-4, atol=1e-5)
