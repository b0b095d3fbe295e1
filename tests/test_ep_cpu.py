"""Expert-parallel exchange on CPU (2 gloo ranks, no GPU).

Each rank routes its own tokens, groups its rows by expert, and the ranks
exchange rows in the engine's receive layout (oracle.ep): rank d computes its
own experts on what it received, and every rank combines its outputs back by
the row_base formula.  The per-rank result must equal the whole-model MoE of
that rank's tokens (oracle.moe.moe_ffn), and the layout must account for
every (token, choice) row exactly once."""

import multiprocessing as mp
import os
import socket
import traceback

import numpy as np

from oracle import ep
from oracle.moe import moe_ffn, permute, route_topk, swiglu_mlp


def _weights(rng, H=48, E=8, Im=32):
    def n(*s):
        return (rng.standard_normal(s) * 0.1).astype(np.float32)

    return n(E, H) * 5, [{"gate_w": n(Im, H), "up_w": n(Im, H), "down_w": n(H, Im)} for _ in range(E)]


def _tokens(r, H=48):
    return np.random.default_rng(100 + r).standard_normal((13 + 9 * r, H)).astype(np.float32)


def _rank(r, P, port, q):
    try:
        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=r, world_size=P)
        router, experts = _weights(np.random.default_rng(7))
        E, k = len(experts), 2
        El = E // P
        x = _tokens(r)
        ids, w = route_topk(x @ router.T, k)
        offs, pos, src = permute(ids, E)
        send = x[src]  # rows grouped by expert
        allv = [None] * P
        dist.all_gather_object(allv, (offs, send))
        offs_all = [a[0] for a in allv]
        order, ro = ep.receive_layout(offs_all, r)
        recv = np.stack([allv[s][1][row] for s, row in order]) if order else np.zeros((0, x.shape[1]), np.float32)
        y = np.zeros_like(recv)
        for j in range(El):  # this rank's experts on what it received
            a, b = ro[j], ro[j + 1]
            if b > a:
                e = experts[r * El + j]
                y[a:b] = swiglu_mlp(recv[a:b], e["gate_w"], e["up_w"], e["down_w"])
        ally = [None] * P
        dist.all_gather_object(ally, y)
        base = ep.row_base(offs_all, r)
        out = np.zeros_like(x)
        for t in range(x.shape[0]):
            for c in range(k):
                e = ids[t, c]
                row = base[e] + pos[t * k + c] - offs[e]
                out[t] += w[t, c] * ally[e // El][row]
        ref, _, _ = moe_ffn(x, router, experts, k)
        dist.destroy_process_group()
        q.put((r, out, ref, len(order), int(offs[-1])))
    except Exception:
        q.put((r, traceback.format_exc(), None, 0, 0))


def test_ep2_exchange_matches_whole_moe():
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, rest) for r, *rest in (q.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(res[r][0], str), res[r][0]
        np.testing.assert_allclose(res[r][0], res[r][1], rtol=1e-5, atol=1e-6)
    # every (token, choice) row is received exactly once across the ranks
    assert res[0][2] + res[1][2] == res[0][3] + res[1][3]


def test_dispatch_layout_properties():
    rng = np.random.default_rng(3)
    P, E, k = 4, 8, 2
    ids = [np.array([rng.choice(E, k, replace=False) for _ in range(n)], np.int64).reshape(n, k)
           for n in (5, 0, 17, 9)]
    rows = [rng.standard_normal((len(i), 6)).astype(np.float32) for i in ids]
    out = ep.dispatch(ids, rows, E)
    offs = [permute(i, E)[0] for i in ids]
    total = sum(len(i) * k for i in ids)
    assert sum(len(o[0]) for o in out) == total
    for d, (recv, ro, base) in enumerate(out):
        assert ro[0] == 0 and ro[-1] == len(recv) and np.all(np.diff(ro) >= 0)
        # row_base of source s for expert e points at s's block inside the owner's receive buffer
        for s in range(P):
            b = ep.row_base(offs, s)
            for e in range(E):
                n = offs[s][e + 1] - offs[s][e]
                if n and e // (E // P) == d:
                    own_recv, own_ro, _ = out[d]
                    src_tokens = permute(ids[s], E)[2][offs[s][e]:offs[s][e + 1]]
                    np.testing.assert_array_equal(own_recv[b[e]:b[e] + n], rows[s][src_tokens])
