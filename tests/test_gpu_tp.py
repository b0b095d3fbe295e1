"""Tensor-parallel engine on 2 GPUs (skipped with fewer): column-parallel
q/k/v and gate/up, row-parallel o and down with the fused peer-memory
all-reduce (+ residual + RMSNorm) for decode and NCCL for prefill, and the
vocabulary-parallel argmax, against the numpy whole-model oracle.  The dense
Qwen3 layout and both mixture-of-experts layouts (Mixtral, Qwen3-MoE: every
expert's width split across the ranks, the router replicated, the weighted
combine all-reduced) run the same packed prefill + greedy decode steps.

Bar: the concatenated logits shards have cosine >= 0.999 with the oracle's
logits; every rank returns the same greedy tokens, equal to the oracle's
wherever its top-2 margin exceeds the bf16 noise; the device error word stays
clear (no timed-out flag wait).
"""

import multiprocessing as mp
import socket

import numpy as np
import pytest
import torch

from oracle.model import forward_last_logits

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gpu_util as G  # noqa: F401  (makes the library's device helpers importable)
    import test_gpu_engine as dense
    import test_gpu_engine_moe as moe


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dense_case():
    C = dict(dense.NARROW, vocab_size=1200)
    w = dense.make_weights(C, 3)
    items = [("model.embed_tokens.weight", w["embed"]), ("lm_head.weight", w["lm_head"]),
             ("model.norm.weight", w["norm"])]
    for i, lw in enumerate(w["layers"]):
        items += [(f"model.layers.{i}.{hf}.weight", lw[k]) for k, hf in dense.HF_NAMES.items()]
    return C, w, items, dense.oracle_cfg(C)


def _moe_case(base):
    C = dict(base, vocab_size=1024)  # 512 vocabulary rows per rank (a multiple of 8)
    w = moe.make_weights(C, 21)
    return C, w, list(moe.weight_items(C, w)), moe.ocfg(C)


def _run_tp2(C, items, seqs, steps, limits=None):
    import tp_worker

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=tp_worker.run, args=(r, 2, port, C, items, seqs, steps, "tp", q, limits))
             for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, out = q.get(timeout=600)
        res[rank] = out
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
        assert res[r]["errors"] == 0
    return res


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("kind", ["dense", "mixtral", "qwen3_moe"])
def test_tp2_prefill_and_decode(kind):
    if kind == "dense":
        C, w, items, ocfg = _dense_case()
    else:
        C, w, items, ocfg = _moe_case(moe.MIXTRAL if kind == "mixtral" else moe.QWEN3_MOE)
    rng = np.random.default_rng(12)
    seqs = [rng.integers(0, C["vocab_size"], n) for n in (7, 40, 230)]
    res = _run_tp2(C, items, seqs, 3)

    def check(shards, toks, prefixes):
        full = np.concatenate(shards, axis=1)
        for i, s in enumerate(prefixes):
            ref = forward_last_logits(s, w, ocfg)
            assert G.cosine(full[i], ref) >= 0.999, (i, G.cosine(full[i], ref))
            top2 = np.sort(ref)[-2:]
            if top2[1] - top2[0] > 0.05 * np.abs(ref).max():
                assert int(toks[i]) == int(np.argmax(ref)), i
        # the exchange compares the same bf16 logits: exactly the global argmax (lowest id on ties)
        np.testing.assert_array_equal(toks, np.argmax(full, 1))

    (l0, t0), (l1, t1) = res[0]["prefill"], res[1]["prefill"]
    np.testing.assert_array_equal(t0, t1)
    check([l0, l1], t0, seqs)
    prefixes = [s.copy() for s in seqs]
    for step in range(3):  # eager, captured, replayed
        (a0, fed0, o0), (a1, fed1, o1) = res[0]["decode"][step], res[1]["decode"][step]
        np.testing.assert_array_equal(o0, o1)
        prefixes = [np.append(p, t) for p, t in zip(prefixes, fed0)]
        check([a0, a1], o0, prefixes)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_wait_times_out_without_hanging(monkeypatch):
    """Failure detection without a GPU fault: one rank enters the fused
    all-reduce, its peer never does.  The bounded flag wait gives up after about
    two seconds, sets DEV_ERR_WAIT_TIMEOUT (bit 0) in the device error word and
    the kernel returns; the context keeps running kernels."""
    import tp_worker

    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=tp_worker.wait_timeout, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
    assert res[0]["timeout_bits"] & 1, res[0]
    assert 1.0 < res[0]["seconds"] < 30.0, res[0]
    assert res[0]["context_ok"]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_long_prefill():
    """A packed prefill of 2100 tokens (two prompts of 1100 and 1000): the
    row-parallel projections take their prefill tiles and the NCCL all-reduce
    path (beyond the fused peer all-reduce's 256 rows); the logits must match
    the oracle as for short prompts."""
    C, w, items, ocfg = _dense_case()
    rng = np.random.default_rng(31)
    seqs = [rng.integers(0, C["vocab_size"], n) for n in (1100, 1000)]
    res = _run_tp2(C, items, seqs, 1, limits=(4, 1152, 2304))
    (l0, t0), (l1, t1) = res[0]["prefill"], res[1]["prefill"]
    np.testing.assert_array_equal(t0, t1)
    full = np.concatenate([l0, l1], axis=1)
    for i, s in enumerate(seqs):
        ref = forward_last_logits(s, w, ocfg)
        assert G.cosine(full[i], ref) >= 0.999, (i, G.cosine(full[i], ref))
    np.testing.assert_array_equal(t0, np.argmax(full, 1))
