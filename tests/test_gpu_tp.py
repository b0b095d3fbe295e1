"""Tensor-parallel engine on 2 GPUs (skipped with fewer): column-parallel
q/k/v and gate/up, row-parallel o and down with the fused peer-memory
all-reduce (+ residual + RMSNorm) for decode and NCCL for prefill, and the
vocabulary-parallel argmax, against the numpy whole-model oracle.

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
    from test_gpu_engine import NARROW, make_weights, oracle_cfg


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_prefill_and_decode():
    import tp_worker

    C = dict(NARROW, vocab_size=1200)
    w = make_weights(C, 3)
    rng = np.random.default_rng(12)
    seqs = [rng.integers(0, C["vocab_size"], n) for n in (7, 40, 230)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=tp_worker.run, args=(r, 2, port, C, w, seqs, 3, q)) for r in range(2)]
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

    def check(shards, toks, prefixes):
        full = np.concatenate(shards, axis=1)
        for i, s in enumerate(prefixes):
            ref = forward_last_logits(s, w, oracle_cfg(C))
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
    for step in range(3):
        (a0, fed0, o0), (a1, fed1, o1) = res[0]["decode"][step], res[1]["decode"][step]
        np.testing.assert_array_equal(o0, o1)
        prefixes = [np.append(p, t) for p, t in zip(prefixes, fed0)]
        check([a0, a1], o0, prefixes)
