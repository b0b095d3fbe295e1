"""The allocation-free decode-attention entry point, through the C ABI.

b200_paged_decode_noalloc serves callers that may not call cudaMalloc (an
operator inside a framework that owns the GPU memory pool, a serving loop
with a frozen memory plan): its split-KV scratch is a fixed array inside the
library.  The GPU test checks it against the regular entry point
(b200_paged_decode with a caller workspace) and against the oracle's paged
decode attention, on two calls in a row — the second call reuses the array
with the first call's leftovers in it.  The CPU tests check that a problem
needing more scratch than the array holds is refused before launch, and that
both entry points return the same code for a shape the kernel does not run.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test.  Tolerance: the per-op bar of the
other kernel tests (cosine >= 0.9999, max |err| <= 2 % of max |ref|).
"""

import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

import oracle

if torch.cuda.is_available():
    import gpu_util as G

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _case(seed, B, ctx):
    rng = np.random.default_rng(seed)
    nq, nkv, hd, bs = 32, 8, 128, 128
    maxb = int((max(ctx) + bs - 1) // bs)
    nblk = B * maxb
    kc = rng.standard_normal((nblk, nkv, bs, hd)).astype(np.float32)
    vc = rng.standard_normal((nblk, nkv, bs, hd)).astype(np.float32)
    tables = rng.permutation(nblk).reshape(B, maxb)
    q = rng.standard_normal((B, nq * hd)).astype(np.float32)
    return dict(q=q, kc=kc, vc=vc, tables=tables, ctx=np.asarray(ctx), B=B, nq=nq, nkv=nkv, hd=hd, bs=bs,
                maxb=maxb, nblk=nblk, max_ctx=int(max(ctx)))


def _run(c, dev, noalloc):
    L = G.L()
    out = torch.empty(c["B"], c["nq"] * c["hd"], dtype=torch.bfloat16, device=G.DEV)
    args = (dev["q"].data_ptr(), c["nq"] * c["hd"], dev["kc"].data_ptr(), dev["vc"].data_ptr(),
            dev["tables"].data_ptr(), c["maxb"], dev["ctx"].data_ptr(), c["B"], c["nq"], c["nkv"], c["hd"], c["bs"],
            c["nblk"], 1.0 / np.sqrt(c["hd"]), out.data_ptr(), c["nq"] * c["hd"])
    if noalloc:
        G.check(L.b200_paged_decode_noalloc(*args, c["max_ctx"], G.stream()), "paged_decode_noalloc")
    else:
        wsb = L.b200_paged_decode_workspace_bytes(c["B"], c["nq"], c["hd"], c["max_ctx"])
        ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=G.DEV)
        G.check(L.b200_paged_decode(*args, ws.data_ptr(), wsb, c["max_ctx"], G.stream()), "paged_decode")
    torch.cuda.synchronize()
    return G.host(out).reshape(c["B"], c["nq"], c["hd"])


@pytest.mark.gpu
def test_noalloc_decode_matches_workspace_entry_point_and_oracle_twice():
    L = G.L()
    assert L.b200_paged_decode_noalloc_max_scratch_bytes() == 8 << 20
    # two different problems back to back: the second finds the first's data in
    # the scratch.  Small batches (8 and 16 sequences x 8 kv heads leave SMs
    # idle) so the kernel splits the KV range and really uses the scratch.
    for seed, B, ctx in ((11, 8, [2048] * 7 + [5]), (12, 16, [1, 64, 65, 777] * 4)):
        c = _case(seed, B, ctx)
        dev = dict(q=G.bf16(c["q"]), kc=G.bf16(c["kc"]), vc=G.bf16(c["vc"]), tables=G.i32(c["tables"]),
                   ctx=G.i32(c["ctx"]))
        assert L.b200_paged_decode_workspace_bytes(B, 32, 128, c["max_ctx"]) > 0
        ora = oracle.paged_decode_attention(G.rounded(c["q"]).reshape(B, c["nq"], c["hd"]), G.rounded(c["kc"]),
                                            G.rounded(c["vc"]), c["tables"], c["ctx"])
        ref = _run(c, dev, noalloc=False)
        for _ in range(2):
            got = _run(c, dev, noalloc=True)
            for b in range(B):
                for want in (ref[b], ora[b]):
                    assert G.cosine(got[b], want) >= 0.9999, b
                    assert G.max_rel_err(got[b], want) <= 0.02, b
    assert G.device_errors() == 0


def _in_subprocess(body, env_extra):
    """Run `body` against the library in a fresh interpreter (the split
    override is read once per process); returns its stdout."""
    env = dict(os.environ, **env_extra)
    code = textwrap.dedent("""
        import sys
        sys.path.insert(0, %r)
        from atb_llm_study_b200 import capi
        L = capi.lib()
    """ % ROOT) + textwrap.dedent(body)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    return r.stdout


def test_noalloc_rejects_problem_larger_than_its_scratch():
    # A supported shape (32 q / 8 kv heads, batch 64, context 32768) with the
    # split count forced to 32: 64 x 32 heads x 32 splits x 129 x 4 B = 33.8 MB
    # of scratch > 8 MiB.  The size check returns before any CUDA call, so this
    # runs without a GPU; the pointers are never dereferenced.
    out = _in_subprocess("""
        B, nq, nkv, hd, max_ctx, d = 64, 32, 8, 128, 32768, 256
        print(L.b200_paged_decode_noalloc(d, nq * hd, d, d, d, 256, d, B, nq, nkv, hd, 128, 16384, 0.1, d, nq * hd,
                                          max_ctx, None))
        print(L.b200_paged_decode_noalloc_max_scratch_bytes())
    """, {"B200_DECODE_SPLITS": "32"})
    rc, cap = (int(x) for x in out.split())
    assert cap == 8 << 20
    assert rc == -1  # B200_ERROR_INVALID_PARAM


def test_noalloc_and_workspace_entry_points_agree_on_unsupported_shapes():
    # Shapes the decode kernel does not run (a GQA group above 16, head_dim 64,
    # block size 32) give ERROR_UNSUPPORTED from both entry points, before any
    # CUDA call; a missing pointer gives ERROR_INVALID_PARAM from both.
    out = _in_subprocess("""
        d = 256
        for nq, nkv, hd, bs, qp in ((64, 1, 128, 128, d), (32, 8, 64, 128, d), (32, 8, 128, 32, d),
                                    (32, 8, 128, 128, 0)):
            a = L.b200_paged_decode_noalloc(qp, nq * hd, d, d, d, 256, d, 4, nq, nkv, hd, bs, 16384, 0.1, d, nq * hd,
                                            1024, None)
            b = L.b200_paged_decode(qp, nq * hd, d, d, d, 256, d, 4, nq, nkv, hd, bs, 16384, 0.1, d, nq * hd, None, 0,
                                    1024, None)
            print(a, b)
    """, {})
    rows = [tuple(int(x) for x in line.split()) for line in out.strip().splitlines()]
    assert rows == [(-7, -7), (-7, -7), (-7, -7), (-1, -1)]
