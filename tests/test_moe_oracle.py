"""Self-consistency of the MoE restatement (the reference has no MoE
implementation or goldens, so its parity is unpinned): one expert routed with
top-1 is the dense SwiGLU MLP; equal logits go to the lower expert index; the
permutation is a stable sort by expert; renormalised weights sum to one."""

import numpy as np

from oracle import moe, swiglu_mlp


def test_single_expert_is_dense_mlp():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((9, 32)).astype(np.float32)
    ew = {"gate_w": rng.standard_normal((48, 32)).astype(np.float32) * 0.1,
          "up_w": rng.standard_normal((48, 32)).astype(np.float32) * 0.1,
          "down_w": rng.standard_normal((32, 48)).astype(np.float32) * 0.1}
    out, ids, w = moe.moe_ffn(x, np.zeros((1, 32), np.float32), [ew], 1)
    np.testing.assert_allclose(out, swiglu_mlp(x, ew["gate_w"], ew["up_w"], ew["down_w"]), rtol=1e-5, atol=1e-6)
    assert (ids == 0).all() and np.allclose(w, 1.0)


def test_topk_ties_go_to_lower_index():
    lg = np.array([[1.0, 3.0, 3.0, 2.0, 3.0]], np.float32)
    ids, w = moe.route_topk(lg, 3)
    assert ids.tolist() == [[1, 2, 4]]
    np.testing.assert_allclose(w.sum(), 1.0, rtol=1e-6)
    ids, w = moe.route_topk(lg, 2, renormalize=False, scale=2.0)
    p = moe.softmax(lg)[0]
    np.testing.assert_allclose(w[0], 2.0 * p[[1, 2]], rtol=1e-6)


def test_permute_is_stable_sort():
    rng = np.random.default_rng(1)
    ids = rng.integers(0, 8, (50, 2)).astype(np.int32)
    off, pos, src = moe.permute(ids, 8)
    flat = ids.reshape(-1)
    assert off[-1] == flat.size and (np.diff(off) == np.bincount(flat, minlength=8)).all()
    for e in range(8):
        entries = np.nonzero(flat == e)[0]
        assert (pos[entries] == np.arange(off[e], off[e + 1])).all()
        assert (src[off[e]:off[e + 1]] == entries // 2).all()
