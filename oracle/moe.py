"""Mixture-of-experts restatement (numpy fp32 / int64).

The reference declares MoE only as stubs (MoeBuilder,
atb_cpp_llm/src/components/common/mlp_builder.h:73-82; MoEMlpGraph,
atb_cpp_llm/src/components/moe/moe_mlp_graph.h:22-29; MlpConfig.num_experts /
top_k, atb_cpp_llm/include/atb_llm/layer_desc.h:59-60), so this follows the
published gates of the two target families instead:

* Mixtral-8x7B: fp32 softmax over the 8 router logits, top-2, weights
  renormalised over the chosen two;
* DeepSeek-V2-Lite: softmax over 64 routed experts, greedy top-6, weights
  times routed_scaling_factor (no renormalisation), plus always-on shared
  experts (a dense SwiGLU MLP of width n_shared * moe_intermediate).

Parity is unpinned by the reference (no implementation, no goldens).  The
restatement is checked against self-consistency properties instead: a single
expert with top-1 equals the dense SwiGLU MLP; the permutation is a stable sort
by expert; top-k ties go to the lower expert index.
"""

import numpy as np

from .layers import swiglu_mlp


def softmax(x):
    x = np.asarray(x, np.float32)
    e = np.exp(x - x.max(-1, keepdims=True))
    return (e / e.sum(-1, keepdims=True)).astype(np.float32)


def route_topk(logits, k, renormalize=True, scale=1.0):
    """``logits [T, E]`` -> ``(ids [T, k] int32, weights [T, k] fp32)``: the k
    largest logits (descending; ties to the lower index), their softmax
    probabilities renormalised over the k (``renormalize``) or times ``scale``."""
    lg = np.asarray(logits, np.float32)
    T, E = lg.shape
    p = softmax(lg)
    # lexsort: last key primary -> sort by -logit, then by index
    idx = np.arange(E)
    ids = np.empty((T, k), np.int32)
    for t in range(T):
        order = np.lexsort((idx, -lg[t]))
        ids[t] = order[:k]
    w = np.take_along_axis(p, ids.astype(np.int64), 1)
    if renormalize:
        w = w / w.sum(-1, keepdims=True)
    else:
        w = w * np.float32(scale)
    return ids, w.astype(np.float32)


def permute(ids, num_experts):
    """Stable grouping of the (token, choice) entries by expert.

    Returns ``offsets [E+1]``, ``pos [T*k]`` (slot of entry t*k+j) and
    ``src [T*k]`` (token of each slot); within an expert, slots follow entry
    order."""
    flat = np.asarray(ids, np.int64).reshape(-1)
    k = np.asarray(ids).shape[1]
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=num_experts)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    pos = np.empty(len(flat), np.int32)
    pos[order] = np.arange(len(flat), dtype=np.int32)
    src = (order // k).astype(np.int32)
    return offsets, pos, src


def moe_ffn(x, gate_w, experts, k, renormalize=True, scale=1.0, shared=None, logits=None):
    """Routed experts (+ shared experts) of one MoE MLP.

    ``experts``: list of dicts ``gate_w up_w down_w`` (each ``[I, H]`` /
    ``[H, I]``); ``shared``: optional dict of the same keys.  Returns
    ``(out [T, H], ids, weights)``; ``logits`` overrides the router GEMV."""
    x = np.asarray(x, np.float32)
    lg = x @ np.asarray(gate_w, np.float32).T if logits is None else np.asarray(logits, np.float32)
    ids, w = route_topk(lg, k, renormalize, scale)
    out = np.zeros_like(x)
    for e, ew in enumerate(experts):
        rows, slot = np.nonzero(ids == e)
        if len(rows) == 0:
            continue
        y = swiglu_mlp(x[rows], ew["gate_w"], ew["up_w"], ew["down_w"])
        out[rows] += w[rows, slot][:, None] * y
    if shared is not None:
        out += swiglu_mlp(x, shared["gate_w"], shared["up_w"], shared["down_w"])
    return out.astype(np.float32), ids, w
