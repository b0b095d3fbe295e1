"""Whole-model oracle for a dense GQA decoder (Qwen3 family).

embedding -> N x decoder_layer -> final RMSNorm -> lm_head, greedy next token.
The layer math is ``layers.decoder_layer`` (pinned to the reference's decoder
layer goldens); the stack mirrors the reference's text stage
(atb_cpp_llm/src/adapters/qwen3vl_embedding/qwen3vl_model.cpp:685-768: layer loop,
FinalNorm, last-token selection).  Qwen3-8B itself is not implemented by the
reference, so whole-model parity at that size is unpinned; the tests use
small configurations of the same architecture.
"""

import numpy as np

from .layers import decoder_layer, linear, rms_norm
from .positions import rope1d_cos_sin


def forward_last_logits(ids, w, cfg):
    """Logits of the last token of one sequence ``ids`` (1-D int array).

    ``w``: dict with ``embed [V,H]``, ``lm_head [V,H]``, ``norm [H]`` and a
    list ``layers`` of per-layer dicts (q_w k_w v_w o_w qn_w kn_w gate_w up_w
    down_w iln_w pln_w; a mixture-of-experts layer has ``router``, ``experts``
    and optionally ``shared`` instead of the MLP weights).  ``cfg``: heads,
    kv_heads, head_dim, eps, theta (+ top_k, renorm, scale for MoE layers).
    """
    from .moe import moe_ffn

    ids = np.asarray(ids, np.int64)
    x = w["embed"][ids].astype(np.float32)
    cos, sin = rope1d_cos_sin(np.arange(len(ids)), cfg["head_dim"], cfg["theta"])
    for lw in w["layers"]:
        mlp = None
        if "experts" in lw:
            def mlp(n2, lw=lw):
                return moe_ffn(n2, lw["router"], lw["experts"], cfg["top_k"], cfg.get("renorm", True),
                               cfg.get("scale", 1.0), lw.get("shared"))[0]
        x = decoder_layer(x, lw, cos, sin, cfg["heads"], cfg["kv_heads"], cfg["head_dim"], cfg["eps"], causal=True,
                          mlp=mlp)
    h = rms_norm(x[-1:], w["norm"], cfg["eps"])
    return linear(h, w["lm_head"])[0]


def embed_forward(ids, w, cfg, position_ids=None, vis_rows=None, vis_embeds=None, deepstack=(), pool_row=None,
                  normalize=True):
    """Pooled embedding of one sequence: the Qwen3-VL embedding text stage.

    Token embedding, the rows ``vis_rows`` replaced by ``vis_embeds``, the
    decoder layers with mrope (``position_ids [3, S]``; ``cfg["mrope"]``
    sections) or 1-D rope, ``deepstack[i]`` added to the same rows after layer
    i, final RMSNorm, the row ``pool_row`` (default last), L2-normalised with
    ``sqrt(sum(x^2) + 1e-12)``.  Mirrors Qwen3VLModel::ForwardWithTiming's text
    stage and pooling (qwen3vl_model.cpp:576-800; DeepstackFusion::InjectFeatures,
    deepstack_fusion.cpp:143-201; BaseModel::RunPooling, base_model.cpp:137-199).
    Returns ``(embedding [H], final-normed hidden [S, H])``.
    """
    from .positions import mrope_cos_sin

    ids = np.asarray(ids, np.int64)
    S = len(ids)
    V = w["embed"].shape[0]
    x = np.where(((ids >= 0) & (ids < V))[:, None], w["embed"][np.clip(ids, 0, V - 1)], 0).astype(np.float32)
    if vis_rows is not None and len(vis_rows):
        x[np.asarray(vis_rows)] = vis_embeds
    if cfg.get("mrope"):
        pid = np.arange(S)[None].repeat(3, 0) if position_ids is None else np.asarray(position_ids, np.int64)
        cos, sin = mrope_cos_sin(pid[:, None, :], cfg["head_dim"], cfg["theta"], tuple(cfg["mrope"]))
        cos, sin = cos[0], sin[0]
    else:
        cos, sin = rope1d_cos_sin(np.arange(S), cfg["head_dim"], cfg["theta"])
    for i, lw in enumerate(w["layers"]):
        x = decoder_layer(x, lw, cos, sin, cfg["heads"], cfg["kv_heads"], cfg["head_dim"], cfg["eps"], causal=True)
        if i < len(deepstack):
            x[np.asarray(vis_rows)] += deepstack[i]
    h = rms_norm(x, w["norm"], cfg["eps"])
    p = h[S - 1 if pool_row is None else pool_row]
    if normalize:
        p = p / np.sqrt(np.sum(p * p) + np.float32(1e-12))
    return p.astype(np.float32), h


def forward_last_logits_mla(ids, w, cfg):
    """Logits of the last token of ``ids`` for a DeepSeek-V2-style model:
    latent attention (oracle.mla, decompressed form) and dense or routed +
    shared expert MLPs.  ``w`` layers carry q_w kva_w kv_norm kvb_w o_w iln_w
    pln_w and either gate_w up_w down_w or router experts shared; ``cfg`` is an
    oracle.mla config plus top_k, renorm, scale."""
    from .layers import swiglu_mlp
    from .mla import mla_attention
    from .moe import moe_ffn

    ids = np.asarray(ids, np.int64)
    x = w["embed"][ids].astype(np.float32)
    pos = np.arange(len(ids))
    for lw in w["layers"]:
        h = x + mla_attention(rms_norm(x, lw["iln_w"], cfg["eps"]), lw, pos, cfg)
        n2 = rms_norm(h, lw["pln_w"], cfg["eps"])
        if "experts" in lw:
            m = moe_ffn(n2, lw["router"], lw["experts"], cfg["top_k"], cfg.get("renorm", False), cfg.get("scale", 1.0),
                        lw.get("shared"))[0]
        else:
            m = swiglu_mlp(n2, lw["gate_w"], lw["up_w"], lw["down_w"])
        x = h + m
    return linear(rms_norm(x[-1:], w["norm"], cfg["eps"]), w["lm_head"])[0]
