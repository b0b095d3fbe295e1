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
    down_w iln_w pln_w).  ``cfg``: heads, kv_heads, head_dim, eps, theta.
    """
    ids = np.asarray(ids, np.int64)
    x = w["embed"][ids].astype(np.float32)
    cos, sin = rope1d_cos_sin(np.arange(len(ids)), cfg["head_dim"], cfg["theta"])
    for lw in w["layers"]:
        x = decoder_layer(x, lw, cos, sin, cfg["heads"], cfg["kv_heads"], cfg["head_dim"], cfg["eps"], causal=True)
    h = rms_norm(x[-1:], w["norm"], cfg["eps"])
    return linear(h, w["lm_head"])[0]
