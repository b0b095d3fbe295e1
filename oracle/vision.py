"""fp32 numpy restatement of the Qwen3-VL vision tower pieces.

Each function restates the reference generator's golden path
(atb_cpp_llm/tests/python_reference/gen_cpu_reference.py) and names the
reference graph builder it pins.  Token order is the merge-block order of
``positions.merge_order``; attention is bidirectional within each image.
"""

import numpy as np

from .layers import gelu_tanh, layer_norm, linear, rope_half, sdpa_gqa


def vision_attention(x, qkv_w, qkv_b, proj_w, proj_b, cos, sin, nh, hd, cu_seqlens=None):
    """qkv Linear(+bias) -> (N, 3, nh, hd) split -> rope(q, k) -> SDPA (no mask)
    -> proj Linear(+bias).  gen_cpu_reference.py:1790-1885; VisionAttentionGraph::Build
    (atb_cpp_llm/src/components/vision/vision_attention_graph.cpp:12-127)."""
    N = x.shape[0]
    qkv = linear(x, qkv_w, qkv_b).reshape(N, 3, nh, hd)
    q = rope_half(qkv[:, 0], cos, sin)
    k = rope_half(qkv[:, 1], cos, sin)
    v = qkv[:, 2]
    cu = [0, N] if cu_seqlens is None else list(cu_seqlens)
    out = np.concatenate([sdpa_gqa(q[a:b], k[a:b], v[a:b], nh, nh) for a, b in zip(cu[:-1], cu[1:])])
    return linear(out.reshape(N, nh * hd), proj_w, proj_b)


def vision_mlp(x, fc1_w, fc1_b, fc2_w, fc2_b):
    """fc1(+bias) -> GELU(tanh) -> fc2(+bias).  gen_cpu_reference.py:1888-1944;
    VisionMlpGraph::Build (atb_cpp_llm/src/components/vision/vision_mlp_graph.cpp:10-40)."""
    return linear(gelu_tanh(linear(x, fc1_w, fc1_b)), fc2_w, fc2_b)


def vision_block(x, w, cos, sin, nh, hd, eps=1e-6, cu_seqlens=None):
    """x + attn(LN1(x)); + mlp(LN2(.)).  gen_cpu_reference.py:1947-2080;
    VisionBlockGraph::Build (atb_cpp_llm/src/components/vision/vision_block_graph.cpp:12-79).
    ``w``: qkv_w qkv_b proj_w proj_b fc1_w fc1_b fc2_w fc2_b n1_w n1_b n2_w n2_b."""
    h = layer_norm(x, w["n1_w"], w["n1_b"], eps)
    r1 = x + vision_attention(h, w["qkv_w"], w["qkv_b"], w["proj_w"], w["proj_b"], cos, sin, nh, hd, cu_seqlens)
    h2 = layer_norm(r1, w["n2_w"], w["n2_b"], eps)
    return r1 + vision_mlp(h2, w["fc1_w"], w["fc1_b"], w["fc2_w"], w["fc2_b"])


def patch_embed(pixels, w, b):
    """Flattened patches [N, C*tp*p*p] -> Linear(+bias).  gen_cpu_reference.py:2083-2129;
    PatchEmbedGraph::Build (atb_cpp_llm/src/components/vision/patch_embed_graph.cpp:9-49)."""
    return linear(pixels, w, b)


def vision_merger(x, n_w, n_b, f1_w, f1_b, f2_w, f2_b, merge=2, deepstack=False, eps=1e-6):
    """main: LN(hidden) -> reshape groups of merge^2 tokens -> fc1 -> GELU -> fc2;
    deepstack: reshape first, LN over the grouped width.  gen_cpu_reference.py:2132-2205;
    VisionMergerGraph::Build (atb_cpp_llm/src/components/vision/vision_merger_graph.cpp:11-87)."""
    N, H = x.shape
    g = merge * merge
    if deepstack:
        h = layer_norm(x.reshape(N // g, H * g), n_w, n_b, eps)
    else:
        h = layer_norm(x, n_w, n_b, eps).reshape(N // g, H * g)
    return linear(gelu_tanh(linear(h, f1_w, f1_b)), f2_w, f2_b)


def vision_tower(pixels, grid_thw, w, cfg):
    """Whole vision tower: patch embed + interpolated position embedding, the
    blocks (attention within each temporal frame of each image), a deepstack
    merger after each block listed in ``cfg["deepstack"]``, the main merger.
    Returns ``(merged [N/m^2, out], [deepstack_i [N/m^2, out], ...])``.

    Composes the pinned pieces above the way Qwen3VLModel::ForwardWithTiming's
    vision stage runs them (atb_cpp_llm/src/adapters/qwen3vl_embedding/
    qwen3vl_model.cpp:384-575; first layer = patch embed + pos embed + block 0,
    vision_runner.cpp:57-113; deepstack taps deepstack_fusion.cpp:55-105).
    ``w``: patch_w patch_b pos_table, ``blocks`` (list of vision_block dicts),
    ``merger`` and ``deepstack_mergers`` (dicts n_w n_b f1_w f1_b f2_w f2_b).
    ``cfg``: heads, merge, eps, deepstack (block indexes), num_grid.
    """
    from .positions import pos_embed_interp, vision_rope_cos_sin

    grid = np.asarray(grid_thw, np.int64)
    hidden = w["patch_w"].shape[0]
    nh = cfg["heads"]
    hd = hidden // nh
    m = cfg["merge"]
    eps = cfg.get("eps", 1e-6)
    x = patch_embed(np.asarray(pixels, np.float32), w["patch_w"], w["patch_b"])
    x = x + pos_embed_interp(w["pos_table"], grid, cfg["num_grid"], m)
    cos, sin = vision_rope_cos_sin(grid, hd, m)
    cu = [0]
    for t, h, ww in grid:
        for _ in range(int(t)):
            cu.append(cu[-1] + int(h * ww))
    ds = []
    for i, bw in enumerate(w["blocks"]):
        x = vision_block(x, bw, cos, sin, nh, hd, eps, cu_seqlens=cu)
        if i in cfg["deepstack"]:
            mw = w["deepstack_mergers"][cfg["deepstack"].index(i)]
            ds.append(vision_merger(x, *(mw[k] for k in ("n_w", "n_b", "f1_w", "f1_b", "f2_w", "f2_b")), merge=m,
                                    deepstack=True, eps=eps))
    mw = w["merger"]
    merged = vision_merger(x, *(mw[k] for k in ("n_w", "n_b", "f1_w", "f1_b", "f2_w", "f2_b")), merge=m, eps=eps)
    return merged, ds
