"""Multi-head latent attention restatement (numpy fp32), DeepSeek-V2 / V2-Lite.

The reference declares MLA only as a stub (MlaAttentionBuilder,
atb_cpp_llm/src/components/common/attention_builder.h:60-69; AttnConfig.
kv_lora_rank / q_lora_rank, atb_cpp_llm/include/atb_llm/layer_desc.h:47-49),
so this restates the published DeepSeek-V2 attention (no q-LoRA, the V2-Lite
form):

  q      = x Wq^T                      per head [qk_nope | qk_rope]
  kv_a   = x Wkva^T                    [kv_lora | qk_rope]
  c      = RMSNorm(kv_a[:kv_lora]) * w_kv_norm
  k_pe   = rope(kv_a[kv_lora:])        shared by every head
  kv     = c Wkvb^T                    per head [k_nope | v]
  score  = (q_nope . k_nope + rope(q_pe) . k_pe) * softmax_scale
  out    = o_proj(softmax(score) v)

Rope uses YaRN-scaled frequencies and rotates the interleaved pairs (2i, 2i+1)
of the projection, producing the de-interleaved layout; softmax_scale =
qk_head_dim^-0.5 * mscale(factor, mscale_all_dim)^2.

Parity is unpinned by the reference (no implementation, no goldens).  The
restatement is checked for self-consistency: the absorbed form (W_UK folded
into the query, W_UV into the output projection, attention over the 576-wide
latent cache) equals the decompressed form.
"""

import math

import numpy as np

from .layers import linear, rms_norm


def yarn_get_mscale(scale=1.0, mscale=1.0):
    return 1.0 if scale <= 1 else 0.1 * mscale * math.log(scale) + 1.0


def yarn_inv_freq(dim, base, factor, orig_max_pos, beta_fast=32, beta_slow=1):
    """YaRN frequencies: per dim pair, the interpolated frequency (base freq /
    factor) blended with the original by a linear ramp between the correction
    dims of beta_fast and beta_slow rotations over the original context."""
    def corr_dim(num_rot):
        return (dim * math.log(orig_max_pos / (num_rot * 2 * math.pi))) / (2 * math.log(base))

    low = max(math.floor(corr_dim(beta_fast)), 0)
    high = min(math.ceil(corr_dim(beta_slow)), dim - 1)
    if low == high:
        high += 0.001
    exps = np.arange(0, dim, 2, dtype=np.float32) / np.float32(dim)
    freq_extra = (1.0 / np.power(np.float32(base), exps)).astype(np.float32)
    freq_inter = (1.0 / (np.float32(factor) * np.power(np.float32(base), exps))).astype(np.float32)
    ramp = np.clip((np.arange(dim // 2, dtype=np.float32) - np.float32(low)) / np.float32(high - low), 0, 1)
    mask = (1.0 - ramp).astype(np.float32)
    return (freq_inter * (1 - mask) + freq_extra * mask).astype(np.float32)


def rope_cfg_tables(positions, cfg):
    """cos, sin [T, rope_dim] for positions (1-D) under cfg's rope (YaRN when
    cfg has "yarn"), including the cos/sin mscale."""
    d = cfg["qk_rope"]
    y = cfg.get("yarn")
    if y:
        inv = yarn_inv_freq(d, cfg["theta"], y["factor"], y["orig_max_pos"], y["beta_fast"], y["beta_slow"])
        ms = yarn_get_mscale(y["factor"], y["mscale"]) / yarn_get_mscale(y["factor"], y["mscale_all_dim"])
    else:
        inv = (1.0 / np.power(np.float32(cfg["theta"]), np.arange(0, d, 2, dtype=np.float32) / np.float32(d)))
        ms = 1.0
    f = np.asarray(positions, np.int64)[:, None].astype(np.float32) * inv.astype(np.float32)
    emb = np.concatenate([f, f], -1)
    return (np.cos(emb) * ms).astype(np.float32), (np.sin(emb) * ms).astype(np.float32)


def softmax_scale(cfg):
    s = (cfg["qk_nope"] + cfg["qk_rope"]) ** -0.5
    y = cfg.get("yarn")
    if y:
        m = yarn_get_mscale(y["factor"], y["mscale_all_dim"])
        s = s * m * m
    return s


def rope_deinterleave(x, cos, sin):
    """x [..., T, d] (or [T, ..., d] broadcast by the caller): pairs (2i, 2i+1)
    rotated, output out[i] = x0 cos - x1 sin, out[d/2+i] = x1 cos + x0 sin."""
    d = x.shape[-1]
    x0, x1 = x[..., 0::2], x[..., 1::2]
    c, s = cos[..., : d // 2], sin[..., : d // 2]
    return np.concatenate([x0 * c - x1 * s, x1 * c + x0 * s], -1).astype(np.float32)


def mla_project(x, w, cos, sin, cfg):
    """Per-token projections: q_nope [T,nh,nope], q_pe roped [T,nh,rope],
    c [T,kv_lora], k_pe roped [T,rope]."""
    T = x.shape[0]
    nh, dn, dr, R = cfg["heads"], cfg["qk_nope"], cfg["qk_rope"], cfg["kv_lora"]
    q = linear(x, w["q_w"]).reshape(T, nh, dn + dr)
    kv_a = linear(x, w["kva_w"])
    c = rms_norm(kv_a[:, :R], w["kv_norm"], cfg["eps"])
    k_pe = rope_deinterleave(kv_a[:, R:], cos, sin)
    q_pe = rope_deinterleave(q[:, :, dn:], cos[:, None, :], sin[:, None, :])
    return q[:, :, :dn], q_pe, c, k_pe


def mla_attention(x, w, positions, cfg, cu_seqlens=None):
    """Decompressed causal MLA over packed sequences -> o_proj output [T, H]."""
    T = x.shape[0]
    nh, dn, dv = cfg["heads"], cfg["qk_nope"], cfg["v_head"]
    cos, sin = rope_cfg_tables(positions, cfg)
    q_nope, q_pe, c, k_pe = mla_project(x, w, cos, sin, cfg)
    kv = linear(c, w["kvb_w"]).reshape(T, nh, dn + dv)
    k_nope, v = kv[:, :, :dn], kv[:, :, dn:]
    sc = softmax_scale(cfg)
    out = np.zeros((T, nh, dv), np.float32)
    cu = [0, T] if cu_seqlens is None else list(cu_seqlens)
    for a, b in zip(cu[:-1], cu[1:]):
        L = b - a
        s = (np.einsum("qhd,khd->hqk", q_nope[a:b], k_nope[a:b])
             + np.einsum("qhd,kd->hqk", q_pe[a:b], k_pe[a:b])) * np.float32(sc)
        s = np.where(np.triu(np.ones((L, L), bool), 1)[None], -np.inf, s)
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        out[a:b] = np.einsum("hqk,khd->qhd", p, v[a:b])
    return linear(out.reshape(T, nh * dv), w["o_w"])


def absorbed_weights(w, cfg):
    """W_qabs [nh*(kv_lora+rope), H]: per head W_UK^T Wq_nope then the rope
    rows of Wq; W_oabs [H, nh*kv_lora]: per head Wo_h W_UV."""
    nh, dn, dr, dv, R = cfg["heads"], cfg["qk_nope"], cfg["qk_rope"], cfg["v_head"], cfg["kv_lora"]
    H = w["q_w"].shape[1]
    wq = w["q_w"].reshape(nh, dn + dr, H)
    kvb = w["kvb_w"].reshape(nh, dn + dv, R)
    wo = w["o_w"].reshape(H, nh, dv)
    qabs = np.concatenate([np.einsum("hdc,hdj->hcj", kvb[:, :dn], wq[:, :dn]), wq[:, dn:]], 1)
    oabs = np.einsum("jhd,hdc->jhc", wo, kvb[:, dn:])
    return qabs.reshape(nh * (R + dr), H).astype(np.float32), oabs.reshape(H, nh * R).astype(np.float32)


def latent_decode(q_abs, cache, ctx, nh, scale):
    """Absorbed decode attention: q_abs [B, nh*576], cache rows per sequence
    (list of [ctx_b, 576]) -> [B, nh*512]."""
    B = q_abs.shape[0]
    out = np.zeros((B, nh * 512), np.float32)
    for b in range(B):
        q = q_abs[b].reshape(nh, 576)
        C = cache[b][: ctx[b]]
        s = (q @ C.T) * np.float32(scale)
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        out[b] = (p @ C[:, :512]).reshape(-1)
    return out


def mla_decode_absorbed(x, w, positions, cfg, cache_c, cache_kpe):
    """Absorbed single-token attention for the last row of each prefix: x [B,
    H] at positions [B], with cache_c / cache_kpe lists of the earlier tokens'
    c and k_pe ([ctx_b - 1, R] / [ctx_b - 1, rope]).  Returns o_proj output."""
    nh, R, dr = cfg["heads"], cfg["kv_lora"], cfg["qk_rope"]
    qabs, oabs = absorbed_weights(w, cfg)
    cos, sin = rope_cfg_tables(positions, cfg)
    B = x.shape[0]
    q = linear(x, qabs).reshape(B, nh, R + dr)
    q[:, :, R:] = rope_deinterleave(q[:, :, R:], cos[:, None, :], sin[:, None, :])
    kv_a = linear(x, w["kva_w"])
    c = rms_norm(kv_a[:, :R], w["kv_norm"], cfg["eps"])
    k_pe = rope_deinterleave(kv_a[:, R:], cos, sin)
    caches = [np.concatenate([np.concatenate([cache_c[b], c[b:b + 1]]),
                              np.concatenate([cache_kpe[b], k_pe[b:b + 1]])], 1) for b in range(B)]
    lat = latent_decode(q.reshape(B, -1), caches, [len(cc) for cc in caches], nh, softmax_scale(cfg))
    return linear(lat, oabs)
