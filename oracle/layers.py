"""fp32 numpy restatement of the reference's decoder-layer math.

Each function cites the reference code it restates.  All arithmetic is fp32
(the reference's torch-CPU golden path is fp32 on fp16-rounded inputs).
"""

import numpy as np


def fp16_round(a):
    """fp32 -> fp16 -> fp32 round trip (gen_cpu_reference.py:975-977)."""
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def bf16_round(a):
    """fp32 -> bf16 (round-to-nearest-even) -> fp32 (gen_cpu_reference.py:103-113)."""
    f = np.ascontiguousarray(np.asarray(a, np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = (u.astype(np.uint32) << 16).view(np.float32)
    # keep NaN payloads NaN
    nan = np.isnan(f)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out.reshape(f.shape)


def rms_norm(x, w, eps):
    """RMSNorm over the last dim: x * rsqrt(mean(x^2) + eps) * w.

    Restates ``_rms_norm_torch`` (gen_cpu_reference.py:1475-1478) and the
    NORM / PRENORM / POSTNORM cases of ``gen_rms_norm`` (:753-833), which the
    reference's ``RmsNormOp::Create`` (atb_cpp_llm/src/ops/rms_norm_op.cpp:7-19)
    is gated against.
    """
    x = np.asarray(x, np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    return (x * (1.0 / np.sqrt(var + np.float32(eps)))).astype(np.float32) * np.asarray(w, np.float32)


def layer_norm(x, g, b, eps):
    """LayerNorm over the last dim (gen_cpu_reference.py:847-878, F.layer_norm)."""
    x = np.asarray(x, np.float32)
    mu = x.mean(-1, keepdims=True, dtype=np.float32)
    xc = x - mu
    var = (xc * xc).mean(-1, keepdims=True, dtype=np.float32)
    return xc / np.sqrt(var + np.float32(eps)) * g + b


def rope_half(x, cos, sin):
    """Contiguous-half rotation ``x*cos + cat(-x2, x1)*sin``.

    Restates ``_apply_rope_half`` (gen_cpu_reference.py:1178-1194), the math of
    ``RopeOp::Create(rotaryCoeff=2)`` (atb_cpp_llm/src/ops/rope_op.cpp:7-18).
    ``x`` is ``[T, heads, d]``; ``cos``/``sin`` are ``[T, d]``.
    """
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return x * cos[:, None, :] + rot * sin[:, None, :]


def sdpa_gqa(q, k, v, nh, kvh, mask=None, causal=False):
    """softmax(q k^T / sqrt(d) + mask) v with K/V heads repeated for GQA.

    Restates ``_sdpa_gqa`` (gen_cpu_reference.py:1481-1497) and the
    ``SelfAttentionOp`` math (atb_cpp_llm/src/ops/self_attention_op.cpp:8-30):
    q ``[S, nh, d]``, k/v ``[S, kvh, d]``, additive ``mask [S, S]`` or
    ``causal=True`` for the in-kernel causal rule ``j > i`` masked.
    """
    S, _, d = q.shape
    rep = nh // kvh
    kk = np.repeat(k, rep, axis=1)
    vv = np.repeat(v, rep, axis=1)
    scores = np.einsum("qhd,khd->hqk", q, kk).astype(np.float32) / np.float32(np.sqrt(d))
    if mask is not None:
        scores = scores + mask[None, :, :]
    if causal:
        Sk = k.shape[0]
        off = Sk - S
        m = np.arange(Sk)[None, :] > (np.arange(S)[:, None] + off)
        scores = np.where(m[None], -np.inf, scores)
    scores = scores - scores.max(-1, keepdims=True)
    p = np.exp(scores)
    p = p / p.sum(-1, keepdims=True)
    return np.einsum("hqk,khd->qhd", p, vv).astype(np.float32)


def silu(x):
    """x * sigmoid(x) (F.silu; gen_cpu_reference.py:950-952)."""
    x = np.asarray(x, np.float32)
    return x / (1.0 + np.exp(-x))


def gelu_tanh(x):
    """tanh-approximate GELU (gen_cpu_reference.py:1764-1766)."""
    x = np.asarray(x, np.float32)
    return 0.5 * x * (1.0 + np.tanh(np.float32(0.7978845608028654) * (x + np.float32(0.044715) * x * x * x)))


def linear(x, w, b=None):
    """y = x W^T (+ b), W stored ``[N, K]`` (LinearOp transB=true,
    atb_cpp_llm/src/ops/linear_op.cpp:7-20; gen_cpu_reference.py:883-919)."""
    y = np.asarray(x, np.float32) @ np.asarray(w, np.float32).T
    if b is not None:
        y = y + b
    return y


def swiglu_mlp(x, gate_w, up_w, down_w):
    """down(silu(gate x) * up x) (SwiGluBuilder::Build,
    atb_cpp_llm/src/components/common/mlp_builder.cpp:12-56;
    gen_cpu_reference.py:1415-1452)."""
    return linear(silu(linear(x, gate_w)) * linear(x, up_w), down_w)


def decoder_layer(x, w, cos, sin, nh, kvh, hd, eps=1e-6, mask=None, causal=False, mlp=None):
    """One pre-norm decoder layer.

    ``h1 = x + O(attn(rope(qknorm(QKV(rmsnorm(x))))))``;
    ``out = h1 + SwiGLU(rmsnorm(h1))``.

    Restates ``gen_text_decoder_layer`` (gen_cpu_reference.py:1567-1596), the
    golden for ``TextDecoderLayerGraph::Build``
    (atb_cpp_llm/src/components/text/decoder_layer_graph.cpp:13-154) and
    ``GqaAttentionBuilder::Build``
    (atb_cpp_llm/src/components/common/gqa_attention_builder.cpp:13-185).
    ``w`` holds ``q_w k_w v_w o_w qn_w kn_w gate_w up_w down_w iln_w pln_w``
    (``qn_w``/``kn_w`` may be None to skip the per-head norm); ``mlp``, when
    given, replaces the SwiGLU MLP (a mixture-of-experts block).
    """
    S = x.shape[0]
    normed = rms_norm(x, w["iln_w"], eps)
    q = linear(normed, w["q_w"]).reshape(S, nh, hd)
    k = linear(normed, w["k_w"]).reshape(S, kvh, hd)
    v = linear(normed, w["v_w"]).reshape(S, kvh, hd)
    if w.get("qn_w") is not None:
        q = rms_norm(q, w["qn_w"], eps)
        k = rms_norm(k, w["kn_w"], eps)
    q = rope_half(q, cos, sin)
    k = rope_half(k, cos, sin)
    a = sdpa_gqa(q, k, v, nh, kvh, mask=mask, causal=causal)
    h1 = x + linear(a.reshape(S, nh * hd), w["o_w"])
    n2 = rms_norm(h1, w["pln_w"], eps)
    if mlp is not None:
        return h1 + mlp(n2)
    return h1 + swiglu_mlp(n2, w["gate_w"], w["up_w"], w["down_w"])
