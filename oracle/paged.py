"""Paged KV cache and the attention forms built on it.

The reference has no paged KV cache: ``KVCacheManager::IsAvailable()`` is
always false (atb_cpp_llm/include/atb_llm/kv_cache.h:23-35), the richer
interface in atb_cpp_llm/src/core/kv_cache_manager.h:25-76 is pure virtual,
and ``IRuntime::AllocKVCache`` returns nullptr
(atb_cpp_llm/include/atb_llm/runtime.h:45-54).  Parity here is therefore
unpinned by the reference; these functions restate the standard block-table
scheme and are checked against the dense attention of ``layers.sdpa_gqa``
(a paged decode over the cache equals dense causal attention's last row).

Cache layout: ``cache[num_blocks, kv_heads, block_size, head_dim]``.
"""

import numpy as np

from .layers import sdpa_gqa


def slot_mapping(block_table, positions, block_size):
    """``slot = block_table[pos // bs] * bs + pos % bs`` (int64, bit-exact)."""
    bt = np.asarray(block_table, np.int64)
    p = np.asarray(positions, np.int64)
    return bt[p // block_size] * block_size + p % block_size


def kv_cache_write(cache, x, slots):
    """Scatter ``x [T, kvh, d]`` into ``cache`` at ``slots [T]`` (in place)."""
    bs = cache.shape[2]
    for t, s in enumerate(np.asarray(slots, np.int64)):
        if s < 0:
            continue
        cache[s // bs, :, s % bs, :] = x[t]
    return cache


def paged_decode_attention(q, k_cache, v_cache, block_tables, context_lens, scale=None):
    """Single-token GQA attention of ``q [B, nq, d]`` over each sequence's
    first ``context_lens[b]`` cached positions; returns ``[B, nq, d]`` fp32."""
    B, nq, d = q.shape
    kvh, bs = k_cache.shape[1], k_cache.shape[2]
    rep = nq // kvh
    scale = np.float32(1.0 / np.sqrt(d)) if scale is None else np.float32(scale)
    out = np.zeros((B, nq, d), np.float32)
    for b in range(B):
        L = int(context_lens[b])
        pos = np.arange(L)
        blk = np.asarray(block_tables[b], np.int64)[pos // bs]
        off = pos % bs
        k = k_cache[blk, :, off, :].astype(np.float32)  # [L, kvh, d]
        v = v_cache[blk, :, off, :].astype(np.float32)
        kk = np.repeat(k, rep, axis=1)
        vv = np.repeat(v, rep, axis=1)
        s = np.einsum("hd,lhd->hl", q[b].astype(np.float32), kk) * scale
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(-1, keepdims=True)
        out[b] = np.einsum("hl,lhd->hd", p, vv)
    return out


def varlen_causal_attention(q, k, v, cu_seqlens, nh, kvh):
    """Causal GQA attention over packed sequences (prefill).

    ``q [T, nh, d]``, ``k/v [T, kvh, d]``; sequence ``i`` owns rows
    ``cu_seqlens[i]:cu_seqlens[i+1]``.  Per sequence this is ``sdpa_gqa`` with
    the causal rule ``j > i`` masked — the reference's ``PA_ENCODER`` call with
    ``MakeCausalMaskFp16`` (atb_cpp_llm/src/ops/self_attention_op.cpp:8-30,
    atb_cpp_llm/src/runners/text_runner.cpp:74-85).
    """
    out = np.zeros(q.shape, np.float32)
    cu = np.asarray(cu_seqlens, np.int64)
    for i in range(len(cu) - 1):
        a, b = int(cu[i]), int(cu[i + 1])
        if b > a:
            out[a:b] = sdpa_gqa(q[a:b], k[a:b], v[a:b], nh, kvh, causal=True)
    return out
