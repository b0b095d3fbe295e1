"""End-to-end parity of the C++ engine (b200_engine_* C ABI): prefill of
several packed sequences into the paged KV cache, then greedy decode steps
(eager first, CUDA-graph replays after), against the numpy whole-model oracle.

Three configurations: "narrow" (every projection runs unsplit), "wide"
(decode-sized projections split K, so the fused consumers — QK-norm/rope over
split-K partials, residual + RMSNorm over split-K partials, SwiGLU reduce —
are on the path) and "wide-mlp" (150 gate/up weight tiles: the decode gate/up
runs stream-K, cut tiles finished from their head's partial).

Bar: cosine >= 0.999 of every last-token logit row; the greedy token must
match the oracle's wherever the oracle's top-2 margin exceeds the bf16 noise.
"""

import ctypes
import json

import numpy as np
import pytest
import torch

from oracle.model import forward_last_logits

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gpu_util as G


class EngineConfig(ctypes.Structure):
    _fields_ = [("model_dir", ctypes.c_char_p), ("config_json", ctypes.c_char_p), ("device_id", ctypes.c_int),
                ("max_batch", ctypes.c_int), ("max_context", ctypes.c_int), ("max_prefill_tokens", ctypes.c_int),
                ("kv_block_size", ctypes.c_int), ("init_seed", ctypes.c_uint64), ("init_std", ctypes.c_float)]


NARROW = dict(model_type="qwen3", hidden_size=512, num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2,
              head_dim=128, intermediate_size=1024, vocab_size=1200, rms_norm_eps=1e-6, rope_theta=1e6,
              tie_word_embeddings=False)
WIDE = dict(NARROW, hidden_size=2048, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
            intermediate_size=4096)
# 2 x 9600 / 128 = 150 weight tiles >= 148 SMs: the decode gate/up runs stream-K, 8 k-blocks a tile, so
# nearly every SM's run cuts a tile (head / tail pieces, flags reset by every launch: 4 decode steps)
WIDE_MLP = dict(NARROW, num_hidden_layers=2, intermediate_size=9600)


def make_weights(C, seed=0):
    rng = np.random.default_rng(seed)
    H, I, V, hd = C["hidden_size"], C["intermediate_size"], C["vocab_size"], C["head_dim"]
    nq, nkv = C["num_attention_heads"], C["num_key_value_heads"]

    def n(*s, std=0.05):
        return G.rounded(rng.standard_normal(s).astype(np.float32) * std)

    std = 0.05 if H <= 512 else 0.02
    w = {"embed": n(V, H, std=1.0), "lm_head": n(V, H, std=std), "norm": G.rounded(1 + n(H, std=0.1)), "layers": []}
    for _ in range(C["num_hidden_layers"]):
        w["layers"].append({
            "q_w": n(nq * hd, H, std=std), "k_w": n(nkv * hd, H, std=std), "v_w": n(nkv * hd, H, std=std),
            "o_w": n(H, nq * hd, std=std), "qn_w": G.rounded(1 + n(hd, std=0.1)), "kn_w": G.rounded(1 + n(hd, std=0.1)),
            "gate_w": n(I, H, std=std), "up_w": n(I, H, std=std), "down_w": n(H, I, std=std),
            "iln_w": G.rounded(1 + n(H, std=0.1)), "pln_w": G.rounded(1 + n(H, std=0.1)),
        })
    return w


HF_NAMES = {"q_w": "self_attn.q_proj", "k_w": "self_attn.k_proj", "v_w": "self_attn.v_proj",
            "o_w": "self_attn.o_proj", "qn_w": "self_attn.q_norm", "kn_w": "self_attn.k_norm",
            "gate_w": "mlp.gate_proj", "up_w": "mlp.up_proj", "down_w": "mlp.down_proj",
            "iln_w": "input_layernorm", "pln_w": "post_attention_layernorm"}


def create_engine(C, w, max_batch=8, max_context=512, block=128):
    L = G.L()
    cfg = EngineConfig(None, json.dumps(C).encode(), 0, max_batch, max_context, 1024, block, 7, 0.02)
    eng = ctypes.c_void_p()
    G.check(L.b200_engine_create(ctypes.byref(cfg), ctypes.byref(eng)), "engine_create")

    def put(name, a):
        a = np.ascontiguousarray(a, np.float32)
        G.check(L.b200_engine_set_weight(eng, name.encode(), a.ctypes.data, 2, a.size), name)

    put("model.embed_tokens.weight", w["embed"])
    put("lm_head.weight", w["lm_head"])
    put("model.norm.weight", w["norm"])
    for i, lw in enumerate(w["layers"]):
        for k, hf in HF_NAMES.items():
            put(f"model.layers.{i}.{hf}.weight", lw[k])
    return eng


def oracle_cfg(C):
    return dict(heads=C["num_attention_heads"], kv_heads=C["num_key_value_heads"], head_dim=C["head_dim"],
                eps=C["rms_norm_eps"], theta=C["rope_theta"])


def check_rows(C, logits, seqs, w):
    for i, s in enumerate(seqs):
        ref = forward_last_logits(s, w, oracle_cfg(C))
        got = logits[i]
        assert G.cosine(got, ref) >= 0.999, (i, G.cosine(got, ref))
        top2 = np.sort(ref)[-2:]
        if top2[1] - top2[0] > 0.05 * np.abs(ref).max():
            assert int(np.argmax(got)) == int(np.argmax(ref)), i


@pytest.mark.parametrize("C,block", [(NARROW, 128), (NARROW, 64), (WIDE, 128), (WIDE_MLP, 128)],
                         ids=["narrow-128", "narrow-64", "wide", "wide-mlp-stream-k"])
def test_engine_prefill_then_decode(C, block):
    w = make_weights(C)
    eng = create_engine(C, w, block=block)
    L = G.L()
    try:
        if C is WIDE:  # the decode projections really split K in this configuration
            assert L.b200_gemm_workspace_bytes(4, 2 * C["intermediate_size"], C["hidden_size"], 3) > 0
        rng = np.random.default_rng(3)
        lens = [5, 17, 130, 64]
        slots = [2, 0, 5, 7]
        seqs = [rng.integers(0, C["vocab_size"], n) for n in lens]
        ids = np.concatenate(seqs).astype(np.int64)
        nxt = np.zeros(len(lens), np.int64)
        V = C["vocab_size"]
        logits = torch.empty(len(lens), V, dtype=torch.bfloat16, device=G.DEV)
        lens_a, slots_a = np.array(lens, np.int32), np.array(slots, np.int32)  # kept alive across the call
        G.check(L.b200_engine_prefill(eng, ids.ctypes.data, 0, lens_a.ctypes.data, slots_a.ctypes.data, len(lens),
                                      None, nxt.ctypes.data, 0, logits.data_ptr()), "prefill")
        torch.cuda.synchronize()
        lg = G.host(logits)
        check_rows(C, lg, seqs, w)
        np.testing.assert_array_equal(nxt, np.argmax(lg, 1))
        # decode 4 steps, feeding back the greedy tokens; slot order shuffled
        order = [3, 0, 2, 1]
        for step in range(4):
            b_slots = np.array([slots[i] for i in order], np.int32)
            b_ids = np.array([nxt[i] for i in order], np.int64)
            out = np.zeros(len(order), np.int64)
            lgd = torch.empty(len(order), V, dtype=torch.bfloat16, device=G.DEV)
            G.check(L.b200_engine_decode(eng, b_ids.ctypes.data, 0, b_slots.ctypes.data, len(order), out.ctypes.data,
                                         0, lgd.data_ptr()), f"decode {step}")
            torch.cuda.synchronize()
            for j, i in enumerate(order):
                seqs[i] = np.append(seqs[i], nxt[i])
            check_rows(C, G.host(lgd), [seqs[i] for i in order], w)
            for j, i in enumerate(order):
                nxt[i] = out[j]
                n = ctypes.c_int64()
                G.check(L.b200_engine_context_len(eng, slots[i], ctypes.byref(n)))
                assert n.value == len(seqs[i])
        assert G.device_errors() == 0
    finally:
        L.b200_engine_destroy(eng)


def test_engine_rejects_bad_requests():
    w = make_weights(NARROW, 1)
    eng = create_engine(NARROW, w, max_batch=4, max_context=128)
    L = G.L()
    try:
        ids = np.zeros(8, np.int64)
        nxt = np.zeros(2, np.int64)
        INVALID = -1
        # duplicate slot, slot out of range, empty sequence, too long
        for lens, slots in (([4, 4], [1, 1]), ([4, 4], [0, 9]), ([0, 8], [0, 1]), ([200, 1], [0, 1])):
            lens_a, slots_a = np.array(lens, np.int32), np.array(slots, np.int32)
            rc = L.b200_engine_prefill(eng, ids.ctypes.data, 0, lens_a.ctypes.data, slots_a.ctypes.data, 2, None,
                                       nxt.ctypes.data, 0, None)
            assert rc == INVALID, (lens, slots, rc)
        # decode on a slot that holds no sequence
        one = np.array([3], np.int32)
        rc = L.b200_engine_decode(eng, ids.ctypes.data, 0, one.ctypes.data, 1, nxt.ctypes.data, 0, None)
        assert rc == INVALID
        # unknown model type is refused at create
        cfg = EngineConfig(None, json.dumps(dict(NARROW, model_type="mystery", num_local_experts=8)).encode(), 0, 1,
                           16, 16, 128, 0, 0.02)
        e2 = ctypes.c_void_p()
        assert L.b200_engine_create(ctypes.byref(cfg), ctypes.byref(e2)) == -7
    finally:
        L.b200_engine_destroy(eng)
