"""End-to-end parity of the engine on mixture-of-experts decoders (Mixtral
and Qwen3-MoE layouts, small configurations of the same architectures):
prefill of packed sequences, then greedy decode steps (eager, captured,
replayed), against the numpy whole-model oracle with oracle.moe routing.

Bar: cosine >= 0.999 of every last-token logit row (the routing of the test
tokens is clear of fp32 near-ties for these seeds), the greedy token equal to
the oracle's wherever its top-2 margin exceeds the bf16 noise.
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
    from test_gpu_engine import EngineConfig

MIXTRAL = dict(model_type="mixtral", hidden_size=512, num_hidden_layers=2, num_attention_heads=4,
               num_key_value_heads=2, intermediate_size=512, num_local_experts=8, num_experts_per_tok=2,
               vocab_size=1000, rms_norm_eps=1e-5, rope_theta=1e6, tie_word_embeddings=False)
QWEN3_MOE = dict(model_type="qwen3_moe", hidden_size=512, num_hidden_layers=2, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=128, intermediate_size=768, moe_intermediate_size=256,
                 num_experts=16, num_experts_per_tok=4, norm_topk_prob=True, vocab_size=1000, rms_norm_eps=1e-6,
                 rope_theta=1e6, tie_word_embeddings=False)


def make_weights(C, seed):
    rng = np.random.default_rng(seed)
    H, V, hd = C["hidden_size"], C["vocab_size"], 128
    nq, nkv = C["num_attention_heads"], C["num_key_value_heads"]
    E = C.get("num_local_experts", C.get("num_experts"))
    Im = C.get("moe_intermediate_size", C["intermediate_size"])

    def n(*s, std=0.05):
        return G.rounded(rng.standard_normal(s).astype(np.float32) * std)

    def one(*s):
        return G.rounded(1 + n(*s, std=0.1))

    w = {"embed": n(V, H, std=1.0), "lm_head": n(V, H), "norm": one(H), "layers": []}
    for _ in range(C["num_hidden_layers"]):
        lw = {"q_w": n(nq * hd, H), "k_w": n(nkv * hd, H), "v_w": n(nkv * hd, H), "o_w": n(H, nq * hd),
              "iln_w": one(H), "pln_w": one(H), "router": n(E, H, std=0.5),
              "experts": [{"gate_w": n(Im, H), "up_w": n(Im, H), "down_w": n(H, Im)} for _ in range(E)]}
        if C["model_type"] == "qwen3_moe":
            lw["qn_w"], lw["kn_w"] = one(hd), one(hd)
        w["layers"].append(lw)
    return w


def weight_items(C, w):
    """(HF name, fp32 array) of every weight of the model, in the checkpoint's naming."""
    yield "model.embed_tokens.weight", w["embed"]
    yield "lm_head.weight", w["lm_head"]
    yield "model.norm.weight", w["norm"]
    mix = C["model_type"] == "mixtral"
    for i, lw in enumerate(w["layers"]):
        p = f"model.layers.{i}."
        for k, nm in (("q_w", "q_proj"), ("k_w", "k_proj"), ("v_w", "v_proj"), ("o_w", "o_proj")):
            yield p + f"self_attn.{nm}.weight", lw[k]
        if "qn_w" in lw:
            yield p + "self_attn.q_norm.weight", lw["qn_w"]
            yield p + "self_attn.k_norm.weight", lw["kn_w"]
        yield p + "input_layernorm.weight", lw["iln_w"]
        yield p + "post_attention_layernorm.weight", lw["pln_w"]
        m = p + ("block_sparse_moe." if mix else "mlp.")
        yield m + "gate.weight", lw["router"]
        for e, ew in enumerate(lw["experts"]):
            names = (("gate_w", "w1"), ("up_w", "w3"), ("down_w", "w2")) if mix else \
                (("gate_w", "gate_proj"), ("up_w", "up_proj"), ("down_w", "down_proj"))
            for k, nm in names:
                yield m + f"experts.{e}.{nm}.weight", ew[k]


def create(C, w, max_batch=8):
    L = G.L()
    cfg = EngineConfig(None, json.dumps(C).encode(), 0, max_batch, 256, 512, 128, 5, 0.02)
    eng = ctypes.c_void_p()
    G.check(L.b200_engine_create(ctypes.byref(cfg), ctypes.byref(eng)), "engine_create")
    for name, a in weight_items(C, w):
        a = np.ascontiguousarray(a, np.float32)
        G.check(L.b200_engine_set_weight(eng, name.encode(), a.ctypes.data, 2, a.size), name)
    return eng


def ocfg(C):
    return dict(heads=C["num_attention_heads"], kv_heads=C["num_key_value_heads"], head_dim=128,
                eps=C["rms_norm_eps"], theta=C["rope_theta"], top_k=C["num_experts_per_tok"], renorm=True)


def check_rows(C, logits, seqs, w):
    for i, s in enumerate(seqs):
        ref = forward_last_logits(s, w, ocfg(C))
        assert G.cosine(logits[i], ref) >= 0.999, (i, G.cosine(logits[i], ref))
        top2 = np.sort(ref)[-2:]
        if top2[1] - top2[0] > 0.05 * np.abs(ref).max():
            assert int(np.argmax(logits[i])) == int(np.argmax(ref)), i


@pytest.mark.parametrize("C", [MIXTRAL, QWEN3_MOE], ids=["mixtral", "qwen3_moe"])
def test_moe_engine_prefill_then_decode(C):
    w = make_weights(C, 21)
    eng = create(C, w)
    L = G.L()
    try:
        rng = np.random.default_rng(4)
        lens, slots = [6, 40, 150], [1, 4, 0]
        seqs = [rng.integers(0, C["vocab_size"], n) for n in lens]
        ids = np.concatenate(seqs).astype(np.int64)
        nxt = np.zeros(3, np.int64)
        V = C["vocab_size"]
        logits = torch.empty(3, V, dtype=torch.bfloat16, device=G.DEV)
        la, sa = np.array(lens, np.int32), np.array(slots, np.int32)
        G.check(L.b200_engine_prefill(eng, ids.ctypes.data, 0, la.ctypes.data, sa.ctypes.data, 3, None,
                                      nxt.ctypes.data, 0, logits.data_ptr()), "prefill")
        torch.cuda.synchronize()
        check_rows(C, G.host(logits), seqs, w)
        for step in range(3):  # eager, captured, replayed
            out = np.zeros(3, np.int64)
            lg = torch.empty(3, V, dtype=torch.bfloat16, device=G.DEV)
            G.check(L.b200_engine_decode(eng, nxt.ctypes.data, 0, sa.ctypes.data, 3, out.ctypes.data, 0,
                                         lg.data_ptr()), f"decode {step}")
            torch.cuda.synchronize()
            seqs = [np.append(s, t) for s, t in zip(seqs, nxt)]
            check_rows(C, G.host(lg), seqs, w)
            nxt = out
        assert G.device_errors() == 0
    finally:
        L.b200_engine_destroy(eng)
