"""End-to-end parity of the engine on a DeepSeek-V2-style decoder (small
configuration of the V2-Lite architecture: 16 latent-attention heads with
kv_lora 512 / rope 64 and YaRN rope, a dense first layer, then 16 routed
experts top-4 + 2 shared experts): prefill of packed sequences (decompressed
heads, latent cache written), then absorbed-latent decode steps (eager,
captured, replayed), against oracle.model.forward_last_logits_mla.

Bar: cosine >= 0.999 of every last-token logit row; the greedy token equal to
the oracle's wherever its top-2 margin exceeds the bf16 noise.
"""

import ctypes
import json

import numpy as np
import pytest
import torch

from oracle.model import forward_last_logits_mla

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gpu_util as G
    from test_gpu_engine import EngineConfig

YARN = dict(type="yarn", factor=40.0, original_max_position_embeddings=4096, beta_fast=32, beta_slow=1, mscale=0.707,
            mscale_all_dim=0.707)
DSV2 = dict(model_type="deepseek_v2", hidden_size=512, num_hidden_layers=2, num_attention_heads=16,
            num_key_value_heads=16, q_lora_rank=None, kv_lora_rank=512, qk_nope_head_dim=128, qk_rope_head_dim=64,
            v_head_dim=128, intermediate_size=768, moe_intermediate_size=128, n_routed_experts=16,
            num_experts_per_tok=4, n_shared_experts=2, first_k_dense_replace=1, norm_topk_prob=False,
            routed_scaling_factor=1.0, topk_method="greedy", scoring_func="softmax", moe_layer_freq=1,
            vocab_size=1000, rms_norm_eps=1e-6, rope_theta=10000.0, rope_scaling=YARN, tie_word_embeddings=False)
OCFG = dict(heads=16, qk_nope=128, qk_rope=64, v_head=128, kv_lora=512, eps=1e-6, theta=10000.0, top_k=4,
            renorm=False, scale=1.0,
            yarn=dict(factor=40.0, orig_max_pos=4096, beta_fast=32, beta_slow=1, mscale=0.707, mscale_all_dim=0.707))


def make_weights(seed=31):
    rng = np.random.default_rng(seed)
    H, V, nh = 512, 1000, 16

    def n(*s, std=0.05):
        return G.rounded(rng.standard_normal(s).astype(np.float32) * std)

    def one(*s):
        return G.rounded(1 + n(*s, std=0.1))

    w = {"embed": n(V, H, std=1.0), "lm_head": n(V, H), "norm": one(H), "layers": []}
    for li in range(2):
        lw = {"q_w": n(nh * 192, H), "kva_w": n(576, H), "kv_norm": one(512), "kvb_w": n(nh * 256, 512, std=0.03),
              "o_w": n(H, nh * 128, std=0.03), "iln_w": one(H), "pln_w": one(H)}
        if li == 0:
            lw.update(gate_w=n(768, H), up_w=n(768, H), down_w=n(H, 768))
        else:
            lw["router"] = n(16, H, std=0.5)
            lw["experts"] = [{"gate_w": n(128, H), "up_w": n(128, H), "down_w": n(H, 128)} for _ in range(16)]
            lw["shared"] = {"gate_w": n(256, H), "up_w": n(256, H), "down_w": n(H, 256)}
        w["layers"].append(lw)
    return w


def weight_items(w):
    """(HF name, fp32 array) of every weight, in DeepSeek-V2 checkpoint naming."""
    yield "model.embed_tokens.weight", w["embed"]
    yield "lm_head.weight", w["lm_head"]
    yield "model.norm.weight", w["norm"]
    mlp3 = (("gate_w", "gate_proj"), ("up_w", "up_proj"), ("down_w", "down_proj"))
    for i, lw in enumerate(w["layers"]):
        p = f"model.layers.{i}."
        yield p + "self_attn.q_proj.weight", lw["q_w"]
        yield p + "self_attn.kv_a_proj_with_mqa.weight", lw["kva_w"]
        yield p + "self_attn.kv_a_layernorm.weight", lw["kv_norm"]
        yield p + "self_attn.kv_b_proj.weight", lw["kvb_w"]
        yield p + "self_attn.o_proj.weight", lw["o_w"]
        yield p + "input_layernorm.weight", lw["iln_w"]
        yield p + "post_attention_layernorm.weight", lw["pln_w"]
        if "gate_w" in lw:
            for k, nm in mlp3:
                yield p + f"mlp.{nm}.weight", lw[k]
        else:
            yield p + "mlp.gate.weight", lw["router"]
            for e, ew in enumerate(lw["experts"]):
                for k, nm in mlp3:
                    yield p + f"mlp.experts.{e}.{nm}.weight", ew[k]
            for k, nm in mlp3:
                yield p + f"mlp.shared_experts.{nm}.weight", lw["shared"][k]


def create(w, block):
    L = G.L()
    cfg = EngineConfig(None, json.dumps(DSV2).encode(), 0, 8, 256, 512, block, 5, 0.02)
    eng = ctypes.c_void_p()
    G.check(L.b200_engine_create(ctypes.byref(cfg), ctypes.byref(eng)), "engine_create")
    for name, a in weight_items(w):
        a = np.ascontiguousarray(a, np.float32)
        G.check(L.b200_engine_set_weight(eng, name.encode(), a.ctypes.data, 2, a.size), name)
    return eng


def check_rows(logits, seqs, w):
    for i, s in enumerate(seqs):
        ref = forward_last_logits_mla(s, w, OCFG)
        assert G.cosine(logits[i], ref) >= 0.999, (i, G.cosine(logits[i], ref))
        top2 = np.sort(ref)[-2:]
        if top2[1] - top2[0] > 0.05 * np.abs(ref).max():
            assert int(np.argmax(logits[i])) == int(np.argmax(ref)), i


@pytest.mark.parametrize("block", [64, 128])
def test_mla_engine_prefill_then_decode(block):
    w = make_weights()
    eng = create(w, block)
    L = G.L()
    try:
        rng = np.random.default_rng(8)
        lens, slots = [5, 70, 129], [2, 0, 7]
        seqs = [rng.integers(0, 1000, n) for n in lens]
        ids = np.concatenate(seqs).astype(np.int64)
        nxt = np.zeros(3, np.int64)
        logits = torch.empty(3, 1000, dtype=torch.bfloat16, device=G.DEV)
        la, sa = np.array(lens, np.int32), np.array(slots, np.int32)
        G.check(L.b200_engine_prefill(eng, ids.ctypes.data, 0, la.ctypes.data, sa.ctypes.data, 3, None,
                                      nxt.ctypes.data, 0, logits.data_ptr()), "prefill")
        torch.cuda.synchronize()
        check_rows(G.host(logits), seqs, w)
        for step in range(3):
            out = np.zeros(3, np.int64)
            lg = torch.empty(3, 1000, dtype=torch.bfloat16, device=G.DEV)
            G.check(L.b200_engine_decode(eng, nxt.ctypes.data, 0, sa.ctypes.data, 3, out.ctypes.data, 0,
                                         lg.data_ptr()), f"decode {step}")
            torch.cuda.synchronize()
            seqs = [np.append(s, t) for s, t in zip(seqs, nxt)]
            check_rows(G.host(lg), seqs, w)
            nxt = out
        assert G.device_errors() == 0
    finally:
        L.b200_engine_destroy(eng)
