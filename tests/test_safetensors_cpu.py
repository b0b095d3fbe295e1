"""Per-rank weight slicing from a safetensors file, on CPU (2 gloo ranks, no
GPU): every rank asks the library for its part of every tensor of the file
(b200_weight_shard_file: the engine's own placement plan, the same code its
b200_engine_create_tp / _create_ep upload runs), the parts are all-gathered,
and rank 0 checks that they reassemble the whole tensor: row blocks for the
column-parallel q / k / v, gate / up and lm_head, column blocks for the
row-parallel o / down, each expert on exactly its owner under expert
parallelism, replicated tensors whole on every rank.  The file is written in
bf16, fp16 and fp32; the reassembled values must equal the whole tensor's bf16
rounding bit for bit.  Key names follow the HF checkpoints the reference loads
(qwen3vl_weights.cpp:23-78: ``model.language_model.layers.{i}.self_attn.q_proj``
...; Mixtral ``block_sparse_moe.experts.{e}.w1``)."""

import ctypes
import json
import multiprocessing as mp
import os
import socket
import traceback

import numpy as np
import pytest

import safetensors_util as stu

DENSE = dict(model_type="qwen3", hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
             head_dim=128, intermediate_size=512, vocab_size=512, rms_norm_eps=1e-6, rope_theta=1e6,
             tie_word_embeddings=False)
MIXTRAL = dict(model_type="mixtral", hidden_size=256, num_hidden_layers=1, num_attention_heads=4,
               num_key_value_heads=2, head_dim=128, intermediate_size=256, num_local_experts=4,
               num_experts_per_tok=2, vocab_size=512, rms_norm_eps=1e-5, rope_theta=1e6, tie_word_embeddings=False)

ROWS = ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj", "w1", "w3", "lm_head")
COLS = ("o_proj", "down_proj", "w2")


def tensors(C, rng, vl_names=False):
    H, V, hd = C["hidden_size"], C["vocab_size"], C["head_dim"]
    nq, nkv, I = C["num_attention_heads"] * hd, C["num_key_value_heads"] * hd, C["intermediate_size"]
    base = "model.language_model." if vl_names else "model."

    def n(*s):
        return (rng.standard_normal(s) * 0.05).astype(np.float32)

    out = [(base + "embed_tokens.weight", n(V, H)), ("lm_head.weight", n(V, H)), (base + "norm.weight", 1 + n(H))]
    for i in range(C["num_hidden_layers"]):
        p = f"{base}layers.{i}."
        out += [(p + "self_attn.q_proj.weight", n(nq, H)), (p + "self_attn.k_proj.weight", n(nkv, H)),
                (p + "self_attn.v_proj.weight", n(nkv, H)), (p + "self_attn.o_proj.weight", n(H, nq)),
                (p + "input_layernorm.weight", 1 + n(H)), (p + "post_attention_layernorm.weight", 1 + n(H))]
        if C["model_type"] == "qwen3":
            out += [(p + "self_attn.q_norm.weight", 1 + n(hd)), (p + "self_attn.k_norm.weight", 1 + n(hd)),
                    (p + "mlp.gate_proj.weight", n(I, H)), (p + "mlp.up_proj.weight", n(I, H)),
                    (p + "mlp.down_proj.weight", n(H, I))]
        else:
            E = C["num_local_experts"]
            out.append((p + "block_sparse_moe.gate.weight", n(E, H)))
            for e in range(E):
                q = p + f"block_sparse_moe.experts.{e}."
                out += [(q + "w1.weight", n(I, H)), (q + "w3.weight", n(I, H)), (q + "w2.weight", n(H, I))]
    return out


def _rank(r, P, port, cfg, path, names, mode, q):
    try:
        import torch.distributed as dist

        from atb_llm_study_b200 import capi

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=r, world_size=P)
        L = capi.lib()
        tp, ep = (P, 1) if mode == "tp" else (1, P)
        parts = {}
        for name, numel in names:
            out = np.zeros(numel, np.uint16)
            got = ctypes.c_int64()
            rc = L.b200_weight_shard_file(json.dumps(cfg).encode(), path.encode(), name.encode(), tp,
                                          r if mode == "tp" else 0, ep, r if mode == "ep" else 0, out.ctypes.data,
                                          numel, ctypes.byref(got))
            parts[name] = (rc, out[:got.value].tobytes())
        gathered = [None] * P
        dist.all_gather_object(gathered, parts)
        dist.destroy_process_group()
        q.put((r, gathered if r == 0 else None))
    except Exception:
        q.put((r, traceback.format_exc()))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather(cfg, path, items, mode, P=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    names = [(n, int(a.size)) for n, a in items]
    procs = [ctx.Process(target=_rank, args=(r, P, port, cfg, path, names, mode, q)) for r in range(P)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(P))
    for p in procs:
        p.join(timeout=60)
    for r in range(P):
        assert not isinstance(res[r], str), res[r]
    return res[0]


def _leaf(name):
    return name.split(".")[-2]


@pytest.mark.parametrize("case,dtype", [("dense-tp", "BF16"), ("dense-tp", "F16"), ("dense-tp", "F32"),
                                        ("mixtral-tp", "BF16"), ("mixtral-ep", "BF16"), ("mixtral-ep", "F16"),
                                        ("vl-names-tp", "BF16")])
def test_two_ranks_reassemble_every_tensor_from_file(tmp_path, case, dtype):
    C = MIXTRAL if case.startswith("mixtral") else DENSE
    mode = case.split("-")[-1]
    # "vl-names": the text decoder's tensors under model.language_model. (the Qwen3-VL checkpoint naming)
    items = tensors(C, np.random.default_rng(len(case)), vl_names=case.startswith("vl"))
    cfg = C
    path = str(tmp_path / "model.safetensors")
    stu.write(path, items, dtype)
    parts = _gather(cfg, path, items, mode)
    E = C.get("num_local_experts", 0)
    for name, a in items:
        whole = stu.as_loaded(a, dtype).reshape(a.shape)
        rcs = [parts[r][name][0] for r in range(2)]
        assert rcs == [0, 0], (name, rcs)
        got = [np.frombuffer(parts[r][name][1], np.uint16) for r in range(2)]
        leaf = _leaf(name)
        if mode == "ep" and ".experts." in name:
            e = int(name.split(".experts.")[1].split(".")[0])
            owner = e // (E // 2)
            assert got[1 - owner].size == 0, name
            np.testing.assert_array_equal(got[owner].reshape(a.shape), whole, err_msg=name)
        elif mode == "tp" and leaf in ROWS:
            np.testing.assert_array_equal(np.concatenate([g.reshape(-1, a.shape[1]) for g in got]), whole,
                                          err_msg=name)
            assert got[0].size == got[1].size == a.size // 2
        elif mode == "tp" and leaf in COLS:
            np.testing.assert_array_equal(np.concatenate([g.reshape(a.shape[0], -1) for g in got], 1), whole,
                                          err_msg=name)
        else:
            for g in got:
                np.testing.assert_array_equal(g.reshape(a.shape), whole, err_msg=name)


def test_shard_query_reports_unknown_names_and_sizes(tmp_path):
    from atb_llm_study_b200 import capi

    L = capi.lib()
    cfg = json.dumps(DENSE).encode()
    a = np.zeros(256 * 256, np.uint16)
    out = np.zeros(a.size, np.uint16)
    got = ctypes.c_int64()
    # a name the model does not use, a wrong element count, a tensor-parallel width that does not divide
    assert L.b200_weight_shard(cfg, 1, 0, 1, 0, b"model.layers.0.mystery.weight", a.ctypes.data, 0, a.size,
                               out.ctypes.data, out.size, ctypes.byref(got)) == -3
    assert L.b200_weight_shard(cfg, 2, 0, 1, 0, b"model.layers.0.self_attn.q_proj.weight", a.ctypes.data, 0,
                               a.size - 8, out.ctypes.data, out.size, ctypes.byref(got)) == -1
    assert L.b200_weight_shard(cfg, 3, 0, 1, 0, b"model.norm.weight", a.ctypes.data, 0, 256, out.ctypes.data,
                               out.size, ctypes.byref(got)) == -7
    # a missing file
    assert L.b200_weight_shard_file(cfg, str(tmp_path / "none.safetensors").encode(), b"model.norm.weight", 1, 0, 1,
                                    0, out.ctypes.data, out.size, ctypes.byref(got)) != 0
