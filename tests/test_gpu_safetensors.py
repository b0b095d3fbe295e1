"""Engine creation from a model directory (config.json + model.safetensors,
the layout LLMEngine::Create / LoadQwen3VLWeights read: qwen3vl_weights.cpp:
79-264, weight_helpers.cpp:16-76) against the same weights given one by one
through b200_engine_set_weight, for files in bf16, fp16 and fp32.

Both engines must produce the same bits: prefill and decode logits of a dense
Qwen3 decoder, and the pooled embedding (+ every hidden row) of a Qwen3-VL
embedding model whose checkpoint carries the vision tower
(model.visual.*) and the text decoder (model.language_model.*).  The dense
file engine is also checked against the oracle (cosine >= 0.999 per logit
row)."""

import ctypes
import json

import numpy as np
import pytest
import torch

import safetensors_util as stu

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gpu_util as G
    import test_gpu_vl_embed as vl
    from test_gpu_engine import HF_NAMES, NARROW, EngineConfig, check_rows, make_weights

DTYPE_ID = {"BF16": 0, "F16": 1, "F32": 2}


def dense_items(w):
    out = [("model.embed_tokens.weight", w["embed"]), ("lm_head.weight", w["lm_head"]), ("model.norm.weight", w["norm"])]
    for i, lw in enumerate(w["layers"]):
        out += [(f"model.layers.{i}.{hf}.weight", lw[k]) for k, hf in HF_NAMES.items()]
    return out


def vl_items(vis, txt):
    out = [("model.visual.patch_embed.proj.weight", vis["patch_w"].reshape(256, 3, 2, 4, 4)),
           ("model.visual.patch_embed.proj.bias", vis["patch_b"]), ("model.visual.pos_embed.weight", vis["pos_table"])]
    for i, b in enumerate(vis["blocks"]):
        out += [(f"model.visual.blocks.{i}.{nm}", b[k]) for k, nm in vl.VIS_NAMES.items()]
    for k, nm in vl.MERGER_NAMES.items():
        out.append((f"model.visual.merger.{nm}", vis["merger"][k]))
        out += [(f"model.visual.deepstack_merger_list.{i}.{nm}", m[k]) for i, m in enumerate(vis["deepstack_mergers"])]
    out += [("model.language_model.embed_tokens.weight", txt["embed"]),
            ("model.language_model.norm.weight", txt["norm"])]
    for i, lw in enumerate(txt["layers"]):
        out += [(f"model.language_model.layers.{i}.{hf}.weight", lw[k]) for k, hf in HF_NAMES.items()]
    return out


def encoded(a, dtype):
    """The host array b200_engine_set_weight gets for the same stored values."""
    if dtype == "BF16":
        return stu.bf16_bits(a)
    if dtype == "F16":
        return np.asarray(a, np.float32).astype(np.float16)
    return np.ascontiguousarray(a, np.float32)


def from_dir(C, items, dtype, tmp_path):
    d = tmp_path / f"model_{dtype}"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(C))
    stu.write(str(d / "model.safetensors"), items, dtype)
    cfg = EngineConfig(str(d).encode(), None, 0, 4, 512, 512, 128, 99, 0.02)
    eng = ctypes.c_void_p()
    G.check(G.L().b200_engine_create(ctypes.byref(cfg), ctypes.byref(eng)), "engine_create(model_dir)")
    return eng


def from_set_weight(C, items, dtype):
    cfg = EngineConfig(None, json.dumps(C).encode(), 0, 4, 512, 512, 128, 99, 0.02)
    eng = ctypes.c_void_p()
    L = G.L()
    G.check(L.b200_engine_create(ctypes.byref(cfg), ctypes.byref(eng)), "engine_create")
    for name, a in items:
        h = np.ascontiguousarray(encoded(a, dtype))
        G.check(L.b200_engine_set_weight(eng, name.encode(), h.ctypes.data, DTYPE_ID[dtype], h.size), name)
    return eng


def run_dense(eng, V, seqs):
    L = G.L()
    ids = np.concatenate(seqs).astype(np.int64)
    lens, slots = np.array([len(s) for s in seqs], np.int32), np.arange(len(seqs), dtype=np.int32)
    nxt = np.zeros(len(seqs), np.int64)
    lg = torch.empty(len(seqs), V, dtype=torch.bfloat16, device=G.DEV)
    G.check(L.b200_engine_prefill(eng, ids.ctypes.data, 0, lens.ctypes.data, slots.ctypes.data, len(seqs), None,
                                  nxt.ctypes.data, 0, lg.data_ptr()), "prefill")
    torch.cuda.synchronize()
    outs = [G.host(lg).copy()]
    for _ in range(2):
        out = np.zeros(len(seqs), np.int64)
        G.check(L.b200_engine_decode(eng, nxt.ctypes.data, 0, slots.ctypes.data, len(seqs), out.ctypes.data, 0,
                                     lg.data_ptr()), "decode")
        torch.cuda.synchronize()
        outs.append(G.host(lg).copy())
        nxt = out
    return outs


@pytest.mark.parametrize("dtype", ["BF16", "F16", "F32"])
def test_dense_engine_from_safetensors_equals_set_weight(tmp_path, dtype):
    C = dict(NARROW)
    w = make_weights(C, 4)
    items = dense_items(w)
    rng = np.random.default_rng(6)
    seqs = [rng.integers(0, C["vocab_size"], n) for n in (9, 70, 33)]
    L = G.L()
    a, b = from_dir(C, items, dtype, tmp_path), from_set_weight(C, items, dtype)
    try:
        got_file, got_set = run_dense(a, C["vocab_size"], seqs), run_dense(b, C["vocab_size"], seqs)
    finally:
        L.b200_engine_destroy(a)
        L.b200_engine_destroy(b)
    for x, y in zip(got_file, got_set):
        np.testing.assert_array_equal(x, y)  # bf16 logits, bit for bit
    if dtype != "F16":  # the bf16 / fp32 files hold exactly the oracle's (bf16-rounded) weights
        check_rows(C, got_file[0], seqs, w)
    assert G.device_errors() == 0


@pytest.mark.parametrize("dtype", ["BF16", "F32"])
def test_qwen3vl_embedding_from_safetensors_equals_set_weight(tmp_path, dtype):
    vis, txt = vl._weights()
    items = vl_items(vis, txt)
    L = G.L()
    g = np.array([[1, 8, 8]], np.int64)
    px = vl._pixels(g, 3)
    ids = [5, 17, vl.VS] + [vl.IMG] * 16 + [9, 33, 2]
    ids = np.array(ids, np.int64)
    res = []
    for make in (lambda: from_dir(vl.CONFIG, items, dtype, tmp_path), lambda: from_set_weight(vl.CONFIG, items, dtype)):
        eng = make()
        try:
            out = np.zeros(512, np.float32)
            hid = torch.empty(len(ids), 512, dtype=torch.bfloat16, device=G.DEV)
            G.check(L.b200_engine_embed(eng, ids.ctypes.data, len(ids), None, px.ctypes.data, 2, 0, len(px),
                                        g.ctypes.data, 1, 1, out.ctypes.data, hid.data_ptr()), "embed")
            torch.cuda.synchronize()
            res.append((out, G.host(hid)))
        finally:
            L.b200_engine_destroy(eng)
    np.testing.assert_array_equal(res[0][0], res[1][0])
    np.testing.assert_array_equal(res[0][1], res[1][1])
    assert G.device_errors() == 0
