"""End-to-end parity of the Qwen3-VL embedding path through the engine C ABI
(b200_engine_vision, b200_engine_embed) against the oracle's composition of
the pinned pieces (oracle.vision.vision_tower, oracle.model.embed_forward),
at a small configuration of the same architecture: vision tower (patch embed
+ interpolated position table, ViT blocks with 2-D rope, deepstack mergers,
main merger), image rows replaced in the text embeddings, mrope position ids,
deepstack features added after the first text layers, final RMSNorm, last-token
pooling + L2 norm.

Bar: cosine >= 0.999 of every compared tensor; max |err| <= 3 % of max |ref|
(bf16 activations through 4 vision blocks, 2 mergers and 3 text layers).
"""

import ctypes
import json

import numpy as np
import pytest
import torch

import oracle
from oracle.model import embed_forward
from oracle.vision import vision_tower

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gpu_util as G
    from test_gpu_engine import HF_NAMES, EngineConfig

IMG, VS = 1100, 1101
TEXT = dict(hidden_size=512, num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=2, head_dim=128,
            intermediate_size=1024, vocab_size=1200, rms_norm_eps=1e-6, rope_theta=5e6,
            rope_scaling=dict(mrope_section=[24, 20, 20], mrope_interleaved=True))
VISION = dict(hidden_size=256, num_heads=4, intermediate_size=512, depth=4, in_channels=3, temporal_patch_size=2,
              patch_size=4, spatial_merge_size=2, num_position_embeddings=64, out_hidden_size=512,
              deepstack_visual_indexes=[1, 2])
CONFIG = dict(model_type="qwen3_vl", text_config=TEXT, vision_config=VISION, image_token_id=IMG,
              vision_start_token_id=VS, tie_word_embeddings=True)
VCFG = dict(heads=4, merge=2, eps=1e-6, deepstack=[1, 2], num_grid=8)
TCFG = dict(heads=4, kv_heads=2, head_dim=128, eps=1e-6, theta=5e6, mrope=[24, 20, 20])
PATCH_DIM = 3 * 2 * 4 * 4


def _weights(seed=0):
    rng = np.random.default_rng(seed)

    def n(*s, std=0.05):
        return G.rounded(rng.standard_normal(s).astype(np.float32) * std)

    def one(*s):
        return G.rounded(1 + rng.standard_normal(s).astype(np.float32) * 0.1)

    H, I, D, O = 256, 512, 1024, 512
    vis = {"patch_w": n(H, PATCH_DIM, std=0.1), "patch_b": n(H, std=0.05), "pos_table": n(64, H, std=0.5),
           "blocks": [], "deepstack_mergers": []}
    for _ in range(4):
        vis["blocks"].append({
            "qkv_w": n(3 * H, H), "qkv_b": n(3 * H), "proj_w": n(H, H), "proj_b": n(H),
            "fc1_w": n(I, H), "fc1_b": n(I), "fc2_w": n(H, I), "fc2_b": n(H),
            "n1_w": one(H), "n1_b": n(H), "n2_w": one(H), "n2_b": n(H)})

    def merger(nd):
        return {"n_w": one(nd), "n_b": n(nd), "f1_w": n(D, D, std=0.03), "f1_b": n(D), "f2_w": n(O, D, std=0.03),
                "f2_b": n(O)}

    vis["merger"] = merger(H)
    vis["deepstack_mergers"] = [merger(D), merger(D)]
    Ht, It, V = 512, 1024, 1200
    txt = {"embed": n(V, Ht, std=1.0), "norm": one(Ht), "layers": []}
    txt["lm_head"] = txt["embed"]
    for _ in range(3):
        txt["layers"].append({
            "q_w": n(512, Ht), "k_w": n(256, Ht), "v_w": n(256, Ht), "o_w": n(Ht, 512), "qn_w": one(128),
            "kn_w": one(128), "gate_w": n(It, Ht), "up_w": n(It, Ht), "down_w": n(Ht, It), "iln_w": one(Ht),
            "pln_w": one(Ht)})
    return vis, txt


VIS_NAMES = {"qkv_w": "attn.qkv.weight", "qkv_b": "attn.qkv.bias", "proj_w": "attn.proj.weight",
             "proj_b": "attn.proj.bias", "fc1_w": "mlp.linear_fc1.weight", "fc1_b": "mlp.linear_fc1.bias",
             "fc2_w": "mlp.linear_fc2.weight", "fc2_b": "mlp.linear_fc2.bias", "n1_w": "norm1.weight",
             "n1_b": "norm1.bias", "n2_w": "norm2.weight", "n2_b": "norm2.bias"}
MERGER_NAMES = {"n_w": "norm.weight", "n_b": "norm.bias", "f1_w": "linear_fc1.weight", "f1_b": "linear_fc1.bias",
                "f2_w": "linear_fc2.weight", "f2_b": "linear_fc2.bias"}


@pytest.fixture(scope="module")
def engine():
    vis, txt = _weights()
    L = G.L()
    cfg = EngineConfig(None, json.dumps(CONFIG).encode(), 0, 2, 512, 512, 128, 3, 0.02)
    eng = ctypes.c_void_p()
    G.check(L.b200_engine_create(ctypes.byref(cfg), ctypes.byref(eng)), "engine_create")
    held = []

    def put(name, a):
        a = np.ascontiguousarray(a, np.float32)
        held.append(a)
        G.check(L.b200_engine_set_weight(eng, name.encode(), a.ctypes.data, 2, a.size), name)

    put("model.visual.patch_embed.proj.weight", vis["patch_w"].reshape(256, 3, 2, 4, 4))
    put("model.visual.patch_embed.proj.bias", vis["patch_b"])
    put("model.visual.pos_embed.weight", vis["pos_table"])
    for i, b in enumerate(vis["blocks"]):
        for k, nm in VIS_NAMES.items():
            put(f"model.visual.blocks.{i}.{nm}", b[k])
    for k, nm in MERGER_NAMES.items():
        put(f"model.visual.merger.{nm}", vis["merger"][k])
        for i, m in enumerate(vis["deepstack_mergers"]):
            put(f"model.visual.deepstack_merger_list.{i}.{nm}", m[k])
    put("model.language_model.embed_tokens.weight", txt["embed"])
    put("model.language_model.norm.weight", txt["norm"])
    for i, lw in enumerate(txt["layers"]):
        for k, hf in HF_NAMES.items():
            put(f"model.language_model.layers.{i}.{hf}.weight", lw[k])
    has = ctypes.c_int64()
    G.check(L.b200_engine_query(eng, 7, ctypes.byref(has)))
    assert has.value == 1
    yield eng, vis, txt
    L.b200_engine_destroy(eng)


def close(got, ref, tol=0.03):
    assert G.cosine(got, ref) >= 0.999, G.cosine(got, ref)
    assert G.max_rel_err(got, ref) <= tol, G.max_rel_err(got, ref)


def _pixels(grid, seed):
    N = int(sum(t * h * w for t, h, w in grid))
    return np.random.default_rng(seed).uniform(-1, 1, (N, PATCH_DIM)).astype(np.float32)


@pytest.mark.parametrize("grid", [[[1, 8, 8]], [[1, 4, 8], [2, 4, 4]], [[1, 2, 6]]])
def test_vision_tower(engine, grid):
    eng, vis, _ = engine
    L = G.L()
    px = _pixels(grid, 11)
    g = np.array(grid, np.int64)
    Nm = len(px) // 4
    merged = torch.empty(Nm, 512, dtype=torch.bfloat16, device=G.DEV)
    ds = torch.empty(2, Nm, 512, dtype=torch.bfloat16, device=G.DEV)
    nm = ctypes.c_int64()
    ref_m, ref_ds = vision_tower(G.rounded(px), g, vis, VCFG)
    # eager pass, captured pass, replayed graph (device pixels on the last one)
    px_dev = G.bf16(px)
    for rep in range(3):
        merged.zero_()
        ds.zero_()
        torch.cuda.synchronize()  # the engine runs on its own stream
        if rep < 2:
            G.check(L.b200_engine_vision(eng, px.ctypes.data, 2, 0, len(px), g.ctypes.data, len(g),
                                         merged.data_ptr(), ds.data_ptr(), ctypes.byref(nm)), "engine_vision")
        else:
            G.check(L.b200_engine_vision(eng, px_dev.data_ptr(), 0, 1, len(px), g.ctypes.data, len(g),
                                         merged.data_ptr(), ds.data_ptr(), ctypes.byref(nm)), "engine_vision")
        torch.cuda.synchronize()
        assert nm.value == Nm
        close(G.host(merged), ref_m)
        for i in range(2):
            close(G.host(ds[i]), ref_ds[i])
    assert G.device_errors() == 0


def _embed(eng, ids, mask=None, px=None, grid=None, hidden=True, normalize=1):
    L = G.L()
    ids = np.ascontiguousarray(ids, np.int64)
    out = np.zeros(512, np.float32)
    hid = torch.empty(len(ids), 512, dtype=torch.bfloat16, device=G.DEV) if hidden else None
    m = None if mask is None else np.ascontiguousarray(mask, np.int64)
    g = None if grid is None else np.ascontiguousarray(grid, np.int64)
    rc = L.b200_engine_embed(eng, ids.ctypes.data, len(ids), None if m is None else m.ctypes.data,
                             None if px is None else px.ctypes.data, 2, 0, 0 if px is None else len(px),
                             None if g is None else g.ctypes.data, 0 if g is None else len(g), normalize,
                             out.ctypes.data, G.ptr(hid))
    torch.cuda.synchronize()
    return rc, out, None if hid is None else G.host(hid)


def test_embed_text_only(engine):
    eng, _, txt = engine
    ids = np.random.default_rng(5).integers(0, 1000, 37)
    rc, out, hid = _embed(eng, ids)
    assert rc == 0
    ref, ref_h = embed_forward(ids, txt, TCFG)
    close(hid, ref_h)
    close(out, ref)
    assert abs(float(np.linalg.norm(out)) - 1.0) < 1e-3
    rc, raw, _ = _embed(eng, ids, hidden=False, normalize=0)
    assert rc == 0
    close(raw, ref_h[-1])


@pytest.mark.parametrize("grid", [[[1, 8, 8]], [[1, 4, 8], [2, 4, 4]]])
def test_embed_with_image(engine, grid):
    eng, vis, txt = engine
    rng = np.random.default_rng(9)
    g = np.array(grid, np.int64)
    ids = []
    for t, h, w in grid:
        ids += list(rng.integers(0, 1000, 5)) + [VS] + [IMG] * (t * h * w // 4)
    ids = np.array(ids + list(rng.integers(0, 1000, 7)), np.int64)
    px = _pixels(grid, 12)
    rc, out, hid = _embed(eng, ids, px=px, grid=g)
    assert rc == 0
    merged, ds = vision_tower(G.rounded(px), g, vis, VCFG)
    pid = oracle.get_rope_index(ids[None], g, image_token_id=IMG, vision_start_token_id=VS)[:, 0]
    rows = np.nonzero(ids == IMG)[0]
    ref, ref_h = embed_forward(ids, txt, TCFG, pid, rows, merged, ds)
    close(hid, ref_h)
    close(out, ref)


def test_embed_repeated_shapes_replay_graph(engine):
    """A repeated request shape runs eagerly, is captured as a CUDA graph on its
    second call and replayed after: every call, with fresh ids (and pixels),
    matches the oracle."""
    eng, vis, txt = engine
    rng = np.random.default_rng(21)
    for _ in range(4):
        ids = rng.integers(0, 1000, 29)
        rc, out, _ = _embed(eng, ids, hidden=False)
        assert rc == 0
        ref, _ = embed_forward(ids, txt, TCFG)
        close(out, ref)
    grid = [[1, 8, 8]]
    g = np.array(grid, np.int64)
    for i in range(3):
        ids = np.array(list(rng.integers(0, 1000, 5)) + [VS] + [IMG] * 16 + list(rng.integers(0, 1000, 4)), np.int64)
        px = _pixels(grid, 30 + i)
        rc, out, _ = _embed(eng, ids, px=px, grid=g, hidden=False)
        assert rc == 0
        merged, ds = vision_tower(G.rounded(px), g, vis, VCFG)
        pid = oracle.get_rope_index(ids[None], g, image_token_id=IMG, vision_start_token_id=VS)[:, 0]
        rows = np.nonzero(ids == IMG)[0]
        ref, _ = embed_forward(ids, txt, TCFG, pid, rows, merged, ds)
        close(out, ref)
    assert G.device_errors() == 0


def test_embed_pools_last_unmasked_token(engine):
    eng, _, txt = engine
    ids = np.random.default_rng(6).integers(0, 1000, 24)
    mask = np.ones(24, np.int64)
    mask[19:] = 0
    rc, out, _ = _embed(eng, ids, mask=mask, hidden=False)
    assert rc == 0
    pid = oracle.get_rope_index(ids[None], None, None, mask[None])[:, 0]
    ref, _ = embed_forward(ids, txt, TCFG, pid, pool_row=18)
    close(out, ref)


def test_embed_rejects_image_token_mismatch(engine):
    eng, _, _ = engine
    grid = [[1, 8, 8]]
    ids = np.array([3, 4, VS] + [IMG] * 15 + [5], np.int64)  # 15 image tokens, 16 merged
    rc, _, _ = _embed(eng, ids, px=_pixels(grid, 1), grid=np.array(grid, np.int64), hidden=False)
    assert rc == -1
    rc, _, _ = _embed(eng, np.zeros(0, np.int64), hidden=False)
    assert rc == -1
