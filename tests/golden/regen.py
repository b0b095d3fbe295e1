"""Re-create the large golden INPUTS from their seeds.

The reference generator (atb_cpp_llm/tests/python_reference/gen_cpu_reference.py)
draws its inputs from seeded numpy / torch generators.  Weight tensors of the
larger cases are tens of MB, too big to commit, so the fixtures keep only the
outputs plus a sha256 of every omitted input; the functions below replay the
generator's draws in the same order, and ``tests/test_golden_oracle.py``
checks each replayed array against its recorded sha256 before use.
"""

import hashlib

import numpy as np


def _f16(a):
    return a.astype(np.float16)


def decoder_layer_inputs(S, nh, kvh, hd, I, seed):
    """Draw order of ``gen_text_decoder_layer._make`` (gen_cpu_reference.py:1518-1540),
    returned fp16-rounded (``_fp16_roundtrip``, :1552-1560)."""
    rng = np.random.default_rng(seed)
    H, Hkv = nh * hd, kvh * hd
    f32 = np.float32
    d = {}
    d["x"] = rng.standard_normal((S, H)).astype(f32) * 0.1
    d["q_w"] = rng.standard_normal((H, H)).astype(f32) * 0.05
    d["k_w"] = rng.standard_normal((Hkv, H)).astype(f32) * 0.05
    d["v_w"] = rng.standard_normal((Hkv, H)).astype(f32) * 0.05
    d["o_w"] = rng.standard_normal((H, H)).astype(f32) * 0.05
    d["qn_w"] = rng.standard_normal((hd,)).astype(f32) * 0.1 + 1.0
    d["kn_w"] = rng.standard_normal((hd,)).astype(f32) * 0.1 + 1.0
    d["gate_w"] = rng.standard_normal((I, H)).astype(f32) * 0.05
    d["up_w"] = rng.standard_normal((I, H)).astype(f32) * 0.05
    d["down_w"] = rng.standard_normal((H, I)).astype(f32) * 0.05
    d["iln_w"] = rng.standard_normal((H,)).astype(f32) * 0.1 + 1.0
    d["pln_w"] = rng.standard_normal((H,)).astype(f32) * 0.1 + 1.0
    ang = rng.standard_normal((S, hd // 2)).astype(f32) * 0.5
    emb = np.concatenate([ang, ang], axis=-1)
    d["cos"] = np.cos(emb)
    d["sin"] = np.sin(emb)
    return {k: _f16(v) for k, v in d.items()}


def swiglu_inputs(S, H, I, seed):
    """Draw order of ``gen_swiglu_mlp._make`` (gen_cpu_reference.py:1431-1443)."""
    rng = np.random.default_rng(seed)
    f32 = np.float32
    d = {
        "x": rng.standard_normal((S, H)).astype(f32) * 0.1,
        "gate_w": rng.standard_normal((I, H)).astype(f32) * 0.05,
        "up_w": rng.standard_normal((I, H)).astype(f32) * 0.05,
        "down_w": rng.standard_normal((H, I)).astype(f32) * 0.05,
    }
    return {k: _f16(v) for k, v in d.items()}


def vision_block_inputs(N, nh, hd, inter, seed):
    """Draw order of ``gen_vision_block._build_case`` (gen_cpu_reference.py:1969-1983)."""
    rng = np.random.default_rng(seed)
    hidden = nh * hd
    f32 = np.float32
    d = {}
    d["x"] = rng.standard_normal((N, hidden)).astype(f32) * 0.2
    d["qkv_w"] = rng.standard_normal((3 * hidden, hidden)).astype(f32) * 0.1
    d["qkv_b"] = rng.standard_normal((3 * hidden,)).astype(f32) * 0.05
    d["proj_w"] = rng.standard_normal((hidden, hidden)).astype(f32) * 0.1
    d["proj_b"] = rng.standard_normal((hidden,)).astype(f32) * 0.05
    d["fc1_w"] = rng.standard_normal((inter, hidden)).astype(f32) * 0.1
    d["fc1_b"] = rng.standard_normal((inter,)).astype(f32) * 0.05
    d["fc2_w"] = rng.standard_normal((hidden, inter)).astype(f32) * 0.1
    d["fc2_b"] = rng.standard_normal((hidden,)).astype(f32) * 0.05
    d["n1_w"] = rng.standard_normal((hidden,)).astype(f32) * 0.1 + 1.0
    d["n1_b"] = rng.standard_normal((hidden,)).astype(f32) * 0.05
    d["n2_w"] = rng.standard_normal((hidden,)).astype(f32) * 0.1 + 1.0
    d["n2_b"] = rng.standard_normal((hidden,)).astype(f32) * 0.05
    return {k: _f16(v) for k, v in d.items()}


def vision_mlp_inputs(N, hidden, inter, seed, zero_bias=False):
    """Draw order of ``gen_vision_mlp._make`` (gen_cpu_reference.py:1909-1918)."""
    rng = np.random.default_rng(seed)
    f32 = np.float32
    d = {"x": rng.standard_normal((N, hidden)).astype(f32) * 0.2,
         "fc1_w": rng.standard_normal((inter, hidden)).astype(f32) * 0.1,
         "fc2_w": rng.standard_normal((hidden, inter)).astype(f32) * 0.1}
    if zero_bias:
        d["fc1_b"] = np.zeros((inter,), f32)
        d["fc2_b"] = np.zeros((hidden,), f32)
    else:
        d["fc1_b"] = rng.standard_normal((inter,)).astype(f32) * 0.05
        d["fc2_b"] = rng.standard_normal((hidden,)).astype(f32) * 0.05
    return {k: _f16(v) for k, v in d.items()}


def patch_embed_inputs(N, K, embed_dim, seed):
    """Draw order of ``gen_patch_embed._make`` (gen_cpu_reference.py:2104-2107)."""
    rng = np.random.default_rng(seed)
    f32 = np.float32
    d = {"pixels": rng.standard_normal((N, K)).astype(f32) * 0.2,
         "w": rng.standard_normal((embed_dim, K)).astype(f32) * 0.05,
         "b": rng.standard_normal((embed_dim,)).astype(f32) * 0.05}
    return {k: _f16(v) for k, v in d.items()}


def linear_inputs(S, K, N):
    """Draw order of ``gen_linear._make_tb`` (gen_cpu_reference.py:898-902)."""
    import torch

    torch.manual_seed(7 + S + K + N)
    x = torch.randn(S, K, dtype=torch.float32) * 0.1
    w = torch.randn(N, K, dtype=torch.float32) * 0.1
    return {"input": x.numpy(), "weight": w.numpy()}


def sha256(a):
    a = np.ascontiguousarray(a)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode())
    h.update(str(a.shape).encode())
    h.update(a.tobytes())
    return h.hexdigest()
