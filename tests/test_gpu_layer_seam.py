"""The layer-graph seam through the C ABI: b200_text_decoder_layer and
b200_vision_block take one layer's inputs in the reference's variant-pack
order (TextDecoderLayerGraph::Build, decoder_layer_graph.cpp:30-52: 15 inputs,
16 with the mask; VisionBlockGraph::Build, vision_block_graph.cpp:22-28: 16
inputs) and a caller-sized workspace, as a caller replacing those graph
builders would call them.

GPU: the reference's three decoder-layer goldens and three vision-block
goldens through the seam (cosine >= 0.999 against the golden, and against the
oracle on the same bf16-rounded inputs with max |err| <= 2 % of max |ref|; the
real-size vision block 4 %, as in the composed-kernel tests), and the
Qwen3-VL-2B text layer config with two packed sequences, each causal on its
own.  CPU: the argument checks (input count, sequence lengths, workspace size)
return ERROR_INVALID_PARAM before any CUDA call.
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from conftest import DEC_CASES, checked_inputs, decoder_case, load_fixture
from oracle import vision

F = np.float32

if torch.cuda.is_available():
    import gpu_util as G


def _pack(ptrs):
    arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
    return arr, ctypes.addressof(arr)


def text_layer(x, w, cos, sin, nh, kvh, hd, lens, use_mask, qk_norm=True, eps=1e-6):
    L = G.L()
    T, H = x.shape
    I = w["gate_w"].shape[0]
    d = {k: G.bf16(v) for k, v in w.items()}
    xd = G.bf16(x)
    out = torch.empty_like(xd)
    seqlen = np.asarray(lens, np.int32)
    ptrs = [xd.data_ptr(), d["q_w"].data_ptr(), d["k_w"].data_ptr(), d["v_w"].data_ptr(), d["o_w"].data_ptr()]
    if qk_norm:
        ptrs += [d["qn_w"].data_ptr(), d["kn_w"].data_ptr()]
    ptrs += [d["gate_w"].data_ptr(), d["up_w"].data_ptr(), d["down_w"].data_ptr(), d["iln_w"].data_ptr(),
             d["pln_w"].data_ptr(), G.f32(cos).data_ptr(), G.f32(sin).data_ptr()]
    if use_mask:  # the reference's additive causal mask: accepted in its slot, the rule is applied in-kernel
        m = np.triu(np.full((T, T), -65504.0, F), 1)
        ptrs.append(G.bf16(m).data_ptr())
    ptrs.append(seqlen.ctypes.data)
    assert len(ptrs) == (16 if use_mask else 15) - (0 if qk_norm else 2)
    wsb = L.b200_text_decoder_layer_workspace_bytes(T, H, nh, kvh, hd, I)
    ws = torch.empty(wsb, dtype=torch.uint8, device=G.DEV)
    arr, addr = _pack(ptrs)
    G.check(L.b200_text_decoder_layer(addr, len(ptrs), out.data_ptr(), T, len(lens), H, nh, kvh, hd, I, eps,
                                      int(qk_norm), int(use_mask), ws.data_ptr(), wsb, G.stream()), "text_decoder_layer")
    torch.cuda.synchronize()
    return G.host(out)


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(DEC_CASES))
def test_text_decoder_layer_seam_golden(name):
    c = decoder_case(name)
    inp = {k: v.astype(F) for k, v in c["inputs"].items()}
    w = {k: inp[k] for k in inp if k.endswith("_w")}
    use_mask = c["mask"] is not None
    S = inp["x"].shape[0]
    out = text_layer(inp["x"], w, inp["cos"], inp["sin"], c["nh"], c["kvh"], c["hd"], [S], use_mask)
    assert G.cosine(out, c["out_ref"].astype(F)) >= 0.999
    wr = {k: G.rounded(v) for k, v in w.items()}
    orc = oracle.decoder_layer(G.rounded(inp["x"]), wr, inp["cos"], inp["sin"], c["nh"], c["kvh"], c["hd"], 1e-6,
                               causal=use_mask)
    assert G.cosine(out, orc) >= 0.999
    assert G.max_rel_err(out, orc) < 0.02
    assert G.device_errors() == 0


@pytest.mark.gpu
def test_text_decoder_layer_seam_qwen3vl_two_packed_sequences():
    S, H, nh, kvh, hd, I = 256, 2048, 16, 8, 128, 6144
    rw = np.random.default_rng(0)
    w = {"q_w": rw.standard_normal((nh * hd, H), F) * 0.02, "k_w": rw.standard_normal((kvh * hd, H), F) * 0.02,
         "v_w": rw.standard_normal((kvh * hd, H), F) * 0.02, "o_w": rw.standard_normal((H, nh * hd), F) * 0.02,
         "qn_w": 1 + rw.standard_normal(hd, F) * 0.02, "kn_w": 1 + rw.standard_normal(hd, F) * 0.02,
         "gate_w": rw.standard_normal((I, H), F) * 0.02, "up_w": rw.standard_normal((I, H), F) * 0.02,
         "down_w": rw.standard_normal((H, I), F) * 0.02, "iln_w": 1 + rw.standard_normal(H, F) * 0.02,
         "pln_w": 1 + rw.standard_normal(H, F) * 0.02}
    x = np.random.default_rng(1).standard_normal((S, H), F)
    lens = [100, 156]
    pos = np.concatenate([np.arange(n) for n in lens])
    cos, sin = oracle.mrope_cos_sin(np.stack([pos, pos, pos])[:, None, :], hd, 5e6, (24, 20, 20))
    out = text_layer(x, w, cos[0], sin[0], nh, kvh, hd, lens, True)
    wr = {k: G.rounded(v) for k, v in w.items()}
    xr = G.rounded(x)
    a = 0
    for n in lens:
        ref = oracle.decoder_layer(xr[a:a + n], wr, cos[0][a:a + n], sin[0][a:a + n], nh, kvh, hd, 1e-6, causal=True)
        assert G.cosine(out[a:a + n], ref) >= 0.999
        assert G.max_rel_err(out[a:a + n], ref) < 0.02
        a += n
    assert G.device_errors() == 0


BLOCK_CASES = {"": 5301, "real_small_": 5302, "real_typical_": 5303}
BLOCK_ORDER = ["qkv_w", "qkv_b", "proj_w", "proj_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "n1_w", "n1_b", "n2_w",
               "n2_b"]


@pytest.mark.gpu
@pytest.mark.parametrize("case", list(BLOCK_CASES))
def test_vision_block_seam_golden(case):
    import regen

    L = G.L()
    fx = load_fixture("vision_block")
    N, nh, hd, inter = (int(v) for v in fx[case + "meta"])
    inp = regen.vision_block_inputs(N, nh, hd, inter, BLOCK_CASES[case])
    checked_inputs("vision_block", case, inp)
    w = {k: v.astype(F) for k, v in inp.items() if k != "x"}
    cos, sin = fx[case + "cos"].astype(F), fx[case + "sin"].astype(F)
    H = nh * hd
    xd = G.bf16(inp["x"].astype(F))
    out = torch.empty_like(xd)
    seq = np.array([N], np.int32)
    ptrs = [xd.data_ptr()] + [G.bf16(w[k]).data_ptr() for k in BLOCK_ORDER] + [G.f32(cos).data_ptr(),
                                                                               G.f32(sin).data_ptr(),
                                                                               seq.ctypes.data]
    wsb = L.b200_vision_block_workspace_bytes(N, H, inter)
    ws = torch.empty(wsb, dtype=torch.uint8, device=G.DEV)
    arr, addr = _pack(ptrs)
    G.check(L.b200_vision_block(addr, 16, out.data_ptr(), N, 1, H, nh, hd, inter, 1e-6, ws.data_ptr(), wsb,
                                G.stream()), "vision_block")
    torch.cuda.synchronize()
    got = G.host(out)
    tol = 0.04 if hd * nh >= 1024 else 0.02
    ref = fx[case + "ref"].astype(F)
    assert G.cosine(got, ref) >= 0.999 and G.max_rel_err(got, ref) <= tol
    wr = {k: G.rounded(v) for k, v in w.items()}
    orc = vision.vision_block(G.rounded(inp["x"].astype(F)), wr, cos, sin, nh, hd)
    assert G.cosine(got, orc) >= 0.999 and G.max_rel_err(got, orc) <= tol
    assert G.device_errors() == 0


def test_seam_argument_checks_before_any_launch():
    """Wrong input counts, lengths that do not sum to T and short workspaces
    are ERROR_INVALID_PARAM; nothing is dereferenced or launched."""
    from atb_llm_study_b200 import capi

    L = capi.lib()
    d = 256  # never dereferenced
    T, H, nh, kvh, hd, I = 64, 256, 2, 1, 128, 512
    need = L.b200_text_decoder_layer_workspace_bytes(T, H, nh, kvh, hd, I)
    assert need >= T * H * 2 + T * (nh + 2 * kvh) * hd * 2
    seq_ok, seq_bad = np.array([T], np.int32), np.array([T - 1], np.int32)

    def call(n_in, seq, wsb, mask=0):
        ptrs = [d] * (n_in - 1) + [seq.ctypes.data]
        arr, addr = _pack(ptrs)
        return L.b200_text_decoder_layer(addr, n_in, d, T, 1, H, nh, kvh, hd, I, 1e-6, 1, mask, d, wsb, None)

    assert call(14, seq_ok, need) == -1  # 15 expected without the mask
    assert call(15, seq_ok, need, mask=1) == -1  # 16 expected with it
    assert call(15, seq_bad, need) == -1  # lengths sum to 63, not 64
    assert call(15, seq_ok, need - 256) == -1  # workspace too small
    vneed = L.b200_vision_block_workspace_bytes(T, H, I)
    assert vneed > 0
    ptrs = [d] * 15 + [seq_ok.ctypes.data]
    arr, addr = _pack(ptrs)
    assert L.b200_vision_block(addr, 15, d, T, 1, H, 2, 128, I, 1e-6, d, vneed, None) == -1
    assert L.b200_vision_block(addr, 16, d, T, 1, H, 2, 64, I, 1e-6, d, vneed, None) == -1  # heads x dim != H
    assert L.b200_vision_block(addr, 16, d, T, 1, H, 2, 128, I, 1e-6, d, vneed - 256, None) == -1
