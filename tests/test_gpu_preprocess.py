"""Image preprocessing on the GPU against PIL (through the reference
generator's golden data) and the oracle.

* b200_bicubic_resize_u8: the generator's small cases and its production-size
  images (416x672 identity, 720x1280 -> 704x1280 vertical only, 1080x1920 and
  1440x2560 -> 992x1792 both passes), bit-exact uint8 (sha256 of PIL's
  output), plus odd up/down sizes against the oracle.
* b200_preprocess_image: the three PreprocessImage cases, fp16 pixel values
  bit-exact with the PIL chain, grid and patch count; bf16 output equal to
  the oracle's float32 values rounded to bf16; and frames that take each
  variant of the fused kernel (rows not a multiple of 16 bytes, so byte-load
  staging; 8- and 16-tap windows; a >2x downscale) bit-exact with the oracle.
"""

import ctypes
import hashlib
import os

import numpy as np
import pytest
import torch

from oracle import preprocess as P

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gpu_util as G

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "preprocess.npz"))


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def resize(x, oh, ow):
    L = G.L()
    C, H, W = x.shape
    xd = torch.from_numpy(np.ascontiguousarray(x)).to(G.DEV)
    out = torch.empty(C, oh, ow, dtype=torch.uint8, device=G.DEV)
    wsb = L.b200_preprocess_workspace_bytes(C, H, W, oh, ow)
    ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device=G.DEV)
    G.check(L.b200_bicubic_resize_u8(xd.data_ptr(), C, H, W, oh, ow, out.data_ptr(), ws.data_ptr(), wsb, G.stream()),
            "bicubic_resize_u8")
    torch.cuda.synchronize()
    return out.cpu().numpy()


def preprocess(x, dtype=1):
    L = G.L()
    C, H, W = x.shape
    nh, nw = ctypes.c_int(), ctypes.c_int()
    G.check(L.b200_smart_resize(H, W, 32, 4096, 1843200, ctypes.byref(nh), ctypes.byref(nw)), "smart_resize")
    n = (nh.value // 16) * (nw.value // 16)
    pv = torch.empty(n, C * 2 * 16 * 16, dtype=torch.float16 if dtype == 1 else torch.bfloat16, device=G.DEV)
    wsb = L.b200_preprocess_workspace_bytes(C, H, W, nh.value, nw.value)
    ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device=G.DEV)
    xd = torch.from_numpy(np.ascontiguousarray(x)).to(G.DEV)
    npatch = ctypes.c_int64()
    grid = (ctypes.c_int64 * 3)()
    G.check(L.b200_preprocess_image(xd.data_ptr(), C, H, W, 16, 2, 2, 4096, 1843200, None, None, dtype, pv.data_ptr(),
                                    pv.numel(), ctypes.byref(npatch), grid, ws.data_ptr(), wsb, G.stream()),
            "preprocess_image")
    torch.cuda.synchronize()
    return pv, npatch.value, tuple(grid)


@pytest.mark.parametrize("name", ["2x2_to_4x4", "4x4_to_2x2", "random_8x8_to_16x16_3ch"])
def test_bicubic_small_cases(name):
    x, y = GOLD[f"bicubic_{name}__input"], GOLD[f"bicubic_{name}__pil"]
    np.testing.assert_array_equal(resize(x, y.shape[1], y.shape[2]), y)


def test_bicubic_production_sizes_match_pil():
    rs = np.random.RandomState(2026)  # the generator's draws, in its order
    for h, w in [(416, 672), (720, 1280), (1080, 1920), (1440, 2560)]:
        x = np.clip(np.round((rs.rand(3, h, w) * 255.0).astype(np.float32)), 0, 255).astype(np.uint8)
        key = f"bicubic_prod_{h}x{w}"
        assert _sha(x) == str(GOLD[f"{key}__in_sha256"])
        oh, ow = (int(v) for v in GOLD[f"{key}__out_shape"][1:])
        assert _sha(resize(x, oh, ow)) == str(GOLD[f"{key}__out_sha256"]), key
    assert G.device_errors() == 0


@pytest.mark.parametrize("shape", [(3, 37, 53, 64, 96), (1, 300, 200, 100, 150), (3, 17, 700, 40, 90),
                                   (2, 5, 5, 1, 1), (3, 1000, 31, 320, 31)])
def test_bicubic_odd_sizes_vs_oracle(shape):
    C, H, W, oh, ow = shape
    x = np.random.default_rng(H * W).integers(0, 256, (C, H, W), dtype=np.uint8)
    np.testing.assert_array_equal(resize(x, oh, ow), P.resample_u8(x, oh, ow))


@pytest.mark.parametrize("name", ["gradient_64x64", "random_96x96", "down_144x272"])
def test_preprocess_chain_matches_pil(name):
    x = GOLD[f"preprocess_{name}__input"]
    pv, n, grid = preprocess(x)
    np.testing.assert_array_equal(np.array([grid]), GOLD[f"preprocess_{name}__grid"])
    assert n == GOLD[f"preprocess_{name}__pil"].shape[0]
    np.testing.assert_array_equal(pv.cpu().numpy().view(np.uint16), GOLD[f"preprocess_{name}__pil"].view(np.uint16))


def test_preprocess_bf16_and_large_image():
    x = np.random.default_rng(9).integers(0, 256, (3, 1080, 1920), dtype=np.uint8)
    pv, n, grid = preprocess(x, dtype=0)
    ref16, rgrid = P.preprocess_image(x)
    assert grid == rgrid and n == ref16.shape[0]
    # bf16 of the same float32 values: compare through the oracle's fp32 chain
    nh, nw = P.smart_resize(1080, 1920)
    r = P.resample_u8(x, nh, nw)
    norm = ((r.astype(np.float32) / np.float32(255.0)) - np.float32(0.5)) / np.float32(0.5)
    want = torch.from_numpy(P.patchify(norm)).to(torch.bfloat16)
    assert torch.equal(pv.cpu(), want)
    assert G.device_errors() == 0


@pytest.mark.parametrize("h,w", [(37, 53), (500, 333), (2400, 3000), (2400, 3008)])
def test_preprocess_chain_fused_variants_vs_oracle(h, w):
    # 37x53 -> 64x96 and 500x333 -> 512x320: unaligned rows, up to 7 taps;
    # 2400x3000 / 2400x3008 -> 1184x1504: 9 / 11 taps (the 16-tap kernel), unaligned / aligned rows
    x = np.random.default_rng(h * 7 + w).integers(0, 256, (3, h, w), dtype=np.uint8)
    pv, n, grid = preprocess(x)
    ref, rgrid = P.preprocess_image(x)
    assert grid == rgrid and n == ref.shape[0]
    np.testing.assert_array_equal(pv.cpu().numpy().view(np.uint16), ref.view(np.uint16))
    assert G.device_errors() == 0
