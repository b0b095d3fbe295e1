"""GetRopeIndex on the GPU (b200_get_rope_index_device) against the host
implementation, itself bit-exact with the reference's GetRopeIndex goldens:
the six reference cases, then random batches with attention masks, several
images per row, image runs cut off by the sequence end and more vision-start
tokens than grids.  Bar: identical int64 position planes, clear error word."""

import ctypes
import json
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    import gpu_util as G

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "mrope.npz"))
IMG, VS = 151655, 151652


def host(ids, mask, grid, merge=2):
    B, S = ids.shape
    out = np.zeros((3, B, S), np.int64)
    ids = np.ascontiguousarray(ids, np.int64)
    m = None if mask is None else np.ascontiguousarray(mask, np.int64)
    g = None if grid is None else np.ascontiguousarray(grid, np.int64)
    assert G.L().b200_get_rope_index(ids.ctypes.data, B, S, None if m is None else m.ctypes.data,
                                     None if g is None else g.ctypes.data, 0 if g is None else len(g), IMG, VS, merge,
                                     out.ctypes.data) == 0
    return out


def device(ids, mask, grid, merge=2):
    L = G.L()
    B, S = ids.shape
    d_ids = torch.from_numpy(np.ascontiguousarray(ids, np.int64)).to(G.DEV)
    d_mask = None if mask is None else torch.from_numpy(np.ascontiguousarray(mask, np.int64)).to(G.DEV)
    d_grid = None if grid is None else torch.from_numpy(np.ascontiguousarray(grid, np.int64)).to(G.DEV)
    out = torch.full((3, B, S), -7, dtype=torch.int64, device=G.DEV)
    wsb = L.b200_rope_index_workspace_bytes(S)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=G.DEV)
    G.check(L.b200_get_rope_index_device(d_ids.data_ptr(), B, S, None if d_mask is None else d_mask.data_ptr(),
                                         None if d_grid is None else d_grid.data_ptr(),
                                         0 if grid is None else len(grid), IMG, VS, merge, out.data_ptr(),
                                         ws.data_ptr(), wsb, G.stream()), "get_rope_index_device")
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("case", ["simple", "no_img", "image_text", "multi_img", "chat_template", "boundary"])
def test_reference_cases(case):
    k = f"rope_index_{case}"
    ids = GOLD[f"{k}__input_ids"]
    grid = GOLD[f"{k}__image_grid_thw"] if f"{k}__image_grid_thw" in GOLD.files else None
    mask = GOLD[f"{k}__attention_mask"] if f"{k}__attention_mask" in GOLD.files else None
    kw = json.loads(str(GOLD[f"{k}__kw"]))
    merge = int(kw.get("spatial_merge_size", 2))
    got = device(ids, mask, grid, merge)
    np.testing.assert_array_equal(got, host(ids, mask, grid, merge))
    np.testing.assert_array_equal(got, GOLD[f"{k}__position_ids"])
    assert G.device_errors() == 0


def _prompt(rng, S, grids):
    toks = list(rng.integers(0, 150000, rng.integers(0, 20)))
    for g in grids:
        toks += [VS] + [IMG] * int(g[0] * (g[1] // 2) * (g[2] // 2)) + list(rng.integers(0, 150000, rng.integers(0, 30)))
    toks = (toks + list(rng.integers(0, 150000, S)))[:S]
    return toks


@pytest.mark.parametrize("seed", range(6))
def test_random_batches(seed):
    rng = np.random.default_rng(seed)
    B, S = int(rng.integers(1, 5)), int(rng.integers(50, 3000))
    grids, rows = [], []
    for _ in range(B):
        g = [(int(rng.integers(1, 3)), 2 * int(rng.integers(1, 12)), 2 * int(rng.integers(1, 12)))
             for _ in range(int(rng.integers(0, 4)))]
        rows.append(_prompt(rng, S, g))
        grids += g
    ids = np.array(rows, np.int64)
    if seed % 2:  # one grid short: the last announced image has none
        grids = grids[:-1] if grids else grids
    mask = None
    if seed % 3 == 0:
        mask = np.ones((B, S), np.int64)
        for b in range(B):
            mask[b, : int(rng.integers(0, 40))] = 0  # left padding
    grid = np.array(grids, np.int64) if grids else None
    np.testing.assert_array_equal(device(ids, mask, grid), host(ids, mask, grid))
    assert G.device_errors() == 0
