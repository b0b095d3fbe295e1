import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(autouse=True)
def _release_device_buffers(request):
    yield
    if "gpu_util" in sys.modules:
        sys.modules["gpu_util"].release()


def load_fixture(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


def manifest():
    with open(os.path.join(GOLDEN, "manifest.json")) as fh:
        return json.load(fh)


DEC_CASES = {
    # name: (S, nh, kvh, hd, I, use_mask, seed) — gen_cpu_reference.py:1627-1629
    "small_nomask": (4, 4, 4, 32, 64, False, 6001),
    "gqa_mask": (8, 12, 4, 64, 256, True, 6002),
    "mha_causal": (16, 32, 32, 128, 1024, True, 6003),
}


def decoder_case(name):
    """Inputs (fp16 numpy) + golden output of one reference decoder-layer case,
    rebuilding omitted weights from their seeds and checking their sha256."""
    import regen

    fx = load_fixture("decoder_layer")
    S, nh, kvh, hd, I, use_mask, seed = DEC_CASES[name]
    meta = fx[f"{name}_meta"]
    assert list(meta) == [S, nh, kvh, hd, I, int(use_mask)]
    rebuilt = regen.decoder_layer_inputs(S, nh, kvh, hd, I, seed)
    man = manifest()
    inp = {}
    for k, v in rebuilt.items():
        key = f"{name}_{k}"
        if key in fx:
            np.testing.assert_array_equal(fx[key], v)
        else:
            entry = man[f"decoder_layer/{key}"]
            assert regen.sha256(v) == entry["sha256"], key
        inp[k] = v
    mask = fx.get(f"{name}_mask")
    return dict(S=S, nh=nh, kvh=kvh, hd=hd, I=I, inputs=inp, mask=mask,
                out_ref=fx[f"{name}_out_ref"])


def checked_inputs(fixture, prefix, rebuilt):
    """Rebuilt (seed-replayed) inputs of one golden case, each checked against
    the committed array or, for arrays too large to commit, the sha256 the
    reference run recorded.  ``prefix`` is the case's key prefix ('' or 'x_')."""
    import regen

    fx = load_fixture(fixture)
    man = manifest()
    for k, v in rebuilt.items():
        key = f"{prefix}{k}"
        if key in fx:
            np.testing.assert_array_equal(fx[key], v, err_msg=key)
        else:
            assert regen.sha256(v) == man[f"{fixture}/{key}"]["sha256"], key
    return fx


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))
