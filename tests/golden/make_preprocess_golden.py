"""Generate ``preprocess.npz``: golden data for the image preprocessing path,
made by running the REFERENCE generator's ``smart_resize`` and
``bicubic_preprocess`` stages (atb_cpp_llm/tests/python_reference/
gen_cpu_reference.py:360-393, :550-680), whose ground truth is real PIL
``Image.resize(BICUBIC)`` per channel and the reference Python
``smart_resize``.

Packed: the SmartResize quadruples (h, w, new_h, new_w); every bicubic case's
uint8 input and PIL output (the production-size cases, several MB each, only
as shape + sha256 of input and output — their inputs are seeded draws the
tests regenerate); the PreprocessImage cases' uint8 input, PIL-chain fp16
pixel values and grid.

Usage (in a container that has the reference checkout and PIL):
    python tests/golden/make_preprocess_golden.py --reference <checkout>   (or ATB_LLM_REFERENCE=<checkout>)
"""

import argparse
import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PROD = [(416, 672), (720, 1280), (1080, 1920), (1440, 2560)]  # the generator's draw order (seed 2026)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def prod_inputs():
    """The production-size inputs exactly as the generator draws them."""
    rs = np.random.RandomState(2026)
    for h, w in PROD:
        img = (rs.rand(3, h, w) * 255.0).astype(np.float32)
        yield (h, w), np.clip(np.round(img), 0.0, 255.0).astype(np.uint8)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ATB_LLM_REFERENCE"),
                    required="ATB_LLM_REFERENCE" not in os.environ)
    args = ap.parse_args()
    tests_dir = os.path.join(args.reference, "atb_cpp_llm", "tests")
    sys.path.insert(0, os.path.join(tests_dir, "python_reference"))
    sys.path.insert(0, tests_dir)
    sys.path.insert(0, args.reference)
    os.environ.setdefault("QWEN3VL_EMB_MODEL_DIR", "/nonexistent-checkpoint")
    import gen_cpu_reference as gen  # noqa: E402
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle.golden_io import read_bin, read_i32s  # noqa: E402

    out = {}
    with tempfile.TemporaryDirectory(dir=HERE) as tmp:
        gen.OUTPUT_DIR = tmp
        gen.STAGES["smart_resize"]()
        gen.STAGES["bicubic_preprocess"]()
        out["smart_resize"] = np.asarray(read_i32s(os.path.join(tmp, "cpu_smart_resize.bin")), np.int32).reshape(-1, 4)
        prod = dict(prod_inputs())
        for f in sorted(os.listdir(tmp)):
            if f.startswith("bicubic_") and f.endswith("_pil_output.bin"):
                name = f[len("bicubic_"):-len("_pil_output.bin")]
                x = read_bin(os.path.join(tmp, f"bicubic_{name}_input.bin"), "f32").astype(np.uint8)
                y = read_bin(os.path.join(tmp, f), "f32").astype(np.uint8)
                if name.startswith("prod_"):
                    h, w = (int(v) for v in name[5:].split("x"))
                    assert sha(prod[(h, w)]) == sha(x), name  # the regenerated draw is the generator's input
                    out[f"bicubic_{name}__in_shape"] = np.array(x.shape, np.int32)
                    out[f"bicubic_{name}__out_shape"] = np.array(y.shape, np.int32)
                    out[f"bicubic_{name}__in_sha256"] = np.array(sha(x))
                    out[f"bicubic_{name}__out_sha256"] = np.array(sha(y))
                else:
                    out[f"bicubic_{name}__input"] = x
                    out[f"bicubic_{name}__pil"] = y
            if f.startswith("preprocess_") and f.endswith("_pil_output.bin"):
                name = f[len("preprocess_"):-len("_pil_output.bin")]
                x = read_bin(os.path.join(tmp, f"preprocess_{name}_input.bin"), "f32").astype(np.uint8)
                out[f"preprocess_{name}__input"] = x
                out[f"preprocess_{name}__pil"] = read_bin(os.path.join(tmp, f), "fp16")
                out[f"preprocess_{name}__grid"] = read_bin(os.path.join(tmp, f"preprocess_{name}_grid.bin"), "i64")
    np.savez_compressed(os.path.join(HERE, "preprocess.npz"), **out)
    print(f"preprocess.npz: {len(out)} arrays")


if __name__ == "__main__":
    main()
