"""Generate the committed golden fixtures by running the REFERENCE generator.

Runs ``atb_cpp_llm/tests/python_reference/gen_cpu_reference.py`` from a
reference checkout (``--reference`` or ``ATB_LLM_REFERENCE``; it is imported, never copied)
into a scratch directory, then packs the files that pin the decoder-layer hot
path into compact ``.npz`` fixtures next to this script:

* arrays up to ``--max-bytes`` are stored verbatim;
* larger arrays (the weights of the bigger cases) are omitted and recorded in
  ``manifest.json`` with shape, dtype and sha256; ``regen.py`` replays the
  generator's seeded draws to rebuild them and the tests check the hash.

The inputs of the ``GetRopeIndex`` cases are not written by the generator,
so ``get_rope_index`` is wrapped while the stages run to record its arguments.

Usage (where a reference checkout exists; the tests read only the fixtures):
    python tests/golden/make_golden.py --reference <checkout>   (or ATB_LLM_REFERENCE=<checkout>)
"""

import argparse
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import regen  # noqa: E402

STAGES = [
    "text_decoder_layer", "op_rms_norm", "op_linear", "op_rope",
    "op_self_attention", "swiglu_mlp", "mrope_cos_sin", "mrope_pid_simple",
    "mrope_pid_no_img", "mrope_pid_image_text", "mrope_pid_multi_img",
    "mrope_pid_chat_template", "mrope_pid_boundary", "op_activation",
    "vision_rope", "vision_attention", "vision_mlp", "vision_block", "patch_embed",
    "vision_merger",
]


def main():
    # the generator seeds its activation cases with hash(name): pin str hashing
    if os.environ.get("PYTHONHASHSEED") != "0":
        os.execve(sys.executable, [sys.executable] + sys.argv, dict(os.environ, PYTHONHASHSEED="0"))
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ATB_LLM_REFERENCE"),
                    required="ATB_LLM_REFERENCE" not in os.environ)
    ap.add_argument("--max-bytes", type=int, default=600_000)
    args = ap.parse_args()

    tests_dir = os.path.join(args.reference, "atb_cpp_llm", "tests")
    sys.path.insert(0, os.path.join(tests_dir, "python_reference"))
    sys.path.insert(0, tests_dir)
    # The generator's env shim demands a checkpoint path even for stages that
    # never read it; none of the stages above touches it.
    os.environ.setdefault("QWEN3VL_EMB_MODEL_DIR", "/nonexistent-checkpoint")
    import gen_cpu_reference as gen  # noqa: E402
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle.golden_io import read_bin, read_i32s  # noqa: E402

    calls = {}
    real = gen.get_rope_index

    def recording(input_ids, image_grid_thw=None, video_grid_thw=None,
                  attention_mask=None, **kw):
        out = real(input_ids, image_grid_thw, video_grid_thw, attention_mask, **kw)
        calls[current[0]] = dict(
            input_ids=input_ids.numpy().copy(),
            image_grid_thw=None if image_grid_thw is None else image_grid_thw.numpy().copy(),
            attention_mask=None if attention_mask is None else attention_mask.numpy().copy(),
            kw=kw, position_ids=out[0].numpy().copy())
        return out

    gen.get_rope_index = recording
    current = [None]
    with tempfile.TemporaryDirectory(dir=HERE) as tmp:
        gen.OUTPUT_DIR = tmp
        for s in STAGES:
            current[0] = s
            gen.STAGES[s]()
        files = sorted(os.listdir(tmp))
        pack(tmp, files, calls, args.max_bytes, read_bin, read_i32s)


def pack(tmp, files, calls, max_bytes, read_bin, read_i32s):
    groups = {
        "decoder_layer": "cpu_dec_", "rms_norm": "cpu_op_rms_norm_",
        "linear": "cpu_op_linear_", "rope": "cpu_op_rope_",
        "self_attention": "cpu_op_sa_", "swiglu": "cpu_swiglu_mlp_",
        "activation": "cpu_op_activation_", "mrope": "cpu_mrope_",
        "vision_rope": ("cpu_vision_rope_", "cpu_vision_freq_table"),
        "vision_attn": "cpu_vision_attn_", "vision_mlp": "cpu_vision_mlp",
        "vision_block": "cpu_vision_block", "patch_embed": "cpu_patch_embed",
        "vision_merger": "cpu_vision_merger_",
    }
    fp16_fixtures = ("decoder_layer", "rope", "self_attention", "swiglu", "vision_attn", "vision_mlp",
                     "vision_block", "patch_embed", "vision_merger")
    manifest = {}
    for fixture, prefixes in groups.items():
        prefixes = prefixes if isinstance(prefixes, tuple) else (prefixes,)
        arrays = {}
        for f in files:
            prefix = next((p for p in prefixes if f.startswith(p)), None)
            if prefix is None or not f.endswith(".bin"):
                continue
            key = f[len("cpu_vision_"):-4] if fixture == "vision_rope" else f[len(prefix):-4]
            key = key.lstrip("_")
            path = os.path.join(tmp, f)
            if fixture == "activation" and "fast_gelu" in key:
                continue
            if key == "meta" or key.endswith("_meta"):
                arrays[key] = read_i32s(path)
                continue
            if fixture in fp16_fixtures:
                a = read_bin(path, "fp16")
            elif fixture == "mrope" and key.startswith("pid"):
                a = read_bin(path, "i64")
            else:
                a = read_bin(path, "f32")
            if a.nbytes > max_bytes:
                manifest[f"{fixture}/{key}"] = dict(
                    shape=list(a.shape), dtype=str(a.dtype), sha256=regen.sha256(a))
                continue
            arrays[key] = a
        if fixture == "mrope":
            for stage, c in calls.items():
                name = stage.replace("mrope_pid_", "rope_index_")
                arrays[f"{name}__input_ids"] = c["input_ids"]
                if c["image_grid_thw"] is not None:
                    arrays[f"{name}__image_grid_thw"] = c["image_grid_thw"]
                if c["attention_mask"] is not None:
                    arrays[f"{name}__attention_mask"] = c["attention_mask"]
                arrays[f"{name}__kw"] = np.array(json.dumps(c["kw"]))
                arrays[f"{name}__position_ids"] = c["position_ids"]
        np.savez_compressed(os.path.join(HERE, f"{fixture}.npz"), **arrays)
        print(f"{fixture}.npz: {len(arrays)} arrays")
    with open(os.path.join(HERE, "manifest.json"), "w") as fh:
        json.dump(manifest, fh, indent=1, sort_keys=True)
    print(f"manifest.json: {len(manifest)} omitted arrays")


if __name__ == "__main__":
    main()
