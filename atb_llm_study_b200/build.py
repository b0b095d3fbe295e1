"""Build libb200_llm.so in-tree with nvcc for sm_100a.

    python -m atb_llm_study_b200.build [-v] [--force]

Every ``csrc/**/*.cu`` and ``csrc/**/*.cpp`` is compiled to an object under
``_build/`` (rebuilt only when the source or any header is newer) and linked
into ``atb_llm_study_b200/libb200_llm.so``.  No GPU is needed to build.
"""

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT_DIR = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libb200_llm.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          f"-I{os.path.join(ROOT, 'include')}", f"-I{CSRC}"]
CU_FLAGS = ARCH + COMMON + ["--expt-relaxed-constexpr", "-Xptxas", "-warn-spills",
                            "-DB200_BUILD"]
CPP_FLAGS = COMMON + ["-DB200_BUILD"]


def _sources():
    srcs = sorted(glob.glob(os.path.join(CSRC, "**", "*.cu"), recursive=True))
    srcs += sorted(glob.glob(os.path.join(CSRC, "**", "*.cpp"), recursive=True))
    return srcs


def _headers():
    hs = glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True)
    hs += glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True)
    hs += glob.glob(os.path.join(ROOT, "include", "*.h"))
    return hs


def _obj(src):
    rel = os.path.relpath(src, CSRC).replace(os.sep, "__")
    return os.path.join(OUT_DIR, rel + ".o")


def _compile(src, force, verbose):
    obj = _obj(src)
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in _headers()])
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep:
        return obj, None
    flags = CU_FLAGS if src.endswith(".cu") else CPP_FLAGS
    cmd = [NVCC] + flags + ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, f"{' '.join(cmd)}\n{r.stdout}\n{r.stderr}"
    if verbose and (r.stdout.strip() or r.stderr.strip()):
        print(r.stdout, r.stderr, flush=True)
    return obj, None


def build(force=False, verbose=False, jobs=None):
    """Compile and link; returns the path of the shared library."""
    os.makedirs(OUT_DIR, exist_ok=True)
    srcs = _sources()
    jobs = jobs or min(8, os.cpu_count() or 4)
    errors = []
    objs = []
    with cf.ThreadPoolExecutor(jobs) as ex:
        for obj, err in ex.map(lambda s: _compile(s, force, verbose), srcs):
            objs.append(obj)
            if err:
                errors.append(err)
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n\n".join(errors))
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart_static", "-lrt", "-lpthread", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    sys.exit(main())
