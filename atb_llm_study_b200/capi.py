"""ctypes binding of libb200_llm.so, generated from include/b200_llm.h.

Every ``B200_API`` declaration in the header becomes an attribute of
:data:`lib` with matching ``argtypes`` / ``restype``; pointer arguments take
plain integers (``tensor.data_ptr()``), streams take the raw ``cudaStream_t``
(``torch.cuda.current_stream().cuda_stream``).  Loading fails loudly when the
library has not been built: there is no fallback implementation.
"""

import ctypes
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
HEADER = os.path.join(ROOT, "include", "b200_llm.h")
LIB_PATH = os.path.join(PKG, "libb200_llm.so")

STATUS = {
    0: "B200_OK", -1: "B200_ERROR_INVALID_PARAM", -2: "B200_ERROR_FILE_NOT_FOUND",
    -3: "B200_ERROR_WEIGHT_LOAD", -4: "B200_ERROR_GRAPH_BUILD", -5: "B200_ERROR_DEVICE_MEMORY",
    -6: "B200_ERROR_INFERENCE", -7: "B200_ERROR_UNSUPPORTED",
}

_SCALARS = {
    "int": ctypes.c_int, "int32_t": ctypes.c_int32, "int64_t": ctypes.c_int64, "float": ctypes.c_float,
    "double": ctypes.c_double, "unsigned": ctypes.c_uint, "uint64_t": ctypes.c_uint64, "void": None,
    "size_t": ctypes.c_size_t,
}


def _ctype(decl):
    decl = decl.strip()
    words = decl.replace("const ", "").replace("*", " * ").split()
    if "*" in words:
        return ctypes.c_char_p if words[0] == "char" else ctypes.c_void_p
    if words[0].startswith("b200_"):  # opaque handles and the stream type
        return ctypes.c_void_p
    return _SCALARS[words[0]]


def parse_header(path=HEADER):
    """Return {name: (restype, [argtypes])} for every B200_API function."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for m in re.finditer(r"B200_API\s+([\w\s\*]+?)\s*\b(b200_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.S):
        ret, name, args = m.group(1), m.group(2), m.group(3).strip()
        restype = _ctype(ret) if ret.strip() != "void" else None
        argtypes = []
        if args and args != "void":
            for a in args.split(","):
                a = " ".join(a.split())
                # drop the parameter name
                t = re.sub(r"\b\w+$", "", a).strip()
                argtypes.append(_ctype(t))
        out[name] = (restype, argtypes)
    return out


class B200Error(RuntimeError):
    pass


def _load():
    if not os.path.exists(LIB_PATH):
        raise B200Error(f"{LIB_PATH} is not built; run `python -m atb_llm_study_b200.build`")
    lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_LOCAL)
    for name, (res, args) in parse_header().items():
        fn = getattr(lib, name)  # AttributeError = symbol missing from the library
        fn.restype = res
        fn.argtypes = args
    return lib


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def check(rc, what=""):
    """Raise B200Error for a non-zero status code."""
    if rc != 0:
        name = STATUS.get(rc, f"B200_ERROR_CUDA_BASE-{-1000 - rc}" if rc <= -1000 else str(rc))
        raise B200Error(f"{what} failed: {name} ({rc})")
    return rc
