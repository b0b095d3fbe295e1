"""Readers for the reference's golden binary formats.

Format follows ``atb_cpp_llm/tests/python_reference/gen_cpu_reference.py:54-122``:

* tensor files: ``[int64 ndim][int64 shape[ndim]][data]`` with data in
  f32 / i64 / fp16 / bf16 (the dtype is implied by the file's role);
* meta files: ``[int64 count][int32 values[count]]``.
"""

import numpy as np

_DTYPES = {"f32": np.float32, "i64": np.int64, "fp16": np.float16, "bf16": np.uint16}


def read_bin(path, dtype="f32"):
    """Read one ``[ndim][shape][data]`` file (gen_cpu_reference.py:54-100)."""
    raw = open(path, "rb").read()
    ndim = int(np.frombuffer(raw, np.int64, 1, 0)[0])
    shape = tuple(int(v) for v in np.frombuffer(raw, np.int64, ndim, 8))
    data = np.frombuffer(raw, _DTYPES[dtype], offset=8 + 8 * ndim)
    return data.reshape(shape).copy()


def read_i32s(path):
    """Read one ``[count][int32...]`` meta file (gen_cpu_reference.py:116-122)."""
    raw = open(path, "rb").read()
    n = int(np.frombuffer(raw, np.int64, 1, 0)[0])
    return np.frombuffer(raw, np.int32, n, 8).copy()
