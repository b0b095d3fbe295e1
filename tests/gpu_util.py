"""Helpers for the GPU parity tests: device buffers through torch (plumbing
only), calls through the C ABI, comparison metrics."""

import numpy as np
import torch

from atb_llm_study_b200 import capi

DEV = "cuda:0"


def L():
    return capi.lib()


def stream():
    return torch.cuda.current_stream().cuda_stream


# Device tensors made by the helpers below stay referenced here until
# release() (called after every test): a kernel is often handed
# `bf16(x).data_ptr()`, and without this reference the temporary would go back
# to torch's caching allocator — and be reused — before the kernel runs.
_held = []


def _keep(t):
    _held.append(t)
    return t


def release():
    torch.cuda.synchronize()
    _held.clear()


def bf16(a):
    """numpy fp32/fp16 -> bf16 device tensor (round to nearest even)."""
    return _keep(torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32))).to(DEV).to(torch.bfloat16))


def f32(a):
    return _keep(torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32))).to(DEV))


def i64(a):
    return _keep(torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.int64))).to(DEV))


def i32(a):
    return _keep(torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.int32))).to(DEV))


def host(t):
    return t.detach().float().cpu().numpy()


def rounded(a):
    """The bf16 value a kernel actually sees for numpy input a."""
    return host(bf16(a))


def ptr(t):
    return 0 if t is None else t.data_ptr()


def check(rc, what=""):
    capi.check(rc, what)


def device_errors(clear=True):
    import ctypes

    bits = ctypes.c_uint(0)
    check(L().b200_device_error_read(ctypes.addressof(bits), int(clear), stream()), "device_error_read")
    return bits.value


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def max_rel_err(out, ref):
    """max |out - ref| / max |ref| — the layer-level error measure used in the tests."""
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(out - ref)) / (np.max(np.abs(ref)) + 1e-30))


def gemm(A, B, epi=0, bias=None, R=None, out=None, ws=True):
    """C = epi(A @ B^T) through b200_gemm_bf16 (torch bf16 device tensors).
    ws: True = a fresh zeroed split-K workspace, False = none, or a tensor to reuse."""
    M, K = A.shape
    N = B.shape[0]
    outN = N // 2 if epi == 3 else N
    if out is None:
        out = torch.empty(M, outN, dtype=torch.bfloat16, device=DEV)
    if isinstance(ws, torch.Tensor):
        wst, wsb = ws, ws.numel()
    else:
        wsb = L().b200_gemm_workspace_bytes(M, N, K, epi) if ws else 0
        wst = torch.zeros(max(wsb, 16), dtype=torch.uint8, device=DEV) if wsb else None
    check(L().b200_gemm_bf16(A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), out.data_ptr(), out.stride(0),
                             M, N, K, epi, ptr(bias), ptr(R), 0 if R is None else R.stride(0), ptr(wst), wsb,
                             stream()), "gemm")
    return out
