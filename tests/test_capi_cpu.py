"""CPU checks of the C-ABI boundary: the library loads without a GPU, exports
every symbol the header declares, and rejects invalid arguments with
B200_ERROR_INVALID_PARAM before touching the device (the reference's
forward-error-path contract, atb_cpp_llm/tests/level4_e2e/test_forward_error_paths.cpp:49-150)."""

import ctypes
import os

import pytest

from atb_llm_study_b200 import capi


def test_header_parses():
    fns = capi.parse_header()
    assert "b200_gemm_bf16" in fns and "b200_paged_decode" in fns
    assert len(fns) >= 15


def test_library_exports_every_declared_symbol():
    if not os.path.exists(capi.LIB_PATH):
        pytest.skip("library not built")
    lib = ctypes.CDLL(capi.LIB_PATH)
    missing = [n for n in capi.parse_header() if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version_and_invalid_params_without_gpu():
    if not os.path.exists(capi.LIB_PATH):
        pytest.skip("library not built")
    L = capi.lib()
    assert L.b200_abi_version() == 100
    INVALID = -1
    # null pointers / bad shapes are rejected on the host, no device call made
    assert L.b200_rmsnorm(None, None, None, None, None, 4, 64, 64, 1e-6, None) == INVALID
    assert L.b200_rmsnorm(16, None, 16, 16, None, 4, 60, 64, 1e-6, None) == INVALID  # dim % 8
    assert L.b200_gemm_bf16(16, 8, 16, 8, 16, 8, 4, 8, 12, 0, None, None, 0, None, 0, None) == INVALID  # K % 8
    assert L.b200_gemm_bf16(16, 64, 16, 64, 16, 64, 4, 64, 64, 9, None, None, 0, None, 0, None) == INVALID
    assert L.b200_gemm_bf16(16, 64, 16, 64, 16, 64, 4, 64, 64, 1, None, None, 0, None, 0, None) == INVALID  # bias missing
    assert L.b200_flash_prefill(16, 64, 16, 16, 64, 16, 64, 16, 1, 8, 3, 2, 64, 0.1, 1, None) == INVALID  # nq % nkv
    assert L.b200_qk_norm_rope(16, 4, 4, 4, 32, 10, None, None, 1e-6, 16, 16, None, None, None, 0, 0, None) == INVALID
    assert L.b200_paged_decode(16, 128, 16, 16, 16, 4, 16, 2, 8, 3, 128, 128, 8, 0.1, 16, 128, None, 0, 64,
                               None) == INVALID
    assert L.b200_embedding(None, 4, 16, 10, 64, 16, None) == INVALID
    assert L.b200_argmax(16, 2, 10, 5, 16, None) == INVALID  # ld < vocab
    assert L.b200_gemm_workspace_bytes(0, 8, 8, 0) == 0


def test_gemm_plan_split_heuristic():
    if not os.path.exists(capi.LIB_PATH):
        pytest.skip("library not built")
    L = capi.lib()
    # decode-shaped projections want split-K workspace on 148 SMs; prefill shapes do not
    assert L.b200_gemm_workspace_bytes(64, 4096, 4096, 0) > 0
    assert L.b200_gemm_workspace_bytes(16384, 6144, 4096, 0) == 0
