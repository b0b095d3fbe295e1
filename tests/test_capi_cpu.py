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


def test_newer_entry_points_reject_invalid_params_without_gpu():
    if not os.path.exists(capi.LIB_PATH):
        pytest.skip("library not built")
    L = capi.lib()
    INVALID = -1
    # tcgen05 prefill attention: nq % nkv, unaligned stride (checked before any tensor map is built)
    assert L.b200_flash_prefill_packed(16, 128, 128, 16, 128, 128, 16, 128, 128, 16, 128, 128, 16, 1, 8, 8, 3, 2,
                                       128, 128, 0.1, 1, None) == INVALID
    assert L.b200_flash_prefill_packed(16, 130, 128, 16, 128, 128, 16, 128, 128, 16, 128, 128, 16, 1, 8, 8, 2, 2,
                                       128, 128, 0.1, 1, None) == INVALID
    # expert-parallel exchange without a communicator
    assert L.b200_ep_dispatch(None, 16, 16, 8, 8, 64, 16, 64, 16, 16, None) == INVALID
    assert L.b200_ep_combine(None, 16, 64, 16, 16, 16, 16, 16, 4, 2, 8, 64, None, None, 16, None, None, 1e-6,
                             None) == INVALID
    # image preprocessing: zero-sized image, more than 3 channels, unknown output dtype
    grid = (ctypes.c_int64 * 3)()
    n = ctypes.c_int64()
    assert L.b200_preprocess_image(16, 3, 0, 32, 16, 2, 2, 4096, 1843200, None, None, 1, 16, 1 << 20,
                                   ctypes.byref(n), grid, 16, 1 << 20, None) == INVALID
    assert L.b200_preprocess_image(16, 4, 32, 32, 16, 2, 2, 4096, 1843200, None, None, 1, 16, 1 << 20,
                                   ctypes.byref(n), grid, 16, 1 << 20, None) == INVALID
    assert L.b200_preprocess_image(16, 3, 32, 32, 16, 2, 2, 4096, 1843200, None, None, 5, 16, 1 << 20,
                                   ctypes.byref(n), grid, 16, 1 << 20, None) == INVALID
    assert L.b200_bicubic_resize_u8(None, 3, 8, 8, 4, 4, None, None, 0, None) == INVALID
    assert L.b200_preprocess_workspace_bytes(3, 0, 8, 4, 4) == 0
    # device position ids: missing workspace
    assert L.b200_get_rope_index_device(16, 1, 8, None, None, 0, 1, 2, 2, 16, None, 0, None) == INVALID
    assert L.b200_rope_index_workspace_bytes(100) == 800


def test_gemm_split_plan_for_the_measured_shapes():
    """Host-side split-K plan of the shapes the benchmarks run (split count =
    workspace bytes / (M x N x 4)): decode projections split until their
    128-row weight tiles cover the 148 SMs; the 16384-token prefill GEMM and
    the lm_head (1187 tiles) never split; the few-hundred-token vision / text
    projections split only where their output tiles leave SMs idle."""
    L = capi.lib()
    want = {
        (64, 6144, 4096): 3,      # Qwen3-8B decode qkv: 48 tiles x 3
        (64, 4096, 4096): 4,      # o
        (64, 24576, 4096): 3,     # gate/up: 192 tiles x 3
        (64, 4096, 12288): 4,     # down
        (64, 151936, 4096): 0,    # lm_head
        (16384, 24576, 4096): 0,  # prefill gate/up
        (784, 1024, 1024): 2,     # vision proj
        (784, 1024, 4096): 5,     # vision fc2
        (784, 4096, 1024): 0,     # vision fc1
        (256, 2048, 6144): 9,     # Qwen3-VL text down
    }
    for (M, N, K), splits in want.items():
        assert L.b200_gemm_workspace_bytes(M, N, K, 0) == splits * M * N * 4, (M, N, K)
