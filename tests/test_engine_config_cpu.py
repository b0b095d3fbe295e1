"""Host-side config resolution and validation of the engine (no GPU): every
architecture the engine runs is accepted with the registry entry it maps to,
and configurations outside what the kernels support are refused with the
reference's status codes (the model registry's exact-match-then-compatibility
lookup, atb_cpp_llm/src/engine/model_registry.cpp:90-121)."""

import ctypes
import json
import os

import pytest

import bench
from atb_llm_study_b200 import capi
from test_gpu_engine import NARROW, WIDE
from test_gpu_engine_mla import DSV2
from test_gpu_engine_moe import MIXTRAL, QWEN3_MOE
from test_gpu_vl_embed import CONFIG as VL_SMALL

pytestmark = pytest.mark.skipif(not os.path.exists(capi.LIB_PATH), reason="library not built")

DEEPSEEK_V2_LITE = dict(DSV2, hidden_size=2048, num_hidden_layers=27, intermediate_size=10944,
                        moe_intermediate_size=1408, n_routed_experts=64, num_experts_per_tok=6, vocab_size=102400)


def check(cfg):
    buf = ctypes.create_string_buffer(64)
    rc = capi.lib().b200_engine_config_check(json.dumps(cfg).encode(), buf, 64)
    return rc, buf.value.decode()


@pytest.mark.parametrize("cfg,kind", [
    (bench.QWEN3_8B, "qwen3"), (bench.QWEN3VL_2B, "qwen3_vl"), (bench.MIXTRAL_8X7B, "mixtral"),
    (DEEPSEEK_V2_LITE, "deepseek_v2"), (NARROW, "qwen3"), (WIDE, "qwen3"), (MIXTRAL, "mixtral"),
    (QWEN3_MOE, "qwen3_moe"), (DSV2, "deepseek_v2"), (VL_SMALL, "qwen3_vl"),
])
def test_supported_configs(cfg, kind):
    assert check(cfg) == (0, kind)


def test_refused_configs():
    assert check(dict(NARROW, model_type="mystery", num_local_experts=8))[0] == -7  # unknown type
    assert check(dict(NARROW, head_dim=96))[0] == -7                                  # GQA heads are 128 wide
    assert check(dict(DSV2, q_lora_rank=1536))[0] == -7                               # query LoRA (full V2)
    assert check(dict(DSV2, num_attention_heads=20))[0] == -7                         # latent heads in groups of 16
    assert check(dict(DSV2, topk_method="group_limited_greedy"))[0] == -7
    assert check(dict(MIXTRAL, num_experts_per_tok=9))[0] == -1
    assert check(dict(NARROW, hidden_size=0))[0] == -1
    assert capi.lib().b200_engine_config_check(b"{not json", None, 0) == -1
