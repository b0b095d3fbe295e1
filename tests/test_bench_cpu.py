"""bench.py's algorithmic work per step (the numerators of every roofline
fraction it prints) against counts made here from the model shapes, and the
region clock sampler on a machine without a GPU."""

import bench


def _close(a, b, rel=1e-3):
    return abs(a - b) <= rel * abs(b)


def test_mixtral_decode_and_prefill_work():
    H, I, E, L, V, kv = 4096, 14336, 8, 32, 32000, 8
    attn = H * (H + 2 * kv * 128) + H * H  # q | k | v, o
    experts = E * 3 * H * I                  # w1, w3, w2 of every expert (batch 32 x top-2 reaches all 8)
    layer_weights = attn + experts + H * E + 2 * H  # + router + two norms
    kv_bytes = 32 * 4096 * L * 2 * kv * 128 * 2  # batch 32 at context 4096
    want = (L * layer_weights + V * H) * 2 + kv_bytes
    assert _close(bench.MX_DECODE_BYTES, want), (bench.MX_DECODE_BYTES, want)
    assert _close(bench.MX_DECODE_BYTES, 110.3e9)
    assert _close(bench.MX_PREFILL_FLOP, 208.9e12)


def test_deepseek_decode_bytes():
    assert _close(bench.ds_decode_bytes(), 33.84e9)


def test_qwen3vl_request_flops():
    # vision: 24 blocks over 784 patches (qkv, proj, fc1, fc2; QK^T and PV at 16 heads x 64)
    N, D, Iv = 784, 1024, 4096
    vision = 24 * (2 * N * (3 * D * D + D * D + 2 * Iv * D) + 4 * N * N * D)
    # text: 28 layers over 256 tokens (q | k | v, o, gate | up | down; causal attention counted whole)
    S, H, It = 256, 2048, 6144
    text = 28 * (2 * S * (H * (H + 2 * 1024) + H * H + 3 * H * It) + 2 * S * S * H)
    assert bench.VL_VISION_FLOP >= vision and _close(bench.VL_VISION_FLOP, 575.9e9)
    assert _close(bench.VL_TEXT_FLOP, text) and _close(bench.VL_TEXT_FLOP, 729.1e9)


def test_moe_decode_bytes_shrink_with_expert_parallelism():
    one = bench.moe_decode_bytes(bench.MIXTRAL_8X7B, 1, 32, 4096)
    two = bench.moe_decode_bytes(bench.MIXTRAL_8X7B, 2, 32, 4096)
    assert _close(two, 65.2e9, rel=2e-3)
    assert two < one


def test_region_clock_without_gpu_reports_none():
    with bench.RegionClock(0) as c:
        pass
    assert c.median() is None or c.median() > 0
