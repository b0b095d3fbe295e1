"""Qwen3-8B bf16 decode & prefill throughput on B200 through the engine's C ABI.

Workload (synthetic, seeded, random-init N(0, 0.02) weights generated on the
device; no checkpoint or dataset):
  * model: hidden 4096, 36 layers, 32 q / 8 kv heads x 128, intermediate
    12288, vocab 151936, QK-norm, rope theta 1e6;
  * prefill: 8 sequences x 2048 tokens per step (token ids U[0, vocab));
    8 such steps fill a 64-slot paged KV cache (block 128);
  * decode (the headline `value`): batch 64, one token per sequence per step,
    every sequence at context 2048 (+ the tokens decoded so far).

`value` = decode tokens/s with inputs resident in HBM (device ids in, device
next tokens out), timed with CUDA events on the engine stream, max over ranks.
`e2e` = the same decode steps through the same C call with host token ids in
and host next tokens out (pinned staging, H2D + D2H inside the timed region).
Multi-GPU: one independent replica per GPU (data parallel, weak scaling).

`--impl reference` times the CPU restatement of the same decode step (numpy
fp32, one layer timed and scaled to 36 layers + lm_head) on the host cores.
"""

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

QWEN3_8B = dict(model_type="qwen3", hidden_size=4096, num_hidden_layers=36, num_attention_heads=32,
                num_key_value_heads=8, head_dim=128, intermediate_size=12288, vocab_size=151936,
                rms_norm_eps=1e-6, rope_theta=1e6, tie_word_embeddings=False)
METRIC = "Qwen3-8B bf16 decode & prefill tok/s at 1/2/4/8 B200; kernel % of roofline"
PREFILL_SEQS, PREFILL_LEN, DECODE_BATCH, DECODE_CTX, BLOCK = 8, 2048, 64, 2048, 128
# DRAM bytes (read + write) of one paged-decode launch at the bench shape, from
# an ncu capture of `bench.py --profile-kernel decode_attention`.
DECODE_ATTN_DRAM_BYTES = 537.43744e6 + 4.910592e6


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p.get("bf16_tflops_sustained", p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "200"], stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 8 and f[1].replace(".", "").isdigit():
                    rows.append(f)
        except Exception:
            pass
        finally:
            if self.path and os.path.exists(self.path):
                os.remove(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = [n for i, n in enumerate(names) if any(r[4 + i].lower().startswith("active") for r in rows)]
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


class RegionClock:
    """Median SM clock over a short timed region: NVML clock reads (read only)
    every 5 ms from a thread; None where NVML is unavailable."""

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.mhz = []
        self.stop = None
        self.thread = None

    def __enter__(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
        except Exception:
            return self
        self.stop = threading.Event()

        def run():
            while not self.stop.is_set():
                try:
                    self.mhz.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                except Exception:
                    return
                time.sleep(0.005)

        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *a):
        if self.thread:
            self.stop.set()
            self.thread.join(1.0)

    def median(self):
        return statistics.median(self.mhz) if self.mhz else None


# --------------------------------------------------------------------- CPU leg

def cpu_decode_layer_setup():
    """One Qwen3-8B decode layer (batch 64, context 2048) of the numpy oracle with
    its inputs built once: returns (layer, head) callables; head runs 1/8 of the
    lm_head rows (its time scales x8)."""
    import numpy as np

    import oracle

    c = QWEN3_8B
    H, nq, nkv, hd, I = c["hidden_size"], c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"], c[
        "intermediate_size"]
    rng = np.random.default_rng(0)
    B, ctx = DECODE_BATCH, DECODE_CTX
    f = np.float32
    w = {
        "q_w": rng.standard_normal((nq * hd, H), f) * 0.02, "k_w": rng.standard_normal((nkv * hd, H), f) * 0.02,
        "v_w": rng.standard_normal((nkv * hd, H), f) * 0.02, "o_w": rng.standard_normal((H, nq * hd), f) * 0.02,
        "gate_w": rng.standard_normal((I, H), f) * 0.02, "up_w": rng.standard_normal((I, H), f) * 0.02,
        "down_w": rng.standard_normal((H, I), f) * 0.02, "qn_w": np.ones(hd, f), "kn_w": np.ones(hd, f),
        "iln_w": np.ones(H, f), "pln_w": np.ones(H, f),
    }
    nblk = ctx // BLOCK + 1
    kc = rng.standard_normal((B * nblk, nkv, BLOCK, hd), f)
    vc = rng.standard_normal((B * nblk, nkv, BLOCK, hd), f)
    tables = np.arange(B * nblk).reshape(B, nblk)
    x = rng.standard_normal((B, H), f)
    cos, sin = oracle.rope1d_cos_sin(np.full(B, ctx), hd, c["rope_theta"])
    lm = rng.standard_normal((c["vocab_size"] // 8, H), f) * 0.02  # 1/8 of lm_head, scaled x8

    def layer():
        n = oracle.rms_norm(x, w["iln_w"], 1e-6)
        q = oracle.rms_norm(oracle.linear(n, w["q_w"]).reshape(B, nq, hd), w["qn_w"], 1e-6)
        k = oracle.rms_norm(oracle.linear(n, w["k_w"]).reshape(B, nkv, hd), w["kn_w"], 1e-6)
        v = oracle.linear(n, w["v_w"]).reshape(B, nkv, hd)
        q, k = oracle.rope_half(q, cos, sin), oracle.rope_half(k, cos, sin)
        slots = oracle.slot_mapping(tables[0], np.array([ctx]), BLOCK)  # representative cache write
        oracle.kv_cache_write(kc, k[:1], slots)
        oracle.kv_cache_write(vc, v[:1], slots)
        a = oracle.paged_decode_attention(q, kc, vc, tables, np.full(B, ctx + 1))
        h = x + oracle.linear(a.reshape(B, -1), w["o_w"])
        return h + oracle.swiglu_mlp(oracle.rms_norm(h, w["pln_w"], 1e-6), w["gate_w"], w["up_w"], w["down_w"])

    def head():
        return oracle.linear(x, lm)

    return layer, head


def cpu_decode_layer_seconds(threads_note):
    """Time one decode layer (batch 64, context 2048) of the numpy oracle."""
    layer, head = cpu_decode_layer_setup()
    layer()  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        layer()
        reps += 1
        if time.perf_counter() - t0 > 4.0 or reps >= 5:
            break
    t_layer = (time.perf_counter() - t0) / reps
    t0 = time.perf_counter()
    head()
    t_head = (time.perf_counter() - t0) * 8
    return t_layer, t_head, reps


def blas_threads():
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return max(n)
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_baseline():
    t_layer, t_head, reps = cpu_decode_layer_seconds(None)
    step = 36 * t_layer + t_head
    return {"value": DECODE_BATCH / step, "unit": "tok/s", "cores": blas_threads(), "kind": "port",
            "sample": f"numpy fp32 oracle: one decode layer (batch 64, context 2048) timed x{reps}, "
                      f"scaled to 36 layers + lm_head (extrapolated); {t_layer * 1e3:.1f} ms/layer"}


# --------------------------------------------------------------------- GPU leg

class EngineConfig(ctypes.Structure):
    _fields_ = [("model_dir", ctypes.c_char_p), ("config_json", ctypes.c_char_p), ("device_id", ctypes.c_int),
                ("max_batch", ctypes.c_int), ("max_context", ctypes.c_int), ("max_prefill_tokens", ctypes.c_int),
                ("kv_block_size", ctypes.c_int), ("init_seed", ctypes.c_uint64), ("init_std", ctypes.c_float)]


def check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what} failed with status {rc}")


def kernel_roofline_decode_attention(L, torch, dev, reps=20):
    """Paged decode attention alone at the decode shape (B 64, ctx 2048, 32/8 heads):
    algorithmic bytes = K + V of every context token = 64*2048*8*128*2*2 B."""
    B, nq, nkv, hd, ctx = DECODE_BATCH, 32, 8, 128, DECODE_CTX
    nblk_seq = (ctx + BLOCK - 1) // BLOCK
    nblk = B * nblk_seq
    g = torch.Generator(device=dev).manual_seed(0)
    kc = (torch.randn(nblk, nkv, BLOCK, hd, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    vc = (torch.randn(nblk, nkv, BLOCK, hd, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    tables = torch.randperm(nblk, device=dev, generator=g).to(torch.int32).reshape(B, nblk_seq)
    ctxl = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    q = torch.randn(B, nq * hd, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty_like(q)
    wsb = L.b200_paged_decode_workspace_bytes(B, nq, hd, ctx)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev)

    def run():
        check(L.b200_paged_decode(q.data_ptr(), nq * hd, kc.data_ptr(), vc.data_ptr(), tables.data_ptr(), nblk_seq,
                                  ctxl.data_ptr(), B, nq, nkv, hd, BLOCK, nblk, hd ** -0.5, out.data_ptr(), nq * hd,
                                  ws.data_ptr(), wsb, ctx, st.cuda_stream), "paged_decode")

    for _ in range(3):
        run()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(st)
    for _ in range(reps):
        run()
    e1.record(st)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps
    algo = B * ctx * nkv * hd * 2 * 2
    del kc, vc
    return ms, algo


def _time_launches(torch, dev, run, reps):
    st = torch.cuda.current_stream(dev)
    for _ in range(3):
        run(st)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(st)
    for _ in range(reps):
        run(st)
    e1.record(st)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / reps


def kernel_roofline_mla_decode(L, torch, dev, reps=20):
    """Absorbed-latent decode attention alone at the DeepSeek-V2-Lite decode
    shape (batch 32, 16 heads, context 4096, block 128): algorithmic bytes =
    the latent rows of every context token = 32*4096*576*2 B (+ q and out)."""
    B, nh, ctx, blk = DS_BATCH, 16, DS_CTX, BLOCK
    nbs = ctx // blk
    nblk = B * nbs
    g = torch.Generator(device=dev).manual_seed(3)
    cache = (torch.randn(nblk * blk, 576, device=dev, generator=g)).to(torch.bfloat16)
    tables = torch.randperm(nblk, device=dev, generator=g).to(torch.int32).reshape(B, nbs)
    ctxl = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    q = (torch.randn(B, nh * 576, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    out = torch.empty(B, nh * 512, dtype=torch.bfloat16, device=dev)
    wsb = L.b200_mla_decode_workspace_bytes(B, nh, ctx)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)

    def run(st):
        check(L.b200_mla_decode(q.data_ptr(), nh * 576, cache.data_ptr(), tables.data_ptr(), nbs, ctxl.data_ptr(), B,
                                nh, blk, nblk, 0.1, out.data_ptr(), nh * 512, ws.data_ptr(), wsb, ctx, st.cuda_stream),
              "mla_decode")

    ms = _time_launches(torch, dev, run, reps)
    del cache
    return ms, B * ctx * 576 * 2 + B * nh * (576 + 512) * 2


def kernel_roofline_moe_gemm(L, torch, dev, reps=10):
    """Grouped expert gate/up GEMM (SwiGLU epilogue) at the Mixtral-8x7B decode
    shape: 64 (token, expert) rows over 8 experts of [2 x 14336, 4096]:
    algorithmic bytes = every expert's weights = 8*28672*4096*2 B (+ tokens)."""
    import numpy as np

    E, N, K, rows = 8, 2 * 14336, 4096, 64
    g = torch.Generator(device=dev).manual_seed(4)
    W = (torch.randn(E * N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    A = torch.randn(rows, K, device=dev, generator=g).to(torch.bfloat16)
    C = torch.empty(rows, N // 2, dtype=torch.bfloat16, device=dev)
    off = torch.from_numpy(np.arange(0, rows + 1, rows // E, dtype=np.int32)).to(dev)

    def run(st):
        check(L.b200_grouped_gemm_bf16(A.data_ptr(), K, W.data_ptr(), K, C.data_ptr(), N // 2, off.data_ptr(), E, rows,
                                       N, K, 3, st.cuda_stream), "grouped_gemm")

    ms = _time_launches(torch, dev, run, reps)
    del W
    return ms, E * N * K * 2 + rows * K * 2 + rows * N // 2 * 2


def kernel_roofline_image_preprocess(L, torch, dev, reps=20):
    """Image preprocessing of the bench_preprocess frame (seeded 3x1080x1920
    uint8, resident on the device) into fp16 pixel values: the coefficient
    kernel + preprocess_fused_kernel per image.  Algorithmic bytes = the uint8
    frame read + the fp16 pixel values written."""
    import numpy as np

    C = 3
    img = np.random.default_rng(11).integers(0, 256, (C, PP_H, PP_W), dtype=np.uint8)
    nh, nw = ctypes.c_int(), ctypes.c_int()
    check(L.b200_smart_resize(PP_H, PP_W, 32, 4096, 1843200, ctypes.byref(nh), ctypes.byref(nw)), "smart_resize")
    n = (nh.value // 16) * (nw.value // 16)
    pv = torch.empty(n, C * 2 * 16 * 16, dtype=torch.float16, device=dev)
    wsb = L.b200_preprocess_workspace_bytes(C, PP_H, PP_W, nh.value, nw.value)
    ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device=dev)
    src = torch.from_numpy(img).to(dev)
    npatch = ctypes.c_int64()
    grid = (ctypes.c_int64 * 3)()

    def run(st):
        check(L.b200_preprocess_image(src.data_ptr(), C, PP_H, PP_W, 16, 2, 2, 4096, 1843200, None, None, 1,
                                      pv.data_ptr(), pv.numel(), ctypes.byref(npatch), grid, ws.data_ptr(), wsb,
                                      st.cuda_stream), "preprocess_image")

    ms = _time_launches(torch, dev, run, reps)
    return ms, img.nbytes + pv.numel() * 2


def kernel_roofline_prefill_attention(L, torch, dev, reps=10):
    """tcgen05 causal prefill attention alone at the Qwen3-8B prefill shape (8
    sequences x 2048, 32 query / 8 kv heads of 128, the engine's packed q|k|v
    rows): 2*S^2*d*nq flops per sequence (the causal half of QK^T and PV)."""
    import numpy as np

    S, B, nq, nkv, hd = PREFILL_LEN, PREFILL_SEQS, 32, 8, 128
    T, W = S * B, (nq + 2 * nkv) * hd
    g = torch.Generator(device=dev).manual_seed(5)
    d = torch.randn(T, W, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(T, nq * hd, dtype=torch.bfloat16, device=dev)
    cu = torch.from_numpy(np.arange(0, T + 1, S, dtype=np.int32)).to(dev)

    def run(st):
        check(L.b200_flash_prefill_packed(d.data_ptr(), W, hd, d.data_ptr() + nq * hd * 2, W, hd,
                                          d.data_ptr() + (nq + nkv) * hd * 2, W, hd, out.data_ptr(), nq * hd, hd,
                                          cu.data_ptr(), B, S, T, nq, nkv, hd, hd, 1.0 / hd ** 0.5, 1, st.cuda_stream),
              "flash_prefill_packed")

    ms = _time_launches(torch, dev, run, reps)
    del d, out
    return ms, 2.0 * S * S * hd * nq * B


def kernel_roofline_prefill_gemm(L, torch, dev, reps=10):
    """gate/up projection with the fused SwiGLU epilogue at the prefill shape
    (M 16384, N 2 x 12288, K 4096): 2*M*N*K flops per launch."""
    M, N, K = PREFILL_SEQS * PREFILL_LEN, 2 * 12288, 4096
    g = torch.Generator(device=dev).manual_seed(1)
    A = (torch.randn(M, K, device=dev, generator=g)).to(torch.bfloat16)
    B = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    C = torch.empty(M, N // 2, dtype=torch.bfloat16, device=dev)
    st = torch.cuda.current_stream(dev)

    def run():
        check(L.b200_gemm_bf16(A.data_ptr(), K, B.data_ptr(), K, C.data_ptr(), N // 2, M, N, K, 3, None, None, 0,
                               None, 0, st.cuda_stream), "gemm")

    for _ in range(3):
        run()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(st)
    for _ in range(reps):
        run()
    e1.record(st)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps
    del A, B, C
    return ms, 2.0 * M * N * K


def kernel_roofline_decode_gemm(L, torch, dev, reps=20):
    """The Qwen3-8B decode gate/up projection on its own: M 64 tokens, N 2 x
    12288, K 4096, swapped split-K tcgen05 GEMM + the SwiGLU reduce, one of 36
    weight copies per launch (every launch streams from HBM, 7.2 GB > L2):
    algorithmic bytes = the 201 MB of weights."""
    M, N, K, copies = DECODE_BATCH, 2 * 12288, 4096, 36
    g = torch.Generator(device=dev).manual_seed(4)
    W = torch.empty(copies, N, K, dtype=torch.bfloat16, device=dev).normal_(0, 0.02, generator=g)
    A = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    C = torch.empty(M, N // 2, dtype=torch.bfloat16, device=dev)
    wsb = L.b200_gemm_workspace_bytes(M, N, K, 3)
    ws = torch.zeros(max(wsb, 16), dtype=torch.uint8, device=dev)
    i = [0]

    def run(st):
        check(L.b200_gemm_bf16(A.data_ptr(), K, W[i[0] % copies].data_ptr(), K, C.data_ptr(), N // 2, M, N, K, 3,
                               None, None, 0, ws.data_ptr(), wsb, st.cuda_stream), "decode gemm")
        i[0] += 1

    ms = _time_launches(torch, dev, run, reps)
    del W
    return ms, N * K * 2


def bandwidth_kernels(L, torch, dev, reps=20):
    """Achieved HBM GB/s of the bandwidth-bound ops on their own, at the shapes
    the benchmarked models run them, inputs larger than L2 where the shape has
    that much data: bytes = every byte the op must read and write once."""
    import numpy as np

    hbm, _, _, src = peaks()
    g = torch.Generator(device=dev).manual_seed(5)
    out = {}

    def line(name, shape, nbytes, run):
        ms = _time_launches(torch, dev, run, reps)
        out[name] = {"shape": shape, "ms": ms, "bytes": nbytes, "GBps": nbytes / (ms / 1e3) / 1e9,
                     "frac": nbytes / (ms / 1e3) / 1e9 / hbm, "peak_source": f"{src} copy bandwidth"}

    # RMSNorm at the Qwen3-8B prefill shape: read x, write out
    T, H = PREFILL_SEQS * PREFILL_LEN, 4096
    x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    w = torch.ones(H, dtype=torch.bfloat16, device=dev)
    y = torch.empty_like(x)
    line("rmsnorm", f"{T}x{H}", 2 * T * H * 2,
         lambda s: check(L.b200_rmsnorm(x.data_ptr(), None, w.data_ptr(), y.data_ptr(), None, T, H, H, 1e-6,
                                        s.cuda_stream), "rmsnorm"))
    # QK RMSNorm + rope in place on q|k|v rows + the paged K/V write, Qwen3-8B prefill shape
    nq, nkv, hd = 32, 8, 128
    W = (nq + 2 * nkv) * hd
    qkv = torch.randn(T, W, device=dev, generator=g).to(torch.bfloat16)
    cos = torch.rand(T, hd, device=dev, generator=g)
    sin = torch.rand(T, hd, device=dev, generator=g)
    nblk = T // BLOCK
    kc = torch.empty(nblk, nkv, BLOCK, hd, dtype=torch.bfloat16, device=dev)
    vc = torch.empty_like(kc)
    slots = torch.arange(T, dtype=torch.int64, device=dev)
    nw = torch.ones(hd, dtype=torch.bfloat16, device=dev)
    line("qk_norm_rope_kv_write", f"{T}x(32+8+8)x128",
         T * W * 2 + T * (nq + nkv) * hd * 2 + T * 2 * nkv * hd * 2 + 2 * T * hd * 4,
         lambda s: check(L.b200_qk_norm_rope(qkv.data_ptr(), T, nq, nkv, hd, W, nw.data_ptr(), nw.data_ptr(), 1e-6,
                                             cos.data_ptr(), sin.data_ptr(), slots.data_ptr(), kc.data_ptr(),
                                             vc.data_ptr(), nblk, BLOCK, s.cuda_stream), "qk_norm_rope"))
    del qkv, kc, vc, cos, sin
    # MoE combine at the Mixtral prefill shape (8 x 1024 tokens, top-2), with residual and the next RMSNorm
    Tm, k = MX_PREFILL_SEQS * MX_PREFILL_LEN, 2
    yp = torch.randn(Tm * k, H, device=dev, generator=g).to(torch.bfloat16)
    pos = torch.randperm(Tm * k, device=dev, generator=g).to(torch.int32)
    tw = torch.rand(Tm, k, device=dev, generator=g)
    res = torch.randn(Tm, H, device=dev, generator=g).to(torch.bfloat16)
    o = torch.empty_like(res)
    nrm = torch.empty_like(res)
    line("moe_combine_residual_rmsnorm", f"{Tm}x{k}x{H}", (Tm * k * H + 3 * Tm * H) * 2 + Tm * k * 8,
         lambda s: check(L.b200_moe_combine(yp.data_ptr(), pos.data_ptr(), tw.data_ptr(), Tm, k, H, res.data_ptr(),
                                            None, o.data_ptr(), w.data_ptr(), nrm.data_ptr(), 1e-6, s.cuda_stream),
                         "moe_combine"))
    del yp, res, o, nrm
    # bilinear position-embedding interpolation of the Qwen3-VL vision tower (48x48 table -> 28x28 grid)
    table = torch.randn(2304, 1024, device=dev, generator=g).to(torch.bfloat16)
    pe = torch.empty(784, 1024, dtype=torch.bfloat16, device=dev)
    grid = np.array([[1, 28, 28]], np.int64)
    line("pos_embed_interp", "2304x1024 -> 784x1024", 784 * 1024 * 2 * (4 + 1),
         lambda s: check(L.b200_pos_embed_interp(table.data_ptr(), 48, 1024, grid.ctypes.data, 1, 2, pe.data_ptr(),
                                                 0, s.cuda_stream), "pos_embed_interp"))
    # the Qwen3-8B decode gate/up projection (swapped split-K tcgen05 GEMM + SwiGLU reduce)
    ms, nbytes = kernel_roofline_decode_gemm(L, torch, dev, reps)
    out["decode_gate_up_gemm"] = {"shape": "M64 N24576 K4096 (+ SwiGLU reduce)", "ms": ms, "bytes": nbytes,
                                  "GBps": nbytes / (ms / 1e3) / 1e9, "frac": nbytes / (ms / 1e3) / 1e9 / hbm,
                                  "peak_source": f"{src} copy bandwidth"}
    return out


QWEN3VL_2B = dict(
    model_type="qwen3_vl", image_token_id=151655, vision_start_token_id=151652, tie_word_embeddings=True,
    text_config=dict(hidden_size=2048, num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8,
                     head_dim=128, intermediate_size=6144, vocab_size=151936, rms_norm_eps=1e-6, rope_theta=5e6,
                     rope_scaling=dict(mrope_section=[24, 20, 20], mrope_interleaved=True)),
    vision_config=dict(depth=24, hidden_size=1024, num_heads=16, intermediate_size=4096, patch_size=16,
                       temporal_patch_size=2, in_channels=3, spatial_merge_size=2, out_hidden_size=2048,
                       num_position_embeddings=2304, deepstack_visual_indexes=[5, 11, 17]))
VL_GRID, VL_SEQ = (1, 28, 28), 256
# algorithmic work of one request (2*params*tokens per linear + 2*2*S^2*hidden per attention):
# vision: 24 blocks (qkv, proj, fc1, fc2 over 784 tokens + bidirectional attention over 784) +
# patch embed + main merger + 3 deepstack mergers over 196 merged tokens;
# text: 28 layers over 256 tokens with causal attention counted as half of S^2.
VL_VISION_FLOP = (24 * (2 * 784 * (3 * 1024 * 1024 + 1024 * 1024 + 2 * 4096 * 1024) + 4 * 784 * 784 * 1024)
                  + 2 * 784 * 1536 * 1024 + 4 * 2 * 196 * (4096 * 4096 + 2048 * 4096))
VL_TEXT_FLOP = 28 * (2 * 256 * (2048 * (2048 + 2 * 1024) + 2048 * 2048 + 3 * 2048 * 6144) + 2 * 256 * 256 * 2048)


def bench_qwen3vl_text_layer(L, torch, dev, reps=20, cpu=True):
    """One Qwen3-VL-2B text decoder layer, S = 256 prefill (hidden 2048, 16 q / 8
    kv heads x 128, SwiGLU 6144, QK-norm, interleaved mrope [24, 20, 20] theta
    5e6 at t = h = w = arange(256), causal; weights N(0, 0.02), activations
    N(0, 1)), through the layer-graph seam b200_text_decoder_layer, CUDA events;
    the same layer on the host cores with the numpy fp32 oracle (median of 5
    after a warm-up).  Algorithmic work: 26.04 GFLOP, 100.7 MB of weights."""
    import numpy as np

    import oracle

    S, H, nq, nkv, hd, I = 256, 2048, 16, 8, 128, 6144
    rng = np.random.default_rng(0)
    f = np.float32
    w = {"q_w": rng.standard_normal((nq * hd, H), f) * 0.02, "k_w": rng.standard_normal((nkv * hd, H), f) * 0.02,
         "v_w": rng.standard_normal((nkv * hd, H), f) * 0.02, "o_w": rng.standard_normal((H, nq * hd), f) * 0.02,
         "qn_w": np.ones(hd, f), "kn_w": np.ones(hd, f), "gate_w": rng.standard_normal((I, H), f) * 0.02,
         "up_w": rng.standard_normal((I, H), f) * 0.02, "down_w": rng.standard_normal((H, I), f) * 0.02,
         "iln_w": np.ones(H, f), "pln_w": np.ones(H, f)}
    x = np.random.default_rng(1).standard_normal((S, H), f)
    pos = np.arange(S)
    cos, sin = oracle.mrope_cos_sin(np.stack([pos, pos, pos])[:, None, :], hd, 5e6, (24, 20, 20))
    cos, sin = cos[0], sin[0]
    order = ["q_w", "k_w", "v_w", "o_w", "qn_w", "kn_w", "gate_w", "up_w", "down_w", "iln_w", "pln_w"]
    dw = {k: torch.from_numpy(w[k]).to(dev).to(torch.bfloat16) for k in order}
    xd = torch.from_numpy(x).to(dev).to(torch.bfloat16)
    cd, sd = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    out = torch.empty_like(xd)
    seqlen = np.array([S], np.int32)
    ptrs = [xd.data_ptr()] + [dw[k].data_ptr() for k in order] + [cd.data_ptr(), sd.data_ptr(), seqlen.ctypes.data]
    pack = (ctypes.c_void_p * len(ptrs))(*ptrs)
    wsb = L.b200_text_decoder_layer_workspace_bytes(S, H, nq, nkv, hd, I)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)

    def run(st):
        check(L.b200_text_decoder_layer(ctypes.addressof(pack), len(ptrs), out.data_ptr(), S, 1, H, nq, nkv, hd, I,
                                        1e-6, 1, 0, ws.data_ptr(), wsb, st.cuda_stream), "text_decoder_layer")

    ms = _time_launches(torch, dev, run, reps)
    flop, wbytes = 26.04e9, 100.7e6
    hbm, tf_burst, _, src = peaks()
    res = {"workload": "Qwen3-VL-2B text decoder layer, S=256 prefill (the reference's CPU golden layer config), "
                       "through b200_text_decoder_layer",
           "gpu_ms": ms, "tensor_frac": flop / (ms / 1e3) / 1e12 / tf_burst,
           "hbm_frac": wbytes / (ms / 1e3) / 1e9 / hbm, "peak_source": f"{src} bf16 burst / copy"}
    if cpu:
        layer = lambda: oracle.decoder_layer(x, w, cos, sin, nq, nkv, hd, 1e-6, causal=True)
        layer()
        ts = []
        for _ in range(5):
            t0 = time.perf_counter()
            layer()
            ts.append(time.perf_counter() - t0)
        cms = statistics.median(ts) * 1e3
        res["cpu_baseline"] = {"value": cms, "unit": "ms/layer", "cores": blas_threads(), "kind": "port",
                               "sample": "numpy fp32 oracle decoder layer, S=256, median of 5 after a warm-up"}
        res["speedup_vs_cpu"] = cms / ms
    return res


def bench_qwen3vl(L, torch, dev, steps, warm, stream_of):
    """Qwen3-VL-2B embedding request: 448x448 image (grid 1x28x28 = 784 patches,
    196 merged tokens) inside a 256-token prompt; vision tower alone, then the
    whole embedding forward (vision -> deepstack -> 28 text layers -> pooling)."""
    import numpy as np

    cfg = EngineConfig(None, json.dumps(QWEN3VL_2B).encode(), dev.index, 1, 1024, 1024, BLOCK, 99, 0.02)
    eng = ctypes.c_void_p()
    check(L.b200_engine_create(ctypes.byref(cfg), ctypes.byref(eng)), "engine_create qwen3vl")
    est = stream_of(eng)
    try:
        t, h, w = VL_GRID
        N = t * h * w
        rng = np.random.default_rng(5)
        px_host = rng.uniform(-1, 1, (N, 1536)).astype(np.float32)
        px_dev = torch.from_numpy(px_host).to(dev).to(torch.bfloat16)
        grid = np.array([VL_GRID], np.int64)
        n_img = N // 4
        tail = VL_SEQ - n_img - 31
        ids = np.concatenate([rng.integers(0, 151000, 30), [151652], np.full(n_img, 151655),
                              rng.integers(0, 151000, tail)]).astype(np.int64)
        emb = np.zeros(2048, np.float32)

        def q(k):
            v = ctypes.c_int64()
            check(L.b200_engine_query(eng, k, ctypes.byref(v)), "query")
            return v.value

        def vision(_):
            check(L.b200_engine_vision(eng, px_dev.data_ptr(), 0, 1, N, grid.ctypes.data, 1, None, None, None),
                  "vision")

        def embed_dev(_):
            check(L.b200_engine_embed(eng, ids.ctypes.data, VL_SEQ, None, px_dev.data_ptr(), 0, 1, N,
                                      grid.ctypes.data, 1, 1, emb.ctypes.data, None), "embed")

        def embed_host(_):
            check(L.b200_engine_embed(eng, ids.ctypes.data, VL_SEQ, None, px_host.ctypes.data, 2, 0, N,
                                      grid.ctypes.data, 1, 1, emb.ctypes.data, None), "embed")

        def timed(fn, n):
            for i in range(warm):
                fn(i)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(est)
            for i in range(n):
                fn(i)
            e1.record(est)
            torch.cuda.synchronize(dev)
            return e0.elapsed_time(e1) / n

        vis_ms = timed(vision, steps)
        vis_launches = q(9)
        emb_ms = timed(embed_dev, steps)
        enc_launches = q(10)
        e2e_ms = timed(embed_host, steps)
        assert abs(float(np.linalg.norm(emb)) - 1.0) < 1e-2
        _, tf_burst, _, src = peaks()
        flop = VL_VISION_FLOP + VL_TEXT_FLOP
        return {
            "workload": "Qwen3-VL-2B embedding: 448x448 image (784 patches -> 196 tokens) in a 256-token prompt",
            "vision_ms": vis_ms, "vision_tflops": VL_VISION_FLOP / (vis_ms / 1e3) / 1e12,
            "vision_frac": VL_VISION_FLOP / (vis_ms / 1e3) / 1e12 / tf_burst,
            "embed_ms": emb_ms, "embed_tflops": flop / (emb_ms / 1e3) / 1e12,
            "embed_frac": flop / (emb_ms / 1e3) / 1e12 / tf_burst,
            "requests_per_s": 1e3 / emb_ms, "e2e_ms": e2e_ms, "e2e_requests_per_s": 1e3 / e2e_ms,
            "flop_per_request": flop, "peak_source": f"{src} bf16 burst",
            "launches": {"vision": vis_launches, "text": enc_launches},
        }
    finally:
        L.b200_engine_destroy(eng)


PP_H, PP_W = 1080, 1920  # a 1080p RGB frame, resized to 992 x 1792 (3472 patches)


def bench_preprocess(L, torch, dev, steps, warm, cpu_baseline=True):
    """Qwen3-VL image preprocessing of one 1080x1920 RGB frame on the GPU
    (SmartResize to 992x1792, Pillow-exact bicubic, normalise, patchify into
    fp16 pixel values [3472, 1536]).  value: image resident in HBM; e2e: the
    uint8 frame copied from pinned host memory every step (the pixel values
    stay on the device for the vision tower).  Algorithmic bytes = the uint8
    frame read + the fp16 pixel values written.  cpu_baseline: the oracle
    port of the reference's CPU PreprocessImage on the same frame."""
    import numpy as np

    C = 3
    rng = np.random.default_rng(11)
    img = rng.integers(0, 256, (C, PP_H, PP_W), dtype=np.uint8)
    nh, nw = ctypes.c_int(), ctypes.c_int()
    check(L.b200_smart_resize(PP_H, PP_W, 32, 4096, 1843200, ctypes.byref(nh), ctypes.byref(nw)), "smart_resize")
    n = (nh.value // 16) * (nw.value // 16)
    pdim = C * 2 * 16 * 16
    pv = torch.empty(n, pdim, dtype=torch.float16, device=dev)
    wsb = L.b200_preprocess_workspace_bytes(C, PP_H, PP_W, nh.value, nw.value)
    ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device=dev)
    img_dev = torch.from_numpy(img).to(dev)
    img_pinned = torch.from_numpy(img).pin_memory()
    npatch = ctypes.c_int64()
    grid = (ctypes.c_int64 * 3)()

    def run(src):
        check(L.b200_preprocess_image(src.data_ptr(), C, PP_H, PP_W, 16, 2, 2, 4096, 1843200, None, None, 1,
                                      pv.data_ptr(), pv.numel(), ctypes.byref(npatch), grid, ws.data_ptr(), wsb,
                                      torch.cuda.current_stream(dev).cuda_stream), "preprocess_image")

    staging = torch.empty_like(img_dev)

    def e2e_step():
        staging.copy_(img_pinned, non_blocking=True)
        run(staging)

    def timed(fn, reps):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / reps

    reps = max(20, steps)
    ms = timed(lambda: run(img_dev), reps)
    e2e_ms = timed(e2e_step, reps)
    nbytes = img.nbytes + n * pdim * 2
    hbm, _, _, src = peaks()
    out = {"workload": f"Qwen3-VL image preprocessing: {C}x{PP_H}x{PP_W} uint8 -> {nh.value}x{nw.value} "
                       f"-> fp16 pixel values [{n}, {pdim}]",
           "images_per_s": 1e3 / ms, "ms_per_image": ms, "e2e_images_per_s": 1e3 / e2e_ms,
           "e2e_h2d_bytes": img.nbytes, "gpu_launches_per_image": 2,
           "roofline": {"bound": "hbm", "bytes_per_image": nbytes, "achieved": nbytes / (ms / 1e3) / 1e9,
                        "peak": hbm, "unit": "GB/s", "frac": nbytes / (ms / 1e3) / 1e9 / hbm,
                        "peak_source": f"{src} copy"}}
    if cpu_baseline:
        import time

        from oracle.preprocess import preprocess_image

        t0 = time.perf_counter()
        preprocess_image(img)
        cpu_s = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": 1.0 / cpu_s, "unit": "images/s", "cores": 1, "kind": "port",
                               "sample": "one 1080x1920 frame through the numpy port of the reference's "
                                         "CPU PreprocessImage"}
    del pv, ws, img_dev, staging
    return out


MIXTRAL_8X7B = dict(model_type="mixtral", hidden_size=4096, num_hidden_layers=32, num_attention_heads=32,
                    num_key_value_heads=8, intermediate_size=14336, num_local_experts=8, num_experts_per_tok=2,
                    vocab_size=32000, rms_norm_eps=1e-5, rope_theta=1e6, tie_word_embeddings=False)
MX_PREFILL_SEQS, MX_PREFILL_LEN, MX_BATCH, MX_CTX = 8, 1024, 32, 4096
# per layer: attention 4096*(4096+2*1024+4096) + 8 experts * 3 * 4096*14336 (+ router 8*4096)
MX_LAYER_PARAMS = 4096 * (4096 + 2 * 1024 + 4096) + 8 * 3 * 4096 * 14336 + 8 * 4096
MX_ACTIVE_LAYER_PARAMS = 4096 * (4096 + 2 * 1024 + 4096) + 2 * 3 * 4096 * 14336 + 8 * 4096
# one decode step reads every expert (P(an expert idle over 64 choices) ~ 1e-4), lm_head and the KV of 32 x 4096 tokens
MX_DECODE_BYTES = (32 * MX_LAYER_PARAMS + 32000 * 4096) * 2 + MX_BATCH * MX_CTX * 32 * 2 * 8 * 128 * 2
MX_PREFILL_FLOP = (2 * 32 * MX_ACTIVE_LAYER_PARAMS * MX_PREFILL_SEQS * MX_PREFILL_LEN
                   + 32 * MX_PREFILL_SEQS * 2 * MX_PREFILL_LEN ** 2 * 4096 + 2 * 32000 * 4096 * MX_PREFILL_SEQS)


def _cpu_time(fn, budget_s=6.0, max_reps=3):
    fn()  # warm
    t0, reps = time.perf_counter(), 0
    while True:
        fn()
        reps += 1
        if time.perf_counter() - t0 > budget_s or reps >= max_reps:
            break
    return (time.perf_counter() - t0) / reps, reps


def cpu_moe_decode_baseline(model):
    """The numpy fp32 oracle's decode step for the MoE sections, timed on the
    host cores at the section's shape and scaled to the model's layers (an
    extrapolation, like the headline's): one MoE decode layer (attention over
    the batch's contexts + the routed experts it reaches) x layers + 1/8 of
    lm_head x 8.  Bounded sample: the experts share a few distinct weight
    arrays (each one is read from host DRAM all the same, being far larger than
    the CPU caches), the caches and weights are random."""
    import numpy as np

    import oracle
    from oracle import mla as omla
    from oracle import moe as omoe

    rng = np.random.default_rng(3)
    f = np.float32

    def nrm(*shape, s=0.02):
        return rng.standard_normal(shape, f) * s

    if model == "mixtral":
        c = MIXTRAL_8X7B
        H, nq, nkv, hd, I, E, K = 4096, 32, 8, 128, 14336, 8, 2
        B, ctx, layers, V = MX_BATCH, MX_CTX, 32, 32000
        w = {"q_w": nrm(nq * hd, H), "k_w": nrm(nkv * hd, H), "v_w": nrm(nkv * hd, H), "o_w": nrm(H, nq * hd)}
        pool = [{"gate_w": nrm(I, H), "up_w": nrm(I, H), "down_w": nrm(H, I)} for _ in range(2)]
        experts = [pool[e % 2] for e in range(E)]
        router = nrm(E, H, s=1.0)
        nblk = ctx // BLOCK + 1
        kc = rng.standard_normal((B * nblk, nkv, BLOCK, hd), f)
        vc = rng.standard_normal((B * nblk, nkv, BLOCK, hd), f)
        tables = np.arange(B * nblk).reshape(B, nblk)
        x = rng.standard_normal((B, H), f)
        cos, sin = oracle.rope1d_cos_sin(np.full(B, ctx), hd, c["rope_theta"])
        ones = np.ones(H, f)

        def layer():
            n = oracle.rms_norm(x, ones, 1e-5)
            q = oracle.rope_half(oracle.linear(n, w["q_w"]).reshape(B, nq, hd), cos, sin)
            k = oracle.rope_half(oracle.linear(n, w["k_w"]).reshape(B, nkv, hd), cos, sin)
            v = oracle.linear(n, w["v_w"]).reshape(B, nkv, hd)
            slots = oracle.slot_mapping(tables[0], np.array([ctx]), BLOCK)
            oracle.kv_cache_write(kc, k[:1], slots)
            oracle.kv_cache_write(vc, v[:1], slots)
            a = oracle.paged_decode_attention(q, kc, vc, tables, np.full(B, ctx + 1))
            h = x + oracle.linear(a.reshape(B, -1), w["o_w"])
            y, _, _ = omoe.moe_ffn(oracle.rms_norm(h, ones, 1e-5), router, experts, K, renormalize=True)
            return h + y

        what = (f"numpy fp32 oracle: one Mixtral-8x7B decode layer (batch {B}, context {ctx}: GQA paged attention, "
                f"8 experts top-2, 2 distinct expert weight arrays)")
    else:
        H, nh, R, dr, dn, dv, Im, E, K = 2048, 16, 512, 64, 128, 128, 1408, 64, 6
        B, ctx, layers, V = DS_BATCH, DS_CTX, 27, 102400
        rs = DEEPSEEK_V2_LITE["rope_scaling"]
        cfg = {"heads": nh, "qk_nope": dn, "qk_rope": dr, "v_head": dv, "kv_lora": R, "eps": 1e-6, "theta": 10000.0,
               "yarn": {"factor": rs["factor"], "orig_max_pos": rs["original_max_position_embeddings"],
                        "beta_fast": rs["beta_fast"], "beta_slow": rs["beta_slow"], "mscale": rs["mscale"],
                        "mscale_all_dim": rs["mscale_all_dim"]}}
        w = {"q_w": nrm(nh * (dn + dr), H), "kva_w": nrm(R + dr, H), "kv_norm": np.ones(R, f),
             "kvb_w": nrm(nh * (dn + dv), R), "o_w": nrm(H, nh * dv)}
        qabs, oabs = omla.absorbed_weights(w, cfg)  # folded once, as the engine does at load
        pool = [{"gate_w": nrm(Im, H), "up_w": nrm(Im, H), "down_w": nrm(H, Im)} for _ in range(8)]
        experts = [pool[e % 8] for e in range(E)]
        shared = {"gate_w": nrm(2 * Im, H), "up_w": nrm(2 * Im, H), "down_w": nrm(H, 2 * Im)}
        router = nrm(E, H, s=1.0)
        caches = [rng.standard_normal((ctx + 1, R + dr), f) for _ in range(B)]
        x = rng.standard_normal((B, H), f)
        cos, sin = omla.rope_cfg_tables(np.full(B, ctx), cfg)
        ones = np.ones(H, f)
        scale = omla.softmax_scale(cfg)

        def layer():
            n = oracle.rms_norm(x, ones, 1e-6)
            q = oracle.linear(n, qabs).reshape(B, nh, R + dr)
            q[:, :, R:] = omla.rope_deinterleave(q[:, :, R:], cos[:, None, :], sin[:, None, :])
            kv_a = oracle.linear(n, w["kva_w"])
            cnew = oracle.rms_norm(kv_a[:, :R], w["kv_norm"], 1e-6)
            kpe = omla.rope_deinterleave(kv_a[:, R:], cos, sin)
            for b in range(B):  # the cache write of this token
                caches[b][ctx, :R], caches[b][ctx, R:] = cnew[b], kpe[b]
            lat = omla.latent_decode(q.reshape(B, -1), caches, [ctx + 1] * B, nh, scale)
            h = x + oracle.linear(lat, oabs)
            y, _, _ = omoe.moe_ffn(oracle.rms_norm(h, ones, 1e-6), router, experts, K, renormalize=False,
                                     shared=shared)
            return h + y

        what = (f"numpy fp32 oracle: one DeepSeek-V2-Lite MoE decode layer (batch {B}, context {ctx}: absorbed "
                f"latent attention, 64 experts top-6 + 2 shared, 8 distinct expert weight arrays)")
    lm = nrm(V // 8, H)
    t_layer, reps = _cpu_time(layer)
    t0 = time.perf_counter()
    oracle.linear(x, lm)
    t_head = (time.perf_counter() - t0) * 8
    step = layers * t_layer + t_head
    return {"value": B / step, "unit": "tok/s", "cores": blas_threads(), "kind": "port",
            "sample": f"{what} timed x{reps} = {t_layer * 1e3:.1f} ms/layer, scaled to {layers} layers + lm_head "
                      f"(extrapolated)"}


def bench_mixtral(L, torch, dev, steps, warm, stream_of):
    """Mixtral-8x7B on one GPU (93 GB of bf16 weights): prefill 8 x 1024 per
    step; decode batch 32 at context 4096 (paged KV, block 128)."""
    import numpy as np

    max_ctx = MX_CTX + 2 * (warm + steps) + 16  # device-fed then host-fed decode steps
    cfg = EngineConfig(None, json.dumps(MIXTRAL_8X7B).encode(), dev.index, MX_BATCH, max_ctx,
                       MX_PREFILL_SEQS * MX_PREFILL_LEN, BLOCK, 77, 0.02)
    eng = ctypes.c_void_p()
    check(L.b200_engine_create(ctypes.byref(cfg), ctypes.byref(eng)), "engine_create mixtral")
    est = stream_of(eng)
    try:
        V = MIXTRAL_8X7B["vocab_size"]
        rng = np.random.default_rng(7)
        T = MX_PREFILL_SEQS * MX_PREFILL_LEN
        ids_pf = torch.from_numpy(rng.integers(0, V, T).astype(np.int64)).to(dev)
        lens_pf = np.full(MX_PREFILL_SEQS, MX_PREFILL_LEN, np.int32)
        nxt = torch.empty(MX_BATCH, dtype=torch.int64, device=dev)

        def timed(fn, n):
            for i in range(warm):
                fn(i)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(est)
            for i in range(n):
                fn(i)
            e1.record(est)
            torch.cuda.synchronize(dev)
            return e0.elapsed_time(e1) / n

        def prefill(i):
            slots = np.arange(MX_PREFILL_SEQS, dtype=np.int32) + (i % (MX_BATCH // MX_PREFILL_SEQS)) * MX_PREFILL_SEQS
            check(L.b200_engine_prefill(eng, ids_pf.data_ptr(), 1, lens_pf.ctypes.data, slots.ctypes.data,
                                        MX_PREFILL_SEQS, None, nxt.data_ptr(), 1, None), "prefill")

        pf_ms = timed(prefill, max(3, min(steps, 5)))
        # fill every slot to context 4096 (2 distinct random sequences of 4096 per call)
        check(L.b200_engine_reset(eng), "reset")
        lens_ctx = np.full(2, MX_CTX, np.int32)
        for g in range(MX_BATCH // 2):
            ids_ctx = torch.from_numpy(rng.integers(0, V, 2 * MX_CTX).astype(np.int64)).to(dev)
            slots = np.array([2 * g, 2 * g + 1], np.int32)
            check(L.b200_engine_prefill(eng, ids_ctx.data_ptr(), 1, lens_ctx.ctypes.data, slots.ctypes.data, 2,
                                        None, nxt[2 * g:].data_ptr(), 1, None), "prefill ctx")
        slots_all = np.arange(MX_BATCH, dtype=np.int32)
        # Each step feeds fresh random tokens (teacher forcing) so that routing
        # stays near-uniform across the experts, as with real traffic; greedy
        # feedback from random weights can collapse onto a few tokens.
        feed_host = rng.integers(0, V, (warm + steps + 1, MX_BATCH)).astype(np.int64)
        feed = torch.from_numpy(feed_host).to(dev)
        out_d = torch.empty(MX_BATCH, dtype=torch.int64, device=dev)
        counter = {"i": 0}

        def decode(_):
            i = counter["i"] % len(feed_host)
            counter["i"] += 1
            check(L.b200_engine_decode(eng, feed[i].data_ptr(), 1, slots_all.ctypes.data, MX_BATCH,
                                       out_d.data_ptr(), 1, None), "decode")

        dec_ms = timed(decode, steps)
        host_next = np.zeros(MX_BATCH, np.int64)

        def decode_host(_):
            i = counter["i"] % len(feed_host)
            counter["i"] += 1
            check(L.b200_engine_decode(eng, feed_host[i].ctypes.data, 0, slots_all.ctypes.data, MX_BATCH,
                                       host_next.ctypes.data, 0, None), "decode")

        e2e_ms = timed(decode_host, steps)
        v = ctypes.c_int64()
        check(L.b200_engine_query(eng, 2, ctypes.byref(v)), "query")
        hbm, tf_burst, tf_sus, src = peaks()
        return {
            "workload": "Mixtral-8x7B (46.7 B params, 8 experts top-2) on one GPU: decode batch 32 at context 4096, "
                        "prefill 8x1024",
            "decode_tok_s": MX_BATCH / (dec_ms / 1e3), "decode_ms_per_step": dec_ms,
            "decode_e2e_tok_s": MX_BATCH / (e2e_ms / 1e3),
            "decode_roofline": {"bound": "hbm", "bytes_per_step": MX_DECODE_BYTES,
                                "achieved": MX_DECODE_BYTES / (dec_ms / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                                "frac": MX_DECODE_BYTES / (dec_ms / 1e3) / 1e9 / hbm, "peak_source": f"{src} copy"},
            "prefill_tok_s": MX_PREFILL_SEQS * MX_PREFILL_LEN / (pf_ms / 1e3), "prefill_ms_per_step": pf_ms,
            "prefill_roofline": {"bound": "tensor", "flop_per_step": MX_PREFILL_FLOP,
                                 "achieved": MX_PREFILL_FLOP / (pf_ms / 1e3) / 1e12, "peak": tf_sus,
                                 "unit": "TFLOP/s", "frac": MX_PREFILL_FLOP / (pf_ms / 1e3) / 1e12 / tf_sus,
                                 "peak_source": f"{src} bf16 sustained"},
            "decode_launches_per_step": v.value,
        }
    finally:
        L.b200_engine_destroy(eng)


DEEPSEEK_V2_LITE = dict(
    model_type="deepseek_v2", hidden_size=2048, num_hidden_layers=27, num_attention_heads=16, num_key_value_heads=16,
    q_lora_rank=None, kv_lora_rank=512, qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128,
    intermediate_size=10944, moe_intermediate_size=1408, n_routed_experts=64, num_experts_per_tok=6,
    n_shared_experts=2, first_k_dense_replace=1, norm_topk_prob=False, routed_scaling_factor=1.0,
    topk_method="greedy", scoring_func="softmax", moe_layer_freq=1, vocab_size=102400, rms_norm_eps=1e-6,
    rope_theta=10000.0, tie_word_embeddings=False,
    rope_scaling=dict(type="yarn", factor=40.0, original_max_position_embeddings=4096, beta_fast=32, beta_slow=1,
                      mscale=0.707, mscale_all_dim=0.707))
DS_BATCH, DS_CTX = 32, 4096


def ds_decode_bytes():
    """One decode step's algorithmic bytes, counted conservatively: the plain
    (not absorbed) attention projections, the dense first layer, the routed
    experts the 32 x 6 choices are expected to reach at uniform routing
    (64 * (1 - (58/64)^32) = 61.27 of 64), the shared experts, the router,
    lm_head, plus the latent cache of 32 x 4096 tokens.  The absorbed decode
    projections this engine streams are larger (+0.6 GB a step), uncounted."""
    H, nh, L = 2048, 16, 27
    attn = H * nh * 192 + H * 576 + 512 + nh * 256 * 512 + H * nh * 128
    dense = 3 * H * 10944
    touched = 64 * (1 - (58 / 64) ** DS_BATCH)
    moe = touched * 3 * H * 1408 + 3 * H * 2 * 1408 + 64 * H
    weights = L * attn + dense + (L - 1) * moe + 102400 * H
    cache = DS_BATCH * DS_CTX * L * 576
    return 2 * (weights + cache)


def bench_deepseek(L, torch, dev, steps, warm, stream_of):
    """DeepSeek-V2-Lite on one GPU: decode batch 32 at context 4096 over the
    latent cache (filled by real prefill calls), fresh random tokens each step."""
    import numpy as np

    max_ctx = DS_CTX + 2 * (warm + steps) + 16
    cfg = EngineConfig(None, json.dumps(DEEPSEEK_V2_LITE).encode(), dev.index, DS_BATCH, max_ctx, 2 * DS_CTX, BLOCK,
                       55, 0.02)
    eng = ctypes.c_void_p()
    check(L.b200_engine_create(ctypes.byref(cfg), ctypes.byref(eng)), "engine_create deepseek")
    est = stream_of(eng)
    try:
        V = DEEPSEEK_V2_LITE["vocab_size"]
        rng = np.random.default_rng(9)
        nxt = torch.empty(DS_BATCH, dtype=torch.int64, device=dev)
        lens = np.full(2, DS_CTX, np.int32)
        t0 = time.perf_counter()
        for g in range(DS_BATCH // 2):
            ids = torch.from_numpy(rng.integers(0, V, 2 * DS_CTX).astype(np.int64)).to(dev)
            slots = np.array([2 * g, 2 * g + 1], np.int32)
            check(L.b200_engine_prefill(eng, ids.data_ptr(), 1, lens.ctypes.data, slots.ctypes.data, 2, None,
                                        nxt[2 * g:].data_ptr(), 1, None), "prefill ctx")
        torch.cuda.synchronize(dev)
        fill_s = time.perf_counter() - t0
        # prefill throughput: 2 x 4096-token prompts per call (the fill's shape), CUDA events, after a warm-up call
        pf_ids = torch.from_numpy(rng.integers(0, V, 2 * DS_CTX).astype(np.int64)).to(dev)
        pf_next = torch.empty(2, dtype=torch.int64, device=dev)

        def prefill_call(g):
            sl = np.array([2 * g, 2 * g + 1], np.int32)
            check(L.b200_engine_prefill(eng, pf_ids.data_ptr(), 1, lens.ctypes.data, sl.ctypes.data, 2, None,
                                        pf_next.data_ptr(), 1, None), "prefill")

        check(L.b200_engine_reset(eng), "reset")
        prefill_call(0)
        torch.cuda.synchronize(dev)
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(est)
        for g in range(1, 4):
            prefill_call(g)
        p1.record(est)
        torch.cuda.synchronize(dev)
        pf_ms = p0.elapsed_time(p1) / 3
        # refill the slots the timed calls reused, so every slot again holds a distinct 4096-token context
        check(L.b200_engine_reset(eng), "reset")
        for g in range(DS_BATCH // 2):
            ids = torch.from_numpy(rng.integers(0, V, 2 * DS_CTX).astype(np.int64)).to(dev)
            slots = np.array([2 * g, 2 * g + 1], np.int32)
            check(L.b200_engine_prefill(eng, ids.data_ptr(), 1, lens.ctypes.data, slots.ctypes.data, 2, None,
                                        nxt[2 * g:].data_ptr(), 1, None), "prefill ctx")
        slots_all = np.arange(DS_BATCH, dtype=np.int32)
        feed_host = rng.integers(0, V, (warm + steps + 1, DS_BATCH)).astype(np.int64)
        feed = torch.from_numpy(feed_host).to(dev)
        out_d = torch.empty(DS_BATCH, dtype=torch.int64, device=dev)
        host_next = np.zeros(DS_BATCH, np.int64)
        counter = {"i": 0}

        def decode(on_device):
            i = counter["i"] % len(feed_host)
            counter["i"] += 1
            if on_device:
                check(L.b200_engine_decode(eng, feed[i].data_ptr(), 1, slots_all.ctypes.data, DS_BATCH,
                                           out_d.data_ptr(), 1, None), "decode")
            else:
                check(L.b200_engine_decode(eng, feed_host[i].ctypes.data, 0, slots_all.ctypes.data, DS_BATCH,
                                           host_next.ctypes.data, 0, None), "decode")

        def timed(on_device):
            for _ in range(warm):
                decode(on_device)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(est)
            for _ in range(steps):
                decode(on_device)
            e1.record(est)
            torch.cuda.synchronize(dev)
            return e0.elapsed_time(e1) / steps

        dec_ms = timed(True)
        e2e_ms = timed(False)
        v = ctypes.c_int64()
        check(L.b200_engine_query(eng, 2, ctypes.byref(v)), "query")
        hbm, _, _, src = peaks()
        nbytes = ds_decode_bytes()
        return {
            "workload": "DeepSeek-V2-Lite (15.7 B params, MLA kv_lora 512 + 64 routed experts top-6 + 2 shared) on "
                        "one GPU: decode batch 32 at context 4096 over the latent cache",
            "decode_tok_s": DS_BATCH / (dec_ms / 1e3), "decode_ms_per_step": dec_ms,
            "decode_e2e_tok_s": DS_BATCH / (e2e_ms / 1e3),
            "decode_roofline": {"bound": "hbm", "bytes_per_step": nbytes, "achieved": nbytes / (dec_ms / 1e3) / 1e9,
                                "peak": hbm, "unit": "GB/s", "frac": nbytes / (dec_ms / 1e3) / 1e9 / hbm,
                                "peak_source": f"{src} copy"},
            "prefill_tok_s": 2 * DS_CTX / (pf_ms / 1e3), "prefill_ms_per_step": pf_ms,
            "prefill": "2 x 4096-token prompts per call",
            "prefill_fill_s": fill_s, "decode_launches_per_step": v.value,
        }
    finally:
        L.b200_engine_destroy(eng)


def kernel_roofline_mla_prefill_attention(L, torch, dev, reps=10):
    """Latent attention's prefill (decompressed heads: 192-wide query / key,
    128-wide value, 16 heads) on the tcgen05 kernel at the DeepSeek-V2-Lite
    prefill shape (2 causal sequences of 4096 tokens, the engine's operand
    layouts): flops = 2 * 16 * sum(S^2 / 2) * (192 + 128)."""
    S, nseq, nh = DS_CTX, 2, 16
    T = S * nseq
    NQP, KVB = nh * 192 + 576, nh * 256
    g = torch.Generator(device=dev).manual_seed(6)
    q = torch.randn(T, NQP, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(T, nh * 192, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(T, KVB, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(T, nh * 128, dtype=torch.bfloat16, device=dev)
    cu = torch.tensor([0, S, 2 * S], dtype=torch.int32, device=dev)

    def run(st):
        check(L.b200_flash_prefill_packed(q.data_ptr(), NQP, 192, k.data_ptr(), nh * 192, 192, v.data_ptr() + 256,
                                          KVB, 256, out.data_ptr(), nh * 128, 128, cu.data_ptr(), nseq, S, T, nh, nh,
                                          192, 128, 0.1, 1, st.cuda_stream), "mla prefill attention")

    ms = _time_launches(torch, dev, run, reps)
    return ms, 2.0 * nh * nseq * (S * S / 2) * (192 + 128)


def make_comm(L, dist, world, rank, dev, sym_bytes):
    """A connected b200_comm_t over all ranks (NCCL id and CUDA IPC handles exchanged through `dist`)."""
    uid = ctypes.create_string_buffer(128)
    if rank == 0:
        check(L.b200_comm_unique_id(uid), "comm_unique_id")
    box = [uid.raw]
    dist.broadcast_object_list(box, src=0)
    uid = ctypes.create_string_buffer(box[0], 128)
    comm = ctypes.c_void_p()
    check(L.b200_comm_create(world, rank, dev.index, uid, sym_bytes, ctypes.byref(comm)), "comm_create")
    h = ctypes.create_string_buffer(64)
    check(L.b200_comm_ipc_handle(comm, h), "comm_ipc_handle")
    hs = [None] * world
    dist.all_gather_object(hs, h.raw)
    check(L.b200_comm_connect(comm, ctypes.create_string_buffer(b"".join(hs), 64 * world)), "comm_connect")
    return comm


def moe_decode_bytes(C, P, batch, ctx):
    """Algorithmic bytes one rank streams in one decode step of a
    mixture-of-experts model under P-way expert parallelism (P = 1: one GPU)
    with data-parallel attention: every replicated weight once (attention —
    plain, not absorbed, projections for MLA — dense layers, shared experts,
    routers, lm_head), this rank's share of the routed experts the P * batch
    tokens are expected to reach at uniform routing, and this rank's own KV
    (latent) cache of batch x ctx tokens."""
    H, Lyr, V = C["hidden_size"], C["num_hidden_layers"], C["vocab_size"]
    if C.get("n_routed_experts"):
        E, k, Im = C["n_routed_experts"], C["num_experts_per_tok"], C["moe_intermediate_size"]
        nh, lora, rope, nope, vh = (C["num_attention_heads"], C["kv_lora_rank"], C["qk_rope_head_dim"],
                                    C["qk_nope_head_dim"], C["v_head_dim"])
        attn = H * nh * (nope + rope) + H * (lora + rope) + lora + nh * (nope + vh) * lora + H * nh * vh
        fd = C["first_k_dense_replace"]
        dense = fd * 3 * H * C["intermediate_size"]
        shared = 3 * H * C["n_shared_experts"] * Im
        cache = batch * ctx * Lyr * (lora + rope)
    else:
        E, k, Im = C["num_local_experts"], C["num_experts_per_tok"], C["intermediate_size"]
        nq, nkv, hd = C["num_attention_heads"], C["num_key_value_heads"], H // C["num_attention_heads"]
        attn = H * (nq + 2 * nkv) * hd + H * nq * hd
        fd, dense, shared = 0, 0, 0
        cache = batch * ctx * Lyr * 2 * nkv * hd
    touched = (E / P) * (1 - ((E - k) / E) ** (P * batch))  # this rank's experts reached by P*batch tokens x k
    weights = Lyr * attn + dense + (Lyr - fd) * (touched * 3 * H * Im + shared + E * H) + V * H
    return 2 * (weights + cache)


def sharded_parity(L, torch, dev, dist, world, rank, C, mode, seed=4242):
    """The sharded code path against one GPU: a 2-layer copy of model C at
    full width is built tensor-parallel (mode "tp") or expert-parallel ("ep")
    over all ranks and, on rank 0, whole on one GPU from the same seed (the
    engine's random init gives every shard the whole model's values at its
    positions).  Both get rank 0's two 96-token prompts, then three decode
    steps of fresh random tokens (eager, captured, replayed).  Rank 0 compares
    its logits with the one-GPU engine's (tensor parallel: its vocabulary
    shard) and the greedy tokens.  Collective: every rank calls it."""
    import numpy as np

    Cp = dict(C, num_hidden_layers=2)
    H, V = Cp["hidden_size"], Cp["vocab_size"]
    nseq, plen, steps = 2, 96, 3
    T = nseq * plen
    k = Cp.get("num_experts_per_tok", 1)
    sym = 2 * T * H * 2 + (16 << 20) if mode == "tp" else 2 * ((64 << 10) + world * T * k * H * 2) + (1 << 20)
    cfg = EngineConfig(None, json.dumps(Cp).encode(), dev.index, nseq, plen + steps + 16, T, BLOCK, seed, 0.02)
    rng = np.random.default_rng(900 + (rank if mode == "ep" else 0))  # expert parallel: every rank its own prompts
    prompts = rng.integers(0, V, T).astype(np.int64)
    feed = rng.integers(0, V, (steps, nseq)).astype(np.int64)
    vcols = V // world if mode == "tp" else V

    def run(e, cols):
        lens, slots = np.full(nseq, plen, np.int32), np.arange(nseq, dtype=np.int32)
        nxt = np.zeros(nseq, np.int64)
        lg = torch.empty(nseq, cols, dtype=torch.bfloat16, device=dev)
        check(L.b200_engine_prefill(e, prompts.ctypes.data, 0, lens.ctypes.data, slots.ctypes.data, nseq, None,
                                    nxt.ctypes.data, 0, lg.data_ptr()), "parity prefill")
        torch.cuda.synchronize(dev)
        logits, toks = [lg.float().cpu().numpy()], [nxt.copy()]
        for i in range(steps):
            out = np.zeros(nseq, np.int64)
            check(L.b200_engine_decode(e, feed[i].ctypes.data, 0, slots.ctypes.data, nseq, out.ctypes.data, 0,
                                       lg.data_ptr()), "parity decode")
            torch.cuda.synchronize(dev)
            logits.append(lg.float().cpu().numpy())
            toks.append(out.copy())
        return np.concatenate(logits), np.concatenate(toks)

    comm = make_comm(L, dist, world, rank, dev, sym)
    eng = ctypes.c_void_p()
    create = L.b200_engine_create_tp if mode == "tp" else L.b200_engine_create_ep
    check(create(ctypes.byref(cfg), comm, ctypes.byref(eng)), f"parity engine_create_{mode}")
    try:
        got, got_tok = run(eng, vcols)
        errs = ctypes.c_uint(0)
        check(L.b200_device_error_read(ctypes.addressof(errs), 1, None), "device_error_read")
    finally:
        torch.cuda.synchronize(dev)
        dist.barrier()
        L.b200_engine_destroy(eng)
        L.b200_comm_destroy(comm)
    res = None
    if rank == 0:
        ref_eng = ctypes.c_void_p()
        check(L.b200_engine_create(ctypes.byref(cfg), ctypes.byref(ref_eng)), "parity engine_create")
        try:
            ref, ref_tok = run(ref_eng, V)
        finally:
            L.b200_engine_destroy(ref_eng)
        ref_shard = ref[:, :vcols]
        cos = [float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30)) for a, b in zip(got, ref_shard)]
        top2 = np.sort(ref, 1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > 0.05 * np.abs(ref).max(1)  # greedy token outside the bf16 noise
        same = got_tok == ref_tok
        res = {"layers": 2, "rows": len(cos), "min_cos": round(min(cos), 6),
               "tokens_equal": f"{int(same.sum())}/{len(same)}", "device_errors": errs.value,
               "parity": bool(min(cos) >= 0.999 and same[clear].all() and errs.value == 0)}
    dist.barrier()
    return res


def bench_ep(L, torch, dev, dist, world, rank, steps, warm, stream_of, C, batch, ctx, name):
    """Expert parallel over all ranks: every rank serves its OWN `batch`
    sequences at context `ctx` (data-parallel attention, whole replicas of the
    non-expert weights) and holds E/P routed experts; every MoE layer exchanges
    tokens through the peer-memory dispatch / combine kernels.  Whole-job
    decode tok/s = P * batch / (max over ranks of the step time); fresh random
    tokens each step (own seed per rank)."""
    import numpy as np

    parity = sharded_parity(L, torch, dev, dist, world, rank, C, "ep")
    H, k = C["hidden_size"], C["num_experts_per_tok"]
    T = 2 * ctx  # prefill tokens per call (two whole prompts)
    half = (64 << 10) + world * T * k * H * 2
    comm = make_comm(L, dist, world, rank, dev, 2 * half + (1 << 20))
    max_ctx = ctx + 2 * (warm + steps) + 16
    cfg = EngineConfig(None, json.dumps(C).encode(), dev.index, batch, max_ctx, T, BLOCK, 99, 0.02)
    eng = ctypes.c_void_p()
    check(L.b200_engine_create_ep(ctypes.byref(cfg), comm, ctypes.byref(eng)), "engine_create_ep")
    est = stream_of(eng)
    try:
        V = C["vocab_size"]
        rng = np.random.default_rng(300 + rank)
        nxt = torch.empty(batch, dtype=torch.int64, device=dev)
        lens = np.full(2, ctx, np.int32)

        def timed(fn, n):
            for i in range(warm):
                fn(i)
            dist.barrier()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(est)
            for i in range(n):
                fn(i)
            e1.record(est)
            torch.cuda.synchronize(dev)
            t = torch.tensor([e0.elapsed_time(e1) / n], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        ids_pf = torch.from_numpy(rng.integers(0, V, T).astype(np.int64)).to(dev)

        def prefill(i):
            g = i % max(1, batch // 2)
            sl = np.array([2 * g, 2 * g + 1], np.int32)
            check(L.b200_engine_prefill(eng, ids_pf.data_ptr(), 1, lens.ctypes.data, sl.ctypes.data, 2, None,
                                        nxt[2 * g:].data_ptr(), 1, None), "prefill")

        pf_ms = timed(prefill, 3)
        check(L.b200_engine_reset(eng), "reset")
        for g in range(batch // 2):
            ids = torch.from_numpy(rng.integers(0, V, T).astype(np.int64)).to(dev)
            sl = np.array([2 * g, 2 * g + 1], np.int32)
            check(L.b200_engine_prefill(eng, ids.data_ptr(), 1, lens.ctypes.data, sl.ctypes.data, 2, None,
                                        nxt[2 * g:].data_ptr(), 1, None), "prefill ctx")
        slots_all = np.arange(batch, dtype=np.int32)
        feed = torch.from_numpy(rng.integers(0, V, (warm + steps + 1, batch)).astype(np.int64)).to(dev)
        out_d = torch.empty(batch, dtype=torch.int64, device=dev)
        counter = {"i": 0}

        def decode(_):
            i = counter["i"] % feed.shape[0]
            counter["i"] += 1
            check(L.b200_engine_decode(eng, feed[i].data_ptr(), 1, slots_all.ctypes.data, batch, out_d.data_ptr(),
                                       1, None), "decode")

        dec_ms = timed(decode, steps)
        v = ctypes.c_int64()
        check(L.b200_engine_query(eng, 2, ctypes.byref(v)), "query")
        errs = ctypes.c_uint(0)
        check(L.b200_device_error_read(ctypes.addressof(errs), 1, None), "device_error_read")
        hbm, _, _, src = peaks()
        nbytes = moe_decode_bytes(C, world, batch, ctx)
        return {"ep": world, "workload": f"{name}: {world} ranks x own decode batch {batch} at context {ctx}, "
                                         f"{C.get('n_routed_experts') or C['num_local_experts']} experts split "
                                         f"{world} ways, attention data-parallel",
                "decode_tok_s": world * batch / (dec_ms / 1e3), "decode_ms_per_step": dec_ms,
                "decode_roofline_per_rank": {"bound": "hbm", "bytes_per_step": nbytes,
                                             "achieved": nbytes / (dec_ms / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                                             "frac": nbytes / (dec_ms / 1e3) / 1e9 / hbm,
                                             "peak_source": f"{src} copy"},
                "prefill_tok_s": world * T / (pf_ms / 1e3), "prefill_ms_per_step": pf_ms,
                "prefill": f"{world} ranks x 2x{ctx}",
                "decode_launches_per_step": v.value, "device_errors": errs.value, "parity": parity}
    finally:
        torch.cuda.synchronize(dev)
        dist.barrier()
        L.b200_engine_destroy(eng)
        L.b200_comm_destroy(comm)


def bench_tp(L, torch, dev, dist, world, rank, steps, warm, stream_of, C, seqs, plen, batch, ctx, note):
    """One model tensor-parallel over all ranks: prefill `seqs` x `plen` per
    step, decode `batch` sequences at context `ctx` (slots filled by prefills of
    whole `ctx`-token prompts); two all-reduces per layer (fused peer-memory
    kernel for decode, NCCL for prefill).  Timed with CUDA events, max over
    ranks."""
    import numpy as np

    parity = sharded_parity(L, torch, dev, dist, world, rank, C, "tp")
    T = max(seqs * plen, ctx)
    comm = make_comm(L, dist, world, rank, dev, 2 * T * C["hidden_size"] * 2 + (16 << 20))
    max_ctx = ctx + warm + steps + 16
    cfg = EngineConfig(None, json.dumps(C).encode(), dev.index, batch, max_ctx, T, BLOCK, 4321, 0.02)
    eng = ctypes.c_void_p()
    check(L.b200_engine_create_tp(ctypes.byref(cfg), comm, ctypes.byref(eng)), "engine_create_tp")
    est = stream_of(eng)
    try:
        V = C["vocab_size"]
        rng = np.random.default_rng(2)  # the same prompts on every rank
        lens = np.full(seqs, plen, np.int32)
        ids_pf = torch.from_numpy(rng.integers(0, V, seqs * plen).astype(np.int64)).to(dev)
        nxt = torch.empty(max(batch, seqs), dtype=torch.int64, device=dev)

        def prefill(i):
            g = i % max(1, batch // seqs)
            slots = np.arange(g * seqs, (g + 1) * seqs, dtype=np.int32) % batch
            check(L.b200_engine_prefill(eng, ids_pf.data_ptr(), 1, lens.ctypes.data, slots.ctypes.data,
                                        seqs, None, nxt.data_ptr(), 1, None), "prefill")

        def timed(fn, n):
            for i in range(warm):
                fn(i)
            dist.barrier()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(est)
            for i in range(n):
                fn(i)
            e1.record(est)
            torch.cuda.synchronize(dev)
            t = torch.tensor([e0.elapsed_time(e1) / n], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        pf_ms = timed(prefill, max(1, min(steps, 3)))
        # fill every slot to `ctx` with distinct prompts, as many per call as fit one prefill
        check(L.b200_engine_reset(eng), "reset")
        per = max(1, T // ctx)
        for g0 in range(0, batch, per):
            n = min(per, batch - g0)
            ids_ctx = torch.from_numpy(rng.integers(0, V, n * ctx).astype(np.int64)).to(dev)
            sl = np.arange(g0, g0 + n, dtype=np.int32)
            check(L.b200_engine_prefill(eng, ids_ctx.data_ptr(), 1, np.full(n, ctx, np.int32).ctypes.data,
                                        sl.ctypes.data, n, None, nxt[g0:].data_ptr(), 1, None), "prefill ctx")
        slots_all = np.arange(batch, dtype=np.int32)
        state = {"a": nxt[:batch].clone(), "b": torch.empty(batch, dtype=torch.int64, device=dev)}
        # mixture-of-experts models are fed fresh random tokens (the same on every rank) so that routing stays
        # near-uniform; greedy feedback from random weights can collapse onto a few tokens and experts
        feed = (torch.from_numpy(rng.integers(0, V, (warm + steps, batch)).astype(np.int64)).to(dev)
                if C.get("num_local_experts") or C.get("n_routed_experts") else None)

        def decode(_):
            state["n"] = state.get("n", -1) + 1
            src = state["a"] if feed is None else feed[state["n"] % feed.shape[0]]
            check(L.b200_engine_decode(eng, src.data_ptr(), 1, slots_all.ctypes.data, batch,
                                       state["b"].data_ptr(), 1, None), "decode")
            state["a"], state["b"] = state["b"], state["a"]

        dec_ms = timed(decode, steps)
        v = ctypes.c_int64()
        check(L.b200_engine_query(eng, 2, ctypes.byref(v)), "query")
        errs = ctypes.c_uint(0)
        check(L.b200_device_error_read(ctypes.addressof(errs), 1, None), "device_error_read")
        return {"tp": world, "decode_batch": batch, "decode_ctx": ctx, "decode_tok_s": batch / (dec_ms / 1e3),
                "decode_ms_per_step": dec_ms, "prefill": f"{seqs}x{plen}",
                "prefill_tok_s": seqs * plen / (pf_ms / 1e3), "prefill_ms_per_step": pf_ms,
                "decode_launches_per_step": v.value, "device_errors": errs.value, "note": note, "parity": parity}
    finally:
        torch.cuda.synchronize(dev)
        dist.barrier()
        L.b200_engine_destroy(eng)
        L.b200_comm_destroy(comm)


def run_b200(args, rank, world, local_rank):
    import numpy as np
    import torch

    from atb_llm_study_b200 import capi

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist_mod
        from datetime import timedelta

        dist = dist_mod
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    L = capi.lib()
    steps, warm = args.steps, args.warmup
    max_ctx = DECODE_CTX + warm + 2 * steps + 16
    cfg = EngineConfig(None, json.dumps(QWEN3_8B).encode(), local_rank, DECODE_BATCH, max_ctx,
                       PREFILL_SEQS * PREFILL_LEN, BLOCK, 1234 + rank, 0.02)
    eng = ctypes.c_void_p()
    check(L.b200_engine_create(ctypes.byref(cfg), ctypes.byref(eng)), "engine_create")
    raw = ctypes.c_void_p()
    check(L.b200_engine_stream(eng, ctypes.byref(raw)), "engine_stream")
    est = torch.cuda.ExternalStream(raw.value, device=dev)

    def q(k):
        v = ctypes.c_int64()
        check(L.b200_engine_query(eng, k, ctypes.byref(v)), "query")
        return v.value

    V = QWEN3_8B["vocab_size"]
    rng = np.random.default_rng(2 + rank)
    T = PREFILL_SEQS * PREFILL_LEN
    lens = np.full(PREFILL_SEQS, PREFILL_LEN, np.int32)
    groups = DECODE_BATCH // PREFILL_SEQS
    ids_host = [rng.integers(0, V, T).astype(np.int64) for _ in range(groups)]
    ids_dev = [torch.from_numpy(a).to(dev) for a in ids_host]
    next_dev = torch.empty(DECODE_BATCH, dtype=torch.int64, device=dev)
    filled = set()

    def prefill(step, on_device):
        gi = step % groups
        slots = np.arange(gi * PREFILL_SEQS, (gi + 1) * PREFILL_SEQS, dtype=np.int32)
        nxt = np.zeros(PREFILL_SEQS, np.int64)
        if on_device:
            check(L.b200_engine_prefill(eng, ids_dev[gi].data_ptr(), 1, lens.ctypes.data, slots.ctypes.data,
                                        PREFILL_SEQS, None, next_dev[gi * PREFILL_SEQS:].data_ptr(), 1, None),
                  "prefill")
        else:
            check(L.b200_engine_prefill(eng, ids_host[gi].ctypes.data, 0, lens.ctypes.data, slots.ctypes.data,
                                        PREFILL_SEQS, None, nxt.ctypes.data, 0, None), "prefill")
            next_dev[gi * PREFILL_SEQS:(gi + 1) * PREFILL_SEQS].copy_(torch.from_numpy(nxt))
        filled.add(gi)

    def timed(fn, n, offset):
        """Barrier + sync, CUDA events on the engine stream around n calls, max over ranks."""
        if dist:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(est)
        for i in range(n):
            fn(offset + i)
        e1.record(est)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1)
        if dist:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    # ---- prefill ----
    for i in range(warm):
        prefill(i, True)
    # clocks are sampled from the first timed prefill step to the last timed
    # decode step (the decode region alone is shorter than the 200 ms period)
    clk = ClockSampler(local_rank).__enter__()
    time.sleep(0.5)  # nvidia-smi start-up
    pf_ms = timed(lambda i: prefill(i, True), steps, warm)
    pf_e2e_ms = timed(lambda i: prefill(i, False), max(1, min(steps, 3)), warm + steps)
    for gi in range(groups):
        if gi not in filled:
            prefill(gi, True)
    torch.cuda.synchronize(dev)
    check(L.b200_engine_reset(eng), "reset")  # every slot restarts at context 2048 below
    for gi in range(groups):
        prefill(gi, True)
    torch.cuda.synchronize(dev)

    # ---- decode ----
    slots_all = np.arange(DECODE_BATCH, dtype=np.int32)
    ids_d = next_dev.clone()
    out_d = torch.empty_like(ids_d)
    host_ids = np.zeros(DECODE_BATCH, np.int64)
    host_next = np.zeros(DECODE_BATCH, np.int64)

    def decode_dev(_):
        nonlocal ids_d, out_d
        check(L.b200_engine_decode(eng, ids_d.data_ptr(), 1, slots_all.ctypes.data, DECODE_BATCH, out_d.data_ptr(), 1,
                                   None), "decode")
        ids_d, out_d = out_d, ids_d

    def decode_host(_):
        check(L.b200_engine_decode(eng, host_ids.ctypes.data, 0, slots_all.ctypes.data, DECODE_BATCH,
                                   host_next.ctypes.data, 0, None), "decode")
        host_ids[:] = host_next

    for i in range(warm):
        decode_dev(i)
    with RegionClock(local_rank) as dec_clk:
        dec_ms = timed(decode_dev, steps, 0)
    clk.__exit__(None, None, None)
    clocks = clk.summary()
    clocks["decode_region_sm_mhz"] = dec_clk.median()
    host_ids[:] = ids_d.cpu().numpy()
    with RegionClock(local_rank) as e2e_clk:
        dec_e2e_ms = timed(decode_host, steps, 0)
    launches_per_step = q(2)
    prefill_launches = q(3)

    # ---- dominant-kernel rooflines, measured live on this GPU ----
    hbm, tf_burst, tf_sus, src = peaks()
    att_ms, att_bytes = kernel_roofline_decode_attention(L, torch, dev)
    gemm_ms, gemm_flops = kernel_roofline_prefill_gemm(L, torch, dev)
    fa_ms, fa_flops = kernel_roofline_prefill_attention(L, torch, dev)
    L.b200_engine_destroy(eng)

    def stream_of(e):
        s = ctypes.c_void_p()
        check(L.b200_engine_stream(e, ctypes.byref(s)), "engine_stream")
        return torch.cuda.ExternalStream(s.value, device=dev)

    tp = tp_mx = ep_ds = ep_mx = None
    if dist and not args.no_ep:
        ep_ds = bench_ep(L, torch, dev, dist, world, rank, max(3, min(steps, 10)), warm, stream_of,
                         DEEPSEEK_V2_LITE, DS_BATCH, DS_CTX, "DeepSeek-V2-Lite")
        ep_mx = bench_ep(L, torch, dev, dist, world, rank, max(3, min(steps, 10)), warm, stream_of, MIXTRAL_8X7B,
                         MX_BATCH, MX_CTX, "Mixtral-8x7B")
    if dist and not args.no_tp:
        tp = bench_tp(L, torch, dev, dist, world, rank, steps, warm, stream_of, QWEN3_8B, PREFILL_SEQS, PREFILL_LEN,
                      DECODE_BATCH, DECODE_CTX, "one Qwen3-8B sharded over all ranks (latency-oriented); the headline "
                      "`value` is independent replicas (throughput-oriented)")
        if not args.no_mixtral:
            tp_mx = bench_tp(L, torch, dev, dist, world, rank, max(3, min(steps, 10)), warm, stream_of, MIXTRAL_8X7B,
                             MX_PREFILL_SEQS, MX_PREFILL_LEN, MX_BATCH, MX_CTX,
                             "one Mixtral-8x7B sharded over all ranks: every expert's width split, router replicated")
    vl = None if args.no_vl else bench_qwen3vl(L, torch, dev, max(3, min(steps, 10)), warm, stream_of)
    if vl:
        vl["text_layer"] = bench_qwen3vl_text_layer(L, torch, dev,
                                                    cpu=rank == 0 and world == 1 and not args.no_cpu_baseline)
    pp = None if args.no_vl else bench_preprocess(L, torch, dev, steps, warm,
                                                  cpu_baseline=rank == 0 and not args.no_cpu_baseline)
    mx = None if args.no_mixtral else bench_mixtral(L, torch, dev, max(3, min(steps, 10)), warm, stream_of)
    ds = None if args.no_deepseek else bench_deepseek(L, torch, dev, max(3, min(steps, 10)), warm, stream_of)
    for sec, name in ((mx, "mixtral"), (ds, "deepseek")):
        if sec and rank == 0 and world == 1 and not args.no_cpu_baseline:
            try:
                sec["cpu_baseline"] = cpu_moe_decode_baseline(name)
                sec["speedup_vs_cpu"] = sec["decode_tok_s"] / sec["cpu_baseline"]["value"]
            except Exception as e:  # the baseline is a report, never a reason to lose the GPU line
                sec["cpu_baseline"] = {"value": None, "error": str(e)[:200]}

    def kernel_line(fn, name):
        ms, nbytes = fn(L, torch, dev)
        return {"kernel": name, "bound": "hbm", "ms": ms, "bytes_per_launch": nbytes,
                "achieved": nbytes / (ms / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                "frac": nbytes / (ms / 1e3) / 1e9 / hbm, "peak_source": f"{src} copy bandwidth"}

    if mx:
        mx["kernel_roofline"] = kernel_line(kernel_roofline_moe_gemm,
                                            "grouped expert gate/up GEMM + SwiGLU, 64 rows over 8 x [28672, 4096]")
    if ds:
        ds["kernel_roofline"] = kernel_line(kernel_roofline_mla_decode,
                                            "mla_decode_kernel (+combine), batch 32 x 16 heads, context 4096")
        fa_ms2, fa_fl2 = kernel_roofline_mla_prefill_attention(L, torch, dev)
        ds["prefill_attention_roofline"] = {
            "kernel": "flash_prefill_tc_kernel<192, 128> (tcgen05), causal 2x4096, 16 heads", "bound": "tensor",
            "ms": fa_ms2, "achieved": fa_fl2 / (fa_ms2 / 1e3) / 1e12, "peak": tf_burst, "unit": "TFLOP/s",
            "frac": fa_fl2 / (fa_ms2 / 1e3) / 1e12 / tf_burst, "peak_source": f"{src} bf16 burst"}

    bw = bandwidth_kernels(L, torch, dev) if not args.no_bw_kernels else None
    dec_tok_s = world * DECODE_BATCH * steps / (dec_ms / 1e3)
    pf_tok_s = world * T * steps / (pf_ms / 1e3)
    result = {
        "metric": METRIC,
        "value": dec_tok_s,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warm,
        "ms_per_step": dec_ms / steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: token ids U[0,151936) seeded; random-init N(0,0.02) weights generated on device",
        "config": {
            "workload": "Qwen3-8B decode, batch 64 at context 2048 (paged KV, block 128), greedy; "
                        "prefill 8x2048 per step fills the cache",
            "model": "Qwen3-8B", "global_batch": world * DECODE_BATCH, "seq_len": DECODE_CTX,
            "decode_context": f"{DECODE_CTX}..{DECODE_CTX + warm + steps}",
            "parallelism": f"dp{world} (independent replicas)",
            "l2": "not flushed: each decode step streams 16 GB of weights + 19 GB of KV (> 126 MB L2)",
        },
        "prefill": {
            "value": pf_tok_s, "unit": "tok/s", "ms_per_step": pf_ms / steps, "tokens_per_step": T,
            "e2e_tok_s": world * T * max(1, min(steps, 3)) / (pf_e2e_ms / 1e3),
            "roofline": {"kernel": "gemm_tcgen05 gate/up + SwiGLU epilogue, M16384 N24576 K4096",
                         "bound": "tensor", "achieved": gemm_flops / (gemm_ms / 1e3) / 1e12, "peak": tf_burst,
                         "unit": "TFLOP/s", "frac": gemm_flops / (gemm_ms / 1e3) / 1e12 / tf_burst,
                         "peak_source": f"{src} bf16 burst", "ms": gemm_ms},
            "attention_roofline": {"kernel": "flash_prefill_tc_kernel (tcgen05), causal 8x2048, 32q/8kv, d128",
                                   "bound": "tensor", "achieved": fa_flops / (fa_ms / 1e3) / 1e12, "peak": tf_burst,
                                   "unit": "TFLOP/s", "frac": fa_flops / (fa_ms / 1e3) / 1e12 / tf_burst,
                                   "peak_source": f"{src} bf16 burst", "ms": fa_ms},
        },
        "roofline": {"kernel": "paged_decode_kernel (+combine), B64 ctx2048 32q/8kv", "bound": "hbm",
                     "achieved": att_bytes / (att_ms / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": att_bytes / (att_ms / 1e3) / 1e9 / hbm, "traffic": DECODE_ATTN_DRAM_BYTES,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch at this "
                                       "shape (profiles/paged_decode_b64_ctx2048.md)",
                     "peak_source": f"{src} copy bandwidth", "ms": att_ms, "bytes_per_launch": att_bytes},
        "e2e": {"value": world * DECODE_BATCH * steps / (dec_e2e_ms / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": DECODE_BATCH * 8 + DECODE_BATCH * 4, "d2h_bytes_per_step": DECODE_BATCH * 8,
                # the e2e steps run after the device-resident ones, with a host sync each step; under
                # sw_power_cap their SM clock can differ from the decode region's (clocks.decode_region_sm_mhz)
                "sm_mhz": e2e_clk.median()},
        "gpu_launches": launches_per_step * steps,
        "gpu_launches_note": f"{launches_per_step} kernels per decode step (CUDA graph); prefill step "
                             f"{prefill_launches}",
        "clocks": clocks,
    }
    if tp:
        result["tensor_parallel"] = tp
    if tp_mx:
        result["tensor_parallel_mixtral"] = tp_mx
    if ep_ds:
        result["expert_parallel_deepseek"] = ep_ds
    if ep_mx:
        result["expert_parallel_mixtral"] = ep_mx
    if vl:
        result["qwen3vl_embedding"] = vl
    if pp:
        result["image_preprocess"] = pp
    if mx:
        result["mixtral_8x7b"] = mx
    if ds:
        result["deepseek_v2_lite"] = ds
    if bw:
        result["bandwidth_kernels"] = bw
    if dist:
        # The sharded runs, compact, as the line's last key: speed-up / efficiency
        # against the one-GPU sections of this same run (tensor parallel: one
        # model's decode step, strong scaling; expert parallel: every rank its
        # own batch, weak scaling) and the sharded-vs-one-GPU parity verdict.
        mg = {"n": world}

        def entry(sec, one_ms=None, one_tok_s=None):
            e = {"decode_tok_s": round(sec["decode_tok_s"], 1), "ms": round(sec["decode_ms_per_step"], 3)}
            if one_ms:
                e["speedup_vs_1gpu"] = round(one_ms / sec["decode_ms_per_step"], 3)
                e["eff"] = round(one_ms / sec["decode_ms_per_step"] / world, 3)
            if one_tok_s:
                e["eff"] = round(sec["decode_tok_s"] / (world * one_tok_s), 3)
            par = sec.get("parity") or {}
            e["parity"] = par.get("parity")
            e["min_cos"] = par.get("min_cos")
            return e

        if tp:
            mg["tp_qwen3_8b"] = entry(tp, one_ms=dec_ms / steps)
        if tp_mx:
            mg["tp_mixtral"] = entry(tp_mx, one_ms=mx["decode_ms_per_step"] if mx else None)
        if ep_mx:
            mg["ep_mixtral"] = entry(ep_mx, one_tok_s=mx["decode_tok_s"] if mx else None)
        if ep_ds:
            mg["ep_deepseek"] = entry(ep_ds, one_tok_s=ds["decode_tok_s"] if ds else None)
        result["multi_gpu"] = mg
        dist.barrier()
    if rank == 0:
        if not args.no_cpu_baseline and world == 1:
            try:
                result["cpu_baseline"] = cpu_baseline()
            except Exception as e:  # the CPU leg must not sink the GPU number
                result["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
        print(json.dumps(result), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args, rank):
    if rank != 0:
        return
    # inputs built once; each step is one decode layer of the oracle, scaled to
    # the 36 layers + lm_head of a Qwen3-8B decode step
    layer, head = cpu_decode_layer_setup()
    for _ in range(args.warmup):
        layer()
    t0 = time.perf_counter()
    head()
    t_head = (time.perf_counter() - t0) * 8
    layer_s = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        layer()
        layer_s.append(time.perf_counter() - t0)
    # What ran: `steps` decode layers, one per step, each timed on its own.
    # The tok/s value is that per-layer time extrapolated to a whole decode
    # step (36 layers + lm_head); the extrapolated step time is reported
    # beside the measured one, never in its place.
    layer_mean = statistics.mean(layer_s)
    step_s = 36 * layer_mean + t_head
    val = DECODE_BATCH / step_s
    cb = {"kind": "port", "cores": blas_threads(),
          "sample": f"numpy fp32 oracle: one decode layer (batch 64, context 2048) per step, scaled to 36 layers "
                    f"+ lm_head (extrapolated); {layer_mean * 1e3:.1f} ms/layer"}
    out = {
        "metric": METRIC, "impl": "reference", "value": val, "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": layer_mean * 1e3, "step_unit": "one Qwen3-8B decode layer",
        "extrapolated": True, "ms_per_decode_step_extrapolated": step_s * 1e3, "lm_head_ms": t_head * 1e3,
        "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "Qwen3-8B decode, batch 64 at context 2048 (one layer timed per step; tok/s "
                               "extrapolated to 36 layers + lm_head)",
                   "model": "Qwen3-8B", "global_batch": DECODE_BATCH, "seq_len": DECODE_CTX,
                   "parallelism": "host CPU"},
        "cpu_baseline": {"kind": cb["kind"], "cores": cb["cores"], "sample": cb["sample"], "value": val},
        "e2e": {"value": val, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference (Ascend ATB) cannot run here; this is the repo's numpy restatement of the "
                "reference's CPU decoder-layer math (oracle/), timed on the host cores",
    }
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-vl", action="store_true", help="skip the Qwen3-VL-2B embedding section")
    ap.add_argument("--no-tp", action="store_true", help="skip the tensor-parallel sections (N > 1)")
    ap.add_argument("--no-ep", action="store_true", help="skip the expert-parallel sections (N > 1)")
    ap.add_argument("--vl-only", action="store_true", help="only the Qwen3-VL-2B embedding section")
    ap.add_argument("--no-mixtral", action="store_true", help="skip the Mixtral-8x7B section")
    ap.add_argument("--mixtral-only", action="store_true", help="only the Mixtral-8x7B section")
    ap.add_argument("--no-deepseek", action="store_true", help="skip the DeepSeek-V2-Lite section")
    ap.add_argument("--deepseek-only", action="store_true", help="only the DeepSeek-V2-Lite section")
    ap.add_argument("--no-bw-kernels", action="store_true", help="skip the bandwidth-bound kernel lines")
    ap.add_argument("--profile-kernel", choices=["decode_attention", "prefill_gemm", "prefill_attention", "mla_decode",
                                                 "moe_gemm", "image_preprocess", "decode_gemm", "bw_kernels",
                                                 "mla_prefill_attention"],
                    help="run only this kernel at its bench shape (3 warm-up + 3 launches), for ncu")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.profile_kernel:
        import torch

        from atb_llm_study_b200 import capi

        dev = torch.device("cuda", local_rank)
        if args.profile_kernel == "bw_kernels":
            print(json.dumps(bandwidth_kernels(capi.lib(), torch, dev, reps=3)))
            return
        fn = {"decode_attention": kernel_roofline_decode_attention, "prefill_gemm": kernel_roofline_prefill_gemm,
              "prefill_attention": kernel_roofline_prefill_attention, "mla_decode": kernel_roofline_mla_decode,
              "moe_gemm": kernel_roofline_moe_gemm, "image_preprocess": kernel_roofline_image_preprocess,
              "decode_gemm": kernel_roofline_decode_gemm,
              "mla_prefill_attention": kernel_roofline_mla_prefill_attention}[args.profile_kernel]
        ms, work = fn(capi.lib(), torch, dev, reps=3)
        print(json.dumps({"kernel": args.profile_kernel, "ms": ms, "work_per_launch": work}))
        return
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.vl_only or args.mixtral_only or args.deepseek_only:
        import torch

        from atb_llm_study_b200 import capi

        dev = torch.device("cuda", local_rank)
        torch.cuda.set_device(dev)
        L = capi.lib()

        def stream_of(e):
            s = ctypes.c_void_p()
            check(L.b200_engine_stream(e, ctypes.byref(s)), "engine_stream")
            return torch.cuda.ExternalStream(s.value, device=dev)

        fn = bench_qwen3vl if args.vl_only else bench_mixtral if args.mixtral_only else bench_deepseek
        res = fn(L, torch, dev, args.steps, args.warmup, stream_of)
        if args.vl_only:
            res["text_layer"] = bench_qwen3vl_text_layer(L, torch, dev, cpu=not args.no_cpu_baseline)
            res["image_preprocess"] = bench_preprocess(L, torch, dev, args.steps, args.warmup)
        elif not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_moe_decode_baseline("mixtral" if args.mixtral_only else "deepseek")
            res["speedup_vs_cpu"] = res["decode_tok_s"] / res["cpu_baseline"]["value"]
        print(json.dumps(res), flush=True)
        return
    run_b200(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
