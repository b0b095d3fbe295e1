// Decode chain: the projections of a dense GQA decoder layer between two decode
// attentions, as ONE persistent launch.
//
// A decode step streams every weight once, and a chain of separate launches
// (o GEMM, residual + RMSNorm, gate/up GEMM, SwiGLU reduce, down GEMM,
// residual + RMSNorm, next layer's qkv GEMM, QK-norm + rope + KV write) leaves
// HBM idle at every launch boundary: the tail of one kernel, the prologue of
// the next, the small reduce kernels in between.  Here one CTA per SM runs all
// of it.  The phases follow each other through grid-wide barriers (bounded
// waits), and each CTA's TMA producer keeps loading the NEXT projection's
// weight tiles into its shared-memory ring while the barrier before that
// projection is still pending; only the token tiles (this step's activations)
// wait for it.  So the weight stream never drains between projections.
//
// Roles per CTA (192 threads), as in the tcgen05 GEMM:
//   warp 0      TMA producer: per k-block a 128 x 64 weight tile at once and
//               the 64 x 64 token tile once its phase's inputs are complete
//   warp 1      TMEM allocation; one thread issues tcgen05.mma (M = 128
//               weight rows, N = 64 tokens, K = 16) into a double-buffered
//               TMEM accumulator
//   warps 2-5   epilogue: fp32 split-K partials from TMEM to global memory;
//               between projections the element-wise phases (residual +
//               RMSNorm, SwiGLU over the partials, QK RMSNorm + rope + paged
//               KV write), with the arithmetic of the separate kernels they
//               replace (splitk_residual_rmsnorm, splitk_reduce, qk_norm_rope)
// Every projection splits K so that its units spread over the SMs; a CTA
// with no unit left in a phase moves straight on to the next phase's weights.
// Grid barriers: an arrival counter (release add, acquire poll) that starts at
// zero each launch; the last CTA to leave resets it.  Every wait gives up
// after ~2 s, sets the device error word and a sticky abort word, and the
// kernel unwinds.  No TMA multicast (the library also runs in multi-GPU jobs).
#include <math.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "decode_chain.h"
#include "gemm.h"

using namespace b200;

namespace {

constexpr int BM = 128, BK = 64, BN = 64;
constexpr int kStages = 8;
constexpr int kABytes = BM * BK * 2;  // weight tile
constexpr int kBBytes = BN * BK * 2;  // token tile
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 192;
constexpr int kEpi = 128;  // epilogue threads (warps 2-5)
constexpr uint32_t kTmemCols = 2 * BN;
constexpr uint32_t kIdesc = idesc_bf16_f32(BM, BN);
constexpr int kSmem = kStages * kStageBytes + 1024 + 512;
constexpr int kMaxCh = 8;  // 16-byte chunks per epilogue thread in a row phase: H <= 8 * 8 * 128 = 8192

struct Phase {
  int tiles_m, kb_total, kb_per_split, splits, units;
  int64_t N;
  float* ws;  // [splits][T][N]
};

struct Params {
  int flags;
  int T;
  int64_t H, I;
  int nq, nkv, hd;
  float eps;
  Phase g[4];  // o, gate/up, down, qkv
  const __nv_bfloat16 *post_norm, *next_norm, *q_norm, *k_norm;
  __nv_bfloat16 *hidden, *normed, *act, *qkv;
  const float *cos_tab, *sin_tab;
  const int64_t* slots;
  __nv_bfloat16 *k_cache, *v_cache;
  int64_t num_blocks;
  int block_size;
  unsigned* sync;  // [0] barrier arrivals, [1] CTAs done, [2] abort (sticky)
  unsigned* err;
};

struct Maps {
  CUtensorMap w[4];  // weights [N, K], box 128 rows x 64
  CUtensorMap x[4];  // tokens [T, K], box 64 rows x 64
};

__device__ __forceinline__ bool phase_on(int flags, int g) {
  return g == 0 ? (flags & CHAIN_O) : g == 3 ? (flags & CHAIN_QKV) : (flags & CHAIN_MLP);
}
__device__ __forceinline__ bool later_on(int flags, int g) {
  for (int h = g + 1; h < 4; ++h)
    if (phase_on(flags, h)) return true;
  return false;
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acquire_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
constexpr int kMaxSplits = 8;  // split-K slices an element-wise phase reads (the plans use at most 4 here)
// generic-proxy writes of this thread -> visible to later TMA (async proxy) reads
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Poll the arrival counter (relaxed) until it reaches `target`, then one
// acquire fence; false on the time limit or when another CTA aborted (the
// abort word is then set here too).
__device__ bool wait_count(unsigned* sync, unsigned target, unsigned* err) {
  const uint64_t t0 = global_timer_ns();
#pragma unroll 1
  for (int i = 0;; ++i) {
    if (ld_relaxed_gpu(sync) >= target) {
      fence_acquire_gpu();
      return true;
    }
    if ((i & 63) == 63) {
      if (ld_relaxed_gpu(sync + 2)) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        raise_error(err, DEV_ERR_WAIT_TIMEOUT);
        atomicExch(sync + 2, 1u);
        return false;
      }
    }
  }
}

// Grid barrier `idx` for the 128 epilogue threads of every CTA: every thread
// makes its stores visible at GPU scope (and to the async proxy of later TMA
// reads), the CTA's threads meet, then one of them adds the CTA's arrival and
// polls for everyone's.
__device__ bool grid_barrier(const Params& p, int idx, int et) {
  fence_proxy_async_global();  // this thread's stores -> later TMA reads of other CTAs
  __threadfence();
  epi_sync();
  __shared__ int ok_s;
  if (et == 0) {
    red_release_add(p.sync, 1u);
    ok_s = wait_count(p.sync, (unsigned)(idx + 1) * gridDim.x, p.err) ? 1 : 0;
  }
  epi_sync();
  return ok_s != 0;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.f + __expf(-x)); }

// hidden[r] = bf16(hidden[r] + sum_s ws[s][r]); normed[r] = RMSNorm(hidden[r]) * w
// (w null: the residual add alone).  Rows r = blockIdx.x, + gridDim.x, ...
__device__ void res_norm_phase(const Params& p, const Phase& g, const __nv_bfloat16* w, int et, float* red) {
  const int64_t H = p.H, nchunk = H / 8;
#pragma unroll 1
  for (int r = blockIdx.x; r < p.T; r += gridDim.x) {
    float v[kMaxCh][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxCh; ++c) {
      const int64_t idx = et + (int64_t)c * kEpi;
      if (idx < nchunk) {
        __nv_bfloat16* hp = p.hidden + (int64_t)r * H + idx * 8;
        unpack8(__ldcg(reinterpret_cast<const uint4*>(hp)), v[c]);
#pragma unroll
        for (int s = 0; s < kMaxSplits; ++s) {  // unrolled: every slice's loads in flight together
          if (s < g.splits) {
            const float4* src = reinterpret_cast<const float4*>(g.ws + ((int64_t)s * p.T + r) * H + idx * 8);
            const float4 a = __ldcg(src), b = __ldcg(src + 1);
            v[c][0] += a.x; v[c][1] += a.y; v[c][2] += a.z; v[c][3] += a.w;
            v[c][4] += b.x; v[c][5] += b.y; v[c][6] += b.z; v[c][7] += b.w;
          }
        }
        const uint4 hb = pack8(v[c]);
        __stcg(reinterpret_cast<uint4*>(hp), hb);
        unpack8(hb, v[c]);  // normalise the stored (bf16) residual stream
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
      }
    }
    if (!w) continue;
    ss = warp_sum(ss);
    epi_sync();
    if ((et & 31) == 0) red[et >> 5] = ss;
    epi_sync();
    const float inv = rsqrtf((red[0] + red[1] + red[2] + red[3]) / (float)H + p.eps);
#pragma unroll
    for (int c = 0; c < kMaxCh; ++c) {
      const int64_t idx = et + (int64_t)c * kEpi;
      if (idx < nchunk) {
        float gw[8], o[8];
        unpack8(*reinterpret_cast<const uint4*>(w + idx * 8), gw);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = v[c][i] * inv * gw[i];
        __stcg(reinterpret_cast<uint4*>(p.normed + (int64_t)r * H + idx * 8), pack8(o));
      }
    }
  }
}

// act[t, f/2 ..] = silu(gate) * up over the gate/up partials (rows interleaved).
__device__ void swiglu_phase(const Params& p, const Phase& g, int et) {
  const int64_t N = g.N, n8 = N / 8, total = (int64_t)p.T * n8;
  const int64_t stride = (int64_t)gridDim.x * kEpi;
  constexpr int kItems = 4;  // items per thread per round, all their loads issued together
#pragma unroll 1
  for (int64_t it0 = (int64_t)blockIdx.x * kEpi + et; it0 < total; it0 += kItems * stride) {
    float v[kItems][8];
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = 0.f;
      const int64_t it = it0 + j * stride;
      if (it < total) {
        const int64_t t = it / n8, f0 = (it % n8) * 8;
#pragma unroll
        for (int s = 0; s < kMaxSplits; ++s) {
          if (s < g.splits) {
            const float4* src = reinterpret_cast<const float4*>(g.ws + ((int64_t)s * p.T + t) * N + f0);
            const float4 a = __ldcg(src), b = __ldcg(src + 1);
            v[j][0] += a.x; v[j][1] += a.y; v[j][2] += a.z; v[j][3] += a.w;
            v[j][4] += b.x; v[j][5] += b.y; v[j][6] += b.z; v[j][7] += b.w;
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int64_t it = it0 + j * stride;
      if (it < total) {
        const int64_t t = it / n8, f0 = (it % n8) * 8;
        uint2 o;
        o.x = pack2(silu_f(v[j][0]) * v[j][1], silu_f(v[j][2]) * v[j][3]);
        o.y = pack2(silu_f(v[j][4]) * v[j][5], silu_f(v[j][6]) * v[j][7]);
        __stcg(reinterpret_cast<uint2*>(p.act + t * p.I + f0 / 2), o);
      }
    }
  }
}

// Per (token, head) on one warp: the head's qkv projection summed from the
// partials; q / k: per-head RMSNorm (weights given) and the half rotation
// x*cos + cat(-x2, x1)*sin; k, v into the paged cache at slots[t]; every head
// into the qkv row (the decode attention reads q there).  Head dim 128.
__device__ void qk_rope_phase(const Params& p, const Phase& g, int et) {
  constexpr int HD = 128, E = HD / 32;
  const int lane = et & 31;
  const int nheads = p.nq + 2 * p.nkv;
  const int64_t QKV = (int64_t)nheads * HD;
  const int64_t items = (int64_t)p.T * nheads;
  const float sign = lane < 16 ? -1.f : 1.f;
#pragma unroll 1
  for (int64_t it = (int64_t)blockIdx.x * 4 + (et >> 5); it < items; it += (int64_t)gridDim.x * 4) {
    const int64_t t = it / nheads;
    const int h = (int)(it % nheads);
    float x[E] = {0, 0, 0, 0};
    const float* src = g.ws + t * QKV + (int64_t)h * HD + lane * E;
#pragma unroll
    for (int s = 0; s < kMaxSplits; ++s) {
      if (s < g.splits) {
        const float4 a = __ldcg(reinterpret_cast<const float4*>(src + (int64_t)s * p.T * QKV));
        x[0] += a.x; x[1] += a.y; x[2] += a.z; x[3] += a.w;
      }
    }
    __nv_bfloat16* hp = p.qkv + t * QKV + (int64_t)h * HD + lane * E;
    const bool is_q = h < p.nq, is_k = !is_q && h < p.nq + p.nkv;
    if (!is_q && !is_k) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        hp[e] = f2bf(x[e]);
        x[e] = bf2f(hp[e]);  // the cache holds the same bf16 value as qkv
      }
    } else {
      const __nv_bfloat16* nw = is_q ? p.q_norm : p.k_norm;
      if (nw) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) ss += x[e] * x[e];
        const float inv = rsqrtf(warp_sum(ss) / (float)HD + p.eps);
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = x[e] * inv * bf2f(nw[lane * E + e]);
      }
      float y[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
        y[e] = x[e] * p.cos_tab[t * HD + lane * E + e] + sign * partner * p.sin_tab[t * HD + lane * E + e];
      }
#pragma unroll
      for (int e = 0; e < E; ++e) {
        x[e] = y[e];
        hp[e] = f2bf(y[e]);
      }
    }
    if (!is_q && p.slots) {
      int64_t slot = p.slots[t];
      if (slot >= p.num_blocks * (int64_t)p.block_size) {
        if (lane == 0) raise_error(p.err, DEV_ERR_BAD_INDEX);
        slot = -1;
      }
      if (slot >= 0) {
        const int kh = is_k ? h - p.nq : h - p.nq - p.nkv;
        __nv_bfloat16* cache = is_k ? p.k_cache : p.v_cache;
        const int64_t blk = slot / p.block_size, off = slot % p.block_size;
        __nv_bfloat16* dst = cache + ((blk * p.nkv + kh) * p.block_size + off) * HD + lane * E;
#pragma unroll
        for (int e = 0; e < E; ++e) dst[e] = f2bf(x[e]);
      }
    }
  }
}

// The k-block sequence of this CTA: for every active phase, its units w =
// blockIdx.x, + gridDim.x, ... and their k-blocks.
struct Cursor {
  int g = -1, w = 0, kb = 0, kb1 = 0;
  int tm = 0, split = 0;
};

__device__ bool unit_begin(const Params& p, Cursor& c) {
  const Phase& ph = p.g[c.g];
  if (c.w >= ph.units) return false;
  c.split = c.w / ph.tiles_m;
  c.tm = c.w % ph.tiles_m;
  c.kb = c.split * ph.kb_per_split;
  c.kb1 = min(ph.kb_total, c.kb + ph.kb_per_split);
  return c.kb < c.kb1;
}

// Advance to the first k-block of the next non-empty unit; false at the end.
__device__ bool next_unit(const Params& p, Cursor& c, bool first) {
  if (!first) c.w += gridDim.x;
  while (true) {
    if (c.g >= 0 && c.g < 4 && unit_begin(p, c)) return true;
    if (c.g >= 0 && c.g < 4 && c.w < p.g[c.g].units) {  // empty K range: skip the unit
      c.w += gridDim.x;
      continue;
    }
    do {
      ++c.g;
    } while (c.g < 4 && !phase_on(p.flags, c.g));
    if (c.g >= 4) return false;
    c.w = blockIdx.x;
  }
}

__global__ void __launch_bounds__(kThreads, 1) decode_chain_kernel(const __grid_constant__ Maps maps,
                                                                   const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + kStages * kBBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(tmem_slot + 2);  // [4]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpi);
    }
    *abort_flag = 0;
    fence_barrier_init();
    for (int g = 0; g < 4; ++g) {
      tma_prefetch_desc(&maps.w[g]);
      tma_prefetch_desc(&maps.x[g]);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // the barrier each phase's token tiles wait for (-1: the previous kernel)
  int gate[4] = {-1, -1, -1, -1};
  {
    int nb = 0;
    bool prev = false;
    for (int g = 0; g < 4; ++g) {
      if (!phase_on(p.flags, g)) continue;
      gate[g] = prev ? nb - 1 : -1;
      nb += later_on(p.flags, g) ? 2 : 1;
      prev = true;
    }
  }

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      // k-blocks whose weight half is issued and whose token half waits for its
      // phase's barrier (at most kStages - 1 after each step)
      int pend_g[kStages], pend_kb[kStages], pend_stage[kStages];
      int np = 0, head = 0;
      bool passed[4] = {false, false, false, false};
      bool pdl_done = false;
      auto gate_ok = [&](int g, bool block) -> bool {
        if (passed[g]) return true;
        if (gate[g] < 0) {
          if (!block) return false;
          if (!pdl_done) pdl_wait();
          pdl_done = true;
        } else {
          const unsigned target = (unsigned)(gate[g] + 1) * gridDim.x;
          if (ld_relaxed_gpu(p.sync) < target) {
            if (!block) return false;
            if (!wait_count(p.sync, target, p.err)) return false;
          } else {
            fence_acquire_gpu();
          }
        }
        fence_proxy_async_global();
        passed[g] = true;
        return true;
      };
      auto issue_tokens = [&](bool block) -> bool {
        while (np > 0) {
          const int g = pend_g[head];
          if (!gate_ok(g, block)) return !block;  // non-blocking: leave it pending
          tma_load_2d(sB + pend_stage[head] * kBBytes, &maps.x[g], &full[pend_stage[head]], pend_kb[head] * BK, 0);
          head = (head + 1) % kStages;
          --np;
          if (!block) continue;
        }
        return true;
      };
      // Entering a phase whose inputs are not ready yet: pull this CTA's next
      // kPrefetchTiles weight tiles into L2 first, so HBM keeps streaming
      // through the barrier beyond what the shared-memory ring holds.
      constexpr int kPrefetchTiles = 24;
      auto prefetch_ahead = [&](Cursor from, int kb) {
        int n = 0;
        while (n < kPrefetchTiles) {
          for (; kb < from.kb1 && n < kPrefetchTiles; ++kb, ++n)
            tma_prefetch_l2_2d(&maps.w[from.g], kb * BK, from.tm * BM);
          if (!next_unit(p, from, false)) break;
          kb = from.kb;
        }
      };
      Cursor c;
      int stage = 0, last_g = -1;
      uint32_t phase = 0;
      bool ok = true;
      for (bool more = next_unit(p, c, true); more && ok; more = next_unit(p, c, false)) {
        if (c.g != last_g) {
          last_g = c.g;
          if (!passed[c.g] && gate[c.g] >= 0) prefetch_ahead(c, c.kb);
        }
        for (int kb = c.kb; kb < c.kb1 && ok; ++kb) {
          if (np == kStages - 1) ok = issue_tokens(true) && !*abort_flag;  // ring full of waiting k-blocks
          if (!ok) break;
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          tma_load_2d(sA + stage * kABytes, &maps.w[c.g], &full[stage], kb * BK, c.tm * BM);
          const int slot = (head + np) % kStages;
          pend_g[slot] = c.g;
          pend_kb[slot] = kb;
          pend_stage[slot] = stage;
          ++np;
          issue_tokens(false);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (ok) ok = issue_tokens(true);
      if (!ok) {
        *abort_flag = 1;
        atomicExch(p.sync + 2, 1u);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      Cursor c;
      int stage = 0, local = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (bool more = next_unit(p, c, true); more && ok && !*abort_flag; more = next_unit(p, c, false), ++local) {
        const int acc = local & 1;
        if (!mbar_wait(&tempty[acc], ((local >> 1) & 1) ^ 1, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = c.kb; kb < c.kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * kABytes), b0 = smem_u32(sB + stage * kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(d, smem_desc_k128(a0 + k * 32), smem_desc_k128(b0 + k * 32), kIdesc,
                      (kb > c.kb || k > 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&tfull[acc]);
      }
      if (!ok) {
        *abort_flag = 1;
        atomicExch(p.sync + 2, 1u);
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue + element-wise phases (warps 2-5) ----------------
    pdl_wait();  // partials / activations of the previous launches are complete
    const int et = threadIdx.x - 64;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int rit = q * 32 + lane;
    int local = 0, nb = 0;
    bool ok = true;
    for (int g = 0; g < 4 && ok; ++g) {
      if (!phase_on(p.flags, g)) continue;
      const Phase& ph = p.g[g];
      for (int w = blockIdx.x; w < ph.units && ok; w += gridDim.x) {
        const int split = w / ph.tiles_m, tm = w % ph.tiles_m;
        const int kb0 = split * ph.kb_per_split, kb1 = min(ph.kb_total, kb0 + ph.kb_per_split);
        if (kb0 >= kb1) continue;
        const int acc = local & 1;
        if (*abort_flag || !mbar_wait(&tfull[acc], (local >> 1) & 1, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int64_t row = (int64_t)tm * BM + rit;  // output feature
        float* base = ph.ws + (int64_t)split * p.T * ph.N;
#pragma unroll 1
        for (int ch = 0; ch < BN / 32; ++ch) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + ch * 32, r);
          tmem_ld_wait();
          if (row < ph.N) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int tok = ch * 32 + i;
              if (tok < p.T) __stcg(base + (int64_t)tok * ph.N + row, __uint_as_float(r[i]));
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        ++local;
      }
      if (!ok) break;
      ok = grid_barrier(p, nb++, et);  // this projection's partials are complete
      if (!ok) break;
      if (g == 0) res_norm_phase(p, ph, p.post_norm, et, red);
      else if (g == 1) swiglu_phase(p, ph, et);
      else if (g == 2) res_norm_phase(p, ph, p.next_norm, et, red);
      else qk_rope_phase(p, ph, et);
      if (later_on(p.flags, g)) ok = grid_barrier(p, nb++, et);  // its element-wise outputs are complete
    }
    if (!ok) {
      *abort_flag = 1;
      atomicExch(p.sync + 2, 1u);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0) {
    // the last CTA out resets the arrival counter for the next launch (every
    // CTA has stopped polling it once it counts itself out here)
    __threadfence();
    if (atomicAdd(p.sync + 1, 1u) == gridDim.x - 1) {
      atomicExch(p.sync, 0u);
      atomicExch(p.sync + 1, 0u);
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// bf16 [rows, cols] row-major (row stride = cols), box box_rows x 64, 128-byte swizzle
bool make_map(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev] > 0 ? n[dev] : 148;
}

// Split plan of one projection (the swapped decode GEMM's plan), partials bytes.
Phase plan_phase(int64_t T, int64_t N, int64_t K, int epi, int sms) {
  const GemmPlan g = plan_gemm(T, N, K, epi, sms);
  Phase ph;
  ph.tiles_m = (int)((N + BM - 1) / BM);
  ph.kb_total = (int)((K + BK - 1) / BK);
  ph.splits = std::max(1, g.splits);
  ph.kb_per_split = (ph.kb_total + ph.splits - 1) / ph.splits;
  ph.splits = (ph.kb_total + ph.kb_per_split - 1) / ph.kb_per_split;
  ph.units = ph.tiles_m * ph.splits;
  ph.N = N;
  ph.ws = nullptr;
  return ph;
}

int64_t up256(int64_t b) { return (b + 255) / 256 * 256; }

}  // namespace

namespace b200 {

int64_t chain_workspace_bytes(int64_t T, int64_t H, int64_t I, int nq, int nkv, int hd) {
  if (T <= 0 || T > BN || H <= 0 || H % 128 || H > 8192 || I <= 0 || I % 64 || hd != 128 || nq <= 0 || nkv <= 0)
    return 0;
  const int sms = sm_count();
  const int64_t QKV = (int64_t)(nq + 2 * nkv) * hd, AO = (int64_t)nq * hd;
  const Phase o = plan_phase(T, H, AO, B200_EPI_RESIDUAL, sms), gu = plan_phase(T, 2 * I, H, B200_EPI_SWIGLU, sms);
  const Phase dn = plan_phase(T, H, I, B200_EPI_RESIDUAL, sms), qk = plan_phase(T, QKV, H, B200_EPI_NONE, sms);
  return up256((int64_t)o.splits * T * H * 4) + up256((int64_t)gu.splits * T * 2 * I * 4) +
         up256((int64_t)dn.splits * T * H * 4) + up256((int64_t)qk.splits * T * QKV * 4);
}

int chain_launch(const ChainArgs& a, cudaStream_t stream) {
  const int64_t T = a.T, H = a.H, I = a.I;
  const int64_t need = chain_workspace_bytes(T, H, I, a.nq, a.nkv, a.hd);
  if (!need || !a.workspace || a.workspace_bytes < need || !a.sync || !a.hidden || !a.normed)
    return B200_ERROR_INVALID_PARAM;
  if ((a.flags & CHAIN_O) && (!a.w_o || !a.attn || !a.post_norm)) return B200_ERROR_INVALID_PARAM;
  if ((a.flags & CHAIN_MLP) && (!a.w_gu || !a.w_down || !a.act)) return B200_ERROR_INVALID_PARAM;
  if ((a.flags & CHAIN_QKV) && (!a.w_qkv || !a.qkv || !a.cos_tab || !a.sin_tab)) return B200_ERROR_INVALID_PARAM;
  if (!(a.flags & (CHAIN_O | CHAIN_MLP | CHAIN_QKV))) return B200_OK;
  const int sms = sm_count();
  const int64_t QKV = (int64_t)(a.nq + 2 * a.nkv) * a.hd, AO = (int64_t)a.nq * a.hd;
  Params p;
  p.flags = a.flags;
  p.T = (int)T;
  p.H = H;
  p.I = I;
  p.nq = a.nq;
  p.nkv = a.nkv;
  p.hd = a.hd;
  p.eps = a.eps;
  p.g[0] = plan_phase(T, H, AO, B200_EPI_RESIDUAL, sms);
  p.g[1] = plan_phase(T, 2 * I, H, B200_EPI_SWIGLU, sms);
  p.g[2] = plan_phase(T, H, I, B200_EPI_RESIDUAL, sms);
  p.g[3] = plan_phase(T, QKV, H, B200_EPI_NONE, sms);
  uint8_t* ws = static_cast<uint8_t*>(a.workspace);
  const int64_t ns[4] = {H, 2 * I, H, QKV};
  for (int g = 0; g < 4; ++g) {
    p.g[g].ws = reinterpret_cast<float*>(ws);
    ws += up256((int64_t)p.g[g].splits * T * ns[g] * 4);
  }
  p.post_norm = static_cast<const __nv_bfloat16*>(a.post_norm);
  p.next_norm = static_cast<const __nv_bfloat16*>(a.next_norm);
  p.q_norm = static_cast<const __nv_bfloat16*>(a.q_norm);
  p.k_norm = static_cast<const __nv_bfloat16*>(a.k_norm);
  p.hidden = static_cast<__nv_bfloat16*>(a.hidden);
  p.normed = static_cast<__nv_bfloat16*>(a.normed);
  p.act = static_cast<__nv_bfloat16*>(a.act);
  p.qkv = static_cast<__nv_bfloat16*>(a.qkv);
  p.cos_tab = a.cos_tab;
  p.sin_tab = a.sin_tab;
  p.slots = a.slots;
  p.k_cache = static_cast<__nv_bfloat16*>(a.k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(a.v_cache);
  p.num_blocks = a.num_blocks;
  p.block_size = a.block_size;
  p.sync = a.sync;
  int dev = 0;
  cudaGetDevice(&dev);
  p.err = error_word(dev);
  // every phase gets valid maps (unused phases point at a used operand)
  Maps m;
  const void* ws_[4] = {a.w_o, a.w_gu, a.w_down, a.w_qkv};
  const void* xs[4] = {a.attn, a.normed, a.act, a.normed};
  const int64_t ks[4] = {AO, H, I, H};
  for (int g = 0; g < 4; ++g) {
    const bool on = g == 0 ? (a.flags & CHAIN_O) : g == 3 ? (a.flags & CHAIN_QKV) : (a.flags & CHAIN_MLP);
    const void* w = on ? ws_[g] : a.hidden;
    const void* x = on ? xs[g] : a.hidden;
    const int64_t rows = on ? ns[g] : T, cols = on ? ks[g] : H;
    if (!make_map(&m.w[g], w, rows, cols, BM) || !make_map(&m.x[g], x, on ? T : T, cols, BN))
      return B200_ERROR_UNSUPPORTED;
  }
  static bool attr[64] = {false};
  if (dev < 0 || dev >= 64) return B200_ERROR_UNSUPPORTED;
  if (!attr[dev]) {
    if (cudaFuncSetAttribute(decode_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) !=
        cudaSuccess)
      return B200_ERROR_UNSUPPORTED;
    attr[dev] = true;
  }
  launch_kernel(decode_chain_kernel, dim3(sms), kThreads, kSmem, stream, m, p);
  B200_CHECK_LAUNCH();
  return B200_OK;
}

}  // namespace b200
