// Multi-head latent attention (DeepSeek-V2 / V2-Lite): the per-token latent
// preparation (compressed-KV RMSNorm, decoupled rope, latent cache write), the
// absorbed-latent decode attention over the paged latent cache, and the rope
// tables of YaRN-scaled frequencies.  The reference only declares MLA as a
// stub (MlaAttentionBuilder, atb_cpp_llm/src/components/common/
// attention_builder.h:60-69; AttnConfig.kv_lora_rank / q_lora_rank,
// atb_cpp_llm/include/atb_llm/layer_desc.h:47-49).
//
// Latent cache: [num_blocks * block_size, 576] bf16 per layer — per token the
// 512 normalised compressed-KV values then the 64 roped key dims shared by
// every head.  Decode runs "absorbed": the query of head h arrives already
// projected into the latent space (512 dims, W_UK folded into the query
// projection) followed by its 64 roped dims, so a head's score against token
// t is q_h . cache_t (576 dims) and its output o_h = sum_t p_t cache_t[:512]
// (W_UV is folded into the output projection).  All heads share the latent
// KV, so one CTA streams a token tile once for 16 heads — the 16 heads are the
// 16 rows of every tensor-core tile.
#include <math.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "mla.h"

using namespace b200;

namespace b200 {
unsigned* error_word(int device);
}

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kLat = 512;          // compressed-KV width (kv_lora_rank)
constexpr int kRope = 64;          // decoupled rope width (qk_rope_head_dim)
constexpr int kD = kLat + kRope;   // 576: latent cache row, absorbed query head
constexpr int kTile = 64;          // tokens per tile
constexpr int kStages = 2;
constexpr int kBoxBytes = kTile * 64 * 2;     // one TMA box: 64 tokens x 64 dims (8 KB)
constexpr int kTileBytes = (kD / 64) * kBoxBytes;  // 9 boxes = 72 KB
constexpr int kQBytes = (kD / 64) * 16 * 128;      // 16 heads x 576 dims in 9 boxes of 16 x 64
constexpr int kPBytes = 16 * kTile * 2;            // probabilities of one tile, bf16
constexpr int kThreads = 160;                      // warps 0-3 compute, warp 4 loads
constexpr int kProducer = 4;
constexpr int kSmem = 1024 + kStages * kTileBytes + kQBytes + 2 * kPBytes + 2 * 2 * 4 * 16 * 4 + 64;

// byte offset of 16-byte chunk c (0..71) of row r in a tile of 64-dim boxes
// (row pitch 128 B inside a box, 128-byte swizzle), boxes `box_bytes` apart
__device__ __forceinline__ uint32_t lat_off(int r, int c, int box_bytes) {
  return (uint32_t)((c >> 3) * box_bytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ void bar_compute() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

struct MlaParams {
  const __nv_bfloat16* q;  // [batch, q_stride]: head h at h*576 (512 latent + 64 rope)
  int64_t q_stride;
  const int32_t* block_tables;
  int max_blocks;
  const int32_t* context_lens;
  int nh, block_size;
  int64_t num_blocks;
  float scale_log2;
  int splits, tokens_per_split;
  __nv_bfloat16* out;  // [batch, out_stride]: head h at h*512
  int64_t out_stride;
  float* ws_o;    // [batch][nh][splits][512]
  float* ws_lse;  // [batch][nh][splits]
  unsigned* err;
};

// One CTA per (sequence, 16-head group, KV split).
__global__ void __launch_bounds__(kThreads) mla_decode_kernel(const __grid_constant__ CUtensorMap tmC,
                                                              const MlaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + kStages * kTileBytes;
  uint8_t* sP = sQ + kQBytes;                                            // [2][16 x 64] bf16
  float* red_m = reinterpret_cast<float*>(sP + 2 * kPBytes);            // [2][4][16]
  float* red_l = red_m + 2 * 4 * 16;                                     // [2][4][16]
  uint64_t* full = reinterpret_cast<uint64_t*>(red_l + 2 * 4 * 16);
  uint64_t* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);

  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, hg = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  int ctx = p.context_lens[b];
  if (ctx < 0 || ctx > p.max_blocks * p.block_size) {
    if (threadIdx.x == 0) raise_error(p.err, DEV_ERR_BAD_INDEX);
    ctx = max(0, min(ctx, p.max_blocks * p.block_size));
  }
  const int t_begin = split * p.tokens_per_split;
  const int t_end = min(ctx, t_begin + p.tokens_per_split);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + kTile - 1) / kTile : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kProducer) {
    // ---- producer: tile i = tokens t_begin + 64 i ... (within one cache block) ----
    int myblk = 0;
    for (int i = 0; i < ntiles; ++i) {
      const int s = i % kStages, round = i / kStages;
      bool ok = true;
      if (lane == 0 && round > 0) ok = mbar_wait(&empty[s], (round - 1) & 1, p.err);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      if ((i & 31) == 0) {
        const int ti = i + lane;
        int blk = 0;
        if (ti < ntiles) {
          blk = p.block_tables[(int64_t)b * p.max_blocks + (t_begin + ti * kTile) / p.block_size];
          if (blk < 0 || blk >= p.num_blocks) {
            raise_error(p.err, DEV_ERR_BAD_INDEX);
            blk = 0;
          }
        }
        myblk = blk;
      }
      const int blk = __shfl_sync(0xffffffffu, myblk, i & 31);
      if (lane == 0) {
        const int tok = t_begin + i * kTile;
        const int row = blk * p.block_size + tok % p.block_size;
        uint8_t* dst = smem + s * kTileBytes;
        mbar_arrive_expect_tx(&full[s], kTileBytes);
#pragma unroll 1
        for (int j = 0; j < kD / 64; ++j) tma_load_2d(dst + j * kBoxBytes, &tmC, &full[s], j * 64, row);
      }
      __syncwarp();
    }
    return;
  }

  // ---- compute warps 0-3: all 16 heads; S over tokens 16w..16w+15 of a tile,
  //      O over latent dims 128w..128w+127 ----
  // The 16 query heads of this group, 576 dims each, into the boxed layout,
  // while the TMA warp already streams the first two tiles.
  for (int i = threadIdx.x; i < 16 * (kD / 8); i += 128) {
    const int r = i / (kD / 8), c = i % (kD / 8);
    const uint4 val = *reinterpret_cast<const uint4*>(p.q + (int64_t)b * p.q_stride + (int64_t)(hg * 16 + r) * kD + c * 8);
    *reinterpret_cast<uint4*>(sQ + lat_off(r, c, 16 * 128)) = val;
  }
  bar_compute();
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  for (int i = 0; i < ntiles; ++i) {
    const int s = i % kStages, par = i & 1;
    const bool ok = mbar_wait(&full[s], (i / kStages) & 1, p.err);
    if (!ok) *abort_flag = 1;
    bar_compute();
    if (*abort_flag) break;
    const uint8_t* sC = smem + s * kTileBytes;
    // Four independent accumulator chains over the 36 k-steps (k-step kk feeds
    // chain kk % 4), summed at the end: one warp per scheduler issues these
    // MMAs back to back, and a single chain would wait out every MMA's latency.
    float sc4[4][2][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int j = 0; j < 2; ++j) sc4[a][j][0] = sc4[a][j][1] = sc4[a][j][2] = sc4[a][j][3] = 0.f;
#pragma unroll 4
    for (int kk = 0; kk < kD / 16; ++kk) {
      const int mat = lane >> 3;
      uint32_t qa[4], kb4[4];
      {
        const int r = (lane & 7) + ((mat & 1) ? 8 : 0);
        const int c = kk * 2 + (mat >> 1);
        ldmatrix_x4(qa, smem_u32(sQ + lat_off(r, c, 16 * 128)));
      }
      {
        const int r = warp * 16 + (mat >> 1) * 8 + (lane & 7);
        const int c = kk * 2 + (mat & 1);
        ldmatrix_x4(kb4, smem_u32(sC + lat_off(r, c, kBoxBytes)));
      }
      mma_bf16_16816(sc4[kk & 3][0], qa, kb4);
      mma_bf16_16816(sc4[kk & 3][1], qa, kb4 + 2);
    }
    float sc[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[j][e] = (sc4[0][j][e] + sc4[1][j][e]) + (sc4[2][j][e] + sc4[3][j][e]);
    // scale, mask, tile row max across the four warps
    const int kbase = t_begin + i * kTile + warp * 16;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kj = kbase + j * 8 + 2 * t4 + (e & 1);
        const float x = kj < t_end ? sc[j][e] * p.scale_log2 : -INFINITY;
        sc[j][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float* rm = red_m + par * 64;
    float* rl = red_l + par * 64;
    if (t4 == 0) {
      rm[warp * 16 + g] = mx[0];
      rm[warp * 16 + g + 8] = mx[1];
    }
    bar_compute();
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = g + 8 * r;
      const float tmax = fmaxf(fmaxf(rm[row], rm[16 + row]), fmaxf(rm[32 + row], rm[48 + row]));
      const float m_new = fmaxf(m_run[r], tmax);
      corr[r] = m_new == -INFINITY ? 1.f : exp2f(m_run[r] - m_new);
      m_run[r] = m_new;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float base = m_run[e >> 1] == -INFINITY ? 0.f : m_run[e >> 1];
        const float pv = exp2f(sc[j][e] - base);
        sc[j][e] = pv;
        rs[e >> 1] += pv;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
    }
    // P (bf16) rows = heads, columns = this warp's 16 tokens
    uint8_t* sp = sP + par * kPBytes;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int c = warp * 2 + j;
      *reinterpret_cast<uint32_t*>(sp + g * 128 + ((c ^ (g & 7)) << 4) + 4 * t4) = pack2(sc[j][0], sc[j][1]);
      *reinterpret_cast<uint32_t*>(sp + (g + 8) * 128 + ((c ^ ((g + 8) & 7)) << 4) + 4 * t4) =
          pack2(sc[j][2], sc[j][3]);
    }
    if (t4 == 0) {
      rl[warp * 16 + g] = rs[0];
      rl[warp * 16 + g + 8] = rs[1];
    }
    bar_compute();
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = g + 8 * r;
      l_run[r] = l_run[r] * corr[r] + (rl[row] + rl[16 + row] + rl[32 + row] + rl[48 + row]);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
    // O[:, 128w .. 128w+127] += P (16 x 64) . C[64 tokens, those dims]
#pragma unroll
    for (int kk = 0; kk < kTile / 16; ++kk) {
      const int mat = lane >> 3;
      uint32_t pa[4];
      {
        const int r = (lane & 7) + ((mat & 1) ? 8 : 0);
        const int c = kk * 2 + (mat >> 1);
        ldmatrix_x4(pa, smem_u32(sp + r * 128 + ((c ^ (r & 7)) << 4)));
      }
#pragma unroll
      for (int jp = 0; jp < 8; ++jp) {
        const int r = kk * 16 + (mat & 1) * 8 + (lane & 7);
        const int c = warp * 16 + 2 * jp + (mat >> 1);
        uint32_t vb[4];
        ldmatrix_x4_trans(vb, smem_u32(sC + lat_off(r, c, kBoxBytes)));
        mma_bf16_16816(o[2 * jp], pa, vb);
        mma_bf16_16816(o[2 * jp + 1], pa, vb + 2);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---- outputs: rows g, g+8 (heads), this warp's 128 latent dims ----
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int head = hg * 16 + g + 8 * r;
    const float L = l_run[r];
    const float inv = L > 0.f ? 1.f / L : 0.f;
    if (p.splits == 1) {
      __nv_bfloat16* orow = p.out + (int64_t)b * p.out_stride + (int64_t)head * kLat + warp * 128;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        *reinterpret_cast<uint32_t*>(orow + j * 8 + 2 * t4) = pack2(o[j][2 * r] * inv, o[j][2 * r + 1] * inv);
    } else {
      const int64_t base = ((int64_t)b * p.nh + head) * p.splits + split;
      float* wrow = p.ws_o + base * kLat + warp * 128;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        *reinterpret_cast<float2*>(wrow + j * 8 + 2 * t4) = make_float2(o[j][2 * r] * inv, o[j][2 * r + 1] * inv);
      if (warp == 0 && t4 == 0) p.ws_lse[base] = L > 0.f ? m_run[r] + log2f(L) : -INFINITY;
    }
  }
}

// out[b, h, :512] = sum_s w_s O_s, w_s = 2^(lse_s - max) / sum.
__global__ void mla_combine_kernel(const float* __restrict__ ws_o, const float* __restrict__ ws_lse, int nh,
                                   int splits, __nv_bfloat16* __restrict__ out, int64_t out_stride) {
  pdl_trigger();
  pdl_wait();
  const int bh = blockIdx.x;
  const int b = bh / nh, h = bh % nh;
  const float* lse = ws_lse + (int64_t)bh * splits;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, lse[s]);
  float den = 0.f;
  for (int s = 0; s < splits; ++s) den += lse[s] == -INFINITY ? 0.f : exp2f(lse[s] - M);
  for (int d = threadIdx.x; d < kLat; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s)
      if (lse[s] != -INFINITY) acc += exp2f(lse[s] - M) * ws_o[((int64_t)bh * splits + s) * kLat + d];
    out[(int64_t)b * out_stride + (int64_t)h * kLat + d] = f2bf(den > 0.f ? acc / den : 0.f);
  }
}

// Per token: c = RMSNorm(kv_a[:512]) * w, k_pe = rope(kv_a[512:576]), both into
// the latent cache row `slot` (and ckv_out / kpe_out when given); the 64 rope
// dims of every query head rotated in place.  Rope pairs are the interleaved
// (2i, 2i+1) of the projection, written de-interleaved: out[i] = x[2i] cos_i -
// x[2i+1] sin_i, out[32+i] = x[2i+1] cos_i + x[2i] sin_i (DeepSeek-V2's layout).
constexpr int kPrepThreads = 128;
__global__ void __launch_bounds__(kPrepThreads) mla_prep_kernel(
    __nv_bfloat16* q, int64_t q_stride, int64_t q_hs, int nh, int q_pe_off, const __nv_bfloat16* __restrict__ kva,
    int64_t kva_stride, const __nv_bfloat16* __restrict__ norm_w, float eps, const float* __restrict__ cos_tab,
    const float* __restrict__ sin_tab, const int64_t* __restrict__ slots, __nv_bfloat16* cache, int64_t num_slots,
    __nv_bfloat16* ckv_out, __nv_bfloat16* kpe_out, unsigned* err) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[kPrepThreads / 32];
  __shared__ float qpe[128 * kRope];  // up to 128 heads
  const int64_t t = blockIdx.x;
  const __nv_bfloat16* row = kva + t * kva_stride;
  // compressed KV: 4 values per thread
  float c[4];
  {
    const uint2 u = *reinterpret_cast<const uint2*>(row + threadIdx.x * 4);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 a = __bfloat1622float2(h2[0]), bb = __bfloat1622float2(h2[1]);
    c[0] = a.x, c[1] = a.y, c[2] = bb.x, c[3] = bb.y;
  }
  float ss = c[0] * c[0] + c[1] * c[1] + c[2] * c[2] + c[3] * c[3];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  // query rope inputs of every head into shared memory (rotated below, after the barrier)
  for (int i = threadIdx.x; i < nh * kRope; i += kPrepThreads) {
    const int h = i / kRope, d = i % kRope;
    qpe[i] = bf2f(q[t * q_stride + (int64_t)h * q_hs + q_pe_off + d]);
  }
  __syncthreads();
  const float rstd = rsqrtf((red[0] + red[1] + red[2] + red[3]) / (float)kLat + eps);
  int64_t slot = slots ? slots[t] : -1;
  if (slot >= num_slots) {
    if (threadIdx.x == 0) raise_error(err, DEV_ERR_BAD_INDEX);
    slot = -1;
  }
  {
    float w[4];
    const uint2 u = *reinterpret_cast<const uint2*>(norm_w + threadIdx.x * 4);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 a = __bfloat1622float2(h2[0]), bb = __bfloat1622float2(h2[1]);
    w[0] = a.x, w[1] = a.y, w[2] = bb.x, w[3] = bb.y;
    uint2 o;
    o.x = pack2(c[0] * rstd * w[0], c[1] * rstd * w[1]);
    o.y = pack2(c[2] * rstd * w[2], c[3] * rstd * w[3]);
    if (slot >= 0) *reinterpret_cast<uint2*>(cache + slot * kD + threadIdx.x * 4) = o;
    if (ckv_out) *reinterpret_cast<uint2*>(ckv_out + t * kLat + threadIdx.x * 4) = o;
  }
  const float* ct = cos_tab + t * kRope;
  const float* st = sin_tab + t * kRope;
  if (threadIdx.x < 32) {  // shared key rope dims
    const int i = threadIdx.x;
    const float x0 = bf2f(row[kLat + 2 * i]), x1 = bf2f(row[kLat + 2 * i + 1]);
    const __nv_bfloat16 lo = f2bf(x0 * ct[i] - x1 * st[i]), hi = f2bf(x1 * ct[i] + x0 * st[i]);
    if (slot >= 0) {
      cache[slot * kD + kLat + i] = lo;
      cache[slot * kD + kLat + 32 + i] = hi;
    }
    if (kpe_out) {
      kpe_out[t * kRope + i] = lo;
      kpe_out[t * kRope + 32 + i] = hi;
    }
  }
  for (int i = threadIdx.x; i < nh * 32; i += kPrepThreads) {
    const int h = i / 32, j = i % 32;
    const float x0 = qpe[h * kRope + 2 * j], x1 = qpe[h * kRope + 2 * j + 1];
    __nv_bfloat16* qh = q + t * q_stride + (int64_t)h * q_hs + q_pe_off;
    qh[j] = f2bf(x0 * ct[j] - x1 * st[j]);
    qh[32 + j] = f2bf(x1 * ct[j] + x0 * st[j]);
  }
}

// cos/sin [T, rot_dim] = cos/sin(pos * inv_freq[i mod rot_dim/2]) * mscale.
struct InvFreq {
  float v[128];
};
__global__ void rope_table_freqs_kernel(const int64_t* __restrict__ pos, int64_t T, int rot_dim, InvFreq inv,
                                        float mscale, float* __restrict__ cos_out, float* __restrict__ sin_out) {
  pdl_trigger();
  pdl_wait();
  const int half = rot_dim / 2;
  const int64_t gid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (gid >= T * half) return;
  const int64_t t = gid / half;
  const int i = (int)(gid % half);
  float s, c;
  sincosf((float)pos[t] * inv.v[i], &s, &c);
  cos_out[t * rot_dim + i] = cos_out[t * rot_dim + i + half] = c * mscale;
  sin_out[t * rot_dim + i] = sin_out[t * rot_dim + i + half] = s * mscale;
}

// C[m, n] = sum_k A(m, k) B(k, n) in fp32 with arbitrary strides, z-batched:
// folds W_UK into the query projection and W_UV into the output projection.
__global__ void absorb_kernel(const __nv_bfloat16* __restrict__ A, int64_t a_sm, int64_t a_sk, int64_t a_z,
                              const __nv_bfloat16* __restrict__ B, int64_t b_sk, int64_t b_sn, int64_t b_z,
                              __nv_bfloat16* __restrict__ C, int64_t c_sm, int64_t c_sn, int64_t c_z, int M, int N,
                              int K) {
  __shared__ float sa[32][33], sb[32][33];
  const int z = blockIdx.z;
  A += z * a_z;
  B += z * b_z;
  C += z * c_z;
  const int m0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < K; k0 += 32) {
    for (int r = ty; r < 32; r += 8) {
      const int m = m0 + r, k = k0 + tx;
      sa[r][tx] = (m < M && k < K) ? bf2f(A[m * a_sm + k * a_sk]) : 0.f;
      const int kb = k0 + r, n = n0 + tx;
      sb[r][tx] = (kb < K && n < N) ? bf2f(B[kb * b_sk + n * b_sn]) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = fmaf(sa[ty + 8 * j][kk], sb[kk][tx], acc[j]);
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int m = m0 + ty + 8 * j, n = n0 + tx;
    if (m < M && n < N) C[m * c_sm + n * c_sn] = f2bf(acc[j]);
  }
}

// kbuf[t, h, 0:128] = kvb[t, h*256 + 0:128]; kbuf[t, h, 128:192] = kpe[t, 0:64]
__global__ void mla_build_k_kernel(const __nv_bfloat16* __restrict__ kvb, int64_t kvb_stride,
                                   const __nv_bfloat16* __restrict__ kpe, __nv_bfloat16* __restrict__ kbuf, int nh) {
  pdl_trigger();
  pdl_wait();
  const int64_t t = blockIdx.x;
  for (int i = threadIdx.x; i < nh * 24; i += blockDim.x) {
    const int h = i / 24, c = i % 24;  // 24 chunks of 8 per 192-wide head
    const uint4 v = c < 16 ? *reinterpret_cast<const uint4*>(kvb + t * kvb_stride + (int64_t)h * 256 + c * 8)
                           : *reinterpret_cast<const uint4*>(kpe + t * kRope + (c - 16) * 8);
    *reinterpret_cast<uint4*>(kbuf + (t * nh + h) * 192 + c * 8) = v;
  }
}

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

// The latent cache as a 2-D [rows, 576] bf16 matrix, box = 64 tokens x 64 dims.
bool make_latent_tmap(CUtensorMap* m, const void* ptr, int64_t rows) {
  EncodeTiledFn f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[2] = {(cuuint64_t)kD, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(kD * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)kTile};
  cuuint32_t estr[2] = {1, 1};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int num_sms() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev] > 0 ? n[dev] : 148;
}

// KV splits.  One CTA fills an SM (172 KB of shared memory), so the time of a
// launch is about (waves of CTAs) x (tiles per split); each extra split also
// writes and combines a partial output.  Pick the split count minimising
// waves * tiles_per_split + splits / 2 (e.g. batch 32 x 16 heads at context
// 4096: 4 splits of 16 tiles, 128 CTAs in one wave, rather than 5 splits whose
// 160 CTAs need a second, nearly empty wave).
int mla_splits(int batch, int nh, int max_context) {
  const int64_t pairs = (int64_t)batch * (nh / 16);
  const int64_t sms = num_sms();
  const int ntiles = (max_context + kTile - 1) / kTile;
  const int max_split = std::max(1, std::min(32, ntiles / 2));
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= max_split; ++s) {
    const int tp = (ntiles + s - 1) / s;
    const int eff = (ntiles + tp - 1) / tp;
    const int64_t waves = (pairs * eff + sms - 1) / sms;
    const double cost = (double)waves * tp + (eff > 1 ? 0.5 * eff : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = eff;
    }
  }
  return best;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

namespace b200 {
// engine helper: C = A . B over strided bf16 views (fp32 accumulation), batched over z
int mla_absorb(const void* A, int64_t a_sm, int64_t a_sk, int64_t a_z, const void* B, int64_t b_sk, int64_t b_sn,
               int64_t b_z, void* C, int64_t c_sm, int64_t c_sn, int64_t c_z, int M, int N, int K, int batch,
               cudaStream_t st) {
  dim3 grid((unsigned)((N + 31) / 32), (unsigned)((M + 31) / 32), (unsigned)batch);
  absorb_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(A), a_sm, a_sk, a_z,
                                      static_cast<const __nv_bfloat16*>(B), b_sk, b_sn, b_z,
                                      static_cast<__nv_bfloat16*>(C), c_sm, c_sn, c_z, M, N, K);
  B200_CHECK_LAUNCH();
  return B200_OK;
}
int mla_build_k(const void* kvb, int64_t kvb_stride, const void* kpe, void* kbuf, int64_t T, int nh, cudaStream_t st) {
  if (!kvb || !kpe || !kbuf || T < 0 || nh <= 0 || kvb_stride < (int64_t)nh * 256 || kvb_stride % 8 || !al16(kvb) ||
      !al16(kpe) || !al16(kbuf))
    return B200_ERROR_INVALID_PARAM;
  if (T == 0) return B200_OK;
  launch_kernel(mla_build_k_kernel, dim3((unsigned)T), 128, 0, st, static_cast<const __nv_bfloat16*>(kvb), kvb_stride,
                static_cast<const __nv_bfloat16*>(kpe), static_cast<__nv_bfloat16*>(kbuf), nh);
  B200_CHECK_LAUNCH();
  return B200_OK;
}
}  // namespace b200

extern "C" int b200_rope_table_freqs(const int64_t* positions, int64_t T, int rot_dim, const float* inv_freq,
                                     float mscale, float* cos_out, float* sin_out, b200_stream_t stream) {
  if (!positions || !inv_freq || !cos_out || !sin_out || T < 0 || rot_dim <= 0 || rot_dim % 2 || rot_dim > 256)
    return B200_ERROR_INVALID_PARAM;
  if (T == 0) return B200_OK;
  InvFreq inv;
  for (int i = 0; i < rot_dim / 2; ++i) inv.v[i] = inv_freq[i];
  const int64_t n = T * (rot_dim / 2);
  launch_kernel(rope_table_freqs_kernel, dim3((unsigned)((n + 255) / 256)), 256, 0, stream, positions, T, rot_dim, inv,
                mscale, cos_out, sin_out);
  B200_CHECK_LAUNCH();
  return B200_OK;
}

extern "C" int b200_mla_prep(void* q, int64_t q_stride, int64_t q_head_stride, int num_heads, int q_rope_offset,
                             const void* kv_a, int64_t kv_a_stride, const void* kv_norm_weight, float eps,
                             const float* cos_tab, const float* sin_tab, const int64_t* slot_mapping,
                             void* latent_cache, int64_t num_slots, void* ckv_out, void* kpe_out, int64_t T,
                             b200_stream_t stream) {
  if (!q || !kv_a || !kv_norm_weight || !cos_tab || !sin_tab || T < 0 || num_heads <= 0 || num_heads > 128)
    return B200_ERROR_INVALID_PARAM;
  if (slot_mapping && (!latent_cache || num_slots <= 0)) return B200_ERROR_INVALID_PARAM;
  if (q_rope_offset < 0 || q_rope_offset + kRope > q_head_stride || q_stride < (int64_t)num_heads * q_head_stride ||
      kv_a_stride < kD || kv_a_stride % 4 || !al16(kv_a) || !al16(kv_norm_weight))
    return B200_ERROR_INVALID_PARAM;
  if ((latent_cache && !al16(latent_cache)) || (ckv_out && !al16(ckv_out))) return B200_ERROR_INVALID_PARAM;
  if (T == 0) return B200_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  launch_kernel(mla_prep_kernel, dim3((unsigned)T), kPrepThreads, 0, stream, static_cast<__nv_bfloat16*>(q), q_stride,
                q_head_stride, num_heads, q_rope_offset, static_cast<const __nv_bfloat16*>(kv_a), kv_a_stride,
                static_cast<const __nv_bfloat16*>(kv_norm_weight), eps, cos_tab, sin_tab, slot_mapping,
                static_cast<__nv_bfloat16*>(latent_cache), num_slots, static_cast<__nv_bfloat16*>(ckv_out),
                static_cast<__nv_bfloat16*>(kpe_out), b200::error_word(dev));
  B200_CHECK_LAUNCH();
  return B200_OK;
}

extern "C" int64_t b200_mla_decode_workspace_bytes(int batch, int num_heads, int max_context) {
  if (batch <= 0 || num_heads <= 0 || max_context <= 0) return 0;
  const int s = mla_splits(batch, num_heads, max_context);
  if (s <= 1) return 0;
  return (int64_t)batch * num_heads * s * (kLat + 1) * (int64_t)sizeof(float);
}

extern "C" int b200_mla_decode(const void* q, int64_t q_stride, const void* latent_cache,
                               const int32_t* block_tables, int max_blocks_per_seq, const int32_t* context_lens,
                               int batch, int num_heads, int block_size, int64_t num_blocks, float scale, void* out,
                               int64_t out_stride, void* workspace, int64_t workspace_bytes, int max_context,
                               b200_stream_t stream) {
  if (!q || !latent_cache || !block_tables || !context_lens || !out || batch < 0 || num_heads <= 0 ||
      num_heads % 16 || max_blocks_per_seq <= 0 || num_blocks <= 0 || max_context <= 0)
    return B200_ERROR_INVALID_PARAM;
  if (block_size <= 0 || block_size % kTile) return B200_ERROR_INVALID_PARAM;
  if (q_stride < (int64_t)num_heads * kD || out_stride < (int64_t)num_heads * kLat || q_stride % 8 || out_stride % 2 ||
      !al16(q) || !al16(latent_cache) || !al16(out))
    return B200_ERROR_INVALID_PARAM;
  if (batch == 0) return B200_OK;
  if (num_blocks * block_size > INT32_MAX || batch > 65535) return B200_ERROR_UNSUPPORTED;
  int splits = mla_splits(batch, num_heads, max_context);
  const int64_t need = (int64_t)batch * num_heads * splits * (kLat + 1) * (int64_t)sizeof(float);
  if (splits > 1 && (!workspace || workspace_bytes < need || !al16(workspace))) splits = 1;
  static bool smem_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !smem_set[dev]) {
    if (cudaFuncSetAttribute(mla_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
      return B200_ERROR_UNSUPPORTED;
    smem_set[dev] = true;
  }
  CUtensorMap tm;
  if (!make_latent_tmap(&tm, latent_cache, num_blocks * block_size)) return B200_ERROR_UNSUPPORTED;
  MlaParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_stride = q_stride;
  p.block_tables = block_tables;
  p.max_blocks = max_blocks_per_seq;
  p.context_lens = context_lens;
  p.nh = num_heads;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.scale_log2 = scale * kLog2e;
  p.splits = splits;
  const int per = (max_context + splits - 1) / splits;
  p.tokens_per_split = (per + kTile - 1) / kTile * kTile;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.ws_o = splits > 1 ? static_cast<float*>(workspace) : nullptr;
  p.ws_lse = splits > 1 ? p.ws_o + (int64_t)batch * num_heads * splits * kLat : nullptr;
  p.err = b200::error_word(dev);
  launch_kernel(mla_decode_kernel, dim3(batch, num_heads / 16, splits), kThreads, kSmem, stream, tm, p);
  B200_CHECK_LAUNCH();
  if (splits > 1) {
    launch_kernel(mla_combine_kernel, dim3(batch * num_heads), 128, 0, stream, (const float*)p.ws_o,
                  (const float*)p.ws_lse, num_heads, splits, p.out, out_stride);
    B200_CHECK_LAUNCH();
  }
  return B200_OK;
}
