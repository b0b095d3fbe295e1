// Attention kernels.
//
// flash_prefill: packed variable-length sequences, GQA, causal rule applied
//   in-kernel (no S x S mask tensor).  One CTA = 64 query rows of one head
//   (4 warps x 16 rows); K/V tiles of 64 keys stream through a 2-stage
//   cp.async ring in XOR-swizzled shared memory; QK^T and PV run on
//   m16n8k16 bf16 MMAs with an fp32 online softmax.
//
// paged_decode: one query token per sequence over a paged KV cache
//   [num_blocks, nkv, block_size, head_dim].  One CTA = (sequence, kv head,
//   KV split); the G = nq/nkv query heads that share the kv head form the
//   16-row MMA tile.  64-token K/V tiles arrive by TMA (128-byte swizzle,
//   3-stage mbarrier ring, bounded waits); each warp owns 16 keys of a tile and
//   keeps its own softmax state; warps and then splits are merged by
//   log-sum-exp.
#include <math.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "common.cuh"

using namespace b200;

namespace {

constexpr float kLog2e = 1.4426950408889634f;

// XOR swizzle of 16-byte chunk c in row r of a tile with CH chunks per row.
template <int CH>
__device__ __forceinline__ int swz(int r, int c) {
  if (CH >= 8) return c ^ (r & 7);
  if (CH == 4) return c ^ ((r >> 1) & 3);
  return c;
}

// ===========================================================================
// Prefill
// ===========================================================================
template <int HDK, int HDV>
struct PrefillCfg {
  static constexpr int BM = 64, BN = 64;
  static constexpr int CHK = HDK / 8, CHV = HDV / 8;  // 16-byte chunks per Q/K row, per V row
  static constexpr int TILE_K = BN * HDK * 2, TILE_V = BN * HDV * 2;
  static constexpr int SMEM = BM * HDK * 2 + 2 * TILE_K + 2 * TILE_V;  // Q + 2 stages x (K, V)
};

template <int HD>
__device__ __forceinline__ void load_tile_async(uint8_t* s, const __nv_bfloat16* base, int64_t stride, int row0,
                                                int nrows_valid) {
  constexpr int CH = HD / 8;
  constexpr int TOTAL = 64 * CH;
#pragma unroll
  for (int i = threadIdx.x; i < TOTAL; i += 128) {
    const int r = i / CH, c = i % CH;
    const bool ok = r < nrows_valid;
    const __nv_bfloat16* g = base + (int64_t)(row0 + (ok ? r : 0)) * stride + c * 8;
    cp_async_16(smem_u32(s + r * HD * 2 + swz<CH>(r, c) * 16), g, ok);
  }
}

// Flash attention over packed variable-length sequences (one CTA = 64 query
// rows of one head of one sequence, 4 warps x 16 rows).  Q/K heads are HDK
// wide and V/out heads HDV wide (they differ for MLA's decompressed heads:
// 128 + 64 rope dims against 128 value dims); every operand has its own row
// and head stride.
template <int HDK, int HDV, bool CAUSAL>
__global__ void __launch_bounds__(128) flash_prefill_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t q_stride, int64_t q_hs, const __nv_bfloat16* __restrict__ k,
    int64_t k_stride, int64_t k_hs, const __nv_bfloat16* __restrict__ v, int64_t v_stride, int64_t v_hs,
    __nv_bfloat16* __restrict__ out, int64_t out_stride, int64_t o_hs, const int32_t* __restrict__ cu_seqlens, int nq,
    int nkv, float scale_log2, int m_blocks) {
  using Cf = PrefillCfg<HDK, HDV>;
  constexpr int CHK = Cf::CHK, CHV = Cf::CHV;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK[2] = {smem + Cf::BM * HDK * 2, smem + Cf::BM * HDK * 2 + Cf::TILE_K};
  uint8_t* sV[2] = {smem + Cf::BM * HDK * 2 + 2 * Cf::TILE_K, smem + Cf::BM * HDK * 2 + 2 * Cf::TILE_K + Cf::TILE_V};

  pdl_trigger();
  pdl_wait();
  const int seq = blockIdx.z, h = blockIdx.y;
  const int mb = m_blocks - 1 - blockIdx.x;  // heaviest (latest) query blocks first
  const int s0 = cu_seqlens[seq], len = cu_seqlens[seq + 1] - s0;
  if (mb * Cf::BM >= len) return;
  const int kh = h / (nq / nkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;

  const __nv_bfloat16* qb = q + (int64_t)s0 * q_stride + h * q_hs;
  const __nv_bfloat16* kb = k + (int64_t)s0 * k_stride + kh * k_hs;
  const __nv_bfloat16* vb = v + (int64_t)s0 * v_stride + kh * v_hs;
  const int q0 = mb * Cf::BM;
  load_tile_async<HDK>(sQ, qb, q_stride, q0, min(Cf::BM, len - q0));
  cp_async_commit();

  const int n_blocks = CAUSAL ? min((len + Cf::BN - 1) / Cf::BN, mb + 1) : (len + Cf::BN - 1) / Cf::BN;
  load_tile_async<HDK>(sK[0], kb, k_stride, 0, min(Cf::BN, len));
  load_tile_async<HDV>(sV[0], vb, v_stride, 0, min(Cf::BN, len));
  cp_async_commit();

  cp_async_wait<1>();
  __syncthreads();
  uint32_t qf[HDK / 16][4];
#pragma unroll
  for (int kk = 0; kk < HDK / 16; ++kk) {
    const int mat = lane >> 3;
    const int r = warp * 16 + (lane & 7) + ((mat & 1) ? 8 : 0);
    const int c = kk * 2 + (mat >> 1);
    ldmatrix_x4(qf[kk], smem_u32(sQ + r * HDK * 2 + swz<CHK>(r, c) * 16));
  }

  float o[HDV / 8][4];
#pragma unroll
  for (int j = 0; j < HDV / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int qi0 = q0 + warp * 16 + g;  // query rows of this thread: qi0, qi0 + 8

  for (int nb = 0; nb < n_blocks; ++nb) {
    const int st = nb & 1;
    if (nb + 1 < n_blocks) {
      const int r0 = (nb + 1) * Cf::BN;
      load_tile_async<HDK>(sK[st ^ 1], kb, k_stride, r0, min(Cf::BN, len - r0));
      load_tile_async<HDV>(sV[st ^ 1], vb, v_stride, r0, min(Cf::BN, len - r0));
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HDK / 16; ++kk) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        const int mat = lane >> 3;
        const int r = (2 * jp + (mat >> 1)) * 8 + (lane & 7);
        const int c = kk * 2 + (mat & 1);
        uint32_t bf[4];
        ldmatrix_x4(bf, smem_u32(sK[st] + r * HDK * 2 + swz<CHK>(r, c) * 16));
        mma_bf16_16816(s[2 * jp], qf[kk], bf);
        mma_bf16_16816(s[2 * jp + 1], qf[kk], bf + 2);
      }
    }
    // mask + online softmax (two rows per thread: qi0 and qi0 + 8)
    const int kbase = nb * Cf::BN;
    const bool need_mask = (kbase + Cf::BN > len) || (CAUSAL && nb == mb);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[j][e] * scale_log2;
        if (need_mask) {
          const int kj = kbase + j * 8 + 2 * t4 + (e & 1);
          const int qi = qi0 + ((e >> 1) ? 8 : 0);
          if (kj >= len || (CAUSAL && kj > qi)) x = -INFINITY;
        }
        s[j][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float m_new = fmaxf(m_run[r], mx[r]);
      corr[r] = m_new == -INFINITY ? 1.f : exp2f(m_run[r] - m_new);
      m_run[r] = m_new;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float base = m_run[e >> 1] == -INFINITY ? 0.f : m_run[e >> 1];
        const float p = exp2f(s[j][e] - base);
        s[j][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) l_run[r] = l_run[r] * corr[r] + rs[r];
#pragma unroll
    for (int j = 0; j < HDV / 8; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int jp = 0; jp < HDV / 16; ++jp) {
        const int mat = lane >> 3;
        const int r = kk * 16 + (mat & 1) * 8 + (lane & 7);
        const int c = 2 * jp + (mat >> 1);
        uint32_t bf[4];
        ldmatrix_x4_trans(bf, smem_u32(sV[st] + r * HDV * 2 + swz<CHV>(r, c) * 16));
        mma_bf16_16816(o[2 * jp], pa, bf);
        mma_bf16_16816(o[2 * jp + 1], pa, bf + 2);
      }
    }
    __syncthreads();  // stage st may be overwritten by the next prefetch
  }

  // finalize: row sums across the quad, normalise, store
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = qi0 + r * 8;
    if (qi >= len) continue;
    const float inv = l_run[r] > 0.f ? 1.f / l_run[r] : 0.f;
    __nv_bfloat16* orow = out + (int64_t)(s0 + qi) * out_stride + h * o_hs;
#pragma unroll
    for (int j = 0; j < HDV / 8; ++j)
      *reinterpret_cast<uint32_t*>(orow + j * 8 + 2 * t4) = pack2(o[j][2 * r] * inv, o[j][2 * r + 1] * inv);
  }
}

// ===========================================================================
// Paged decode
// ===========================================================================
constexpr int kDecTile = 64;    // tokens per K/V tile
constexpr int kDecStages = 3;
constexpr int kDecHD = 128;
constexpr int kDecHalfBytes = kDecTile * 64 * 2;        // 64 tokens x 64 dims (one TMA box, 8 KB)
constexpr int kDecTileBytes = 2 * kDecHalfBytes;        // 64 tokens x 128 dims
constexpr int kDecStageBytes = 2 * kDecTileBytes;       // K + V
constexpr int kDecSmem = kDecStages * kDecStageBytes + 16 * kDecHD * 2 + 1024 + 128;

struct DecodeParams {
  const __nv_bfloat16* q;
  int64_t q_stride;
  const int32_t* block_tables;
  int max_blocks;
  const int32_t* context_lens;
  int nq, nkv, G, block_size;
  int64_t num_blocks;
  float scale_log2;
  int splits, tokens_per_split;
  __nv_bfloat16* out;
  int64_t out_stride;
  float* ws_o;    // [batch][nq][splits][HD]
  float* ws_lse;  // [batch][nq][splits]
  unsigned* err;
  // the next projection's weights, pulled into L2 by the CTAs of the last
  // wave (linear CTA index >= pf_first) after their last tile load
  const uint8_t* pf;
  int64_t pf_bytes;
  int pf_first;
};

// byte offset of 16-byte chunk c (0..15) of token row r inside a [64 x 128]
// tile stored as two TMA boxes of [64 x 64] with the 128-byte swizzle
__device__ __forceinline__ uint32_t dec_off(int r, int c) {
  return (uint32_t)((c >> 3) * kDecHalfBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

constexpr int kDecThreads = 160;  // warps 0-3 compute, warp 4 issues the TMA loads
constexpr int kDecProducerWarp = 4;

__global__ void __launch_bounds__(kDecThreads) paged_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                                                           const __grid_constant__ CUtensorMap tmV,
                                                           const DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + kDecStages * kDecStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sQ + 16 * kDecHD * 2);
  uint64_t* empty = full + kDecStages;

  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, kh = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  int ctx = p.context_lens[b];
  if (ctx < 0 || ctx > p.max_blocks * p.block_size) {
    if (threadIdx.x == 0) raise_error(p.err, DEV_ERR_BAD_INDEX);
    ctx = max(0, min(ctx, p.max_blocks * p.block_size));
  }
  const int t_begin = split * p.tokens_per_split;
  const int t_end = min(ctx, t_begin + p.tokens_per_split);
  const int ntiles = t_end > t_begin ? (t_end - t_begin + kDecTile - 1) / kDecTile : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDecStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_barrier_init();
  }
  // Q rows: heads kh*G .. kh*G+G-1, padded with zeros to 16 rows
  for (int i = threadIdx.x; i < 16 * 16; i += blockDim.x) {
    const int r = i >> 4, c = i & 15;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < p.G) val = *reinterpret_cast<const uint4*>(p.q + (int64_t)b * p.q_stride + (kh * p.G + r) * kDecHD + c * 8);
    *reinterpret_cast<uint4*>(sQ + r * 256 + ((c ^ (r & 7)) << 4)) = val;
  }
  __syncthreads();

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  if (warp == kDecProducerWarp) {
    // ---- producer warp: tile i of this split covers tokens t_begin + 64 i ... ----
    // Lane l fetches the block id of tile (32 k + l); lane 0 issues the loads.
    int myblk = 0;
    for (int i = 0; i < ntiles; ++i) {
      const int s = i % kDecStages, round = i / kDecStages;
      bool ok = true;
      if (lane == 0 && round > 0) ok = mbar_wait(&empty[s], (round - 1) & 1, p.err);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      if ((i & 31) == 0) {
        const int ti = i + lane;
        int blk = 0;
        if (ti < ntiles) {
          blk = p.block_tables[(int64_t)b * p.max_blocks + (t_begin + ti * kDecTile) / p.block_size];
          if (blk < 0 || blk >= p.num_blocks) {
            raise_error(p.err, DEV_ERR_BAD_INDEX);
            blk = 0;
          }
        }
        myblk = blk;
      }
      const int blk = __shfl_sync(0xffffffffu, myblk, i & 31);
      if (lane == 0) {
        const int tok = t_begin + i * kDecTile;
        const int row = (blk * p.nkv + kh) * p.block_size + tok % p.block_size;
        uint8_t* dst = smem + s * kDecStageBytes;
        mbar_arrive_expect_tx(&full[s], kDecStageBytes);
        tma_load_2d(dst, &tmK, &full[s], 0, row);
        tma_load_2d(dst + kDecHalfBytes, &tmK, &full[s], 64, row);
        tma_load_2d(dst + kDecTileBytes, &tmV, &full[s], 0, row);
        tma_load_2d(dst + kDecTileBytes + kDecHalfBytes, &tmV, &full[s], 64, row);
      }
      __syncwarp();
    }
    if (lane == 0 && p.pf) {
      const int64_t lin = blockIdx.x + (int64_t)gridDim.x * (blockIdx.y + (int64_t)gridDim.y * blockIdx.z);
      const int64_t total = (int64_t)gridDim.x * gridDim.y * gridDim.z;
      prefetch_l2_share(p.pf, p.pf_bytes, lin - p.pf_first, total - p.pf_first);
    }
  } else {
  // ---- compute warps 0-3 ----
  uint32_t qf[8][4];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int mat = lane >> 3;
    const int r = (lane & 7) + ((mat & 1) ? 8 : 0);
    const int c = kk * 2 + (mat >> 1);
    ldmatrix_x4(qf[kk], smem_u32(sQ + r * 256 + ((c ^ (r & 7)) << 4)));
  }

  for (int i = 0; i < ntiles; ++i) {
    const int s = i % kDecStages;
    if (!mbar_wait(&full[s], (i / kDecStages) & 1, p.err)) break;
    const uint8_t* sK = smem + s * kDecStageBytes;
    const uint8_t* sV = sK + kDecTileBytes;
    // this warp's 16 keys: rows warp*16 .. +15 of the tile
    float sc[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int mat = lane >> 3;
      const int r = warp * 16 + (mat >> 1) * 8 + (lane & 7);
      const int c = kk * 2 + (mat & 1);
      uint32_t bf[4];
      ldmatrix_x4(bf, smem_u32(sK + dec_off(r, c)));
      mma_bf16_16816(sc[0], qf[kk], bf);
      mma_bf16_16816(sc[1], qf[kk], bf + 2);
    }
    const int kbase = t_begin + i * kDecTile + warp * 16;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kj = kbase + j * 8 + 2 * t4 + (e & 1);
        float x = kj < t_end ? sc[j][e] * p.scale_log2 : -INFINITY;
        sc[j][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float m_new = fmaxf(m_run[r], mx[r]);
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
    for (int r = 0; r < 2; ++r) l_run[r] = l_run[r] * corr[r] + rs[r];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
    uint32_t pa[4];
    pa[0] = pack2(sc[0][0], sc[0][1]);
    pa[1] = pack2(sc[0][2], sc[0][3]);
    pa[2] = pack2(sc[1][0], sc[1][1]);
    pa[3] = pack2(sc[1][2], sc[1][3]);
#pragma unroll
    for (int jp = 0; jp < 8; ++jp) {
      const int mat = lane >> 3;
      const int r = warp * 16 + (mat & 1) * 8 + (lane & 7);
      const int c = 2 * jp + (mat >> 1);
      uint32_t bf[4];
      ldmatrix_x4_trans(bf, smem_u32(sV + dec_off(r, c)));
      mma_bf16_16816(o[2 * jp], pa, bf);
      mma_bf16_16816(o[2 * jp + 1], pa, bf + 2);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  }  // compute warps

  // ---- merge the 4 compute warps (each has its own m, l, O over its keys) ----
  __syncthreads();
  float* sm_m = reinterpret_cast<float*>(smem);          // [4][16]
  float* sm_l = sm_m + 64;                               // [4][16]
  float* sm_o = sm_l + 64;                               // [16][128] fp32 accumulator
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  if (t4 == 0 && warp < 4) {
    sm_m[warp * 16 + g] = m_run[0];
    sm_m[warp * 16 + g + 8] = m_run[1];
    sm_l[warp * 16 + g] = l_run[0];
    sm_l[warp * 16 + g + 8] = l_run[1];
  }
  for (int i = threadIdx.x; i < 16 * kDecHD; i += blockDim.x) sm_o[i] = 0.f;
  __syncthreads();
  float fac[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = g + r * 8;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w * 16 + row]);
    fac[r] = (m_run[r] == -INFINITY) ? 0.f : exp2f(m_run[r] - M);
  }
  for (int w = 0; w < 4; ++w) {
    if (warp == w) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        sm_o[g * kDecHD + j * 8 + 2 * t4] += o[j][0] * fac[0];
        sm_o[g * kDecHD + j * 8 + 2 * t4 + 1] += o[j][1] * fac[0];
        sm_o[(g + 8) * kDecHD + j * 8 + 2 * t4] += o[j][2] * fac[1];
        sm_o[(g + 8) * kDecHD + j * 8 + 2 * t4 + 1] += o[j][3] * fac[1];
      }
    }
    __syncthreads();
  }
  // row totals: M (log2 domain) and L = sum_w l_w * 2^(m_w - M)
  for (int i = threadIdx.x; i < p.G * kDecHD; i += blockDim.x) {
    const int row = i / kDecHD, d = i % kDecHD;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w * 16 + row]);
    float L = 0.f;
    for (int w = 0; w < 4; ++w)
      if (sm_m[w * 16 + row] != -INFINITY) L += sm_l[w * 16 + row] * exp2f(sm_m[w * 16 + row] - M);
    const int head = kh * p.G + row;
    const float val = sm_o[row * kDecHD + d];
    if (p.splits == 1) {
      p.out[(int64_t)b * p.out_stride + head * kDecHD + d] = f2bf(L > 0.f ? val / L : 0.f);
    } else {
      const int64_t base = ((int64_t)b * p.nq + head) * p.splits + split;
      p.ws_o[base * kDecHD + d] = L > 0.f ? val / L : 0.f;
      if (d == 0) p.ws_lse[base] = L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
}

// out[b, h] = sum_s w_s O_s with w_s = 2^(lse_s - max) / sum (lse in log2 units)
__global__ void decode_combine_kernel(const float* __restrict__ ws_o, const float* __restrict__ ws_lse, int nq,
                                      int splits, __nv_bfloat16* __restrict__ out, int64_t out_stride) {
  pdl_trigger();
  pdl_wait();
  const int bh = blockIdx.x;  // b * nq + h
  const int b = bh / nq, h = bh % nq;
  const float* lse = ws_lse + (int64_t)bh * splits;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, lse[s]);
  float den = 0.f;
  for (int s = 0; s < splits; ++s) den += lse[s] == -INFINITY ? 0.f : exp2f(lse[s] - M);
  const int d = threadIdx.x;  // 128 threads
  float acc = 0.f;
  for (int s = 0; s < splits; ++s)
    if (lse[s] != -INFINITY) acc += exp2f(lse[s] - M) * ws_o[((int64_t)bh * splits + s) * kDecHD + d];
  out[(int64_t)b * out_stride + h * kDecHD + d] = f2bf(den > 0.f ? acc / den : 0.f);
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

// The cache viewed as a 2-D [rows, 128] bf16 matrix, box = 64 rows x 64 dims.
bool make_cache_tmap(CUtensorMap* m, const void* ptr, int64_t rows) {
  EncodeTiledFn f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[2] = {(cuuint64_t)kDecHD, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(kDecHD * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)kDecTile};
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

// Most splits a decode may use at this context: >= 4 tiles per split, <= 32.
int decode_max_splits(int max_context) {
  return std::max(1, std::min(32, (max_context + 4 * kDecTile - 1) / (4 * kDecTile)));
}

// KV splits per (sequence, kv head).  Splitting costs a CTA prologue per split,
// partial outputs and the combine pass, which measured more than the tail of
// a partly filled last wave (batch 64 x 8 kv heads at context 2048: 95 us
// unsplit, 114 us with 2 splits, 125 us with 4).  So split only when the
// (sequence, kv head) pairs cannot occupy every SM: aim for two CTAs per SM.
int decode_splits(int batch, int nkv, int max_context) {
  static const int forced = [] {  // tuning override: B200_DECODE_SPLITS=<n>
    const char* v = std::getenv("B200_DECODE_SPLITS");
    return v ? std::atoi(v) : 0;
  }();
  if (forced > 0) return std::min(forced, decode_max_splits(max_context));
  const int64_t pairs = (int64_t)batch * nkv;
  const int64_t sms = num_sms();
  if (pairs >= sms) return 1;
  const int64_t want = (2 * sms + pairs - 1) / pairs;
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, decode_max_splits(max_context)));
}

// The split-KV plan of one decode launch: the split count decode_splits picks,
// rounded so every split covers whole K/V tiles, the tokens each split covers
// and the fp32 scratch the splits need (per query head and split: 128 partial
// outputs + one log-sum-exp).  b200_paged_decode, its allocation-free variant
// and the workspace query all size from this one plan.
struct DecodePlan {
  int splits;
  int tokens_per_split;
  int64_t scratch_bytes;  // 0 when unsplit
};

DecodePlan decode_plan(int batch, int nq, int nkv, int max_context) {
  DecodePlan d;
  const int ctx = std::max(1, max_context);
  const int want = decode_splits(batch, nkv, ctx);
  const int tiles_total = (ctx + kDecTile - 1) / kDecTile;
  const int tiles_per_split = (tiles_total + want - 1) / want;
  d.splits = (tiles_total + tiles_per_split - 1) / tiles_per_split;
  d.tokens_per_split = tiles_per_split * kDecTile;
  d.scratch_bytes = d.splits > 1 ? (int64_t)batch * nq * d.splits * (kDecHD + 1) * (int64_t)sizeof(float) : 0;
  return d;
}

// Opt one kernel (a distinct template argument per kernel) into large dynamic
// shared memory, once per device.
template <auto Kernel>
bool set_smem(int bytes) {
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return false;
  if (!done[dev]) done[dev] = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess;
  return done[dev];
}

template <int HDK, int HDV, bool CAUSAL>
int launch_prefill(const void* q, int64_t qs, int64_t qhs, const void* k, int64_t ks, int64_t khs, const void* v,
                   int64_t vs, int64_t vhs, void* out, int64_t os, int64_t ohs, const int32_t* cu, int num_seqs,
                   int max_seqlen, int nq, int nkv, float scale, cudaStream_t st) {
  using Cf = PrefillCfg<HDK, HDV>;
  auto kern = flash_prefill_kernel<HDK, HDV, CAUSAL>;
  if (!set_smem<flash_prefill_kernel<HDK, HDV, CAUSAL>>(Cf::SMEM)) return B200_ERROR_UNSUPPORTED;
  const int mblocks = (max_seqlen + 63) / 64;
  dim3 grid(mblocks, nq, num_seqs);
  launch_kernel(kern, grid, 128, Cf::SMEM, st, static_cast<const __nv_bfloat16*>(q), qs, qhs,
                static_cast<const __nv_bfloat16*>(k), ks, khs, static_cast<const __nv_bfloat16*>(v), vs, vhs,
                static_cast<__nv_bfloat16*>(out), os, ohs, cu, nq, nkv, scale * kLog2e, mblocks);
  B200_CHECK_LAUNCH();
  return B200_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int b200_flash_prefill_ex(const void* q, int64_t q_stride, int64_t q_head_stride, const void* k,
                                     int64_t k_stride, int64_t k_head_stride, const void* v, int64_t v_stride,
                                     int64_t v_head_stride, void* out, int64_t out_stride, int64_t out_head_stride,
                                     const int32_t* cu_seqlens, int num_seqs, int max_seqlen, int nq, int nkv,
                                     int head_dim_qk, int head_dim_v, float scale, int causal, b200_stream_t stream) {
  if (!q || !k || !v || !out || !cu_seqlens || num_seqs < 0 || max_seqlen < 0 || nq <= 0 || nkv <= 0 || nq % nkv)
    return B200_ERROR_INVALID_PARAM;
  for (int64_t s : {q_stride, q_head_stride, k_stride, k_head_stride, v_stride, v_head_stride, out_stride,
                    out_head_stride})
    if (s < 0 || s % 8) return B200_ERROR_INVALID_PARAM;
  if (!al16(q) || !al16(k) || !al16(v) || !al16(out)) return B200_ERROR_INVALID_PARAM;
  if (q_stride < (int64_t)(nq - 1) * q_head_stride + head_dim_qk ||
      k_stride < (int64_t)(nkv - 1) * k_head_stride + head_dim_qk ||
      v_stride < (int64_t)(nkv - 1) * v_head_stride + head_dim_v ||
      out_stride < (int64_t)(nq - 1) * out_head_stride + head_dim_v)
    return B200_ERROR_INVALID_PARAM;
  if (num_seqs == 0 || max_seqlen == 0) return B200_OK;
  if (num_seqs > 65535 || nq > 65535) return B200_ERROR_UNSUPPORTED;
#define B200_PF(HK, HV)                                                                                          \
  return causal ? launch_prefill<HK, HV, true>(q, q_stride, q_head_stride, k, k_stride, k_head_stride, v, v_stride, \
                                               v_head_stride, out, out_stride, out_head_stride, cu_seqlens,        \
                                               num_seqs, max_seqlen, nq, nkv, scale, stream)                     \
                : launch_prefill<HK, HV, false>(q, q_stride, q_head_stride, k, k_stride, k_head_stride, v, v_stride, \
                                                v_head_stride, out, out_stride, out_head_stride, cu_seqlens,       \
                                                num_seqs, max_seqlen, nq, nkv, scale, stream)
  if (head_dim_qk == head_dim_v) {
    switch (head_dim_qk) {
      case 16: B200_PF(16, 16);
      case 32: B200_PF(32, 32);
      case 64: B200_PF(64, 64);
      case 128: B200_PF(128, 128);
      default: return B200_ERROR_UNSUPPORTED;
    }
  }
  if (head_dim_qk == 192 && head_dim_v == 128) B200_PF(192, 128);
  return B200_ERROR_UNSUPPORTED;
#undef B200_PF
}

extern "C" int b200_flash_prefill(const void* q, int64_t q_stride, const void* k, const void* v, int64_t kv_stride,
                                  void* out, int64_t out_stride, const int32_t* cu_seqlens, int num_seqs,
                                  int max_seqlen, int nq, int nkv, int head_dim, float scale, int causal,
                                  b200_stream_t stream) {
  if (head_dim <= 0) return B200_ERROR_INVALID_PARAM;
  return b200_flash_prefill_ex(q, q_stride, head_dim, k, kv_stride, head_dim, v, kv_stride, head_dim, out, out_stride,
                               head_dim, cu_seqlens, num_seqs, max_seqlen, nq, nkv, head_dim, head_dim, scale, causal,
                               stream);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of b200_paged_decode.
//
// Its split-KV scratch (per-split partial outputs and log-sum-exps) lives in
// the file-scope array below instead of a caller-provided workspace.  Every
// GPU that loads this library holds the array until the process exits.  Host
// code cannot use the array's name as a device address, so the first call on
// each device looks the address up with cudaGetSymbolAddress (with that device
// current) and caches it; all later calls on that device reuse it.
// ---------------------------------------------------------------------------
static constexpr int64_t kNoAllocScratchBytes = 8ll << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_paged_decode_scratch[kNoAllocScratchBytes];

namespace {

// Device address of g_paged_decode_scratch on the current device (nullptr on
// failure).  Entries are atomics: host threads that race on a device's first
// call each look the address up and store the same value.  A cached address
// does not survive cudaDeviceReset (the array is re-created with the context).
void* noalloc_scratch(cudaError_t* err) {
  static std::atomic<void*> ptrs[64];
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= 64) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  void* cached = ptrs[dev].load(std::memory_order_acquire);
  if (!cached) {
    *err = cudaGetSymbolAddress(&cached, g_paged_decode_scratch);
    if (*err != cudaSuccess) return nullptr;
    ptrs[dev].store(cached, std::memory_order_release);
  }
  return cached;
}

}  // namespace

extern "C" int64_t b200_paged_decode_noalloc_max_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int b200_paged_decode_noalloc(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                                         const int32_t* block_tables, int max_blocks_per_seq,
                                         const int32_t* context_lens, int batch, int nq, int nkv, int head_dim,
                                         int block_size, int64_t num_blocks, float scale, void* out,
                                         int64_t out_stride, int max_context, b200_stream_t stream) {
  // The argument checks b200_paged_decode makes before its plan, in the same
  // order, so both entry points return the same code for the same bad call.
  if (!q || !k_cache || !v_cache || !block_tables || !context_lens || !out || batch < 0 || nq <= 0 || nkv <= 0 ||
      nq % nkv || max_blocks_per_seq <= 0 || num_blocks <= 0 || max_context < 0)
    return B200_ERROR_INVALID_PARAM;
  if (head_dim != kDecHD || (block_size != 64 && block_size != 128) || nq / nkv > 16) return B200_ERROR_UNSUPPORTED;
  // Reject, before any launch, a problem whose split-KV scratch exceeds the
  // array: the same plan b200_paged_decode runs, so a call that passes here
  // is never silently run unsplit for want of scratch.
  if (batch > 0 && decode_plan(batch, nq, nkv, max_context).scratch_bytes > kNoAllocScratchBytes)
    return B200_ERROR_INVALID_PARAM;
  cudaError_t e = cudaSuccess;
  void* scratch = noalloc_scratch(&e);
  if (!scratch) return B200_ERROR_CUDA_BASE - (int)e;
  return b200_paged_decode(q, q_stride, k_cache, v_cache, block_tables, max_blocks_per_seq, context_lens, batch, nq,
                           nkv, head_dim, block_size, num_blocks, scale, out, out_stride, scratch,
                           kNoAllocScratchBytes, max_context, stream);
}

extern "C" int64_t b200_paged_decode_workspace_bytes(int batch, int nq, int head_dim, int max_context) {
  if (batch <= 0 || nq <= 0 || head_dim != kDecHD || max_context <= 0) return 0;
  // the split count depends on nkv, which this query does not take: size for
  // the most splits any kv-head count can select at this context
  const int s = decode_max_splits(max_context);
  if (s <= 1) return 0;
  return (int64_t)batch * nq * s * (kDecHD + 1) * (int64_t)sizeof(float) + 256;
}

namespace b200 {
int paged_decode_launch(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                        const int32_t* block_tables, int max_blocks_per_seq, const int32_t* context_lens, int batch,
                        int nq, int nkv, int head_dim, int block_size, int64_t num_blocks, float scale, void* out,
                        int64_t out_stride, void* workspace, int64_t workspace_bytes, int max_context,
                        cudaStream_t stream, const void* prefetch, int64_t prefetch_bytes) {
  if (!q || !k_cache || !v_cache || !block_tables || !context_lens || !out || batch < 0 || nq <= 0 || nkv <= 0 ||
      nq % nkv || max_blocks_per_seq <= 0 || num_blocks <= 0 || max_context < 0)
    return B200_ERROR_INVALID_PARAM;
  if (head_dim != kDecHD || (block_size != 64 && block_size != 128) || nq / nkv > 16) return B200_ERROR_UNSUPPORTED;
  if (q_stride % 8 || out_stride % 8 || !al16(q) || !al16(out) || !al16(k_cache) || !al16(v_cache))
    return B200_ERROR_INVALID_PARAM;
  if ((int64_t)max_blocks_per_seq * block_size < max_context) return B200_ERROR_INVALID_PARAM;
  if (batch == 0) return B200_OK;
  const int64_t rows = num_blocks * nkv * block_size;
  if (rows > INT32_MAX) return B200_ERROR_UNSUPPORTED;
  if (nkv > 65535) return B200_ERROR_UNSUPPORTED;

  DecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_stride = q_stride;
  p.block_tables = block_tables;
  p.max_blocks = max_blocks_per_seq;
  p.context_lens = context_lens;
  p.nq = nq;
  p.nkv = nkv;
  p.G = nq / nkv;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.scale_log2 = scale * kLog2e;
  // tokens per split: a multiple of the tile so tiles never straddle splits;
  // without a workspace that holds the plan's scratch the context runs unsplit
  const DecodePlan plan = decode_plan(batch, nq, nkv, max_context);
  int splits = plan.splits;
  p.tokens_per_split = plan.tokens_per_split;
  if (splits > 1 && (!workspace || workspace_bytes < plan.scratch_bytes || !al16(workspace))) {
    splits = 1;
    p.tokens_per_split = ((std::max(1, max_context) + kDecTile - 1) / kDecTile) * kDecTile;
  }
  p.splits = splits;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = out_stride;
  p.ws_o = static_cast<float*>(workspace);
  p.ws_lse = p.ws_o + (int64_t)batch * nq * splits * kDecHD;
  int dev = 0;
  cudaGetDevice(&dev);
  p.err = b200::error_word(dev);
  p.pf = nullptr;
  p.pf_bytes = 0;
  p.pf_first = 0;
  if (prefetch && prefetch_bytes >= 16 && (reinterpret_cast<uintptr_t>(prefetch) & 15u) == 0) {
    const int64_t total = (int64_t)batch * nkv * splits;
    p.pf = static_cast<const uint8_t*>(prefetch);
    p.pf_bytes = prefetch_bytes & ~int64_t(15);
    p.pf_first = (int)std::max<int64_t>(0, total - 2 * (int64_t)num_sms());  // the last wave (2 CTAs per SM)
  }

  CUtensorMap tk, tv;
  if (!make_cache_tmap(&tk, k_cache, rows) || !make_cache_tmap(&tv, v_cache, rows)) return B200_ERROR_UNSUPPORTED;
  if (!set_smem<paged_decode_kernel>(kDecSmem)) return B200_ERROR_UNSUPPORTED;
  dim3 grid(batch, nkv, splits);
  launch_kernel(paged_decode_kernel, grid, kDecThreads, kDecSmem, stream, tk, tv, p);
  B200_CHECK_LAUNCH();
  if (splits > 1) {
    launch_kernel(decode_combine_kernel, dim3(batch * nq), kDecHD, 0, stream, p.ws_o, p.ws_lse, nq, splits, p.out,
                  out_stride);
    B200_CHECK_LAUNCH();
  }
  return B200_OK;
}
}  // namespace b200

extern "C" int b200_paged_decode(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                                 const int32_t* block_tables, int max_blocks_per_seq, const int32_t* context_lens,
                                 int batch, int nq, int nkv, int head_dim, int block_size, int64_t num_blocks,
                                 float scale, void* out, int64_t out_stride, void* workspace, int64_t workspace_bytes,
                                 int max_context, b200_stream_t stream) {
  return b200::paged_decode_launch(q, q_stride, k_cache, v_cache, block_tables, max_blocks_per_seq, context_lens,
                                   batch, nq, nkv, head_dim, block_size, num_blocks, scale, out, out_stride, workspace,
                                   workspace_bytes, max_context, stream, nullptr, 0);
}
