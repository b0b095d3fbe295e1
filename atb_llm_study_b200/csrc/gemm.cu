// bf16 GEMM on the 5th-generation tensor cores: C = epi(A * B^T).
//
// Design (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: 128x64 A tile + BNx64 B tile per stage, 128-byte
//               swizzle, STAGES-deep ring of shared-memory buffers guarded by
//               full/empty mbarriers.
//   warp 1      allocates TMEM, then one thread issues tcgen05.mma
//               (M=128, N=BN, K=16, bf16 -> fp32) into one of two TMEM
//               accumulators and releases stages with tcgen05.commit.
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns, fused
//               bias / residual / SwiGLU / GELU, bf16 stores.
// The accumulator is double-buffered, so tile i's epilogue overlaps tile
// i+1's main loop.
//
// Skinny problems (few token rows, the decode case) run "swapped": the weight
// matrix feeds the 128-row MMA side and the tokens the N side, and the
// epilogue writes the transpose.  When there are too few output tiles to
// cover the SMs the K loop is split: each split stores its fp32 partial tile
// in a workspace slice with plain coalesced stores, and the reduction (with
// the epilogue) runs in the consumer — splitk_reduce for the C ABI call, or a
// kernel that reads the result anyway (residual + RMSNorm, QK-norm + rope).
// A swapped SwiGLU projection with enough k-blocks per SM (the decode
// gate/up) runs "stream-K" instead: every CTA takes an equal, contiguous run
// of the (tile, k-block) sequence, so a tile is cut at most once; the CTA
// holding a tile's head stores its fp32 partial first thing and raises the
// tile's flag, the CTA holding the tail finishes that tile last, adding the
// head's partial (loaded while its own MMAs run) before the SwiGLU epilogue.
// No partial stores for whole tiles and no separate reduce launch.
//
// No TMA multicast is used (the library also runs in multi-GPU jobs).
#include <math.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "gemm.h"

using namespace b200;

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kGroupM = 16;
constexpr int kMaxGroups = 256;                            // experts of one grouped GEMM
constexpr int kGroupTabBytes = 2 * (kMaxGroups + 2) * 4;  // row offsets + unit prefix in shared memory

template <int BN>
struct Cfg {
  static constexpr int STAGES = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int SMEM_GROUPED = SMEM + kGroupTabBytes;
  static constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN);
};

struct Params {
  int64_t rows;    // MMA M extent (rows of A)
  int64_t cols;    // MMA N extent (rows of B)
  int64_t K;
  int tiles_m, tiles_n, splits, kb_total, kb_per_split;
  __nv_bfloat16* C;
  int64_t ldc;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* R;
  int64_t ldr;
  float* ws;  // split-K fp32 partial tiles [splits][tokens][features]
  unsigned* err;
  // Grouped (per-expert) GEMM: the tokens of group g are rows [goff[g],
  // goff[g+1]) of the token operand and its weights are rows [g*gN, (g+1)*gN)
  // of the weight operand; the output row of a token is its token row.
  const int32_t* goff;
  int groups;
  int64_t gN;
  int gF;          // feature tiles per group
  int64_t gRows;   // rows of the token operand (goff is clamped to it)
  // Decode chains: bytes of the NEXT projection's weights this launch pulls
  // into L2 from its tail (each CTA a share, after its last tile load), so HBM
  // keeps streaming across the launch boundary.  pf_bytes % 16 == 0.
  const uint8_t* pf;
  int64_t pf_bytes;
  // Stream-K (swapped SwiGLU only): one flag per tile, zero between launches;
  // ws then holds one 128 x BN fp32 partial per tile, [tile][token][row].
  int* sk_flags;
};

// One output tile: its MMA tile coordinates, K range, the TMA row coordinates
// of both operands and the epilogue's row / column origin and limits.
struct Unit {
  int tm, tn, kb0, kb1;
  int a_row, b_row;
  int64_t row0, col0, row_lim, col_lim;
  int piece;  // stream-K: kPieceWhole, kPieceHead or kPieceTail of tile tm
};
constexpr int kPieceWhole = 0, kPieceHead = 1, kPieceTail = 2;

__device__ __forceinline__ float gelu_tanh_f(float x) {
  return 0.5f * x * (1.f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}
// x * sigmoid(x) with the fast division intrinsic (the epilogue warps are few:
// an IEEE division per element would dominate a decode gate/up epilogue).
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.f + __expf(-x)); }

// Epilogue on 8 consecutive features f0..f0+7 of token `tok` (non-SwiGLU kinds).
template <int EPI>
__device__ __forceinline__ void epi8(float v[8], int64_t tok, int64_t f0, const Params& p) {
  if (EPI == B200_EPI_BIAS || EPI == B200_EPI_BIAS_GELU || EPI == B200_EPI_BIAS_RESIDUAL) {
    float b[8];
    unpack8(*reinterpret_cast<const uint4*>(p.bias + f0), b);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] += b[i];
  }
  if (EPI == B200_EPI_BIAS_GELU) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = gelu_tanh_f(v[i]);
  }
  if (EPI == B200_EPI_RESIDUAL || EPI == B200_EPI_BIAS_RESIDUAL) {
    float r[8];
    unpack8(*reinterpret_cast<const uint4*>(p.R + tok * p.ldr + f0), r);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] += r[i];
  }
}

template <int EPI>
__device__ __forceinline__ float epi1(float v, int64_t tok, int64_t f, const Params& p) {
  if (EPI == B200_EPI_BIAS || EPI == B200_EPI_BIAS_GELU || EPI == B200_EPI_BIAS_RESIDUAL) v += bf2f(p.bias[f]);
  if (EPI == B200_EPI_BIAS_GELU) v = gelu_tanh_f(v);
  if (EPI == B200_EPI_RESIDUAL || EPI == B200_EPI_BIAS_RESIDUAL) v += bf2f(p.R[tok * p.ldr + f]);
  return v;
}

// Store one 32-column chunk of accumulator values for MMA row `row`, columns
// [col0, col0+32), applying the epilogue.  Normal orientation: row = token,
// columns = features (vector stores).  Swapped: row = feature (consecutive
// features in consecutive lanes), columns = tokens.
template <int EPI, bool SWAP>
__device__ __forceinline__ void emit_chunk(float v[32], int64_t row, int64_t col0, int lane, const Params& p) {
  if (!SWAP) {
    if (row >= p.rows) return;
    if (EPI == B200_EPI_SWIGLU) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int64_t c = col0 + g * 8;
        if (c < p.cols) {
          uint2 o;
          o.x = pack2(silu_f(v[8 * g]) * v[8 * g + 1], silu_f(v[8 * g + 2]) * v[8 * g + 3]);
          o.y = pack2(silu_f(v[8 * g + 4]) * v[8 * g + 5], silu_f(v[8 * g + 6]) * v[8 * g + 7]);
          *reinterpret_cast<uint2*>(p.C + row * p.ldc + c / 2) = o;
        }
      }
    } else {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int64_t c = col0 + g * 8;
        if (c < p.cols) {
          float* vv = v + 8 * g;
          epi8<EPI>(vv, row, c, p);
          *reinterpret_cast<uint4*>(p.C + row * p.ldc + c) = pack8(vv);
        }
      }
    }
  } else if (EPI == B200_EPI_SWIGLU) {
    // Lanes 2j / 2j+1 hold the gate / up rows of feature j: the even lane
    // finishes tokens 0..15 of the chunk, the odd lane tokens 16..31, one
    // exchange per token pair (each lane sends what its partner lacks).
    const bool odd = lane & 1;
    const int64_t f = row >> 1;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float other = __shfl_xor_sync(0xffffffffu, odd ? v[i] : v[16 + i], 1);
      const int tok = odd ? 16 + i : i;
      const float o = odd ? silu_f(other) * v[16 + i] : silu_f(v[i]) * other;
      if (row < p.rows && col0 + tok < p.cols) p.C[(col0 + tok) * p.ldc + f] = f2bf(o);
    }
  } else if (row < p.rows) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col0 + i < p.cols) p.C[(col0 + i) * p.ldc + row] = f2bf(epi1<EPI>(v[i], col0 + i, row, p));
  }
}

// Index of (MMA row, MMA column) in the split-K accumulator ws[token][feature].
template <bool SWAP>
__device__ __forceinline__ int64_t ws_index(int64_t row, int64_t col, const Params& p) {
  return SWAP ? col * p.rows + row : row * p.cols + col;
}

__device__ __forceinline__ void decode_unit(int w, const Params& p, int& tm, int& tn, int& kb0, int& kb1) {
  const int tiles = p.tiles_m * p.tiles_n;
  const int split = w / tiles;
  const int t = w % tiles;
  const int group = kGroupM * p.tiles_n;
  const int g = t / group;
  const int first_m = g * kGroupM;
  const int gm = min(p.tiles_m - first_m, kGroupM);
  const int r = t % group;
  tm = first_m + r % gm;
  tn = r / gm;
  kb0 = split * p.kb_per_split;
  kb1 = min(p.kb_total, kb0 + p.kb_per_split);
}

// Unit w of the launch.  Plain GEMM: decode_unit's raster.  Grouped: gtab[0..G]
// holds the groups' token row offsets and gtab[G+1..2G+1] the prefix of their
// unit counts; within a group the token tiles of one feature tile are
// consecutive (they share that weight tile).
template <int BN, bool SWAP, bool GROUPED>
__device__ __forceinline__ Unit get_unit(int w, const Params& p, const int* gtab) {
  Unit u;
  if (!GROUPED) {
    decode_unit(w, p, u.tm, u.tn, u.kb0, u.kb1);
    u.a_row = u.tm * BM;
    u.b_row = u.tn * BN;
    u.row0 = (int64_t)u.tm * BM;
    u.col0 = (int64_t)u.tn * BN;
    u.row_lim = p.rows;
    u.col_lim = p.cols;
    return u;
  }
  const int* up = gtab + p.groups + 1;
  int lo = 0, hi = p.groups;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (up[mid] <= w) lo = mid;
    else hi = mid;
  }
  const int g = lo;
  constexpr int TOKT = SWAP ? BN : BM;
  const int t0 = gtab[g], t1 = gtab[g + 1];
  const int tt = (t1 - t0 + TOKT - 1) / TOKT;
  const int r = w - up[g];
  const int tok = r % tt, feat = r / tt;
  u.kb0 = 0;
  u.kb1 = p.kb_total;
  if (SWAP) {
    u.tm = feat;
    u.tn = tok;
    u.a_row = (int)(g * p.gN) + feat * BM;
    u.b_row = t0 + tok * BN;
    u.row0 = (int64_t)feat * BM;
    u.row_lim = p.gN;
    u.col0 = (int64_t)t0 + (int64_t)tok * BN;
    u.col_lim = t1;
  } else {
    u.tm = tok;
    u.tn = feat;
    u.a_row = t0 + tok * BM;
    u.b_row = (int)(g * p.gN) + feat * BN;
    u.row0 = (int64_t)t0 + (int64_t)tok * BM;
    u.row_lim = t1;
    u.col0 = (int64_t)feat * BN;
    u.col_lim = p.gN;
  }
  return u;
}

// Stream-K schedule of CTA c out of G over tiles_m tiles of kb_total k-blocks
// (tiles_n == 1): the run [c*W/G, (c+1)*W/G) of the tile-major k-block
// sequence, W = tiles_m * kb_total, at least kb_total long, so it cuts at
// most the tile it starts in (a tail piece) and the tile it ends in (a head
// piece).  Order: the head piece first, the whole tiles, the tail piece last.
struct SkRun {
  int s, e, t0, t1, whole0, whole_n;
  bool head, tail;
};

__device__ __forceinline__ SkRun sk_run(const Params& p, int c, int G) {
  SkRun r;
  const int64_t W = (int64_t)p.tiles_m * p.kb_total;
  r.s = (int)(W * c / G);
  r.e = (int)(W * (c + 1) / G);
  r.t0 = r.s / p.kb_total;
  r.t1 = (r.e - 1) / p.kb_total;
  r.tail = r.s % p.kb_total != 0;
  r.head = r.e % p.kb_total != 0;
  r.whole0 = r.tail ? r.t0 + 1 : r.t0;
  r.whole_n = (r.head ? r.t1 - 1 : r.t1) - r.whole0 + 1;
  return r;
}

__device__ __forceinline__ int sk_units(const SkRun& r) { return (int)r.head + r.whole_n + (int)r.tail; }

template <int BN>
__device__ __forceinline__ Unit sk_unit(int i, const SkRun& r, const Params& p) {
  int t;
  if (r.head && i == 0) t = r.t1;
  else if (i - (int)r.head < r.whole_n) t = r.whole0 + i - (int)r.head;
  else t = r.t0;
  Unit u;
  u.tm = t;
  u.tn = 0;
  const int base = t * p.kb_total;
  u.kb0 = max(r.s, base) - base;
  u.kb1 = min(r.e, base + p.kb_total) - base;
  u.piece = u.kb0 > 0 ? kPieceTail : (u.kb1 < p.kb_total ? kPieceHead : kPieceWhole);
  u.a_row = t * BM;
  u.b_row = 0;
  u.row0 = (int64_t)t * BM;
  u.col0 = 0;
  u.row_lim = p.rows;
  u.col_lim = p.cols;
  return u;
}

template <int BN, int EPI, bool SWAP, bool PARTIAL, bool GROUPED = false, bool SK = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const Params p) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + C::STAGES * C::B_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* skbar = tempty + 2;  // stream-K, one-shot: [0] head partial stored (128), [1] tail flag seen (1)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(skbar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  int* gtab = reinterpret_cast<int*>(smem + C::STAGES * C::STAGE_BYTES + 256);  // grouped launches only

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int units = p.tiles_m * p.tiles_n * p.splits;
  pdl_trigger();
  // unit sequence of this CTA: w = w0, w0 + wstep, ... < wend (stream-K: its own run)
  SkRun skr{};
  if (SK) {
    skr = sk_run(p, blockIdx.x, gridDim.x);
    units = sk_units(skr);
  }
  const int w0 = SK ? 0 : blockIdx.x, wstep = SK ? 1 : gridDim.x;
  auto unit_at = [&](int w, const int* gt) { return SK ? sk_unit<BN>(w, skr, p) : get_unit<BN, SWAP, GROUPED>(w, p, gt); };

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(&skbar[0], 128);
    mbar_init(&skbar[1], 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (GROUPED) {
    // the group row offsets come from the previous kernel (the expert permutation)
    pdl_wait();
    if (threadIdx.x == 0) {
      int prev = 0, run = 0;
      for (int g = 0; g <= p.groups; ++g) {
        int v = p.goff[g];
        if (v < prev || v > p.gRows || (g == 0 && v != 0)) {
          raise_error(p.err, DEV_ERR_BAD_INDEX);
          v = min(max(v, prev), (int)p.gRows);
          if (g == 0) v = 0;
        }
        gtab[g] = prev = v;
      }
      constexpr int TOKT = SWAP ? BN : BM;
      for (int g = 0; g < p.groups; ++g) {
        gtab[p.groups + 1 + g] = run;
        run += ((gtab[g + 1] - gtab[g] + TOKT - 1) / TOKT) * p.gF;
      }
      gtab[2 * p.groups + 1] = run;
    }
    __syncthreads();
    units = gtab[2 * p.groups + 1];
  }

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      // The weight operand (A when swapped, B otherwise) is constant: its
      // tiles for the first stages are requested before waiting for the
      // previous kernel on the stream, so the weight stream starts while that
      // kernel drains.  Activation tiles are only loaded after the wait.
      // (Grouped launches already waited: their tiles depend on the offsets.)
      // The first STAGES k-blocks of the CTA's unit sequence (across unit
      // boundaries: a stream-K head piece may be short) are preloaded.
      int pre = 0;
      if (!GROUPED) {
        for (int w = w0; w < units && pre < C::STAGES; w += wstep) {
          const Unit u0 = unit_at(w, gtab);
          for (int kb = u0.kb0; kb < u0.kb1 && pre < C::STAGES; ++kb, ++pre) {
            mbar_arrive_expect_tx(&full[pre], C::STAGE_BYTES);
            if (SWAP) tma_load_2d(sA + pre * C::A_BYTES, &tmA, &full[pre], kb * BK, u0.a_row);
            else tma_load_2d(sB + pre * C::B_BYTES, &tmB, &full[pre], kb * BK, u0.b_row);
          }
        }
      }
      pdl_wait();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;  // k-blocks of the sequence so far
      for (int w = w0; w < units && !*abort_flag; w += wstep) {
        const Unit u = unit_at(w, gtab);
        for (int kb = u.kb0; kb < u.kb1; ++kb, ++issued) {
          if (issued < pre) {
            // stage == issued already expects both halves; add the activation half
            if (SWAP) tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * BK, u.b_row);
            else tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * BK, u.a_row);
          } else {
            if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) {
              *abort_flag = 1;
              break;
            }
            mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
            tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * BK, u.a_row);
            tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * BK, u.b_row);
          }
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!*abort_flag) prefetch_l2_share(p.pf, p.pf_bytes, blockIdx.x, gridDim.x);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int w = w0; w < units && !*abort_flag; w += wstep, ++local) {
        const Unit u = unit_at(w, gtab);
        const int kb0 = u.kb0, kb1 = u.kb1;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.err)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(d_tmem, smem_desc_k128(a0 + k * 32), smem_desc_k128(b0 + k * 32), C::IDESC,
                      (kb > kb0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&tfull[acc]);
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    pdl_wait();  // reads the residual / writes outputs the previous kernel may still use
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int rit = q * 32 + lane;
    int local = 0;
    for (int w = w0; w < units && !*abort_flag; w += wstep, ++local) {
      const Unit u = unit_at(w, gtab);
      const int split = w / (p.tiles_m * p.tiles_n);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      // stream-K tail piece: the head's partial of this tile, loaded before
      // this tile's own accumulator is ready
      float head[SK ? BN : 1];
      if (SK && u.piece == kPieceTail) {
        if (warp == 2 && lane == 0) {
          volatile int* f = p.sk_flags + u.tm;
          const uint64_t t0 = global_timer_ns();
          bool ok = true;
          while (*f == 0) {
            if (global_timer_ns() - t0 > kWaitLimitNs) {
              raise_error(p.err, DEV_ERR_WAIT_TIMEOUT);
              ok = false;
              break;
            }
          }
          __threadfence();
          if (ok) *f = 0;  // flags are zero between launches
          mbar_arrive(&skbar[1]);
        }
        if (!mbar_wait(&skbar[1], 0, p.err)) {
          *abort_flag = 1;
          break;
        }
        const float* hp = p.ws + (int64_t)u.tm * BM * BN + rit;
#pragma unroll
        for (int c = 0; c < BN; ++c) head[c] = __ldcg(hp + c * BM);
      }
      if (!mbar_wait(&tfull[acc], acc_phase, p.err)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int64_t row = u.row0 + rit;
      Params pe = p;  // bounds of this tile's output (a group's rows in grouped launches)
      pe.rows = u.row_lim;
      pe.cols = u.col_lim;
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + ch * 32, r);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        const int64_t col0 = u.col0 + ch * 32;
        if (SK && u.piece == kPieceHead) {
          // this tile's head: fp32 partial [token][row] (coalesced over rows)
          float* hp = p.ws + (int64_t)u.tm * BM * BN + (int64_t)ch * 32 * BM + rit;
#pragma unroll
          for (int i = 0; i < 32; ++i) __stcg(hp + i * BM, v[i]);
          continue;
        }
        if (SK && u.piece == kPieceTail) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] += ch == 0 ? head[i] : head[(BN > 32 ? 32 : 0) + i];  // static indices
        }
        if (PARTIAL) {
          // this K slice's partial tile -> ws[split][token][feature] (plain coalesced stores)
          if (row < p.rows) {
            float* base = p.ws + (int64_t)split * p.rows * p.cols;
            if (!SWAP && col0 + 32 <= p.cols) {
#pragma unroll
              for (int g = 0; g < 8; ++g)
                __stcg(reinterpret_cast<float4*>(base + ws_index<SWAP>(row, col0 + 4 * g, p)),
                       make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]));
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (col0 + i < p.cols) __stcg(base + ws_index<SWAP>(row, col0 + i, p), v[i]);
            }
          }
        } else {
          emit_chunk<EPI, SWAP>(v, row, col0, lane, pe);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (SK && u.piece == kPieceHead) {
        __threadfence();  // every thread's partial stores before the flag
        mbar_arrive(&skbar[0]);
        if (warp == 2 && lane == 0) {
          if (mbar_wait(&skbar[0], 0, p.err)) atomicExch(p.sk_flags + u.tm, 1);
          else *abort_flag = 1;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
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

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with row stride ld,
// box = box_rows x 64 elements (128 bytes, the swizzle span).
bool make_tmap(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeTiledFn f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
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

template <int BN, int EPI, bool SWAP, bool PARTIAL, bool GROUPED = false, bool SK = false>
int launch_t(const CUtensorMap& a, const CUtensorMap& b, const Params& p, int grid, cudaStream_t st) {
  auto k = gemm_tcgen05_kernel<BN, EPI, SWAP, PARTIAL, GROUPED, SK>;
  constexpr int smem = GROUPED ? Cfg<BN>::SMEM_GROUPED : Cfg<BN>::SMEM;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return B200_ERROR_UNSUPPORTED;
    attr_set[dev] = true;
  }
  launch_kernel(k, dim3(grid), kThreads, smem, st, a, b, p);
  B200_CHECK_LAUNCH();
  return B200_OK;
}

// Sum split-K partials ws[s][tok][feat] and apply the epilogue.  One thread per
// 8 features (SwiGLU: 8 interleaved gate/up features -> 4 outputs).
template <int EPI>
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int64_t tokens, int64_t feats,
                                     Params p) {
  pdl_trigger();
  pdl_wait();
  const int64_t nv = feats / 8;
  const int64_t gid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (gid >= tokens * nv) return;
  const int64_t tok = gid / nv, f0 = (gid % nv) * 8;
  float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  constexpr int kBatch = 8;  // the loads of up to 8 splits in flight before they are summed (split order kept)
  for (int s0 = 0; s0 < splits; s0 += kBatch) {
    float4 a[kBatch][2];
#pragma unroll
    for (int i = 0; i < kBatch; ++i)
      if (s0 + i < splits) {
        const float4* src = reinterpret_cast<const float4*>(ws + ((int64_t)(s0 + i) * tokens + tok) * feats + f0);
        a[i][0] = src[0];
        a[i][1] = src[1];
      }
#pragma unroll
    for (int i = 0; i < kBatch; ++i)
      if (s0 + i < splits) {
        v[0] += a[i][0].x; v[1] += a[i][0].y; v[2] += a[i][0].z; v[3] += a[i][0].w;
        v[4] += a[i][1].x; v[5] += a[i][1].y; v[6] += a[i][1].z; v[7] += a[i][1].w;
      }
  }
  if (EPI == B200_EPI_SWIGLU) {
    uint2 o;
    o.x = pack2(silu_f(v[0]) * v[1], silu_f(v[2]) * v[3]);
    o.y = pack2(silu_f(v[4]) * v[5], silu_f(v[6]) * v[7]);
    *reinterpret_cast<uint2*>(p.C + tok * p.ldc + f0 / 2) = o;
  } else {
    epi8<EPI>(v, tok, f0, p);
    *reinterpret_cast<uint4*>(p.C + tok * p.ldc + f0) = pack8(v);
  }
}

template <int BN, bool SWAP, bool PARTIAL>
int launch_epi(int epi, const CUtensorMap& a, const CUtensorMap& b, const Params& p, int grid, cudaStream_t st) {
  // split-K units only store partials: the epilogue runs where they are reduced
  if (PARTIAL) return launch_t<BN, B200_EPI_NONE, SWAP, true>(a, b, p, grid, st);
  switch (epi) {
    case B200_EPI_NONE: return launch_t<BN, B200_EPI_NONE, SWAP, false>(a, b, p, grid, st);
    case B200_EPI_BIAS: return launch_t<BN, B200_EPI_BIAS, SWAP, false>(a, b, p, grid, st);
    case B200_EPI_RESIDUAL: return launch_t<BN, B200_EPI_RESIDUAL, SWAP, false>(a, b, p, grid, st);
    case B200_EPI_SWIGLU: return launch_t<BN, B200_EPI_SWIGLU, SWAP, false>(a, b, p, grid, st);
    case B200_EPI_BIAS_GELU: return launch_t<BN, B200_EPI_BIAS_GELU, SWAP, false>(a, b, p, grid, st);
    case B200_EPI_BIAS_RESIDUAL: return launch_t<BN, B200_EPI_BIAS_RESIDUAL, SWAP, false>(a, b, p, grid, st);
  }
  return B200_ERROR_INVALID_PARAM;
}

Params make_params(const b200::GemmPlan& g, int64_t M, int64_t N, int64_t K, void* Cp, int64_t ldc, const void* bias,
                   const void* R, int64_t ldr, void* ws) {
  Params p;
  p.rows = g.swap ? N : M;
  p.cols = g.swap ? M : N;
  p.K = K;
  p.tiles_m = g.tiles_m;
  p.tiles_n = g.tiles_n;
  p.splits = g.splits;
  p.kb_total = g.kb_total;
  p.kb_per_split = g.kb_per_split;
  p.C = static_cast<__nv_bfloat16*>(Cp);
  p.ldc = ldc;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.R = static_cast<const __nv_bfloat16*>(R);
  p.ldr = ldr;
  p.ws = g.splits > 1 ? static_cast<float*>(ws) : nullptr;
  p.goff = nullptr;
  p.groups = 0;
  p.gN = 0;
  p.gF = 0;
  p.gRows = 0;
  p.pf = nullptr;
  p.pf_bytes = 0;
  p.sk_flags = nullptr;
  int dev = 0;
  cudaGetDevice(&dev);
  p.err = b200::error_word(dev);
  return p;
}

}  // namespace

namespace b200 {

GemmPlan plan_gemm(int64_t M, int64_t N, int64_t K, int epilogue, int sms) {
  GemmPlan g;
  g.swap = M <= 128;
  const int64_t mma_rows = g.swap ? N : M;
  const int64_t mma_cols = g.swap ? M : N;
  if (g.swap) g.bn = mma_cols <= 64 ? 64 : 128;
  else g.bn = mma_cols > 128 ? 256 : 128;
  g.tiles_m = (int)((mma_rows + BM - 1) / BM);
  // Few 256-wide tiles over a short K (the few-hundred-token GEMMs of the
  // vision tower and of short prompts): 128-wide tiles put twice as many CTAs
  // to work; with long K the wider tile's lower bytes per flop wins instead.
  if (!g.swap && g.bn == 256 && 2 * g.tiles_m * ((mma_cols + 255) / 256) < sms && K <= 2048) g.bn = 128;
  g.tiles_n = (int)((mma_cols + g.bn - 1) / g.bn);
  g.kb_total = (int)((K + BK - 1) / BK);
  const int tiles = g.tiles_m * g.tiles_n;
  // Split K only when the output tiles leave SMs idle.  Each split keeps
  // >= 16 k-blocks (its pipeline fill stays small next to its weight stream;
  // 8 when token-major tiles cover under half the SMs) and every extra split
  // is charged 3 % for its partial-tile traffic.
  const int min_kb = (!g.swap && 2 * tiles < sms) ? 8 : 16;
  int best = 1;
  if (tiles < 2 * sms) {
    double best_score = (double)tiles / ((double)sms * ((tiles + sms - 1) / sms)) - 0.03;
    for (int s = 2; s <= 16; ++s) {
      if (g.kb_total / s < min_kb) break;
      const int u = tiles * s;
      const double score = (double)u / ((double)sms * ((u + sms - 1) / sms)) - 0.03 * s;
      if (score > best_score + 0.02) {
        best_score = score;
        best = s;
      }
    }
  }
  static const int forced = [] {  // tuning override for swapped (decode-sized) GEMMs: B200_GEMM_SPLITS=<n>
    const char* v = std::getenv("B200_GEMM_SPLITS");
    return v ? std::atoi(v) : 0;
  }();
  if (forced > 0 && g.swap) best = std::max(1, std::min(forced, g.kb_total));
  g.kb_per_split = (g.kb_total + best - 1) / best;
  g.splits = (g.kb_total + g.kb_per_split - 1) / g.kb_per_split;
  g.ws_bytes = g.splits > 1 ? (int64_t)g.splits * M * N * (int64_t)sizeof(float) : 0;
  (void)epilogue;
  return g;
}

int gemm_launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* Cp, int64_t ldc, int64_t M, int64_t N,
                int64_t K, int epi, const void* bias, const void* R, int64_t ldr, void* ws, int64_t ws_bytes,
                cudaStream_t st, int* splits_out, const void* prefetch, int64_t prefetch_bytes, int* sk_flags,
                int sk_flag_count) {
  if (splits_out) *splits_out = 1;
  if (!A || !B || !Cp || M < 0 || N < 0 || K <= 0) return B200_ERROR_INVALID_PARAM;
  if (epi < B200_EPI_NONE || epi > B200_EPI_BIAS_RESIDUAL) return B200_ERROR_INVALID_PARAM;
  if (K % 8 || lda % 8 || ldb % 8 || ldc % 8 || lda < K || ldb < K || N % 8) return B200_ERROR_INVALID_PARAM;
  const int64_t outN = epi == B200_EPI_SWIGLU ? N / 2 : N;
  if (epi == B200_EPI_SWIGLU && N % 16) return B200_ERROR_INVALID_PARAM;
  if (ldc < outN) return B200_ERROR_INVALID_PARAM;
  const bool needs_bias = epi == B200_EPI_BIAS || epi == B200_EPI_BIAS_GELU || epi == B200_EPI_BIAS_RESIDUAL;
  const bool needs_res = epi == B200_EPI_RESIDUAL || epi == B200_EPI_BIAS_RESIDUAL;
  if ((needs_bias && !bias) || (needs_res && (!R || ldr % 8 || ldr < N))) return B200_ERROR_INVALID_PARAM;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al(A) || !al(B) || !al(Cp) || (bias && !al(bias)) || (R && !al(R)) || (ws && !al(ws)))
    return B200_ERROR_INVALID_PARAM;
  if (M == 0 || N == 0) return B200_OK;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return B200_ERROR_UNSUPPORTED;

  const int sms = num_sms();
  GemmPlan g = plan_gemm(M, N, K, epi, sms);
  if (g.splits > 1 && (!splits_out || !ws || ws_bytes < g.ws_bytes)) {
    g.splits = 1;
    g.kb_per_split = g.kb_total;
  }
  Params p = make_params(g, M, N, K, Cp, ldc, bias, R, ldr, ws);
  if (prefetch && prefetch_bytes >= 16 && (reinterpret_cast<uintptr_t>(prefetch) & 15u) == 0) {
    p.pf = static_cast<const uint8_t*>(prefetch);
    p.pf_bytes = prefetch_bytes & ~int64_t(15);
  }
  CUtensorMap ta, tb;
  const void* mA = g.swap ? B : A;  // operand on the 128-row MMA side
  const void* mB = g.swap ? A : B;
  const int64_t ldmA = g.swap ? ldb : lda, ldmB = g.swap ? lda : ldb;
  if (!make_tmap(&ta, mA, p.rows, K, ldmA, BM) || !make_tmap(&tb, mB, p.cols, K, ldmB, g.bn))
    return B200_ERROR_UNSUPPORTED;
  // Stream-K for a swapped SwiGLU projection over at least one whole tile of
  // k-blocks per SM (the decode gate/up): even runs, no reduce launch.
  const bool sk = sk_flags && g.swap && g.bn == 64 && epi == B200_EPI_SWIGLU && g.tiles_n == 1 &&
                  g.tiles_m >= sms && g.tiles_m <= sk_flag_count && (g.tiles_m % sms) != 0 && ws &&
                  (reinterpret_cast<uintptr_t>(sk_flags) & 3u) == 0 &&
                  ws_bytes >= (int64_t)g.tiles_m * BM * 64 * (int64_t)sizeof(float);
  if (sk) {
    g.splits = 1;
    g.kb_per_split = g.kb_total;
    p = make_params(g, M, N, K, Cp, ldc, bias, R, ldr, ws);
    p.ws = static_cast<float*>(ws);
    p.sk_flags = sk_flags;
    p.pf = prefetch && prefetch_bytes >= 16 && (reinterpret_cast<uintptr_t>(prefetch) & 15u) == 0
               ? static_cast<const uint8_t*>(prefetch) : nullptr;
    p.pf_bytes = p.pf ? (prefetch_bytes & ~int64_t(15)) : 0;
  }
  const int units = g.tiles_m * g.tiles_n * g.splits;
  const int grid = sk ? sms : std::min(units, sms);
  const bool partial = g.splits > 1;
  int rc;
  if (sk) {
    rc = launch_t<64, B200_EPI_SWIGLU, true, false, false, true>(ta, tb, p, grid, st);
    if (rc == B200_OK && splits_out) *splits_out = 1;
    return rc;
  }
  if (g.bn == 256) {
    rc = partial ? launch_epi<256, false, true>(epi, ta, tb, p, grid, st) : launch_epi<256, false, false>(epi, ta, tb, p, grid, st);
  } else if (g.bn == 128) {
    if (g.swap)
      rc = partial ? launch_epi<128, true, true>(epi, ta, tb, p, grid, st) : launch_epi<128, true, false>(epi, ta, tb, p, grid, st);
    else
      rc = partial ? launch_epi<128, false, true>(epi, ta, tb, p, grid, st) : launch_epi<128, false, false>(epi, ta, tb, p, grid, st);
  } else {
    rc = partial ? launch_epi<64, true, true>(epi, ta, tb, p, grid, st) : launch_epi<64, true, false>(epi, ta, tb, p, grid, st);
  }
  if (rc == B200_OK && splits_out) *splits_out = g.splits;
  return rc;
}

int splitk_reduce(const float* ws, int splits, int64_t M, int64_t N, int epi, const void* bias, const void* R,
                  int64_t ldr, void* Cp, int64_t ldc, cudaStream_t st) {
  GemmPlan g;
  g.splits = splits;
  Params p = make_params(g, M, N, 0, Cp, ldc, bias, R, ldr, nullptr);
  const int64_t n = M * (N / 8);
  const unsigned grid = (unsigned)((n + 255) / 256);
  switch (epi) {
    case B200_EPI_NONE: launch_kernel(splitk_reduce_kernel<B200_EPI_NONE>, dim3(grid), 256, 0, st, ws, splits, M, N, p); break;
    case B200_EPI_BIAS: launch_kernel(splitk_reduce_kernel<B200_EPI_BIAS>, dim3(grid), 256, 0, st, ws, splits, M, N, p); break;
    case B200_EPI_RESIDUAL: launch_kernel(splitk_reduce_kernel<B200_EPI_RESIDUAL>, dim3(grid), 256, 0, st, ws, splits, M, N, p); break;
    case B200_EPI_SWIGLU: launch_kernel(splitk_reduce_kernel<B200_EPI_SWIGLU>, dim3(grid), 256, 0, st, ws, splits, M, N, p); break;
    case B200_EPI_BIAS_GELU: launch_kernel(splitk_reduce_kernel<B200_EPI_BIAS_GELU>, dim3(grid), 256, 0, st, ws, splits, M, N, p); break;
    case B200_EPI_BIAS_RESIDUAL: launch_kernel(splitk_reduce_kernel<B200_EPI_BIAS_RESIDUAL>, dim3(grid), 256, 0, st, ws, splits, M, N, p); break;
    default: return B200_ERROR_INVALID_PARAM;
  }
  B200_CHECK_LAUNCH();
  return B200_OK;
}

int grouped_gemm_launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* Cp, int64_t ldc,
                        const int32_t* goff, int groups, int64_t rows, int64_t N, int64_t K, int epi,
                        cudaStream_t st) {
  if (!A || !B || !Cp || !goff || groups <= 0 || groups > kMaxGroups || rows < 0 || N <= 0 || K <= 0)
    return B200_ERROR_INVALID_PARAM;
  if (epi != B200_EPI_NONE && epi != B200_EPI_SWIGLU) return B200_ERROR_INVALID_PARAM;
  if (K % 8 || lda % 8 || ldb % 8 || ldc % 8 || lda < K || ldb < K || N % 8) return B200_ERROR_INVALID_PARAM;
  if (epi == B200_EPI_SWIGLU && N % 16) return B200_ERROR_INVALID_PARAM;
  if (ldc < (epi == B200_EPI_SWIGLU ? N / 2 : N)) return B200_ERROR_INVALID_PARAM;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al(A) || !al(B) || !al(Cp)) return B200_ERROR_INVALID_PARAM;
  if (rows == 0) return B200_OK;
  if (rows > INT32_MAX / 2 || (int64_t)groups * N > INT32_MAX / 2 || K > INT32_MAX) return B200_ERROR_UNSUPPORTED;
  // Few tokens per group (decode): weights on the 128-row MMA side, up to 64
  // tokens of a group on the N side.  Otherwise tokens on the 128-row side.
  const bool swap = rows <= 96LL * groups;
  GemmPlan g;
  g.swap = swap;
  g.bn = swap ? 64 : (N > 128 ? 256 : 128);
  g.kb_total = (int)((K + BK - 1) / BK);
  g.kb_per_split = g.kb_total;
  g.splits = 1;
  const int feat_tile = swap ? BM : g.bn, tok_tile = swap ? g.bn : BM;
  const int gF = (int)((N + feat_tile - 1) / feat_tile);
  // host upper bound of the units: every group's partial token tile + the full ones
  const int64_t max_units = ((rows + tok_tile - 1) / tok_tile + groups) * (int64_t)gF;
  g.tiles_m = swap ? gF : 1;
  g.tiles_n = swap ? 1 : gF;
  Params p = make_params(g, rows, N, K, Cp, ldc, nullptr, nullptr, 0, nullptr);
  p.goff = goff;
  p.groups = groups;
  p.gN = N;
  p.gF = gF;
  p.gRows = rows;
  CUtensorMap tw, tt;  // weights [groups * N, K], tokens [rows, K]
  if (!make_tmap(&tw, B, (int64_t)groups * N, K, ldb, swap ? BM : g.bn) ||
      !make_tmap(&tt, A, rows, K, lda, swap ? g.bn : BM))
    return B200_ERROR_UNSUPPORTED;
  const int grid = (int)std::min<int64_t>(max_units, num_sms());
  if (swap)
    return epi == B200_EPI_SWIGLU ? launch_t<64, B200_EPI_SWIGLU, true, false, true>(tw, tt, p, grid, st)
                                  : launch_t<64, B200_EPI_NONE, true, false, true>(tw, tt, p, grid, st);
  if (g.bn == 256)
    return epi == B200_EPI_SWIGLU ? launch_t<256, B200_EPI_SWIGLU, false, false, true>(tt, tw, p, grid, st)
                                  : launch_t<256, B200_EPI_NONE, false, false, true>(tt, tw, p, grid, st);
  return epi == B200_EPI_SWIGLU ? launch_t<128, B200_EPI_SWIGLU, false, false, true>(tt, tw, p, grid, st)
                                : launch_t<128, B200_EPI_NONE, false, false, true>(tt, tw, p, grid, st);
}

int gemm_run(const void* A, int64_t lda, const void* B, int64_t ldb, void* Cp, int64_t ldc, int64_t M, int64_t N,
             int64_t K, int epi, const void* bias, const void* R, int64_t ldr, void* ws, int64_t ws_bytes,
             cudaStream_t st) {
  int splits = 1;
  int rc = gemm_launch(A, lda, B, ldb, Cp, ldc, M, N, K, epi, bias, R, ldr, ws, ws_bytes, st, &splits);
  if (rc != B200_OK || splits <= 1) return rc;
  return splitk_reduce(static_cast<const float*>(ws), splits, M, N, epi, bias, R, ldr, Cp, ldc, st);
}

}  // namespace b200

extern "C" int b200_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M,
                              int64_t N, int64_t K, int epilogue, const void* bias, const void* residual, int64_t ldr,
                              void* workspace, int64_t workspace_bytes, b200_stream_t stream) {
  return b200::gemm_run(A, lda, B, ldb, C, ldc, M, N, K, epilogue, bias, residual, ldr, workspace, workspace_bytes,
                        stream);
}

extern "C" int b200_grouped_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                                      const int32_t* group_offsets, int groups, int64_t rows, int64_t N, int64_t K,
                                      int epilogue, b200_stream_t stream) {
  return b200::grouped_gemm_launch(A, lda, B, ldb, C, ldc, group_offsets, groups, rows, N, K, epilogue, stream);
}

extern "C" int64_t b200_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int epilogue) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return b200::plan_gemm(M, N, K, epilogue, num_sms()).ws_bytes;
}

