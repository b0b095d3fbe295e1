// Prefill attention on the 5th-generation tensor cores: 64- or 128-wide heads,
// multi-head latent attention's decompressed heads (192-wide query / key:
// 128 no-rope + 64 rope dims, 128-wide value), and 16- / 32-wide heads run as
// 64-wide ones: a 3-D tensor map views every head as its own row of hd
// elements, and the 64-column box fills the columns past hd with zeros, so the
// scores are exact and only the first hd output columns are stored.
//
// One work item = 128 query rows of one head of one sequence; one persistent
// CTA per SM walks its share of the items (heaviest first), 320 threads:
//   warp 0      TMA producer: each item's Q tile, then K and V tiles of 128 keys
//               (64-column boxes, 128-byte swizzle) through rings guarded by
//               full/empty mbarriers: 2 K stages; 2 V stages, 1 for 192-wide
//               query/key heads (their tiles fill shared memory otherwise).
//   warp 1      allocates TMEM; one thread issues tcgen05.mma:
//               S_j = Q K_j^T into one of three TMEM score buffers (M=128,
//               N=128, K=128), and O += P_j V_j into the TMEM output
//               accumulator (P read from tensor memory, where the softmax
//               wrote it over its own scores; V read MN-major so no transpose
//               is ever materialised).  Each step issues P.V of the next tile
//               once its P is ready and then scores up to two tiles ahead, so
//               the tensor core computes S_{j+2} right behind P_j V_j while the
//               softmax warps work on S_{j+1}; a score buffer is reused once
//               the P.V that reads its P is done.
//   warps 2-9   softmax, two threads per query row (TMEM lane = row; warps
//               2-5 take key columns 0-63, warps 6-9 columns 64-127, so each
//               scheduler runs two softmax warps): load the row's scores,
//               mask (causal rule j > i and the sequence end), online max /
//               sum in the log2 domain (the two halves of a row exchange their
//               maxima through shared memory once per tile), write P (bf16
//               pairs) into TMEM over the half's own score columns (keys 0-63
//               at columns 0-31, keys 64-127 at 64-95), the layout the MMA
//               reads as its A operand.  The running max only moves when it grows by more than
//               2^8, so the O rows in TMEM are rescaled rarely; the final 1/l
//               scaling and the bf16 store happen once per item, from TMEM
//               (the next item's first P.V waits for that read; its scores do
//               not).
// Every mbarrier wait is bounded and sets the device error word on timeout.
// No TMA multicast (the library also runs in multi-GPU jobs).
#include <math.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

using namespace b200;

namespace {

constexpr int kThreads = 352;  // warps: 0 TMA, 1 score MMAs, 2-9 softmax, 10 P.V MMAs
constexpr int kPvWarp = 10;
constexpr int kTile = 128;                    // query rows per CTA = keys per tile
constexpr int kBoxBytes = kTile * 128;        // 128 rows x 64 bf16 (one 128-byte swizzle span)
constexpr int kXBytes = (4 + 2) * 128 * 4;    // row-half exchange: maxima [2 tiles][2 halves], sums [2 halves]
// query/key head width HDK (64, 128 or 192) and value width HDV (64 or 128):
// Q and K tiles are HDK / 64 boxes of 128 rows, V tiles HDV / 64 boxes
template <int HDK, int HDV>
struct TcCfg {
  static constexpr int BOXES_QK = HDK / 64, BOXES_V = HDV / 64;
  static constexpr int TILE_QK = BOXES_QK * kBoxBytes, TILE_V = BOXES_V * kBoxBytes;
  static constexpr int V_STAGES = HDK > 128 ? 1 : 2;
  // Q, K x2, V x V_STAGES, P + alignment + barriers
  static constexpr int SMEM = 3 * TILE_QK + V_STAGES * TILE_V + kXBytes + 1024 + 256;
  static constexpr uint32_t IDESC_O = idesc_bf16_f32(128, HDV) | (1u << 16);  // B operand (V) MN-major
};
constexpr uint32_t kTmemCols = 512;           // score / P buffers at [0,128) [128,256) [256,384), O at [384,512)
constexpr int kSBufs = 3;
constexpr uint32_t kOCol = 384;
constexpr float kRescaleLog2 = 8.f;           // move the running max only when it grows by > 2^8
constexpr uint32_t kIdescS = idesc_bf16_f32(128, 128);

// MN-major operand, 128-byte swizzle: 64-element rows of the MN dimension,
// 8-row groups of the K dimension 1024 bytes apart (SBO), the next 64
// MN elements `lbo` bytes away (LBO).
__device__ __forceinline__ uint64_t smem_desc_mn128(uint32_t addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t r[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 2^x on the special-function unit (PTX ex2.approx, relative error ~2^-22)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16: A (M x K, bf16 pairs per
// 32-bit column, row m in lane m) read from tensor memory.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// max(a, b, c) in one instruction (three-input max.f32 of sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Named barrier `id` over `n` threads.
__device__ __forceinline__ void named_bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
// Named barrier `id` over 64 threads returning the OR of `v` over them.
__device__ __forceinline__ bool pair_or(int id, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %2, 0;\n\tbar.red.or.pred q, %1, 64, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(id), "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

// One work item: 128 query rows (tile m) of head h of sequence sq.  Items are
// ordered heaviest first (causal tiles late in a sequence see more keys) and
// dealt round-robin to the persistent CTAs.
struct FaItem {
  int m, h, sq, start, len, m0, ntiles, kvh;
};

template <bool CAUSAL>
__device__ __forceinline__ FaItem fa_item(int w, const int32_t* __restrict__ cu, int nq, int nkv, int nseq,
                                          int mblocks) {
  FaItem it;
  const int per_m = nq * nseq;
  it.m = mblocks - 1 - w / per_m;
  const int r = w % per_m;
  it.h = r % nq;
  it.sq = r / nq;
  it.start = cu[it.sq];
  it.len = cu[it.sq + 1] - it.start;
  it.m0 = it.m * kTile;
  const int kt = (it.len + kTile - 1) / kTile;
  it.ntiles = it.m0 >= it.len ? 0 : (CAUSAL ? min(kt, it.m + 1) : kt);
  it.kvh = it.h / (nq / nkv);
  return it;
}

// First item index >= w of this CTA's sequence (w, w + G, ...) that has work, or W.
template <bool CAUSAL>
__device__ __forceinline__ int fa_next(int w, int W, int G, const int32_t* __restrict__ cu, int nq, int nkv,
                                       int nseq, int mblocks) {
  for (; w < W; w += G)
    if (fa_item<CAUSAL>(w, cu, nq, nkv, nseq, mblocks).ntiles > 0) return w;
  return W;
}

// HEADS3D: the maps are [rows][heads][hd] views (coordinates: column 0, head
// index, row) of heads narrower than the 64-column box; out_cols = hd.
// Persistent: gridDim.x CTAs walk the W = mblocks * nq * num_seqs items; TMEM,
// barriers and the K/V ring live across items, and the producer streams the
// next item's Q / K / V (and the MMA thread its first scores) while the
// current item finishes.
template <int HDK, int HDV, bool CAUSAL, bool HEADS3D = false>
__global__ void __launch_bounds__(kThreads, 1)
    flash_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ out, int64_t os,
                            int64_t ohs, const int32_t* __restrict__ cu, int nq, int nkv, int64_t qhs, int64_t khs,
                            int64_t vhs, float scale_log2, int mblocks, int nseq, int out_cols, unsigned* err) {
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  using Cf = TcCfg<HDK, HDV>;
  constexpr int kTileBytes = Cf::TILE_QK, kVBytes = Cf::TILE_V, VS = Cf::V_STAGES;
  uint8_t* sK = smem + kTileBytes;
  uint8_t* sV = smem + 3 * kTileBytes;
  float* sMx = reinterpret_cast<float*>(sV + VS * kVBytes);  // [tile parity][half][row]
  float* sL = sMx + 4 * 128;                            // [half][row]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sL + 2 * 128);
  uint64_t* q_full = bars;        // Q of the current item landed (once per item)
  uint64_t* q_empty = bars + 1;   // the item's last S issued and done: Q may be replaced
  uint64_t* k_full = bars + 2;    // [2]
  uint64_t* k_empty = bars + 4;   // [2]
  uint64_t* v_full = bars + 6;    // [2]
  uint64_t* v_empty = bars + 8;   // [2]
  uint64_t* s_full = bars + 10;   // [3] scores of the tile in buffer i ready
  uint64_t* p_full = bars + 13;   // [3] P of the tile in buffer i written (256 arrivals)
  uint64_t* pv_done = bars + 16;  // [3] P.V of the tile whose P sits in buffer i done
  uint64_t* o_free = bars + 19;   // the output accumulator read out (256 arrivals)
  uint64_t* drain = bars + 20;    // [2] MMA issuers' teardown after an abort
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int W = mblocks * nq * nseq;
  const int G = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < kSBufs; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 256);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(o_free, 256);
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // q / k / v and the sequence offsets come from earlier kernels
  const int w_first = fa_next<CAUSAL>(blockIdx.x, W, G, cu, nq, nkv, nseq, mblocks);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int g = 0, n = 0;  // K/V tiles and items so far
      for (int w = w_first; w < W && !*abort_flag; w = fa_next<CAUSAL>(w + G, W, G, cu, nq, nkv, nseq, mblocks), ++n) {
        const FaItem it = fa_item<CAUSAL>(w, cu, nq, nkv, nseq, mblocks);
        const int qc = (int)(it.h * qhs), kc = (int)(it.kvh * khs), vc = (int)(it.kvh * vhs);
        bool ok = true;
        for (int j = 0; j < it.ntiles; ++j, ++g) {
          const int st = g & 1;
          const uint32_t ph = (g >> 1) & 1;
          const int row = it.start + j * kTile;
          if (g >= 2 && !mbar_wait_idle(&k_empty[st], ph ^ 1, err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[st], kTileBytes);
          if (HEADS3D) tma_load_3d(sK + st * kTileBytes, &tmK, &k_full[st], 0, it.kvh, row);
          else
            for (int bx = 0; bx < Cf::BOXES_QK; ++bx)
              tma_load_2d(sK + st * kTileBytes + bx * kBoxBytes, &tmK, &k_full[st], kc + 64 * bx, row);
          if (j == 0) {
            // this item's Q, once the previous item's last scores are done with it
            if (n > 0 && !mbar_wait_idle(q_empty, (n - 1) & 1, err)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(q_full, kTileBytes);
            if (HEADS3D) tma_load_3d(sQ, &tmQ, q_full, 0, it.h, it.start + it.m0);
            else
              for (int bx = 0; bx < Cf::BOXES_QK; ++bx)
                tma_load_2d(sQ + bx * kBoxBytes, &tmQ, q_full, qc + 64 * bx, it.start + it.m0);
          }
          const int vst = g % VS;
          const uint32_t vph = (g / VS) & 1;
          if (g >= VS && !mbar_wait_idle(&v_empty[vst], vph ^ 1, err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full[vst], kVBytes);
          if (HEADS3D) tma_load_3d(sV + vst * kVBytes, &tmV, &v_full[vst], 0, it.kvh, row);
          else
            for (int bx = 0; bx < Cf::BOXES_V; ++bx)
              tma_load_2d(sV + vst * kVBytes + bx * kBoxBytes, &tmV, &v_full[vst], vc + 64 * bx, row);
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- score MMA issuer ----------------
    // S_g = Q K_g^T into score buffer g % 3, as soon as K_g has landed and the
    // P.V that read the buffer's previous P (tile g - 3) is done: the scores
    // run up to two tiles ahead of P.V, which warp 10 issues independently.
    if (lane == 0) {
      bool ok = true;
      int g = 0, n = 0;  // tiles and items so far
      for (int w = w_first; w < W && ok && !*abort_flag;
           w = fa_next<CAUSAL>(w + G, W, G, cu, nq, nkv, nseq, mblocks), ++n) {
        const FaItem it = fa_item<CAUSAL>(w, cu, nq, nkv, nseq, mblocks);
        if (!mbar_wait_idle(q_full, n & 1, err)) {  // this item's Q
          ok = false;
          break;
        }
        for (int j = 0; j < it.ntiles; ++j, ++g) {
          const int b = g % kSBufs, u = g / kSBufs;
          if (!mbar_wait_idle(&k_full[g & 1], (g >> 1) & 1, err) ||
              (g >= kSBufs && !mbar_wait_idle(&pv_done[b], (u - 1) & 1, err))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t q0 = smem_u32(sQ), k0 = smem_u32(sK + (g & 1) * kTileBytes);
#pragma unroll
          for (int ks = 0; ks < HDK / 16; ++ks) {
            const uint32_t off = (ks >> 2) * kBoxBytes + (ks & 3) * 32;
            umma_bf16(tmem + b * 128, smem_desc_k128(q0 + off), smem_desc_k128(k0 + off), kIdescS, ks > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[b]);
          umma_commit(&k_empty[g & 1]);
          if (j + 1 == it.ntiles) umma_commit(q_empty);  // Q may be replaced once these scores are done
        }
      }
      if (!ok) {
        *abort_flag = 1;
        umma_commit(&drain[0]);  // every MMA issued by this thread completes before TMEM is freed
        mbar_wait(&drain[0], 0, err);
      }
    }
    __syncwarp();
  } else if (warp == kPvWarp) {
    // ---------------- P.V MMA issuer ----------------
    // O += P_g V_g once the softmax has written P_g (bf16, in TMEM over its
    // own scores: keys 0-63 at columns 0-31, keys 64-127 at columns 64-95 of
    // buffer g % 3, the A operand) and V_g has landed; an item's first P.V
    // also waits until the softmax warps have read out the previous item.
    if (lane == 0) {
      bool ok = true;
      int g = 0, n = 0;
      for (int w = w_first; w < W && ok && !*abort_flag;
           w = fa_next<CAUSAL>(w + G, W, G, cu, nq, nkv, nseq, mblocks), ++n) {
        const FaItem it = fa_item<CAUSAL>(w, cu, nq, nkv, nseq, mblocks);
        for (int j = 0; j < it.ntiles; ++j, ++g) {
          const int b = g % kSBufs, vst = g % VS;
          if (!mbar_wait_idle(&p_full[b], (g / kSBufs) & 1, err) ||
              !mbar_wait_idle(&v_full[vst], (g / VS) & 1, err) ||
              (j == 0 && n >= 1 && !mbar_wait_idle(o_free, (n - 1) & 1, err))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t pa = tmem + b * 128, v0 = smem_u32(sV + vst * kVBytes);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            umma_bf16_ts(tmem + kOCol, pa + (ks >> 2) * 64 + (ks & 3) * 8, smem_desc_mn128(v0 + ks * 2048, kBoxBytes),
                         Cf::IDESC_O, (j > 0 || ks > 0) ? 1u : 0u);
          umma_commit(&pv_done[b]);
          umma_commit(&v_empty[vst]);
        }
      }
      if (!ok) {
        *abort_flag = 1;
        umma_commit(&drain[1]);
        mbar_wait(&drain[1], 0, err);
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax (warps 2..9: two threads per query row) ----------------
    // Warp w owns TMEM lanes 32 (w % 4) ..; warps 2-5 take key columns 0-63 of
    // every score row, warps 6-9 columns 64-127 (and the matching halves of P
    // and O).  The two threads of a row exchange their partial maxima through
    // shared memory once per tile (barrier of the warp pair), so both take the
    // same running-max decisions; row sums stay per thread until the item ends.
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lanes = (uint32_t)(quarter * 32) << 16;
    const int pair_bar = 1 + quarter;  // named barrier of warps (quarter + 2, quarter + 6)
    bool ok = true;
    int g = 0, n = 0;  // tiles and items so far
    for (int w = w_first; w < W && ok; w = fa_next<CAUSAL>(w + G, W, G, cu, nq, nkv, nseq, mblocks), ++n) {
      const FaItem it = fa_item<CAUSAL>(w, cu, nq, nkv, nseq, mblocks);
      const int qpos = it.m0 + row;  // query position within the sequence
      const uint32_t tO = tmem + lanes + kOCol + half * (HDV / 2);
      float mref = -INFINITY, l = 0.f;
      for (int j = 0; j < it.ntiles; ++j, ++g) {
        const int st = g % kSBufs;
        const uint32_t ph = (g / kSBufs) & 1;
        // warp-uniform outcome (the TMEM loads below are warp-collective), and
        // the same for both warps of the pair (they meet at named barriers)
        const bool got = __all_sync(0xffffffffu, ok && !*abort_flag && mbar_wait_idle(&s_full[st], ph, err));
        if (pair_or(pair_bar, !got)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[64];
        tmem_ld_32x32b_x32(tmem + lanes + st * 128 + half * 64, sr);
        tmem_ld_32x32b_x32(tmem + lanes + st * 128 + half * 64 + 32, sr + 32);
        tmem_ld_wait();
        const int kv0 = j * kTile + half * 64;  // first key of this thread's columns
        const bool full_half = kv0 + 64 <= it.len && (!CAUSAL || kv0 + 63 <= it.m0);
        // raw-score max of this half (scale > 0), masked keys set to -inf
        if (!full_half) {
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const int col = kv0 + c;
            if (col >= it.len || (CAUSAL && col > qpos)) sr[c] = __float_as_uint(-INFINITY);
          }
        }
        // eight independent chains of three-input maxima (two scores per instruction)
        float m8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = fmax3(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1]), -INFINITY);
#pragma unroll
        for (int c = 8; c < 32; ++c)
          m8[c & 7] = fmax3(m8[c & 7], __uint_as_float(sr[2 * c]), __uint_as_float(sr[2 * c + 1]));
        float mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        // the row's other half (slots alternate by tile: the partner is at most one tile behind)
        sMx[((g & 1) * 2 + half) * 128 + row] = mx;
        named_bar_sync(pair_bar, 64);
        mx = fmaxf(mx, sMx[((g & 1) * 2 + (half ^ 1)) * 128 + row]);
        mx *= scale_log2;
        // running max (log2 domain): moved only when it grows by more than 2^kRescaleLog2
        float alpha = 1.f;
        bool rescale = false;
        if (mx > mref + kRescaleLog2 || (mref == -INFINITY && mx > -INFINITY)) {
          rescale = mref != -INFINITY;
          alpha = rescale ? ex2(mref - mx) : 0.f;
          l *= alpha;
          mref = mx;
        }
        // P = 2^(s * scale - ref), packed to bf16 pairs in place
        const float ref = mref == -INFINITY ? 0.f : mref;
        float r8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) r8[i] = 0.f;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float p0 = ex2(fmaf(__uint_as_float(sr[2 * c]), scale_log2, -ref));
          const float p1 = ex2(fmaf(__uint_as_float(sr[2 * c + 1]), scale_log2, -ref));
          r8[c & 7] += p0 + p1;
          sr[c] = pack2(p0, p1);
        }
        const float rs = ((r8[0] + r8[1]) + (r8[2] + r8[3])) + ((r8[4] + r8[5]) + (r8[6] + r8[7]));
        if (j > 0 && __any_sync(0xffffffffu, rescale)) {
          // O holds the item's tiles < j once the previous tile's P.V is done
          // (per-buffer barrier: its previous phase, tile g - 4, is complete);
          // a failed wait is acted on at the next tile's pair vote (no exit between pair barriers)
          if (!__all_sync(0xffffffffu, mbar_wait_idle(&pv_done[(g - 1) % kSBufs], ((g - 1) / kSBufs) & 1, err)))
            ok = false;
          tc_fence_after();
          if (ok) {
#pragma unroll 1
            for (int c = 0; c < HDV / 64; ++c) {
              uint32_t r[32];
              tmem_ld_32x32b_x32(tO + c * 32, r);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * (rescale ? alpha : 1.f));
              tmem_st_32x32b_x32(tO + c * 32, r);
            }
            tmem_st_wait();
          }
        }
        // P over this half's own score columns (32 columns of bf16 pairs)
        tmem_st_32x32b_x32(tmem + lanes + st * 128 + half * 64, sr);
        tmem_st_wait();
        l += rs;
        tc_fence_before();
        mbar_arrive(&p_full[st]);
      }
      const bool done = __all_sync(0xffffffffu, ok && !*abort_flag &&
                                                    mbar_wait_idle(&pv_done[(g - 1) % kSBufs], ((g - 1) / kSBufs) & 1, err));
      if (pair_or(pair_bar, !done)) {
        ok = false;
        break;
      }
      // the row sum: both halves
      sL[half * 128 + row] = l;
      named_bar_sync(pair_bar, 64);
      l += sL[(half ^ 1) * 128 + row];
      named_bar_sync(pair_bar, 64);  // sL is rewritten at the next item's end
      // this item's output: O / l from TMEM, bf16 rows (this thread's half of the columns)
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool valid = qpos < it.len;
      __nv_bfloat16* orow =
          out + (int64_t)(it.start + (valid ? qpos : 0)) * os + (int64_t)it.h * ohs + half * (HDV / 2);
#pragma unroll 1
      for (int c = 0; c < HDV / 64; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tO + c * 32, r);
        tmem_ld_wait();
        if (valid) {
#pragma unroll
          for (int g4 = 0; g4 < 4; ++g4) {
            if (HEADS3D && half * (HDV / 2) + c * 32 + g4 * 8 >= out_cols) break;
            float f[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(r[8 * g4 + i]) * inv;
            *reinterpret_cast<uint4*>(orow + c * 32 + g4 * 8) = pack8(f);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(o_free);
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
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

// Row-major bf16 [rows, cols] with row stride ld (elements); box = 128 rows x
// 64 columns, 128-byte swizzle; rows past `rows` read as zeros.
bool make_map(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld) {
  EncodeTiledFn f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)kTile};
  cuuint32_t estr[2] = {1, 1};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [rows][heads][hd] view of a row-major bf16 matrix (row stride ld, head
// stride hs, elements) for heads narrower than 64: box = 64 x 1 head x 128
// rows, the 64 - hd columns past each head and rows past `rows` read as zeros.
bool make_map_heads(CUtensorMap* m, const void* ptr, int64_t rows, int64_t heads, int64_t hd, int64_t hs,
                    int64_t ld) {
  EncodeTiledFn f = encode_fn();
  if (!f) return false;
  cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)heads, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)(hs * 2), (cuuint64_t)(ld * 2)};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)kTile};
  cuuint32_t estr[3] = {1, 1, 1};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int HDK, int HDV, bool CAUSAL, bool HEADS3D = false>
int launch_tc(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, void* out, int64_t os,
              int64_t ohs, const int32_t* cu, int num_seqs, int mblocks, int nq, int nkv, int64_t qhs, int64_t khs,
              int64_t vhs, float scale_log2, int out_cols, cudaStream_t st) {
  auto k = flash_prefill_tc_kernel<HDK, HDV, CAUSAL, HEADS3D>;
  using Cf = TcCfg<HDK, HDV>;
  static_assert(Cf::SMEM <= 227 * 1024, "shared memory");
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return B200_ERROR_UNSUPPORTED;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM) != cudaSuccess)
      return B200_ERROR_UNSUPPORTED;
    attr_set[dev] = true;
  }
  // persistent: one CTA per SM (shared memory allows no second), each walking
  // every G-th work item
  static int sms[64] = {0};
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int64_t items = (int64_t)mblocks * nq * num_seqs;
  if (items > INT32_MAX) return B200_ERROR_UNSUPPORTED;
  const int grid = (int)std::min<int64_t>(items, sms[dev] > 0 ? sms[dev] : 148);
  launch_kernel(k, dim3(grid), kThreads, Cf::SMEM, st, mq, mk, mv, static_cast<__nv_bfloat16*>(out), os, ohs, cu, nq,
                nkv, qhs, khs, vhs, scale_log2, mblocks, num_seqs, out_cols, b200::error_word(dev));
  B200_CHECK_LAUNCH();
  return B200_OK;
}

}  // namespace

extern "C" int b200_flash_prefill_packed(const void* q, int64_t q_stride, int64_t q_head_stride, const void* k,
                                         int64_t k_stride, int64_t k_head_stride, const void* v, int64_t v_stride,
                                         int64_t v_head_stride, void* out, int64_t out_stride,
                                         int64_t out_head_stride, const int32_t* cu_seqlens, int num_seqs,
                                         int max_seqlen, int64_t total_tokens, int nq, int nkv, int head_dim_qk,
                                         int head_dim_v, float scale, int causal, b200_stream_t stream) {
  const bool tc_shape = (head_dim_qk == head_dim_v && (head_dim_qk == 128 || head_dim_qk == 64 ||
                                                      head_dim_qk == 32 || head_dim_qk == 16)) ||
                        (head_dim_qk == 192 && head_dim_v == 128);
  if (!tc_shape || total_tokens <= 0)
    return b200_flash_prefill_ex(q, q_stride, q_head_stride, k, k_stride, k_head_stride, v, v_stride, v_head_stride,
                                 out, out_stride, out_head_stride, cu_seqlens, num_seqs, max_seqlen, nq, nkv,
                                 head_dim_qk, head_dim_v, scale, causal, stream);
  if (!q || !k || !v || !out || !cu_seqlens || num_seqs < 0 || max_seqlen < 0 || nq <= 0 || nkv <= 0 || nq % nkv)
    return B200_ERROR_INVALID_PARAM;
  for (int64_t s : {q_stride, q_head_stride, k_stride, k_head_stride, v_stride, v_head_stride, out_stride,
                    out_head_stride})
    if (s < 0 || s % 8) return B200_ERROR_INVALID_PARAM;
  for (const void* p : {q, k, v, (const void*)out})
    if (reinterpret_cast<uintptr_t>(p) & 15u) return B200_ERROR_INVALID_PARAM;
  const int hd = head_dim_qk, hdv = head_dim_v;
  const int64_t qcols = (int64_t)(nq - 1) * q_head_stride + hd, kcols = (int64_t)(nkv - 1) * k_head_stride + hd,
                vcols = (int64_t)(nkv - 1) * v_head_stride + hdv;
  if (q_stride < qcols || k_stride < kcols || v_stride < vcols ||
      out_stride < (int64_t)(nq - 1) * out_head_stride + hdv)
    return B200_ERROR_INVALID_PARAM;
  if (num_seqs == 0 || max_seqlen == 0) return B200_OK;
  if (num_seqs > 65535 || nq > 65535 || total_tokens > INT32_MAX || qcols > INT32_MAX || kcols > INT32_MAX ||
      vcols > INT32_MAX)
    return B200_ERROR_UNSUPPORTED;
  const int mblocks = (max_seqlen + kTile - 1) / kTile;
  const float sl2 = scale * 1.4426950408889634f;
  // the maps end at the last packed row and at each operand's last head, so
  // no tile reads past the buffers: rows beyond total_tokens read as zeros
  CUtensorMap mq, mk, mv;
  if (hd < 64) {  // narrow heads as 64-wide ones, zero-filled past hd
    if (!make_map_heads(&mq, q, total_tokens, nq, hd, q_head_stride, q_stride) ||
        !make_map_heads(&mk, k, total_tokens, nkv, hd, k_head_stride, k_stride) ||
        !make_map_heads(&mv, v, total_tokens, nkv, hd, v_head_stride, v_stride))
      return B200_ERROR_UNSUPPORTED;
    return causal ? launch_tc<64, 64, true, true>(mq, mk, mv, out, out_stride, out_head_stride, cu_seqlens, num_seqs,
                                                  mblocks, nq, nkv, q_head_stride, k_head_stride, v_head_stride, sl2,
                                                  hd, stream)
                  : launch_tc<64, 64, false, true>(mq, mk, mv, out, out_stride, out_head_stride, cu_seqlens,
                                                   num_seqs, mblocks, nq, nkv, q_head_stride, k_head_stride,
                                                   v_head_stride, sl2, hd, stream);
  }
  if (!make_map(&mq, q, total_tokens, qcols, q_stride) || !make_map(&mk, k, total_tokens, kcols, k_stride) ||
      !make_map(&mv, v, total_tokens, vcols, v_stride))
    return B200_ERROR_UNSUPPORTED;
#define B200_TC(HK, HV, C)                                                                                     \
  launch_tc<HK, HV, C>(mq, mk, mv, out, out_stride, out_head_stride, cu_seqlens, num_seqs, mblocks, nq, nkv,     \
                       q_head_stride, k_head_stride, v_head_stride, sl2, HV, stream)
  if (hd == 192) return causal ? B200_TC(192, 128, true) : B200_TC(192, 128, false);
  if (hd == 128) return causal ? B200_TC(128, 128, true) : B200_TC(128, 128, false);
  return causal ? B200_TC(64, 64, true) : B200_TC(64, 64, false);
#undef B200_TC
}
