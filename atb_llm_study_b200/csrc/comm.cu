// Tensor-parallel communication for the engine: an NCCL communicator for the
// large (prefill-sized) all-reduces, and a symmetric buffer shared by CUDA IPC
// over NVLink for the fused decode-sized ones — one kernel that, on every
// rank, sums the ranks' partial rows straight from peer memory (in rank order,
// so every rank gets identical bits), adds the residual and applies the next
// RMSNorm; plus the vocabulary-parallel argmax exchange.
//
// Symmetric region of each rank: [flags: uint64 per source rank][argmax pairs]
// [partials, parity 0][partials, parity 1].  A call's epoch comes from a
// per-communicator device counter (so replayed CUDA graphs advance it); a rank
// publishes "my partials of epoch e are complete" by storing e into its slot
// of every peer's flag array and waits (bounded) until every slot of its own
// array reaches e.  Partials alternate between two buffers by call parity: a
// rank rewrites parity p only after finishing the next call, which needs every
// peer's signal for it, which each peer sends only after finishing the call
// that read parity p.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

using namespace b200;

namespace b200 {
unsigned* error_word(int device);
}

namespace {

constexpr int kMaxRanks = 8;
constexpr int64_t kFlagBytes = 4096;
constexpr int64_t kArgmaxRows = 8192;
constexpr int64_t kArgmaxBytes = kArgmaxRows * 8;
constexpr int64_t kHeader = kFlagBytes + kArgmaxBytes;

// ---- NCCL, loaded at run time (the library stays loadable without it) ----
struct Nccl {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  bool ok = false;
};

const Nccl& nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    n.GetUniqueId = reinterpret_cast<decltype(n.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    n.CommInitRank = reinterpret_cast<decltype(n.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
    n.AllReduce = reinterpret_cast<decltype(n.AllReduce)>(dlsym(h, "ncclAllReduce"));
    n.AllGather = reinterpret_cast<decltype(n.AllGather)>(dlsym(h, "ncclAllGather"));
    n.CommDestroy = reinterpret_cast<decltype(n.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
    n.ok = n.GetUniqueId && n.CommInitRank && n.AllReduce && n.AllGather && n.CommDestroy;
  });
  return n;
}

struct Peers {
  const uint8_t* base[kMaxRanks];  // every rank's symmetric region (own included)
  uint64_t* flags;                 // this rank's flag array
  int world, rank;
};

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Thread 0 of a CTA: publish epoch `ep` to every rank, then wait (bounded) for
// every rank's publication.  Redundant publications from several CTAs store the
// same value.
__device__ void exchange(const Peers& pp, uint64_t ep, unsigned* err) {
  __threadfence_system();
  for (int r = 0; r < pp.world; ++r) {
    uint64_t* slot = reinterpret_cast<uint64_t*>(const_cast<uint8_t*>(pp.base[r])) + pp.rank;
    st_release_sys(slot, ep);
  }
  const uint64_t t0 = global_timer_ns();
  for (int r = 0; r < pp.world; ++r) {
    while (ld_acquire_sys(pp.flags + r) < ep) {
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        raise_error(err, DEV_ERR_WAIT_TIMEOUT);
        return;
      }
    }
  }
}

// The last CTA to finish advances the communicator's epoch for the next call.
__device__ void finish(uint64_t* epoch, unsigned* done, uint64_t ep) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0;
      *reinterpret_cast<volatile uint64_t*>(epoch) = ep;
      __threadfence();
    }
  }
}

constexpr int kArThreads = 256;

// hidden[t] += sum_r partial_r[t] (ranks in order, fp32, one rounding);
// normed[t] = RMSNorm(hidden[t]) * norm_w when norm_w is not null.
template <int CH>
__global__ void __launch_bounds__(kArThreads) allreduce_rmsnorm_kernel(Peers pp, int64_t buf_off, int64_t T, int64_t H,
                                                                        __nv_bfloat16* hidden,
                                                                        const __nv_bfloat16* __restrict__ norm_w,
                                                                        __nv_bfloat16* normed, float eps,
                                                                        uint64_t* epoch, unsigned* done,
                                                                        unsigned* err) {
  pdl_trigger();
  pdl_wait();
  __shared__ uint64_t ep_s;
  __shared__ float red[kArThreads / 32];
  if (threadIdx.x == 0) {
    ep_s = *reinterpret_cast<volatile uint64_t*>(epoch) + 1;
    exchange(pp, ep_s, err);
  }
  __syncthreads();
  const uint64_t ep = ep_s;
  const int64_t nch = H / 8;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    float v[CH][8];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int64_t idx = threadIdx.x + (int64_t)c * kArThreads;
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] = 0.f;
      if (idx < nch) {
        // every rank's partial requested before the first add (rank order kept):
        // one NVLink round trip, not one per rank
        uint4 part[kMaxRanks];
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
          if (r < pp.world) part[r] = __ldcg(reinterpret_cast<const uint4*>(pp.base[r] + buf_off) + t * nch + idx);
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
          if (r < pp.world) {
            float a[8];
            unpack8(part[r], a);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[c][i] += a[i];
          }
        float res[8];
        unpack8(*reinterpret_cast<const uint4*>(hidden + t * H + idx * 8), res);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] += res[i];
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int64_t idx = threadIdx.x + (int64_t)c * kArThreads;
      if (idx < nch) {
        const uint4 o = pack8(v[c]);
        *reinterpret_cast<uint4*>(hidden + t * H + idx * 8) = o;
        unpack8(o, v[c]);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
      }
    }
    if (norm_w) {
      ss = warp_sum(ss);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
      __syncthreads();
      if (threadIdx.x < 32) {
        float s = threadIdx.x < kArThreads / 32 ? red[threadIdx.x] : 0.f;
        s = warp_sum(s);
        if (threadIdx.x == 0) red[0] = s;
      }
      __syncthreads();
      const float rstd = rsqrtf(red[0] / (float)H + eps);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int64_t idx = threadIdx.x + (int64_t)c * kArThreads;
        if (idx < nch) {
          float g[8];
          unpack8(*reinterpret_cast<const uint4*>(norm_w + idx * 8), g);
#pragma unroll
          for (int i = 0; i < 8; ++i) g[i] *= v[c][i] * rstd;
          *reinterpret_cast<uint4*>(normed + t * H + idx * 8) = pack8(g);
        }
      }
      __syncthreads();  // red[] is reused by the next row
    }
  }
  finish(epoch, done, ep);
}

// Local argmax of each row of this rank's vocabulary shard -> (value, global
// index) pairs in the symmetric argmax area.  One CTA per row.
__global__ void shard_argmax_kernel(const __nv_bfloat16* __restrict__ logits, int64_t V, int64_t ld, int64_t offset,
                                    uint8_t* pairs) {
  pdl_trigger();
  pdl_wait();
  __shared__ float sv[32];
  __shared__ int64_t si[32];
  const int64_t r = blockIdx.x;
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  for (int64_t j = threadIdx.x; j < V; j += blockDim.x) {
    const float x = bf2f(logits[r * ld + j]);
    if (x > bv || (x == bv && j < bi)) {
      bv = x;
      bi = j;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
        bv = sv[w];
        bi = si[w];
      }
    float* p = reinterpret_cast<float*>(pairs + r * 8);
    p[0] = bv;
    reinterpret_cast<int32_t*>(p)[1] = (int32_t)(bi == INT64_MAX ? 0 : bi + offset);
  }
}

// out[r] = the global argmax over every rank's pair (value desc, index asc).
__global__ void gather_argmax_kernel(Peers pp, int64_t rows, int64_t* out, uint64_t* epoch, unsigned* done,
                                     unsigned* err) {
  pdl_trigger();
  pdl_wait();
  __shared__ uint64_t ep_s;
  if (threadIdx.x == 0) {
    ep_s = *reinterpret_cast<volatile uint64_t*>(epoch) + 1;
    exchange(pp, ep_s, err);
  }
  __syncthreads();
  for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) {
    float bv = -INFINITY;
    int32_t bi = INT32_MAX;
    uint2 pr[kMaxRanks];  // every rank's pair requested before the comparisons
#pragma unroll
    for (int k = 0; k < kMaxRanks; ++k)
      if (k < pp.world) pr[k] = __ldcg(reinterpret_cast<const uint2*>(pp.base[k] + kFlagBytes + r * 8));
#pragma unroll
    for (int k = 0; k < kMaxRanks; ++k) {
      if (k >= pp.world) break;
      const uint2 u = pr[k];
      const float v = __uint_as_float(u.x);
      const int32_t i = (int32_t)u.y;
      if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
      }
    }
    out[r] = bi;
  }
  finish(epoch, done, ep_s);
}

// ---- expert parallel: token dispatch and weighted combine over peer memory ----
//
// Each rank routes its own tokens and groups its (token, choice) rows by
// expert (send rows + E+1 group offsets, both in its symmetric region).
// Rank d owns experts [d*El, (d+1)*El).  Dispatch: rank d pulls, for each
// local expert j and each source s in that order, source s's rows of expert
// d*El+j straight from s's symmetric region into a contiguous receive buffer
// (expert-major, then source rank, then the source's row order) and writes
// the El+1 group offsets its grouped GEMMs read.  Combine: every rank pulls
// the expert outputs of its own rows back from the owners' symmetric result
// buffers and sums them with the routing weights, the residual and the
// shared expert, then applies the next RMSNorm.

constexpr int kEpThreads = 256;
constexpr int kEpMaxExperts = 256;
constexpr int kEpMaxTopK = 8;

__device__ __forceinline__ int32_t clampi(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : v > hi ? hi : v; }

// One warp: exclusive scan of v[0..n) in place (n <= 2048), returns the total.
__device__ int32_t warp_exclusive_scan(int32_t* v, int n) {
  const int lane = threadIdx.x & 31;
  int32_t carry = 0;
  for (int base = 0; base < n; base += 32) {
    const int i = base + lane;
    const int32_t x = i < n ? v[i] : 0;
    int32_t inc = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += y;
    }
    if (i < n) v[i] = carry + inc - x;
    carry += __shfl_sync(0xffffffffu, inc, 31);
  }
  return carry;
}

__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(Peers pp, int64_t off_offsets, int64_t off_rows,
                                                                  int E, int El, int64_t H, int32_t send_cap,
                                                                  __nv_bfloat16* __restrict__ recv, int32_t recv_cap,
                                                                  int32_t* __restrict__ recv_offsets,
                                                                  int32_t* __restrict__ row_base, uint64_t* epoch,
                                                                  unsigned* done, unsigned* err) {
  pdl_trigger();
  pdl_wait();
  __shared__ uint64_t ep_s;
  __shared__ int32_t ro[kEpMaxExperts + 1];   // receive offset of group g = j*P + s
  __shared__ int32_t start[kEpMaxExperts];    // first send row of group g at its source
  __shared__ int32_t tot[kEpMaxExperts];      // block 0: rows of expert e over all sources
  __shared__ int32_t before[kEpMaxExperts];   // block 0: rows of expert e from sources < this rank
  if (threadIdx.x == 0) {
    ep_s = *reinterpret_cast<volatile uint64_t*>(epoch) + 1;
    exchange(pp, ep_s, err);
  }
  __syncthreads();
  const int P = pp.world, G = El * P, e0 = pp.rank * El;
  for (int g = threadIdx.x; g < G; g += blockDim.x) {
    const int j = g / P, s = g - j * P;
    const int32_t* o = reinterpret_cast<const int32_t*>(pp.base[s] + off_offsets);
    const int32_t a = clampi(__ldcg(o + e0 + j), 0, send_cap);
    const int32_t b = clampi(__ldcg(o + e0 + j + 1), a, send_cap);
    start[g] = a;
    ro[g] = b - a;
  }
  if (blockIdx.x == 0) {
    // where this rank's rows of every expert land on the expert's owner:
    // row_base[e] = rows of the owner's earlier experts + rows of expert e from lower ranks
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      int32_t t = 0, bsum = 0;
      for (int s = 0; s < P; ++s) {
        const int32_t* o = reinterpret_cast<const int32_t*>(pp.base[s] + off_offsets);
        const int32_t a = clampi(__ldcg(o + e), 0, send_cap);
        const int32_t n = clampi(__ldcg(o + e + 1), a, send_cap) - a;
        t += n;
        if (s < pp.rank) bsum += n;
      }
      tot[e] = t;
      before[e] = bsum;
    }
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int32_t total = warp_exclusive_scan(ro, G);
    if (threadIdx.x == 0) ro[G] = total;
  }
  if (blockIdx.x == 0) {
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      int32_t b = before[e];
      for (int f = (e / El) * El; f < e; ++f) b += tot[f];
      row_base[e] = b;
    }
    for (int j = threadIdx.x; j <= El; j += blockDim.x) recv_offsets[j] = min(ro[j * P], recv_cap);
  }
  __syncthreads();
  int32_t total = ro[G];
  if (total > recv_cap) {
    if (threadIdx.x == 0) raise_error(err, DEV_ERR_BAD_INDEX);
    total = recv_cap;
  }
  // one warp per received row; every lane issues all its remote loads of a
  // row (up to kCopyUnroll 16-byte chunks) before the first store, so a row
  // costs one NVLink round trip rather than one per chunk
  constexpr int kCopyUnroll = 8;
  const int64_t nch = H / 8;
  const int lane = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * (kEpThreads / 32);
  for (int64_t i = (int64_t)blockIdx.x * (kEpThreads / 32) + (threadIdx.x >> 5); i < total; i += nw) {
    int lo = 0, hi = G;  // ro[lo] <= i < ro[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (ro[mid] <= i) lo = mid;
      else hi = mid;
    }
    const int s = lo % P;
    const int64_t src = start[lo] + (i - ro[lo]);
    const uint4* sp = reinterpret_cast<const uint4*>(pp.base[s] + off_rows) + src * nch;
    uint4* dp = reinterpret_cast<uint4*>(recv) + i * nch;
    for (int64_t c0 = lane; c0 < nch; c0 += 32 * kCopyUnroll) {
      uint4 r[kCopyUnroll];
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u)
        if (c0 + u * 32 < nch) r[u] = __ldcg(sp + c0 + u * 32);
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u)
        if (c0 + u * 32 < nch) dp[c0 + u * 32] = r[u];
    }
  }
  finish(epoch, done, ep_s);
}

template <int CH>
__global__ void __launch_bounds__(kEpThreads) ep_combine_kernel(
    Peers pp, int64_t off_results, int32_t recv_cap, const int32_t* __restrict__ row_base,
    const int32_t* __restrict__ own_offsets, const int32_t* __restrict__ ids, const float* __restrict__ w,
    const int32_t* __restrict__ pos, int64_t T, int k, int E, int El, int64_t H, const __nv_bfloat16* residual,
    const __nv_bfloat16* __restrict__ shared, __nv_bfloat16* out, const __nv_bfloat16* __restrict__ norm_w,
    __nv_bfloat16* __restrict__ normed, float eps, uint64_t* epoch, unsigned* done, unsigned* err) {
  pdl_trigger();
  pdl_wait();
  __shared__ uint64_t ep_s;
  __shared__ float red[kEpThreads / 32];
  if (threadIdx.x == 0) {
    ep_s = *reinterpret_cast<volatile uint64_t*>(epoch) + 1;
    exchange(pp, ep_s, err);
  }
  __syncthreads();
  const int64_t nch = H / 8;
  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    float v[CH][8];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int64_t idx = threadIdx.x + (int64_t)c * kEpThreads;
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] = 0.f;
      if (idx < nch) {
        float a[8];
        if (residual) {
          unpack8(*reinterpret_cast<const uint4*>(residual + t * H + idx * 8), a);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[c][i] = a[i];
        }
        if (shared) {
          unpack8(*reinterpret_cast<const uint4*>(shared + t * H + idx * 8), a);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[c][i] += a[i];
        }
      }
    }
    // every choice's source row first, then all the remote loads, then the
    // weighted sum in choice order (one NVLink round trip per token)
    const uint4* yrow[kEpMaxTopK];
    float wj[kEpMaxTopK];
#pragma unroll
    for (int j = 0; j < kEpMaxTopK; ++j) {
      yrow[j] = nullptr;
      wj[j] = 0.f;
      if (j < k) {
        const int32_t p = pos[t * k + j];
        const int32_t e = ids[t * k + j];
        if (p >= 0 && e >= 0 && e < E) {
          const int64_t row = (int64_t)row_base[e] + (p - own_offsets[e]);
          if (row >= 0 && row < recv_cap) {
            yrow[j] = reinterpret_cast<const uint4*>(pp.base[e / El] + off_results) + row * nch;
            wj[j] = w[t * k + j];
          } else if (threadIdx.x == 0) {
            raise_error(err, DEV_ERR_BAD_INDEX);
          }
        }
      }
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int64_t idx = threadIdx.x + (int64_t)c * kEpThreads;
      if (idx < nch) {
        uint4 ys[kEpMaxTopK];
#pragma unroll
        for (int j = 0; j < kEpMaxTopK; ++j)
          if (yrow[j]) ys[j] = __ldcg(yrow[j] + idx);
#pragma unroll
        for (int j = 0; j < kEpMaxTopK; ++j) {
          if (!yrow[j]) continue;
          float a[8];
          unpack8(ys[j], a);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[c][i] = fmaf(wj[j], a[i], v[c][i]);
        }
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int64_t idx = threadIdx.x + (int64_t)c * kEpThreads;
      if (idx < nch) {
        const uint4 o = pack8(v[c]);
        *reinterpret_cast<uint4*>(out + t * H + idx * 8) = o;
        unpack8(o, v[c]);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
      }
    }
    if (norm_w) {
      ss = warp_sum(ss);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
      __syncthreads();
      if (threadIdx.x < 32) {
        float s = threadIdx.x < kEpThreads / 32 ? red[threadIdx.x] : 0.f;
        s = warp_sum(s);
        if (threadIdx.x == 0) red[0] = s;
      }
      __syncthreads();
      const float rstd = rsqrtf(red[0] / (float)H + eps);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int64_t idx = threadIdx.x + (int64_t)c * kEpThreads;
        if (idx < nch) {
          float g[8];
          unpack8(*reinterpret_cast<const uint4*>(norm_w + idx * 8), g);
#pragma unroll
          for (int i = 0; i < 8; ++i) g[i] *= v[c][i] * rstd;
          *reinterpret_cast<uint4*>(normed + t * H + idx * 8) = pack8(g);
        }
      }
      __syncthreads();
    }
  }
  finish(epoch, done, ep_s);
}

}  // namespace

struct b200_comm_s {
  int world = 1, rank = 0, device = 0;
  ncclComm_t nccl = nullptr;
  uint8_t* sym = nullptr;
  int64_t sym_bytes = 0;
  uint8_t* peers[kMaxRanks] = {nullptr};
  bool opened[kMaxRanks] = {false};
  uint64_t* epoch = nullptr;
  unsigned* done = nullptr;
  bool connected = false;
};

namespace {
Peers peers_of(const b200_comm_s* c) {
  Peers p;
  for (int r = 0; r < kMaxRanks; ++r) p.base[r] = r < c->world ? c->peers[r] : nullptr;
  p.flags = reinterpret_cast<uint64_t*>(c->sym);
  p.world = c->world;
  p.rank = c->rank;
  return p;
}
int64_t half_bytes(const b200_comm_s* c) { return ((c->sym_bytes - kHeader) / 2) & ~int64_t(255); }
int cuda_rc(cudaError_t e) { return e == cudaSuccess ? B200_OK : B200_ERROR_CUDA_BASE - (int)e; }
// Offset of [p, p + bytes) inside this rank's symmetric region (every rank's
// copy of it sits at the same offset), or -1 when it is not inside.
int64_t sym_offset(const b200_comm_s* c, const void* p, int64_t bytes) {
  const auto* q = static_cast<const uint8_t*>(p);
  if (!p || q < c->sym + kHeader || bytes < 0 || q + bytes > c->sym + c->sym_bytes) return -1;
  return q - c->sym;
}
}  // namespace

extern "C" int b200_comm_unique_id(void* id_out) {
  if (!id_out) return B200_ERROR_INVALID_PARAM;
  if (!nccl().ok) return B200_ERROR_UNSUPPORTED;
  ncclUniqueId id;
  if (nccl().GetUniqueId(&id) != ncclSuccess) return B200_ERROR_INFERENCE;
  std::memcpy(id_out, &id, sizeof(id));
  return B200_OK;
}

extern "C" int b200_comm_create(int world, int rank, int device, const void* nccl_id, int64_t sym_bytes,
                                b200_comm_t* out) {
  if (!out || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || sym_bytes < kHeader + 2 * 4096)
    return B200_ERROR_INVALID_PARAM;
  *out = nullptr;
  if (cudaSetDevice(device) != cudaSuccess) return B200_ERROR_INVALID_PARAM;
  auto* c = new (std::nothrow) b200_comm_s();
  if (!c) return B200_ERROR_DEVICE_MEMORY;
  c->world = world;
  c->rank = rank;
  c->device = device;
  c->sym_bytes = sym_bytes;
  int rc = cuda_rc(cudaMalloc(&c->sym, (size_t)sym_bytes));
  if (rc == B200_OK) rc = cuda_rc(cudaMemset(c->sym, 0, (size_t)kHeader));
  if (rc == B200_OK) rc = cuda_rc(cudaMalloc(&c->epoch, 64));
  if (rc == B200_OK) rc = cuda_rc(cudaMemset(c->epoch, 0, 64));
  if (rc == B200_OK) c->done = reinterpret_cast<unsigned*>(c->epoch + 1);
  if (rc == B200_OK && world > 1) {
    if (!nccl_id) rc = B200_ERROR_INVALID_PARAM;
    else if (!nccl().ok) rc = B200_ERROR_UNSUPPORTED;
    else {
      ncclUniqueId id;
      std::memcpy(&id, nccl_id, sizeof(id));
      if (nccl().CommInitRank(&c->nccl, world, id, rank) != ncclSuccess) rc = B200_ERROR_INFERENCE;
    }
  }
  c->peers[rank] = c->sym;
  if (world == 1) c->connected = true;
  if (rc == B200_OK) rc = cuda_rc(cudaDeviceSynchronize());
  if (rc != B200_OK) {
    if (c->nccl) nccl().CommDestroy(c->nccl);
    if (c->sym) cudaFree(c->sym);
    if (c->epoch) cudaFree(c->epoch);
    delete c;
    return rc;
  }
  *out = c;
  return B200_OK;
}

extern "C" int b200_comm_ipc_handle(b200_comm_t c, void* handle_out) {
  if (!c || !handle_out) return B200_ERROR_INVALID_PARAM;
  cudaIpcMemHandle_t h;
  cudaSetDevice(c->device);
  const int rc = cuda_rc(cudaIpcGetMemHandle(&h, c->sym));
  if (rc == B200_OK) std::memcpy(handle_out, &h, sizeof(h));
  return rc;
}

extern "C" int b200_comm_connect(b200_comm_t c, const void* handles) {
  if (!c || !handles) return B200_ERROR_INVALID_PARAM;
  cudaSetDevice(c->device);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank || c->opened[r]) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * sizeof(h), sizeof(h));
    void* p = nullptr;
    const int rc = cuda_rc(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    if (rc != B200_OK) return rc;
    c->peers[r] = static_cast<uint8_t*>(p);
    c->opened[r] = true;
  }
  c->connected = true;
  return B200_OK;
}

extern "C" int b200_comm_destroy(b200_comm_t c) {
  if (!c) return B200_OK;
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < kMaxRanks; ++r)
    if (c->opened[r]) cudaIpcCloseMemHandle(c->peers[r]);
  if (c->nccl) nccl().CommDestroy(c->nccl);
  if (c->sym) cudaFree(c->sym);
  if (c->epoch) cudaFree(c->epoch);
  delete c;
  return B200_OK;
}

extern "C" int b200_comm_info(b200_comm_t c, int* world, int* rank, void** buffer0, void** buffer1,
                              int64_t* buffer_bytes) {
  if (!c) return B200_ERROR_INVALID_PARAM;
  if (world) *world = c->world;
  if (rank) *rank = c->rank;
  if (buffer0) *buffer0 = c->sym + kHeader;
  if (buffer1) *buffer1 = c->sym + kHeader + half_bytes(c);
  if (buffer_bytes) *buffer_bytes = half_bytes(c);
  return B200_OK;
}

extern "C" int b200_comm_allreduce_bf16(b200_comm_t c, void* buf, int64_t count, b200_stream_t stream) {
  if (!c || !buf || count < 0) return B200_ERROR_INVALID_PARAM;
  if (c->world == 1 || count == 0) return B200_OK;
  if (!c->nccl) return B200_ERROR_UNSUPPORTED;
  return nccl().AllReduce(buf, buf, (size_t)count, ncclBfloat16, ncclSum, c->nccl, stream) == ncclSuccess
             ? B200_OK
             : B200_ERROR_INFERENCE;
}

extern "C" int b200_comm_allgather_bf16(b200_comm_t c, const void* send, void* recv, int64_t count,
                                        b200_stream_t stream) {
  if (!c || !send || !recv || count < 0) return B200_ERROR_INVALID_PARAM;
  if (count == 0) return B200_OK;
  if (c->world == 1) {
    return cuda_rc(cudaMemcpyAsync(recv, send, (size_t)count * 2, cudaMemcpyDeviceToDevice, stream));
  }
  if (!c->nccl) return B200_ERROR_UNSUPPORTED;
  return nccl().AllGather(send, recv, (size_t)count, ncclBfloat16, c->nccl, stream) == ncclSuccess
             ? B200_OK
             : B200_ERROR_INFERENCE;
}

extern "C" int b200_comm_allreduce_rmsnorm(b200_comm_t c, int parity, int64_t T, int64_t H, void* hidden,
                                           const void* norm_weight, void* normed, float eps, b200_stream_t stream) {
  if (!c || !hidden || T < 0 || H <= 0 || H % 8 || H > 8192 || (parity != 0 && parity != 1))
    return B200_ERROR_INVALID_PARAM;
  if (norm_weight && !normed) return B200_ERROR_INVALID_PARAM;
  if (!c->connected) return B200_ERROR_INVALID_PARAM;
  if ((int64_t)T * H * 2 > half_bytes(c)) return B200_ERROR_INVALID_PARAM;
  if (T == 0) return B200_OK;
  const Peers pp = peers_of(c);
  const int64_t off = kHeader + parity * half_bytes(c);
  const int64_t per = (H / 8 + kArThreads - 1) / kArThreads;
  const unsigned grid = (unsigned)std::min<int64_t>(T, 1024);
  auto hb = static_cast<__nv_bfloat16*>(hidden);
  auto nw = static_cast<const __nv_bfloat16*>(norm_weight);
  auto nb = static_cast<__nv_bfloat16*>(normed);
  unsigned* err = b200::error_word(c->device);
  // every CTA publishes the epoch before it waits, so no CTA depends on
  // another CTA of this rank being resident
  switch (per) {
    case 1: launch_kernel(allreduce_rmsnorm_kernel<1>, dim3(grid), kArThreads, 0, stream, pp, off, T, H, hb, nw, nb, eps, c->epoch, c->done, err); break;
    case 2: launch_kernel(allreduce_rmsnorm_kernel<2>, dim3(grid), kArThreads, 0, stream, pp, off, T, H, hb, nw, nb, eps, c->epoch, c->done, err); break;
    case 3:
    case 4: launch_kernel(allreduce_rmsnorm_kernel<4>, dim3(grid), kArThreads, 0, stream, pp, off, T, H, hb, nw, nb, eps, c->epoch, c->done, err); break;
    default: return B200_ERROR_UNSUPPORTED;
  }
  B200_CHECK_LAUNCH();
  return B200_OK;
}

extern "C" int b200_comm_argmax(b200_comm_t c, const void* logits, int64_t rows, int64_t vocab_local, int64_t ld,
                                int64_t* out, b200_stream_t stream) {
  if (!c || !logits || !out || rows < 0 || vocab_local <= 0 || ld < vocab_local || rows > kArgmaxRows)
    return B200_ERROR_INVALID_PARAM;
  if (!c->connected) return B200_ERROR_INVALID_PARAM;
  if ((int64_t)vocab_local * c->world > INT32_MAX) return B200_ERROR_UNSUPPORTED;
  if (rows == 0) return B200_OK;
  launch_kernel(shard_argmax_kernel, dim3((unsigned)rows), 256, 0, stream, static_cast<const __nv_bfloat16*>(logits),
                vocab_local, ld, (int64_t)c->rank * vocab_local, c->sym + kFlagBytes);
  B200_CHECK_LAUNCH();
  launch_kernel(gather_argmax_kernel, dim3(1), 256, 0, stream, peers_of(c), rows, out, c->epoch, c->done,
                b200::error_word(c->device));
  B200_CHECK_LAUNCH();
  return B200_OK;
}

extern "C" int b200_ep_dispatch(b200_comm_t c, const int32_t* send_offsets, const void* send_rows, int64_t send_cap,
                                int64_t experts, int64_t H, void* recv_rows, int64_t recv_cap, int32_t* recv_offsets,
                                int32_t* row_base, b200_stream_t stream) {
  if (!c || !recv_rows || !recv_offsets || !row_base || experts <= 0 || H <= 0 || H % 8 || send_cap < 0 ||
      recv_cap < 0 || send_cap > INT32_MAX || recv_cap > INT32_MAX)
    return B200_ERROR_INVALID_PARAM;
  if (!c->connected || experts % c->world || experts > kEpMaxExperts) return B200_ERROR_INVALID_PARAM;
  const int64_t oo = sym_offset(c, send_offsets, (experts + 1) * 4);
  const int64_t orow = sym_offset(c, send_rows, send_cap * H * 2);
  if (oo < 0 || orow < 0 || (oo & 3) || (orow & 15) || (reinterpret_cast<uintptr_t>(recv_rows) & 15))
    return B200_ERROR_INVALID_PARAM;
  const int El = (int)(experts / c->world);
  // enough warps to keep NVLink busy for the decode-sized batches, a full wave for prefill
  const int64_t want = (recv_cap + kEpThreads / 32 - 1) / (kEpThreads / 32);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, 2 * 148));
  launch_kernel(ep_dispatch_kernel, dim3(grid), kEpThreads, 0, stream, peers_of(c), oo, orow, (int)experts, El, H,
                (int32_t)send_cap, static_cast<__nv_bfloat16*>(recv_rows), (int32_t)recv_cap, recv_offsets, row_base,
                c->epoch, c->done, b200::error_word(c->device));
  B200_CHECK_LAUNCH();
  return B200_OK;
}

extern "C" int b200_ep_combine(b200_comm_t c, const void* results, int64_t recv_cap, const int32_t* row_base,
                               const int32_t* send_offsets, const int32_t* topk_ids, const float* topk_weights,
                               const int32_t* perm_pos, int64_t T, int top_k, int64_t experts, int64_t H,
                               const void* residual, const void* shared, void* out, const void* norm_weight,
                               void* normed, float eps, b200_stream_t stream) {
  if (!c || !row_base || !send_offsets || !topk_ids || !topk_weights || !perm_pos || !out || T < 0 || top_k <= 0 ||
      top_k > kEpMaxTopK || experts <= 0 || H <= 0 || H % 8 || recv_cap < 0 || recv_cap > INT32_MAX)
    return B200_ERROR_INVALID_PARAM;
  if (norm_weight && !normed) return B200_ERROR_INVALID_PARAM;
  if (!c->connected || experts % c->world || experts > kEpMaxExperts) return B200_ERROR_INVALID_PARAM;
  const int64_t ores = sym_offset(c, results, recv_cap * H * 2);
  if (ores < 0 || (ores & 15)) return B200_ERROR_INVALID_PARAM;
  for (const void* p : {(const void*)out, residual, shared, norm_weight, (const void*)normed})
    if (p && (reinterpret_cast<uintptr_t>(p) & 15)) return B200_ERROR_INVALID_PARAM;
  const int64_t per = (H / 8 + kEpThreads - 1) / kEpThreads;
  // every rank takes part in the exchange even with no tokens of its own
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(T, 1024));
  const int El = (int)(experts / c->world);
  auto rb = static_cast<const __nv_bfloat16*>(residual);
  auto sb = static_cast<const __nv_bfloat16*>(shared);
  auto ob = static_cast<__nv_bfloat16*>(out);
  auto nw = static_cast<const __nv_bfloat16*>(norm_weight);
  auto nb = static_cast<__nv_bfloat16*>(normed);
  unsigned* err = b200::error_word(c->device);
  const Peers pp = peers_of(c);
  switch (per) {
    case 1: launch_kernel(ep_combine_kernel<1>, dim3(grid), kEpThreads, 0, stream, pp, ores, (int32_t)recv_cap, row_base, send_offsets, topk_ids, topk_weights, perm_pos, T, top_k, (int)experts, El, H, rb, sb, ob, nw, nb, eps, c->epoch, c->done, err); break;
    case 2: launch_kernel(ep_combine_kernel<2>, dim3(grid), kEpThreads, 0, stream, pp, ores, (int32_t)recv_cap, row_base, send_offsets, topk_ids, topk_weights, perm_pos, T, top_k, (int)experts, El, H, rb, sb, ob, nw, nb, eps, c->epoch, c->done, err); break;
    case 3:
    case 4: launch_kernel(ep_combine_kernel<4>, dim3(grid), kEpThreads, 0, stream, pp, ores, (int32_t)recv_cap, row_base, send_offsets, topk_ids, topk_weights, perm_pos, T, top_k, (int)experts, El, H, rb, sb, ob, nw, nb, eps, c->epoch, c->done, err); break;
    default: return B200_ERROR_UNSUPPORTED;
  }
  B200_CHECK_LAUNCH();
  return B200_OK;
}
