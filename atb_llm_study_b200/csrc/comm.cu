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
        for (int r = 0; r < pp.world; ++r) {
          const uint4* src = reinterpret_cast<const uint4*>(pp.base[r] + buf_off) + t * nch + idx;
          float a[8];
          unpack8(__ldcg(src), a);
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
    for (int k = 0; k < pp.world; ++k) {
      const uint2 u = __ldcg(reinterpret_cast<const uint2*>(pp.base[k] + kFlagBytes + r * 8));
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
