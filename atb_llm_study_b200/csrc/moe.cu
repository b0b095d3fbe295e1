// Mixture-of-experts plumbing around the grouped tcgen05 GEMM: router
// (gate logits + softmax + top-k), the expert permutation (tokens grouped by
// expert, stable in token order) and the weighted combine back into token
// order.  The reference only declares these as stubs (MoeBuilder,
// atb_cpp_llm/src/components/common/mlp_builder.h:73-82; MoEMlpGraph,
// atb_cpp_llm/src/components/moe/moe_mlp_graph.h:22-29; MlpConfig.num_experts /
// top_k, atb_cpp_llm/include/atb_llm/layer_desc.h:59-60).
//
// Routing follows the published Mixtral / DeepSeek-V2 gates: fp32 logits,
// softmax over the experts, the k largest (ties to the lower expert index),
// weights renormalised over the k chosen (Mixtral) or scaled (DeepSeek).
#include <math.h>

#include "common.cuh"

using namespace b200;

namespace {

constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 8;
constexpr int kPermChunk = 256;  // entries per permutation block (one warp)

// Router: a CTA of 256 threads per TPB tokens.  Each thread accumulates the
// dot products of its H/8-chunks with every expert row (the gate rows are
// read once per CTA for all its tokens), the warps' partial sums meet in
// shared memory, and warp tt finishes token tt: softmax and top-k, with
// expert e's logit in lane e % 32, slot e / 32.
constexpr int kRouteThreads = 256;

template <int EA, int TPB>
__global__ void __launch_bounds__(kRouteThreads) moe_route_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ wg,
    const float* __restrict__ logits_in, int64_t T, int64_t H, int E, int k, int renorm, float scale,
    int32_t* __restrict__ ids, float* __restrict__ wts, float* __restrict__ logits_out) {
  pdl_trigger();
  pdl_wait();
  constexpr int PER = (EA + 31) / 32, NW = kRouteThreads / 32;
  __shared__ float red[NW][TPB][EA];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t0 = (int64_t)blockIdx.x * TPB;
  if (!logits_in) {
    float acc[TPB][EA];
#pragma unroll
    for (int tt = 0; tt < TPB; ++tt)
#pragma unroll
      for (int e = 0; e < EA; ++e) acc[tt][e] = 0.f;
    for (int64_t c = threadIdx.x; c < H / 8; c += kRouteThreads) {
      float xv[TPB][8];
#pragma unroll
      for (int tt = 0; tt < TPB; ++tt) {
        if (t0 + tt < T) {
          unpack8(*reinterpret_cast<const uint4*>(x + (t0 + tt) * ldx + c * 8), xv[tt]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[tt][j] = 0.f;
        }
      }
#pragma unroll
      for (int e = 0; e < EA; ++e) {
        if (e < E) {
          float w[8];
          unpack8(*reinterpret_cast<const uint4*>(wg + (int64_t)e * H + c * 8), w);
#pragma unroll
          for (int tt = 0; tt < TPB; ++tt)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[tt][e] = fmaf(xv[tt][j], w[j], acc[tt][e]);
        }
      }
    }
#pragma unroll
    for (int tt = 0; tt < TPB; ++tt)
#pragma unroll
      for (int e = 0; e < EA; ++e) {
        const float s = warp_sum(acc[tt][e]);
        if (lane == 0) red[warp][tt][e] = s;
      }
    __syncthreads();
  }
  if (warp >= TPB) return;
  const int64_t t = t0 + warp;
  if (t >= T) return;
  float lg[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    if (e >= E) {
      lg[i] = -INFINITY;
    } else if (logits_in) {
      lg[i] = logits_in[t * E + e];
    } else {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) s += red[w][warp][e];
      lg[i] = s;
    }
  }
  if (logits_out) {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (e < E) logits_out[t * E + e] = lg[i];
    }
  }
  // softmax over the experts
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) m = fmaxf(m, lg[i]);
  m = warp_max(m);
  float pr[PER], s = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    pr[i] = lane + 32 * i < E ? __expf(lg[i] - m) : 0.f;
    s += pr[i];
  }
  s = warp_sum(s);
  const float inv = 1.0f / s;
#pragma unroll
  for (int i = 0; i < PER; ++i) pr[i] *= inv;
  // k rounds of warp argmax over the logits (value desc, index asc)
  uint32_t taken = 0;
  int sel_id[kMaxTopK];
  float sel_p[kMaxTopK];
  float sum_sel = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    sel_id[j] = 0;
    sel_p[j] = 0.f;
    if (j >= k) continue;
    float bv = -INFINITY, bp = 0.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !(taken >> i & 1u) && (lg[i] > bv || (lg[i] == bv && e < bi))) {
        bv = lg[i];
        bi = e;
        bp = pr[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const float op = __shfl_xor_sync(0xffffffffu, bp, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
        bp = op;
      }
    }
    if (bi < E && (bi & 31) == lane) taken |= 1u << (bi >> 5);
    sel_id[j] = bi;
    sel_p[j] = bp;
    sum_sel += bp;
  }
#pragma unroll
  for (int j = 0; j < kMaxTopK; ++j) {
    if (j < k && lane == j) {
      ids[t * k + j] = sel_id[j];
      wts[t * k + j] = renorm ? sel_p[j] / sum_sel : sel_p[j] * scale;
    }
  }
}

// Per block of kPermChunk entries: how many go to each expert.
__global__ void moe_count_kernel(const int32_t* __restrict__ ids, int64_t n, int E, int32_t* __restrict__ counts,
                                 unsigned* err) {
  pdl_trigger();
  pdl_wait();
  __shared__ int c[kMaxExperts];
  const int lane = threadIdx.x;
  for (int e = lane; e < E; e += 32) c[e] = 0;
  __syncwarp();
  const int64_t base = (int64_t)blockIdx.x * kPermChunk;
  for (int i = lane; i < kPermChunk && base + i < n; i += 32) {
    const int e = ids[base + i];
    if (e < 0 || e >= E) {
      raise_error(err, DEV_ERR_BAD_INDEX);
      continue;
    }
    atomicAdd(&c[e], 1);
  }
  __syncwarp();
  for (int e = lane; e < E; e += 32) counts[(int64_t)blockIdx.x * E + e] = c[e];
}

// Expert offsets (exclusive scan of the totals) and each block's first slot per expert.
__global__ void moe_scan_kernel(const int32_t* __restrict__ counts, int nb, int E, int32_t* __restrict__ base,
                                int32_t* __restrict__ offsets) {
  pdl_trigger();
  pdl_wait();
  __shared__ int tot[kMaxExperts + 1];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int s = 0;
    for (int b = 0; b < nb; ++b) s += counts[(int64_t)b * E + e];
    tot[e] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      const int v = tot[e];
      tot[e] = run;
      offsets[e] = run;
      run += v;
    }
    offsets[E] = run;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = tot[e];
    for (int b = 0; b < nb; ++b) {
      base[(int64_t)b * E + e] = run;
      run += counts[(int64_t)b * E + e];
    }
  }
}

// Slot of every entry: its expert's offset + the entries of that expert before
// it in entry order (so each expert's rows are in token order).
__global__ void moe_scatter_kernel(const int32_t* __restrict__ ids, int64_t n, int k, int E,
                                   const int32_t* __restrict__ base, int32_t* __restrict__ pos,
                                   int32_t* __restrict__ src) {
  pdl_trigger();
  pdl_wait();
  __shared__ int c[kMaxExperts];
  const int lane = threadIdx.x;
  for (int e = lane; e < E; e += 32) c[e] = base[(int64_t)blockIdx.x * E + e];
  __syncwarp();
  for (int ch = 0; ch < kPermChunk / 32; ++ch) {
    const int64_t i = (int64_t)blockIdx.x * kPermChunk + ch * 32 + lane;
    int e = -1;
    if (i < n) {
      e = ids[i];
      if (e < 0 || e >= E) e = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0) {
      const int p = c[e] + rank;
      pos[i] = p;
      src[p] = (int32_t)(i / k);
    } else if (i < n) {
      pos[i] = -1;
    }
    __syncwarp();
    if (e >= 0 && lane == 31 - __clz(peers)) c[e] += __popc(peers);
    __syncwarp();
  }
}

// x_perm[r] = x[src[r]] for the r < offsets[E] filled slots.
__global__ void moe_gather_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const int32_t* __restrict__ src,
                                  const int32_t* __restrict__ total, int64_t H, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int64_t r = blockIdx.x;
  if (r >= *total) return;
  const uint4* s = reinterpret_cast<const uint4*>(x + (int64_t)src[r] * ldx);
  uint4* d = reinterpret_cast<uint4*>(out + r * H);
  for (int64_t c = threadIdx.x; c < H / 8; c += blockDim.x) d[c] = s[c];
}

// out[t] = residual[t] + shared[t] + sum_j w[t, j] * y[pos[t*k + j]] (fp32,
// one rounding), then optionally normed[t] = RMSNorm(out[t]) * norm_w.
constexpr int kCombineThreads = 256;
template <int CH>
__global__ void __launch_bounds__(kCombineThreads) moe_combine_kernel(
    const __nv_bfloat16* __restrict__ y, const int32_t* __restrict__ pos, const float* __restrict__ w, int k,
    int64_t H, const __nv_bfloat16* residual, const __nv_bfloat16* __restrict__ shared, __nv_bfloat16* out,
    const __nv_bfloat16* __restrict__ norm_w, __nv_bfloat16* __restrict__ normed, float eps) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[kCombineThreads / 32];
  const int64_t t = blockIdx.x;
  const int64_t nch = H / 8;
  float v[CH][8];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kCombineThreads;
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
  // up to 8 choices at a time: their rows' loads all issued before the
  // weighted sum, which keeps choice order
  constexpr int kInFlight = 8;
  for (int j0 = 0; j0 < k; j0 += kInFlight) {
    const uint4* yrow[kInFlight];
    float wj[kInFlight];
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) {
      const int j = j0 + u;
      const int p = j < k ? pos[t * k + j] : -1;
      yrow[u] = p >= 0 ? reinterpret_cast<const uint4*>(y + (int64_t)p * H) : nullptr;
      wj[u] = p >= 0 ? w[t * k + j] : 0.f;
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int64_t idx = threadIdx.x + (int64_t)c * kCombineThreads;
      if (idx < nch) {
        uint4 ys[kInFlight];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u)
          if (yrow[u]) ys[u] = yrow[u][idx];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) {
          if (!yrow[u]) continue;
          float a[8];
          unpack8(ys[u], a);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[c][i] = fmaf(wj[u], a[i], v[c][i]);
        }
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kCombineThreads;
    if (idx < nch) {
      const uint4 o = pack8(v[c]);
      *reinterpret_cast<uint4*>(out + t * H + idx * 8) = o;
      unpack8(o, v[c]);  // the norm sees the stored (rounded) values
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
    }
  }
  if (!norm_w) return;
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float s = threadIdx.x < kCombineThreads / 32 ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) red[0] = s;
  }
  __syncthreads();
  const float rstd = rsqrtf(red[0] / (float)H + eps);
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kCombineThreads;
    if (idx < nch) {
      float g[8];
      unpack8(*reinterpret_cast<const uint4*>(norm_w + idx * 8), g);
#pragma unroll
      for (int i = 0; i < 8; ++i) g[i] *= v[c][i] * rstd;
      *reinterpret_cast<uint4*>(normed + t * H + idx * 8) = pack8(g);
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Gate logits with one warp per (token, expert): the few-token (decode) form,
// which keeps every SM busy where one CTA per token would leave most idle.
__global__ void moe_gate_logits_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                       const __nv_bfloat16* __restrict__ wg, int64_t T, int64_t H, int E,
                                       float* __restrict__ logits) {
  pdl_trigger();
  pdl_wait();
  const int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= T * E) return;
  const int64_t t = w / E;
  const int e = (int)(w % E);
  float acc = 0.f;
  for (int64_t c = lane; c < H / 8; c += 32) {
    float xv[8], wv[8];
    unpack8(*reinterpret_cast<const uint4*>(x + t * ldx + c * 8), xv);
    unpack8(*reinterpret_cast<const uint4*>(wg + (int64_t)e * H + c * 8), wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc = fmaf(xv[j], wv[j], acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) logits[t * E + e] = acc;
}

int route_launch(const void* x, int64_t ldx, const void* wg, const float* logits_in, int64_t T, int64_t H, int E,
                 int k, int renorm, float scale, int32_t* ids, float* wts, float* logits_out, cudaStream_t st) {
  auto xb = static_cast<const __nv_bfloat16*>(x);
  auto wb = static_cast<const __nv_bfloat16*>(wg);
  if (!logits_in && logits_out && T < 1024) {
    // few tokens: logits with a warp per (token, expert), then the selection from them
    const int64_t warps = T * E;
    launch_kernel(moe_gate_logits_kernel, dim3((unsigned)((warps * 32 + 255) / 256)), 256, 0, st, xb, ldx, wb, T, H,
                  E, logits_out);
    B200_CHECK_LAUNCH();
    return route_launch(nullptr, 0, nullptr, logits_out, T, H, E, k, renorm, scale, ids, wts, nullptr, st);
  }
  // Accumulators per thread: experts (rounded up) x tokens per CTA.  Many
  // tokens: several per CTA, so the gate rows are read once for all of them;
  // few (decode): one per CTA, for more CTAs in flight.
  const bool many = T >= 1024;
#define B200_ROUTE(EA, TPB)                                                                                       \
  launch_kernel(moe_route_kernel<EA, TPB>, dim3((unsigned)((T + TPB - 1) / TPB)), kRouteThreads, 0, st, xb, ldx, \
                wb, logits_in, T, H, E, k, renorm, scale, ids, wts, logits_out)
  if (E <= 8) many ? B200_ROUTE(8, 4) : B200_ROUTE(8, 1);
  else if (E <= 16) many ? B200_ROUTE(16, 4) : B200_ROUTE(16, 1);
  else if (E <= 32) many ? B200_ROUTE(32, 2) : B200_ROUTE(32, 1);
  else if (E <= 64) many ? B200_ROUTE(64, 2) : B200_ROUTE(64, 1);
  else if (E <= 128) B200_ROUTE(128, 1);
  else return B200_ERROR_UNSUPPORTED;
#undef B200_ROUTE
  B200_CHECK_LAUNCH();
  return B200_OK;
}

}  // namespace

namespace b200 {
unsigned* error_word(int device);
}

extern "C" int b200_moe_route(const void* x, int64_t ldx, const void* gate_weight, int64_t T, int64_t H,
                              int num_experts, int top_k, int renormalize, float scale, int32_t* topk_ids,
                              float* topk_weights, float* logits, b200_stream_t stream) {
  if (!x || !gate_weight || !topk_ids || !topk_weights || T < 0 || H <= 0 || H % 8 || ldx < H || ldx % 8)
    return B200_ERROR_INVALID_PARAM;
  if (num_experts <= 0 || top_k <= 0 || top_k > kMaxTopK || top_k > num_experts) return B200_ERROR_INVALID_PARAM;
  if (!aligned16(x) || !aligned16(gate_weight)) return B200_ERROR_INVALID_PARAM;
  if (num_experts > 128) return B200_ERROR_UNSUPPORTED;
  if (T == 0) return B200_OK;
  return route_launch(x, ldx, gate_weight, nullptr, T, H, num_experts, top_k, renormalize, scale, topk_ids,
                      topk_weights, logits, stream);
}

extern "C" int b200_moe_topk(const float* logits, int64_t T, int num_experts, int top_k, int renormalize, float scale,
                             int32_t* topk_ids, float* topk_weights, b200_stream_t stream) {
  if (!logits || !topk_ids || !topk_weights || T < 0) return B200_ERROR_INVALID_PARAM;
  if (num_experts <= 0 || top_k <= 0 || top_k > kMaxTopK || top_k > num_experts) return B200_ERROR_INVALID_PARAM;
  if (num_experts > 128) return B200_ERROR_UNSUPPORTED;
  if (T == 0) return B200_OK;
  return route_launch(nullptr, 0, nullptr, logits, T, 8, num_experts, top_k, renormalize, scale, topk_ids,
                      topk_weights, nullptr, stream);
}

extern "C" int64_t b200_moe_permute_workspace_bytes(int64_t T, int top_k, int num_experts) {
  if (T <= 0 || top_k <= 0 || num_experts <= 0) return 0;
  const int64_t nb = (T * top_k + kPermChunk - 1) / kPermChunk;
  return 2 * nb * num_experts * (int64_t)sizeof(int32_t);
}

extern "C" int b200_moe_permute(const int32_t* topk_ids, int64_t T, int top_k, int num_experts, const void* x,
                                int64_t ldx, int64_t H, void* x_perm, int32_t* expert_offsets, int32_t* perm_pos,
                                int32_t* perm_src, void* workspace, int64_t workspace_bytes, b200_stream_t stream) {
  if (!topk_ids || !expert_offsets || !perm_pos || !perm_src || !workspace || T < 0 || top_k <= 0 ||
      num_experts <= 0 || num_experts > kMaxExperts)
    return B200_ERROR_INVALID_PARAM;
  if (x_perm && (!x || H <= 0 || H % 8 || ldx < H || ldx % 8 || !aligned16(x) || !aligned16(x_perm)))
    return B200_ERROR_INVALID_PARAM;
  if (T * top_k > INT32_MAX / 2) return B200_ERROR_UNSUPPORTED;
  if (workspace_bytes < b200_moe_permute_workspace_bytes(T, top_k, num_experts)) return B200_ERROR_INVALID_PARAM;
  const int64_t n = T * top_k;
  const int nb = (int)((n + kPermChunk - 1) / kPermChunk);
  int dev = 0;
  cudaGetDevice(&dev);
  if (n == 0) {
    cudaError_t e = cudaMemsetAsync(expert_offsets, 0, (size_t)(num_experts + 1) * 4, stream);
    return e == cudaSuccess ? B200_OK : B200_ERROR_CUDA_BASE - (int)e;
  }
  int32_t* counts = static_cast<int32_t*>(workspace);
  int32_t* base = counts + (int64_t)nb * num_experts;
  launch_kernel(moe_count_kernel, dim3(nb), 32, 0, stream, topk_ids, n, num_experts, counts, b200::error_word(dev));
  launch_kernel(moe_scan_kernel, dim3(1), 256, 0, stream, (const int32_t*)counts, nb, num_experts, base,
                expert_offsets);
  launch_kernel(moe_scatter_kernel, dim3(nb), 32, 0, stream, topk_ids, n, top_k, num_experts, (const int32_t*)base,
                perm_pos, perm_src);
  if (x_perm)
    launch_kernel(moe_gather_kernel, dim3((unsigned)n), 128, 0, stream, static_cast<const __nv_bfloat16*>(x), ldx,
                  (const int32_t*)perm_src, (const int32_t*)(expert_offsets + num_experts), H,
                  static_cast<__nv_bfloat16*>(x_perm));
  B200_CHECK_LAUNCH();
  return B200_OK;
}

extern "C" int b200_moe_combine(const void* y_perm, const int32_t* perm_pos, const float* topk_weights, int64_t T,
                                int top_k, int64_t H, const void* residual, const void* shared, void* out,
                                const void* norm_weight, void* normed, float eps, b200_stream_t stream) {
  if (!y_perm || !perm_pos || !topk_weights || !out || T < 0 || top_k <= 0 || H <= 0 || H % 8)
    return B200_ERROR_INVALID_PARAM;
  if (norm_weight && !normed) return B200_ERROR_INVALID_PARAM;
  for (const void* p : {y_perm, (const void*)out, residual, shared, norm_weight, (const void*)normed})
    if (p && !aligned16(p)) return B200_ERROR_INVALID_PARAM;
  if (T == 0) return B200_OK;
  const int64_t per = (H / 8 + kCombineThreads - 1) / kCombineThreads;
  auto yb = static_cast<const __nv_bfloat16*>(y_perm);
  auto rb = static_cast<const __nv_bfloat16*>(residual);
  auto sb = static_cast<const __nv_bfloat16*>(shared);
  auto ob = static_cast<__nv_bfloat16*>(out);
  auto nw = static_cast<const __nv_bfloat16*>(norm_weight);
  auto nb = static_cast<__nv_bfloat16*>(normed);
  const dim3 g((unsigned)T);
  switch (per) {
    case 1: launch_kernel(moe_combine_kernel<1>, g, kCombineThreads, 0, stream, yb, perm_pos, topk_weights, top_k, H, rb, sb, ob, nw, nb, eps); break;
    case 2: launch_kernel(moe_combine_kernel<2>, g, kCombineThreads, 0, stream, yb, perm_pos, topk_weights, top_k, H, rb, sb, ob, nw, nb, eps); break;
    case 3:
    case 4: launch_kernel(moe_combine_kernel<4>, g, kCombineThreads, 0, stream, yb, perm_pos, topk_weights, top_k, H, rb, sb, ob, nw, nb, eps); break;
    default: return B200_ERROR_UNSUPPORTED;
  }
  B200_CHECK_LAUNCH();
  return B200_OK;
}
