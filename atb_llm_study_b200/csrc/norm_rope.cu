// Bandwidth-bound kernels of the decoder layer: RMSNorm (+ fused residual add),
// LayerNorm, rope cos/sin tables, per-head QK-RMSNorm + rope + paged-KV write,
// slot mapping, embedding gather, row scatter-add and argmax.
//
// All of them move 16-byte vectors per thread (8 bf16), keep a row in
// registers between the reduction and the write, and reduce with warp
// shuffles plus one shared-memory hop.
#include <math.h>

#include <algorithm>

#include <cstdlib>

#include "common.cuh"

using namespace b200;

namespace {

constexpr int kNormThreads = 128;


template <int NT>
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) t += red[i];
  return t;
}

// One CTA per row.  h = x (+ residual); out = h * rsqrt(mean(h^2) + eps) * w.
template <int CH>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                               const __nv_bfloat16* residual,
                                                               const __nv_bfloat16* __restrict__ w,
                                                               __nv_bfloat16* out, __nv_bfloat16* residual_out,
                                                               int64_t dim, int64_t stride, float eps) {
  __shared__ float red[kNormThreads / 32];
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const int64_t nchunk = dim / 8;
  const __nv_bfloat16* xr = x + row * stride;
  float v[CH][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kNormThreads;
    if (idx < nchunk) {
      unpack8(*reinterpret_cast<const uint4*>(xr + idx * 8), v[c]);
      if (residual) {
        float r[8];
        unpack8(*reinterpret_cast<const uint4*>(residual + row * stride + idx * 8), r);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] += r[i];
        if (residual_out) *reinterpret_cast<uint4*>(residual_out + row * stride + idx * 8) = pack8(v[c]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
    }
  }
  const float tot = block_sum<kNormThreads>(ss, red);
  const float inv = rsqrtf(tot / (float)dim + eps);
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kNormThreads;
    if (idx < nchunk) {
      float g[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(w + idx * 8), g);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = v[c][i] * inv * g[i];
      *reinterpret_cast<uint4*>(out + row * stride + idx * 8) = pack8(o);
    }
  }
}

// One CTA of 512 threads per row (decode has few rows, so each thread owns
// one to four 16-byte chunks and issues all its loads up front):
// h = hidden + sum_s partials[s][row] (a split-K projection finished here),
// hidden = bf16(h), out = rmsnorm(bf16(h)) * w.
constexpr int kRowThreads = 512;
constexpr int kBatchSplits = 8;  // split-K partial loads issued together before they are summed

// v[0..7] += sum over s < splits of the 8 fp32 at p + s * slice (in split
// order): the loads of up to kBatchSplits slices are all in flight before the
// first add, so the L2 latency is paid once, not once per split.
__device__ __forceinline__ void add_split_partials8(float v[8], const float* p, int64_t slice, int splits) {
  for (int s0 = 0; s0 < splits; s0 += kBatchSplits) {
    float4 a[kBatchSplits][2];
#pragma unroll
    for (int i = 0; i < kBatchSplits; ++i)
      if (s0 + i < splits) {
        const float4* src = reinterpret_cast<const float4*>(p + (int64_t)(s0 + i) * slice);
        a[i][0] = src[0];
        a[i][1] = src[1];
      }
#pragma unroll
    for (int i = 0; i < kBatchSplits; ++i)
      if (s0 + i < splits) {
        v[0] += a[i][0].x; v[1] += a[i][0].y; v[2] += a[i][0].z; v[3] += a[i][0].w;
        v[4] += a[i][1].x; v[5] += a[i][1].y; v[6] += a[i][1].z; v[7] += a[i][1].w;
      }
  }
}

template <int CH>
__global__ void __launch_bounds__(kRowThreads) splitk_residual_rmsnorm_kernel(const float* __restrict__ partials,
                                                                              int splits, int64_t rows,
                                                                              __nv_bfloat16* hidden,
                                                                              const __nv_bfloat16* __restrict__ w,
                                                                              __nv_bfloat16* __restrict__ out,
                                                                              int64_t dim, float eps) {
  constexpr int kNormThreads = kRowThreads;
  __shared__ float red[kNormThreads / 32];
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const int64_t nchunk = dim / 8;
  float v[CH][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kNormThreads;
    if (idx < nchunk) {
      unpack8(*reinterpret_cast<const uint4*>(hidden + row * dim + idx * 8), v[c]);
      add_split_partials8(v[c], partials + row * dim + idx * 8, rows * dim, splits);
      const uint4 hb = pack8(v[c]);
      *reinterpret_cast<uint4*>(hidden + row * dim + idx * 8) = hb;
      unpack8(hb, v[c]);  // normalise the stored (bf16) residual stream
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
    }
  }
  uint4 wv[CH];  // the norm weight, loaded while the row sum is reduced
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kNormThreads;
    if (idx < nchunk) wv[c] = *reinterpret_cast<const uint4*>(w + idx * 8);
  }
  const float inv = rsqrtf(block_sum<kNormThreads>(ss, red) / (float)dim + eps);
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kNormThreads;
    if (idx < nchunk) {
      float g[8], o[8];
      unpack8(wv[c], g);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = v[c][i] * inv * g[i];
      *reinterpret_cast<uint4*>(out + row * dim + idx * 8) = pack8(o);
    }
  }
}

template <int CH>
__global__ void __launch_bounds__(kNormThreads) layernorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                                 const __nv_bfloat16* __restrict__ g,
                                                                 const __nv_bfloat16* __restrict__ b,
                                                                 __nv_bfloat16* __restrict__ out, int64_t dim,
                                                                 float eps) {
  __shared__ float red[kNormThreads / 32];
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const int64_t nchunk = dim / 8;
  float v[CH][8];
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kNormThreads;
    if (idx < nchunk) {
      unpack8(*reinterpret_cast<const uint4*>(x + row * dim + idx * 8), v[c]);
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[c][i];
    }
  }
  const float mean = block_sum<kNormThreads>(s, red) / (float)dim;
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kNormThreads;
    if (idx < nchunk) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[c][i] - mean;
        ss += d * d;
      }
    }
  }
  const float inv = rsqrtf(block_sum<kNormThreads>(ss, red) / (float)dim + eps);
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kNormThreads;
    if (idx < nchunk) {
      float gg[8], bb[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(g + idx * 8), gg);
      unpack8(*reinterpret_cast<const uint4*>(b + idx * 8), bb);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = (v[c][i] - mean) * inv * gg[i] + bb[i];
      *reinterpret_cast<uint4*>(out + row * dim + idx * 8) = pack8(o);
    }
  }
}

// One CTA of kNormThreads per row, the thread / chunk mapping of
// layernorm_kernel: h = bf16(sum_s partials[s][row] + bias + hidden[row])
// (the additions in splitk_reduce_kernel's order), hidden[row] = h, then
// layernorm_kernel's arithmetic on h.  Replaces a split-K reduce launch and a
// LayerNorm launch with one.
template <int CH>
__global__ void __launch_bounds__(kNormThreads) splitk_bias_residual_layernorm_kernel(
    const float* __restrict__ partials, int splits, int64_t rows, const __nv_bfloat16* __restrict__ bias,
    __nv_bfloat16* hidden, const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ b,
    __nv_bfloat16* __restrict__ out, int64_t dim, float eps) {
  __shared__ float red[kNormThreads / 32];
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const int64_t nchunk = dim / 8;
  float v[CH][8];
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kNormThreads;
    if (idx < nchunk) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] = 0.f;
      add_split_partials8(v[c], partials + row * dim + idx * 8, rows * dim, splits);
      float t[8];
      unpack8(*reinterpret_cast<const uint4*>(bias + idx * 8), t);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] += t[i];
      unpack8(*reinterpret_cast<const uint4*>(hidden + row * dim + idx * 8), t);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] += t[i];
      const uint4 hb = pack8(v[c]);
      *reinterpret_cast<uint4*>(hidden + row * dim + idx * 8) = hb;
      unpack8(hb, v[c]);  // normalise the stored (bf16) residual stream
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[c][i];
    }
  }
  const float mean = block_sum<kNormThreads>(s, red) / (float)dim;
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kNormThreads;
    if (idx < nchunk) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[c][i] - mean;
        ss += d * d;
      }
    }
  }
  const float inv = rsqrtf(block_sum<kNormThreads>(ss, red) / (float)dim + eps);
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int64_t idx = threadIdx.x + (int64_t)c * kNormThreads;
    if (idx < nchunk) {
      float gg[8], bb[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(g + idx * 8), gg);
      unpack8(*reinterpret_cast<const uint4*>(b + idx * 8), bb);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = (v[c][i] - mean) * inv * gg[i] + bb[i];
      *reinterpret_cast<uint4*>(out + row * dim + idx * 8) = pack8(o);
    }
  }
}

// cos/sin table: one thread per (token, frequency index i < d/2).
// plane(i) selects which position-id plane feeds frequency i: 0 for 1-D rope;
// for interleaved mrope, 1 when i%3==1 && i<3*sec_h, 2 when i%3==2 && i<3*sec_w.
struct InvFreq {
  float v[128];  // head_dim <= 256
};

__global__ void rope_table_kernel(const int64_t* __restrict__ pos, int64_t T, int half, const InvFreq inv_freq,
                                  int mrope, int sec_h, int sec_w, float* __restrict__ cos_out,
                                  float* __restrict__ sin_out) {
  pdl_trigger();
  pdl_wait();
  const int64_t gid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (gid >= T * half) return;
  const int64_t t = gid / half;
  const int i = (int)(gid % half);
  int plane = 0;
  if (mrope) {
    if (i % 3 == 1 && i < 3 * sec_h) plane = 1;
    else if (i % 3 == 2 && i < 3 * sec_w) plane = 2;
  }
  const float p = (float)pos[plane * T + t];
  const float f = p * inv_freq.v[i];
  float s, c;
  sincosf(f, &s, &c);
  const int64_t o = t * 2 * half;
  cos_out[o + i] = c;
  cos_out[o + i + half] = c;
  sin_out[o + i] = s;
  sin_out[o + i + half] = s;
}

// Per-head RMSNorm (q, k) + half-rotation rope (q, k) + paged-KV write (k, v).
// Grid (token, head group); each warp handles one head.  Lane l holds elements
// [l*E, l*E+E) of a head (E = head_dim/32); the rotation partner of element
// i (i +- head_dim/2) sits in lane l^16.
template <int HD>
__global__ void __launch_bounds__(128) qk_norm_rope_kernel(__nv_bfloat16* qkv, int nq, int nkv, int64_t row_stride,
                                                           const __nv_bfloat16* __restrict__ qn_w,
                                                           const __nv_bfloat16* __restrict__ kn_w, float eps,
                                                           const float* __restrict__ cos_tab,
                                                           const float* __restrict__ sin_tab,
                                                           const int64_t* __restrict__ slots,
                                                           __nv_bfloat16* k_cache, __nv_bfloat16* v_cache,
                                                           int64_t num_blocks, int block_size, unsigned* err,
                                                           const float* __restrict__ partials, int splits,
                                                           int64_t p_ld, int64_t p_slice) {
  // partials != null: the projection was split along K and qkv holds nothing
  // yet; every head is summed from the fp32 partial tiles
  // partials[s][t][p_ld] and written to qkv (v too, for prefill attention).
  constexpr int E = HD / 32;
  pdl_trigger();
  pdl_wait();
  const int64_t t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nheads = nq + 2 * nkv;
  __nv_bfloat16* row = qkv + t * row_stride;
  float cs[E], sn[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    cs[e] = cos_tab[t * HD + lane * E + e];
    sn[e] = sin_tab[t * HD + lane * E + e];
  }
  int64_t slot = -1;
  if (slots) {
    slot = slots[t];
    if (slot >= num_blocks * (int64_t)block_size) {
      raise_error(err, DEV_ERR_BAD_INDEX);
      slot = -1;
    }
  }
  const float sign = lane < 16 ? -1.f : 1.f;
  const int wpc = blockDim.x / 32;  // heads of a token are spread over gridDim.y CTAs
  for (int h = blockIdx.y * wpc + warp; h < nheads; h += gridDim.y * wpc) {
    __nv_bfloat16* hp = row + (int64_t)h * HD + lane * E;
    float x[E];
    if (partials) {
#pragma unroll
      for (int e = 0; e < E; ++e) x[e] = 0.f;
      const float* src = partials + t * p_ld + (int64_t)h * HD + lane * E;
      // all splits' loads in flight before the first add (split order kept)
      for (int s0 = 0; s0 < splits; s0 += kBatchSplits) {
        float a[kBatchSplits][E];
#pragma unroll
        for (int i = 0; i < kBatchSplits; ++i)
          if (s0 + i < splits) {
#pragma unroll
            for (int e = 0; e < E; ++e) a[i][e] = src[(int64_t)(s0 + i) * p_slice + e];
          }
#pragma unroll
        for (int i = 0; i < kBatchSplits; ++i)
          if (s0 + i < splits) {
#pragma unroll
            for (int e = 0; e < E; ++e) x[e] += a[i][e];
          }
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) x[e] = bf2f(hp[e]);
    }
    const bool is_q = h < nq, is_k = !is_q && h < nq + nkv;
    if (partials && !is_q && !is_k) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        hp[e] = f2bf(x[e]);
        x[e] = bf2f(hp[e]);  // the cache holds the same bf16 value as qkv
      }
    }
    if (is_q || is_k) {
      const __nv_bfloat16* nw = is_q ? qn_w : kn_w;
      if (nw) {
        float wn[E];
#pragma unroll
        for (int e = 0; e < E; ++e) wn[e] = bf2f(nw[lane * E + e]);
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) ss += x[e] * x[e];
        const float inv = rsqrtf(warp_sum(ss) / (float)HD + eps);
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = x[e] * inv * wn[e];
      }
      float y[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
        y[e] = x[e] * cs[e] + sign * partner * sn[e];
      }
#pragma unroll
      for (int e = 0; e < E; ++e) {
        x[e] = y[e];
        hp[e] = f2bf(y[e]);
      }
    }
    if (slot >= 0 && !is_q) {
      const int kh = is_k ? h - nq : h - nq - nkv;
      __nv_bfloat16* cache = is_k ? k_cache : v_cache;
      const int64_t blk = slot / block_size, off = slot % block_size;
      __nv_bfloat16* dst = cache + ((blk * nkv + kh) * block_size + off) * HD + lane * E;
#pragma unroll
      for (int e = 0; e < E; ++e) dst[e] = f2bf(x[e]);
    }
  }
}

__global__ void slot_mapping_kernel(const int32_t* __restrict__ bt, int max_blocks, const int32_t* __restrict__ seq,
                                    const int64_t* __restrict__ pos, int64_t T, int bs, int64_t* __restrict__ slots,
                                    unsigned* err) {
  pdl_trigger();
  pdl_wait();
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= T) return;
  const int64_t p = pos[t];
  const int64_t bi = p / bs;
  if (p < 0 || bi >= max_blocks) {
    raise_error(err, DEV_ERR_BAD_INDEX);
    slots[t] = -1;
    return;
  }
  slots[t] = (int64_t)bt[(int64_t)seq[t] * max_blocks + bi] * bs + p % bs;
}

__global__ void embedding_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 int64_t vocab, int64_t dim, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int64_t t = blockIdx.x;
  const int64_t id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  const uint4* src = reinterpret_cast<const uint4*>(table + (ok ? id : 0) * dim);
  uint4* dst = reinterpret_cast<uint4*>(out + t * dim);
  for (int64_t c = threadIdx.x; c < dim / 8; c += blockDim.x) dst[c] = ok ? src[c] : make_uint4(0, 0, 0, 0);
}

__global__ void scatter_add_kernel(__nv_bfloat16* hidden, int64_t rows, int64_t dim, const int32_t* __restrict__ idx,
                                   const __nv_bfloat16* __restrict__ feat, float alpha, unsigned* err) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = blockIdx.x;
  const int64_t r = idx[i];
  if (r < 0 || r >= rows) {
    if (threadIdx.x == 0) raise_error(err, DEV_ERR_BAD_INDEX);
    return;
  }
  for (int64_t c = threadIdx.x; c < dim / 8; c += blockDim.x) {
    float h[8], f[8];
    unpack8(*reinterpret_cast<const uint4*>(hidden + r * dim + c * 8), h);
    unpack8(*reinterpret_cast<const uint4*>(feat + i * dim + c * 8), f);
#pragma unroll
    for (int k = 0; k < 8; ++k) h[k] += alpha * f[k];
    *reinterpret_cast<uint4*>(hidden + r * dim + c * 8) = pack8(h);
  }
}

constexpr int kArgmaxThreads = 512;

// One CTA per row.  With 16-byte aligned rows each thread reads 8 logits per
// load; indices a thread visits only increase, so `>` keeps the lowest index
// on ties, and the reductions below break ties toward the lower index.
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const __nv_bfloat16* __restrict__ logits,
                                                                int64_t vocab, int64_t ld, int64_t* __restrict__ out) {
  __shared__ float sv[kArgmaxThreads / 32];
  __shared__ int64_t si[kArgmaxThreads / 32];
  pdl_trigger();
  pdl_wait();
  const int64_t r = blockIdx.x;
  const __nv_bfloat16* row = logits + r * ld;
  float best = -INFINITY;
  int64_t bi = INT64_MAX;
  const bool vec = (vocab % 8 == 0) && (ld % 8 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  if (vec) {
    const uint4* rv = reinterpret_cast<const uint4*>(row);
#pragma unroll 4
    for (int64_t c = threadIdx.x; c < vocab / 8; c += blockDim.x) {
      float f[8];
      unpack8(__ldg(rv + c), f);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (f[i] > best) {
          best = f[i];
          bi = c * 8 + i;
        }
    }
  } else {
    for (int64_t j = threadIdx.x; j < vocab; j += blockDim.x) {
      const float v = bf2f(row[j]);
      if (v > best) {
        best = v;
        bi = j;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < kArgmaxThreads / 32; ++i)
      if (sv[i] > best || (sv[i] == best && si[i] < bi)) {
        best = sv[i];
        bi = si[i];
      }
    out[r] = bi == INT64_MAX ? 0 : bi;
  }
}

// ---------------------------------------------------------------------------
// Device error word, one per device.
// ---------------------------------------------------------------------------
__device__ unsigned g_device_error_word;

}  // namespace

namespace b200 {
static thread_local bool t_pdl_on = true;

bool pdl_enabled() {
  static const bool env_on = [] {
    const char* v = std::getenv("B200_PDL");
    return !(v && v[0] == '0');
  }();
  return env_on && t_pdl_on;
}

void set_pdl(bool on) { t_pdl_on = on; }

unsigned* error_word(int device) {
  static unsigned* ptrs[64] = {nullptr};
  if (device < 0 || device >= 64) return nullptr;
  if (!ptrs[device]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error_word) != cudaSuccess) return nullptr;
    ptrs[device] = static_cast<unsigned*>(p);
  }
  return ptrs[device];
}
}  // namespace b200

static unsigned* current_error_word() {
  int dev = 0;
  cudaGetDevice(&dev);
  return b200::error_word(dev);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" int b200_abi_version(void) { return 100; }

extern "C" int b200_device_error_read(unsigned* out_bits, int clear, b200_stream_t stream) {
  unsigned* w = current_error_word();
  if (!w || !out_bits) return B200_ERROR_INVALID_PARAM;
  cudaError_t e = cudaMemcpyAsync(out_bits, w, sizeof(unsigned), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(w, 0, sizeof(unsigned), stream);
  if (e == cudaSuccess && clear) e = cudaStreamSynchronize(stream);
  return e == cudaSuccess ? B200_OK : B200_ERROR_CUDA_BASE - (int)e;
}

extern "C" int b200_rmsnorm(const void* x, const void* residual, const void* weight, void* out, void* residual_out,
                            int64_t rows, int64_t dim, int64_t stride, float eps, b200_stream_t stream) {
  if (!x || !weight || !out || rows < 0 || dim <= 0 || dim % 8 || stride < dim || stride % 8) return B200_ERROR_INVALID_PARAM;
  if (!aligned16(x) || !aligned16(out) || !aligned16(weight) || (residual && !aligned16(residual)) ||
      (residual_out && !aligned16(residual_out)))
    return B200_ERROR_INVALID_PARAM;
  if (rows == 0) return B200_OK;
  const int64_t per = (dim / 8 + kNormThreads - 1) / kNormThreads;
  auto xb = static_cast<const __nv_bfloat16*>(x);
  auto rb = static_cast<const __nv_bfloat16*>(residual);
  auto wb = static_cast<const __nv_bfloat16*>(weight);
  auto ob = static_cast<__nv_bfloat16*>(out);
  auto rob = static_cast<__nv_bfloat16*>(residual_out);
  dim3 g((unsigned)rows);
  switch (per) {
    case 1: launch_kernel(rmsnorm_kernel<1>, g, kNormThreads, 0, stream, xb, rb, wb, ob, rob, dim, stride, eps); break;
    case 2: launch_kernel(rmsnorm_kernel<2>, g, kNormThreads, 0, stream, xb, rb, wb, ob, rob, dim, stride, eps); break;
    case 3:
    case 4: launch_kernel(rmsnorm_kernel<4>, g, kNormThreads, 0, stream, xb, rb, wb, ob, rob, dim, stride, eps); break;
    case 5: case 6: case 7:
    case 8: launch_kernel(rmsnorm_kernel<8>, g, kNormThreads, 0, stream, xb, rb, wb, ob, rob, dim, stride, eps); break;
    default: return B200_ERROR_UNSUPPORTED;
  }
  B200_CHECK_LAUNCH();
  return B200_OK;
}

extern "C" int b200_layernorm(const void* x, const void* gamma, const void* beta, void* out, int64_t rows, int64_t dim,
                              float eps, b200_stream_t stream) {
  if (!x || !gamma || !beta || !out || rows < 0 || dim <= 0 || dim % 8) return B200_ERROR_INVALID_PARAM;
  if (!aligned16(x) || !aligned16(out) || !aligned16(gamma) || !aligned16(beta)) return B200_ERROR_INVALID_PARAM;
  if (rows == 0) return B200_OK;
  const int64_t per = (dim / 8 + kNormThreads - 1) / kNormThreads;
  auto xb = static_cast<const __nv_bfloat16*>(x);
  auto gb = static_cast<const __nv_bfloat16*>(gamma);
  auto bb = static_cast<const __nv_bfloat16*>(beta);
  auto ob = static_cast<__nv_bfloat16*>(out);
  dim3 g((unsigned)rows);
  switch (per) {
    case 1: launch_kernel(layernorm_kernel<1>, g, kNormThreads, 0, stream, xb, gb, bb, ob, dim, eps); break;
    case 2: launch_kernel(layernorm_kernel<2>, g, kNormThreads, 0, stream, xb, gb, bb, ob, dim, eps); break;
    case 3:
    case 4: launch_kernel(layernorm_kernel<4>, g, kNormThreads, 0, stream, xb, gb, bb, ob, dim, eps); break;
    case 5: case 6: case 7:
    case 8: launch_kernel(layernorm_kernel<8>, g, kNormThreads, 0, stream, xb, gb, bb, ob, dim, eps); break;
    default: return B200_ERROR_UNSUPPORTED;
  }
  B200_CHECK_LAUNCH();
  return B200_OK;
}

// inv_freq[i] = 1 / theta^(2i/d) evaluated in fp32 on the host, the way the
// reference evaluates it (engine_utils.py:426, mrope.cpp:19-24), and passed to
// the kernel by value (no allocation, no copy).
static int rope_table(const int64_t* pos, int64_t T, int head_dim, float theta, int mrope, int sh, int sw, float* c,
                      float* s, b200_stream_t stream) {
  if (!pos || !c || !s || T < 0 || head_dim <= 0 || head_dim % 2) return B200_ERROR_INVALID_PARAM;
  if (head_dim > 256) return B200_ERROR_UNSUPPORTED;
  if (T == 0) return B200_OK;
  InvFreq inv;
  for (int i = 0; i < head_dim / 2; ++i) inv.v[i] = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
  const int half = head_dim / 2;
  const int64_t n = T * half;
  launch_kernel(rope_table_kernel, dim3((unsigned)((n + 255) / 256)), 256, 0, stream, pos, T, half, inv, mrope, sh, sw,
                c, s);
  B200_CHECK_LAUNCH();
  return B200_OK;
}

extern "C" int b200_rope_table_mrope(const int64_t* position_ids, int64_t T, int head_dim, float theta, int section_t,
                                     int section_h, int section_w, float* cos_out, float* sin_out,
                                     b200_stream_t stream) {
  if (section_t < 0 || section_h < 0 || section_w < 0) return B200_ERROR_INVALID_PARAM;
  return rope_table(position_ids, T, head_dim, theta, 1, section_h, section_w, cos_out, sin_out, stream);
}

extern "C" int b200_rope_table_1d(const int64_t* positions, int64_t T, int head_dim, float theta, float* cos_out,
                                  float* sin_out, b200_stream_t stream) {
  return rope_table(positions, T, head_dim, theta, 0, 0, 0, cos_out, sin_out, stream);
}

namespace b200 {

int qk_norm_rope_launch(void* qkv, int64_t T, int nq, int nkv, int head_dim, int64_t row_stride, const void* q_norm_w,
                        const void* k_norm_w, float eps, const float* cos_tab, const float* sin_tab,
                        const int64_t* slot_mapping, void* k_cache, void* v_cache, int64_t num_blocks, int block_size,
                        const float* partials, int splits, cudaStream_t stream) {
  if (!qkv || !cos_tab || !sin_tab || T < 0 || nq <= 0 || nkv <= 0 || nq % nkv ||
      row_stride < (int64_t)(nq + 2 * nkv) * head_dim)
    return B200_ERROR_INVALID_PARAM;
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr)) return B200_ERROR_INVALID_PARAM;
  if (slot_mapping && (!k_cache || !v_cache || block_size <= 0 || num_blocks <= 0)) return B200_ERROR_INVALID_PARAM;
  if (partials && splits <= 0) return B200_ERROR_INVALID_PARAM;
  if (T == 0) return B200_OK;
  auto q = static_cast<__nv_bfloat16*>(qkv);
  auto qn = static_cast<const __nv_bfloat16*>(q_norm_w);
  auto kn = static_cast<const __nv_bfloat16*>(k_norm_w);
  auto kc = static_cast<__nv_bfloat16*>(k_cache);
  auto vc = static_cast<__nv_bfloat16*>(v_cache);
  unsigned* err = current_error_word();
  const int64_t p_ld = row_stride, p_slice = T * row_stride;  // partials [splits][T][row_stride]
  // one CTA (4 warps) per token and head group: with few tokens (decode) every
  // warp gets one head; with many (prefill) one CTA walks all heads of its
  // token, so the grid stays a few CTAs per SM instead of ~12 per token
  const int64_t nh4 = (nq + 2 * nkv + 3) / 4;
  const int64_t gy = std::min<int64_t>(nh4, std::max<int64_t>(1, (8 * 148 + T - 1) / T));
  dim3 g((unsigned)T, (unsigned)gy);
  switch (head_dim) {
    case 32: launch_kernel(qk_norm_rope_kernel<32>, g, 128, 0, stream, q, nq, nkv, row_stride, qn, kn, eps, cos_tab, sin_tab, slot_mapping, kc, vc, num_blocks, block_size, err, partials, splits, p_ld, p_slice); break;
    case 64: launch_kernel(qk_norm_rope_kernel<64>, g, 128, 0, stream, q, nq, nkv, row_stride, qn, kn, eps, cos_tab, sin_tab, slot_mapping, kc, vc, num_blocks, block_size, err, partials, splits, p_ld, p_slice); break;
    case 128: launch_kernel(qk_norm_rope_kernel<128>, g, 128, 0, stream, q, nq, nkv, row_stride, qn, kn, eps, cos_tab, sin_tab, slot_mapping, kc, vc, num_blocks, block_size, err, partials, splits, p_ld, p_slice); break;
    default: return B200_ERROR_UNSUPPORTED;
  }
  B200_CHECK_LAUNCH();
  return B200_OK;
}

int splitk_residual_rmsnorm(const float* partials, int splits, int64_t rows, int64_t dim, void* hidden,
                            const void* weight, void* normed, float eps, cudaStream_t stream) {
  if (!partials || splits <= 0 || !hidden || !weight || !normed || rows < 0 || dim <= 0 || dim % 8)
    return B200_ERROR_INVALID_PARAM;
  if (rows == 0) return B200_OK;
  const int64_t per = (dim / 8 + kRowThreads - 1) / kRowThreads;
  auto h = static_cast<__nv_bfloat16*>(hidden);
  auto w = static_cast<const __nv_bfloat16*>(weight);
  auto o = static_cast<__nv_bfloat16*>(normed);
  dim3 g((unsigned)rows);
  switch (per) {
    case 1: launch_kernel(splitk_residual_rmsnorm_kernel<1>, g, kRowThreads, 0, stream, partials, splits, rows, h, w, o, dim, eps); break;
    case 2: launch_kernel(splitk_residual_rmsnorm_kernel<2>, g, kRowThreads, 0, stream, partials, splits, rows, h, w, o, dim, eps); break;
    case 3:
    case 4: launch_kernel(splitk_residual_rmsnorm_kernel<4>, g, kRowThreads, 0, stream, partials, splits, rows, h, w, o, dim, eps); break;
    default: return B200_ERROR_UNSUPPORTED;
  }
  B200_CHECK_LAUNCH();
  return B200_OK;
}

int splitk_bias_residual_layernorm(const float* partials, int splits, int64_t rows, int64_t dim, const void* bias,
                                   void* hidden, const void* gamma, const void* beta, void* normed, float eps,
                                   cudaStream_t stream) {
  if (!partials || splits <= 0 || !bias || !hidden || !gamma || !beta || !normed || rows < 0 || dim <= 0 || dim % 8)
    return B200_ERROR_INVALID_PARAM;
  if (!aligned16(partials) || !aligned16(bias) || !aligned16(hidden) || !aligned16(gamma) || !aligned16(beta) ||
      !aligned16(normed))
    return B200_ERROR_INVALID_PARAM;
  if (rows == 0) return B200_OK;
  const int64_t per = (dim / 8 + kNormThreads - 1) / kNormThreads;
  auto bs = static_cast<const __nv_bfloat16*>(bias);
  auto h = static_cast<__nv_bfloat16*>(hidden);
  auto gb = static_cast<const __nv_bfloat16*>(gamma);
  auto bb = static_cast<const __nv_bfloat16*>(beta);
  auto o = static_cast<__nv_bfloat16*>(normed);
  dim3 g((unsigned)rows);
  switch (per) {
    case 1: launch_kernel(splitk_bias_residual_layernorm_kernel<1>, g, kNormThreads, 0, stream, partials, splits, rows, bs, h, gb, bb, o, dim, eps); break;
    case 2: launch_kernel(splitk_bias_residual_layernorm_kernel<2>, g, kNormThreads, 0, stream, partials, splits, rows, bs, h, gb, bb, o, dim, eps); break;
    case 3:
    case 4: launch_kernel(splitk_bias_residual_layernorm_kernel<4>, g, kNormThreads, 0, stream, partials, splits, rows, bs, h, gb, bb, o, dim, eps); break;
    default: return B200_ERROR_UNSUPPORTED;
  }
  B200_CHECK_LAUNCH();
  return B200_OK;
}

}  // namespace b200

extern "C" int b200_qk_norm_rope(void* qkv, int64_t T, int nq, int nkv, int head_dim, int64_t row_stride,
                                 const void* q_norm_w, const void* k_norm_w, float eps, const float* cos_tab,
                                 const float* sin_tab, const int64_t* slot_mapping, void* k_cache, void* v_cache,
                                 int64_t num_blocks, int block_size, b200_stream_t stream) {
  return b200::qk_norm_rope_launch(qkv, T, nq, nkv, head_dim, row_stride, q_norm_w, k_norm_w, eps, cos_tab, sin_tab,
                                   slot_mapping, k_cache, v_cache, num_blocks, block_size, nullptr, 0, stream);
}

extern "C" int b200_slot_mapping(const int32_t* block_tables, int max_blocks_per_seq, const int32_t* seq_ids,
                                 const int64_t* positions, int64_t T, int block_size, int64_t* slots,
                                 b200_stream_t stream) {
  if (!block_tables || !seq_ids || !positions || !slots || T < 0 || block_size <= 0 || max_blocks_per_seq <= 0)
    return B200_ERROR_INVALID_PARAM;
  if (T == 0) return B200_OK;
  launch_kernel(slot_mapping_kernel, dim3((unsigned)((T + 255) / 256)), 256, 0, stream, block_tables,
                max_blocks_per_seq, seq_ids, positions, T, block_size, slots, current_error_word());
  B200_CHECK_LAUNCH();
  return B200_OK;
}

extern "C" int b200_embedding(const int64_t* ids, int64_t T, const void* table, int64_t vocab, int64_t dim, void* out,
                              b200_stream_t stream) {
  if (!ids || !table || !out || T < 0 || vocab <= 0 || dim <= 0 || dim % 8) return B200_ERROR_INVALID_PARAM;
  if (!aligned16(table) || !aligned16(out)) return B200_ERROR_INVALID_PARAM;
  if (T == 0) return B200_OK;
  launch_kernel(embedding_kernel, dim3((unsigned)T), 128, 0, stream, ids, static_cast<const __nv_bfloat16*>(table),
                vocab, dim, static_cast<__nv_bfloat16*>(out));
  B200_CHECK_LAUNCH();
  return B200_OK;
}

extern "C" int b200_scatter_add_rows(void* hidden, int64_t rows, int64_t dim, const int32_t* idx, const void* feat,
                                     int64_t n, float alpha, b200_stream_t stream) {
  if (!hidden || !idx || !feat || rows < 0 || n < 0 || dim <= 0 || dim % 8) return B200_ERROR_INVALID_PARAM;
  if (!aligned16(hidden) || !aligned16(feat)) return B200_ERROR_INVALID_PARAM;
  if (n == 0) return B200_OK;
  launch_kernel(scatter_add_kernel, dim3((unsigned)n), 128, 0, stream, static_cast<__nv_bfloat16*>(hidden), rows, dim,
                idx, static_cast<const __nv_bfloat16*>(feat), alpha, current_error_word());
  B200_CHECK_LAUNCH();
  return B200_OK;
}

extern "C" int b200_argmax(const void* logits, int64_t rows, int64_t vocab, int64_t ld, int64_t* out,
                           b200_stream_t stream) {
  if (!logits || !out || rows < 0 || vocab <= 0 || ld < vocab) return B200_ERROR_INVALID_PARAM;
  if (rows == 0) return B200_OK;
  launch_kernel(argmax_kernel, dim3((unsigned)rows), kArgmaxThreads, 0, stream,
                static_cast<const __nv_bfloat16*>(logits), vocab, ld, out);
  B200_CHECK_LAUNCH();
  return B200_OK;
}
