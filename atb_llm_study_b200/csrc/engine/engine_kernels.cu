#include "common.cuh"
#include "engine/engine_kernels.h"

using namespace b200;

namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  // splitmix64 finaliser
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Two normals per hash via Box-Muller.
__global__ void fill_normal_kernel(__nv_bfloat16* x, int64_t n, float mean, float std, uint64_t seed) {
  const int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) * 2;
  if (i >= n) return;
  const uint64_t h = mix64(seed * 0x9E3779B97F4A7C15ull + (uint64_t)i);
  const float u1 = ((float)(h >> 40) + 1.0f) * (1.0f / 16777217.0f);  // (0, 1]
  const float u2 = (float)((h >> 16) & 0xFFFFFFull) * (1.0f / 16777216.0f);
  const float r = sqrtf(-2.0f * logf(u1));
  float s, c;
  sincospif(2.0f * u2, &s, &c);
  x[i] = f2bf(mean + std * r * c);
  if (i + 1 < n) x[i + 1] = f2bf(mean + std * r * s);
}

// Element (r, c) of a rows x cols window takes the value the plain fill gives
// global element gbase + r * gstride + c (pairs share one Box-Muller draw:
// even index = cosine branch, odd = sine branch), so a shard of a matrix
// filled through its window equals the same rows / columns of the whole
// matrix filled at once.
__global__ void fill_normal_window_kernel(__nv_bfloat16* x, int64_t rows, int64_t cols, float mean, float std,
                                          uint64_t seed, int64_t gbase, int64_t gstride) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const int64_t r = i / cols, c = i % cols;
  const uint64_t g = (uint64_t)(gbase + r * gstride + c);
  const uint64_t h = mix64(seed * 0x9E3779B97F4A7C15ull + (g & ~1ull));
  const float u1 = ((float)(h >> 40) + 1.0f) * (1.0f / 16777217.0f);  // (0, 1]
  const float u2 = (float)((h >> 16) & 0xFFFFFFull) * (1.0f / 16777216.0f);
  const float rad = sqrtf(-2.0f * logf(u1));
  float s, co;
  sincospif(2.0f * u2, &s, &co);
  x[i] = f2bf(mean + std * rad * ((g & 1) ? s : co));
}

__global__ void fill_const_kernel(__nv_bfloat16* x, int64_t n, float v) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < n) x[i] = f2bf(v);
}

__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ src, const int32_t* __restrict__ idx,
                                   int64_t dim, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int64_t r = blockIdx.x;
  const uint4* s = reinterpret_cast<const uint4*>(src + (int64_t)idx[r] * dim);
  uint4* d = reinterpret_cast<uint4*>(out + r * dim);
  for (int64_t c = threadIdx.x; c < dim / 8; c += blockDim.x) d[c] = s[c];
}

__global__ void scatter_rows_kernel(__nv_bfloat16* __restrict__ dst, const int32_t* __restrict__ idx, int64_t dim,
                                    const __nv_bfloat16* __restrict__ src) {
  pdl_trigger();
  pdl_wait();
  const int64_t r = blockIdx.x;
  const uint4* s = reinterpret_cast<const uint4*>(src + r * dim);
  uint4* d = reinterpret_cast<uint4*>(dst + (int64_t)idx[r] * dim);
  for (int64_t c = threadIdx.x; c < dim / 8; c += blockDim.x) d[c] = s[c];
}

// out = x / sqrt(sum(x^2) + 1e-12) (fp32 math), or a plain widening copy.
__global__ void pool_l2_kernel(const __nv_bfloat16* __restrict__ x, int64_t dim, int normalize, float* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  float ss = 0.f;
  for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) {
    const float v = bf2f(x[c]);
    ss += v * v;
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = normalize ? 1.0f / sqrtf(red[0] + 1e-12f) : 1.0f;
  for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) out[c] = bf2f(x[c]) * inv;
}

__global__ void decode_prepare_kernel(const int32_t* __restrict__ seq_slots, int B, int32_t* ctx_lens,
                                      const int32_t* __restrict__ bt, int max_blocks, int bs,
                                      int64_t* __restrict__ positions, int64_t* __restrict__ slots,
                                      int32_t* __restrict__ ctx_batch, int32_t* __restrict__ bt_batch,
                                      unsigned* err) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  const int s = seq_slots[b];
  const int p = ctx_lens[s];
  for (int j = threadIdx.x; j < max_blocks; j += blockDim.x)
    bt_batch[(int64_t)b * max_blocks + j] = bt[(int64_t)s * max_blocks + j];
  if (threadIdx.x != 0) return;
  positions[b] = p;
  positions[B + b] = p;
  positions[2 * B + b] = p;
  if (p < 0 || p >= max_blocks * bs) {
    raise_error(err, DEV_ERR_BAD_INDEX);
    slots[b] = -1;
    ctx_batch[b] = max(0, min(p, max_blocks * bs));
    return;
  }
  slots[b] = (int64_t)bt[(int64_t)s * max_blocks + p / bs] * bs + p % bs;
  ctx_batch[b] = p + 1;
  ctx_lens[s] = p + 1;
}

}  // namespace

namespace b200llm {

int FillNormalBf16(void* x, int64_t n, float mean, float std, uint64_t seed, cudaStream_t st) {
  if (n <= 0) return 0;
  const int64_t threads = (n + 1) / 2;
  fill_normal_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(static_cast<__nv_bfloat16*>(x), n, mean, std,
                                                                        seed);
  return cudaGetLastError() == cudaSuccess ? 0 : B200_ERROR_INFERENCE;
}

int FillNormalWindowBf16(void* x, int64_t rows, int64_t cols, float mean, float std, uint64_t seed, int64_t gbase,
                         int64_t gstride, cudaStream_t st) {
  if (rows <= 0 || cols <= 0) return 0;
  const int64_t n = rows * cols;
  fill_normal_window_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(static_cast<__nv_bfloat16*>(x), rows, cols,
                                                                          mean, std, seed, gbase, gstride);
  return cudaGetLastError() == cudaSuccess ? 0 : B200_ERROR_INFERENCE;
}

int FillConstBf16(void* x, int64_t n, float value, cudaStream_t st) {
  if (n <= 0) return 0;
  fill_const_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(static_cast<__nv_bfloat16*>(x), n, value);
  return cudaGetLastError() == cudaSuccess ? 0 : B200_ERROR_INFERENCE;
}

int GatherRows(const void* src, const int32_t* idx, int64_t n, int64_t dim, void* out, cudaStream_t st) {
  if (n <= 0) return 0;
  launch_kernel(gather_rows_kernel, dim3((unsigned)n), 128, 0, st, static_cast<const __nv_bfloat16*>(src), idx, dim,
                static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : B200_ERROR_INFERENCE;
}

int ScatterRows(void* dst, const int32_t* idx, int64_t n, int64_t dim, const void* src, cudaStream_t st) {
  if (n <= 0) return 0;
  launch_kernel(scatter_rows_kernel, dim3((unsigned)n), 128, 0, st, static_cast<__nv_bfloat16*>(dst), idx, dim,
                static_cast<const __nv_bfloat16*>(src));
  return cudaGetLastError() == cudaSuccess ? 0 : B200_ERROR_INFERENCE;
}

int PoolL2(const void* x, int64_t dim, int normalize, float* out, cudaStream_t st) {
  if (dim <= 0) return 0;
  launch_kernel(pool_l2_kernel, dim3(1), 512, 0, st, static_cast<const __nv_bfloat16*>(x), dim, normalize, out);
  return cudaGetLastError() == cudaSuccess ? 0 : B200_ERROR_INFERENCE;
}

int DecodePrepare(const int32_t* seq_slots, int B, int32_t* ctx_lens, const int32_t* block_tables, int max_blocks,
                  int block_size, int64_t* positions, int64_t* slots, int32_t* ctx_batch, int32_t* bt_batch,
                  unsigned* err, cudaStream_t st) {
  if (B <= 0) return 0;
  launch_kernel(decode_prepare_kernel, dim3(B), 64, 0, st, seq_slots, B, ctx_lens, block_tables, max_blocks,
                block_size, positions, slots, ctx_batch, bt_batch, err);
  return cudaGetLastError() == cudaSuccess ? 0 : B200_ERROR_INFERENCE;
}

}  // namespace b200llm
