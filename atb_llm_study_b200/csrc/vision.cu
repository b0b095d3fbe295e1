// Vision-tower kernels: 2-D vision rope table, plain half-rotation rope for
// any head size, and the bilinear position-embedding interpolation (fused
// with the add onto the patch embeddings).
//
// Token order everywhere is the merge-block order of the vision tower: for
// each image, merge blocks row-major, the merge x merge patches of a block
// row-major, the whole grid repeated over t.  A token's (row, col) patch
// coordinate is decoded on the fly from its index, so no index tables are
// built on the host.
#include <math.h>

#include "common.cuh"

using namespace b200;

namespace {

constexpr int kMaxImages = 64;

struct Grids {
  int n;
  int64_t start[kMaxImages + 1];  // first token of image i (prefix sums of t*h*w)
  int h[kMaxImages], w[kMaxImages];
};

// (row, col) of token `tok` in its image's patch grid; image index in *img.
__device__ __forceinline__ void token_rc(const Grids& g, int merge, int64_t tok, int* img, int* row, int* col) {
  int i = 0;
  while (i + 1 < g.n && tok >= g.start[i + 1]) ++i;
  const int64_t hw = (int64_t)g.h[i] * g.w[i];
  const int64_t r = (tok - g.start[i]) % hw;  // position inside one temporal slice
  const int mm = merge * merge;
  const int64_t blk = r / mm, in = r % mm;
  const int mw = g.w[i] / merge;
  *img = i;
  *row = (int)(blk / mw) * merge + (int)(in / merge);
  *col = (int)(blk % mw) * merge + (int)(in % merge);
}

struct InvFreqV {
  float v[64];
};

// cos/sin [T, head_dim]: freq = cat(row * inv, col * inv) (head_dim/2 values),
// emb = cat(freq, freq).  One thread per (token, j < head_dim/2).
__global__ void rope_table_vision_kernel(Grids g, int merge, int head_dim, InvFreqV inv, int64_t T, float* cos_out,
                                         float* sin_out) {
  pdl_trigger();
  pdl_wait();
  const int half = head_dim / 2, quarter = head_dim / 4;
  const int64_t gid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (gid >= T * half) return;
  const int64_t t = gid / half;
  const int j = (int)(gid % half);
  int img, row, col;
  token_rc(g, merge, t, &img, &row, &col);
  const float pos = (float)(j < quarter ? row : col);
  float s, c;
  sincosf(pos * inv.v[j % quarter], &s, &c);
  cos_out[t * head_dim + j] = c;
  cos_out[t * head_dim + j + half] = c;
  sin_out[t * head_dim + j] = s;
  sin_out[t * head_dim + j + half] = s;
}

// In place x*cos + cat(-x2, x1)*sin on `nheads` heads of each row.  One
// thread per (token, head, i < head_dim/2) rotating the pair (i, i + half).
__global__ void rope_apply_kernel(__nv_bfloat16* x, int64_t T, int nheads, int head_dim, int64_t stride,
                                  const float* __restrict__ cos_tab, const float* __restrict__ sin_tab) {
  pdl_trigger();
  pdl_wait();
  const int half = head_dim / 2;
  const int64_t gid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (gid >= T * nheads * half) return;
  const int i = (int)(gid % half);
  const int64_t th = gid / half;
  const int64_t t = th / nheads;
  const int h = (int)(th % nheads);
  __nv_bfloat16* p = x + t * stride + (int64_t)h * head_dim;
  const float x1 = bf2f(p[i]), x2 = bf2f(p[i + half]);
  const float c1 = cos_tab[t * head_dim + i], s1 = sin_tab[t * head_dim + i];
  const float c2 = cos_tab[t * head_dim + i + half], s2 = sin_tab[t * head_dim + i + half];
  p[i] = f2bf(x1 * c1 - x2 * s1);
  p[i + half] = f2bf(x2 * c2 + x1 * s2);
}

// out[t, :] (+)= bilinear interpolation of table at token t's patch position.
// fy = float(row) * (G-1) / (h-1) etc. in fp32, the expression order of the
// reference's CPU interpolation.  One CTA per token, 8 features per thread.
__global__ void pos_embed_interp_kernel(const __nv_bfloat16* __restrict__ table, int num_grid, Grids g, int merge,
                                        int64_t dim, __nv_bfloat16* out, int accumulate) {
  pdl_trigger();
  pdl_wait();
  const int64_t t = blockIdx.x;
  int img, row, col;
  token_rc(g, merge, t, &img, &row, &col);
  const int h = g.h[img], w = g.w[img];
  const float G1 = (float)(num_grid - 1);
  const float fy = h <= 1 ? 0.f : __fdiv_rn(__fmul_rn((float)row, G1), (float)(h - 1));
  const float fx = w <= 1 ? 0.f : __fdiv_rn(__fmul_rn((float)col, G1), (float)(w - 1));
  const int y0 = (int)fy, x0 = (int)fx;
  const int y1 = min(y0 + 1, num_grid - 1), x1 = min(x0 + 1, num_grid - 1);
  const float dy = __fsub_rn(fy, (float)y0), dx = __fsub_rn(fx, (float)x0);
  const float ody = __fsub_rn(1.f, dy), odx = __fsub_rn(1.f, dx);
  const __nv_bfloat16* r00 = table + ((int64_t)y0 * num_grid + x0) * dim;
  const __nv_bfloat16* r01 = table + ((int64_t)y0 * num_grid + x1) * dim;
  const __nv_bfloat16* r10 = table + ((int64_t)y1 * num_grid + x0) * dim;
  const __nv_bfloat16* r11 = table + ((int64_t)y1 * num_grid + x1) * dim;
  for (int64_t c = threadIdx.x; c < dim / 8; c += blockDim.x) {
    float a[8], b[8], cc[8], d[8], o[8];
    unpack8(*reinterpret_cast<const uint4*>(r00 + c * 8), a);
    unpack8(*reinterpret_cast<const uint4*>(r01 + c * 8), b);
    unpack8(*reinterpret_cast<const uint4*>(r10 + c * 8), cc);
    unpack8(*reinterpret_cast<const uint4*>(r11 + c * 8), d);
    if (accumulate) unpack8(*reinterpret_cast<const uint4*>(out + t * dim + c * 8), o);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float v = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(__fmul_rn(a[k], ody), odx), __fmul_rn(__fmul_rn(b[k], ody), dx)),
                                          __fmul_rn(__fmul_rn(cc[k], dy), odx)),
                                __fmul_rn(__fmul_rn(d[k], dy), dx));
      o[k] = accumulate ? o[k] + v : v;
    }
    *reinterpret_cast<uint4*>(out + t * dim + c * 8) = pack8(o);
  }
}

// Host-side grid table (grid_thw is host metadata, as in the reference).
int make_grids(const int64_t* grid_thw, int n, int merge, Grids* g, int64_t* total) {
  if (!grid_thw || n <= 0 || n > kMaxImages || merge <= 0) return B200_ERROR_INVALID_PARAM;
  g->n = n;
  g->start[0] = 0;
  for (int i = 0; i < n; ++i) {
    const int64_t t = grid_thw[3 * i], h = grid_thw[3 * i + 1], w = grid_thw[3 * i + 2];
    if (t <= 0 || h <= 0 || w <= 0 || h % merge || w % merge || h > (1 << 20) || w > (1 << 20))
      return B200_ERROR_INVALID_PARAM;
    g->h[i] = (int)h;
    g->w[i] = (int)w;
    g->start[i + 1] = g->start[i] + t * h * w;
  }
  *total = g->start[n];
  return B200_OK;
}

}  // namespace

extern "C" int b200_rope_table_vision(const int64_t* grid_thw, int num_images, int merge_size, int head_dim,
                                      float theta, float* cos_out, float* sin_out, b200_stream_t stream) {
  if (!cos_out || !sin_out || head_dim <= 0 || head_dim % 4 || head_dim > 256) return B200_ERROR_INVALID_PARAM;
  Grids g;
  int64_t T = 0;
  int rc = make_grids(grid_thw, num_images, merge_size, &g, &T);
  if (rc != B200_OK) return rc;
  // inv_freq over dim = head_dim/2 with step 2: 1 / theta^(2j / dim), j < head_dim/4
  InvFreqV inv;
  const int dim = head_dim / 2;
  for (int j = 0; j < head_dim / 4; ++j) inv.v[j] = 1.0f / powf(theta, (float)(2 * j) / (float)dim);
  const int64_t n = T * (head_dim / 2);
  launch_kernel(rope_table_vision_kernel, dim3((unsigned)((n + 255) / 256)), 256, 0, stream, g, merge_size, head_dim,
                inv, T, cos_out, sin_out);
  B200_CHECK_LAUNCH();
  return B200_OK;
}

extern "C" int b200_rope_apply(void* x, int64_t T, int nheads, int head_dim, int64_t stride, const float* cos_tab,
                               const float* sin_tab, b200_stream_t stream) {
  if (!x || !cos_tab || !sin_tab || T < 0 || nheads <= 0 || head_dim <= 0 || head_dim % 2 ||
      stride < (int64_t)nheads * head_dim)
    return B200_ERROR_INVALID_PARAM;
  if (T == 0) return B200_OK;
  const int64_t n = T * nheads * (head_dim / 2);
  launch_kernel(rope_apply_kernel, dim3((unsigned)((n + 255) / 256)), 256, 0, stream, static_cast<__nv_bfloat16*>(x),
                T, nheads, head_dim, stride, cos_tab, sin_tab);
  B200_CHECK_LAUNCH();
  return B200_OK;
}

extern "C" int b200_pos_embed_interp(const void* table, int num_grid, int64_t dim, const int64_t* grid_thw,
                                     int num_images, int merge_size, void* out, int accumulate, b200_stream_t stream) {
  if (!table || !out || num_grid <= 0 || dim <= 0 || dim % 8) return B200_ERROR_INVALID_PARAM;
  if ((reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(out)) & 15) return B200_ERROR_INVALID_PARAM;
  Grids g;
  int64_t T = 0;
  int rc = make_grids(grid_thw, num_images, merge_size, &g, &T);
  if (rc != B200_OK) return rc;
  if (T > INT32_MAX) return B200_ERROR_UNSUPPORTED;
  launch_kernel(pos_embed_interp_kernel, dim3((unsigned)T), 128, 0, stream, static_cast<const __nv_bfloat16*>(table),
                num_grid, g, merge_size, dim, static_cast<__nv_bfloat16*>(out), accumulate);
  B200_CHECK_LAUNCH();
  return B200_OK;
}
