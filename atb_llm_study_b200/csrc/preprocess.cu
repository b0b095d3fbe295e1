// Qwen3-VL image preprocessing on the GPU: SmartResize (host), Pillow's
// 8-bit antialiased BICUBIC resample, (x/255 - mean)/std and the merge-block
// patchify with the temporal duplicate, written straight into the vision
// tower's pixel_values (fp16 or bf16).
//
// Replaces the reference's CPU PreprocessImage / BicubicResize /
// SmartResize (atb_cpp_llm/src/adapters/qwen3vl_embedding/
// qwen3vl_preprocess.cpp:52-366) and its device pipeline
// PreprocessImageNpu (:369-824), bit for bit: the resample keeps Pillow's
// fixed-point arithmetic (coefficients quantised to 22 fractional bits,
// int32 accumulation from 2^21, clip of >> 22), so results equal PIL's.
//
// Work per image: the fixed-point coefficients of both axes (one small
// kernel, FMA-free double arithmetic identical to the host's).  Then, when
// every window has at most 16 taps (downscales up to about 3.5x, every
// upscale) and a block's input rows fit in shared memory, one
// preprocess_fused_kernel that runs the horizontal pass into shared memory
// and the vertical pass plus normalise/patchify from there.  Otherwise one
// horizontal-pass kernel (one thread per output sample, uint8 intermediate
// [C, H, out_w]) and one vertical-pass kernel that also
// normalises and scatters each value to its patch positions (frame 0 and the
// duplicated frames).  An axis whose size does not change is not resampled
// (the horizontal pass is skipped; the vertical pass runs with one unit tap,
// which reproduces the input byte exactly).  HBM-bound byte work, no tensor
// cores: 2-D grids (256 samples of one row per block) keep the index math in
// 32-bit and the row reads coalesced.
#include <cuda_fp16.h>
#include <math.h>

#include <algorithm>

#include "common.cuh"

using namespace b200;

namespace {

constexpr int kPrecisionBits = 22;
constexpr int kThreads = 256;
constexpr int kRowsPerBlock = 8;  // image rows one block walks through

__device__ __forceinline__ uint8_t clip8(int v) {
  const int s = v >> kPrecisionBits;  // arithmetic shift
  return (uint8_t)(s < 0 ? 0 : (s > 255 ? 255 : s));
}

// out[c][y][xx] = clip8(2^21 + sum_x in[c][y][xmin + x] * k[xx][x]);
// grid (out_w / 256, C*H): 256 consecutive output samples of one row per
// block; the input bytes their windows cover (monotone in xx) are staged in
// shared memory once.
template <int KMAX>
__global__ void __launch_bounds__(kThreads) resample_h_kernel(const uint8_t* __restrict__ in, int rows, int W,
                                                               int out_w, int ksize, const int* __restrict__ bounds,
                                                               const int* __restrict__ coef, uint8_t* __restrict__ out,
                                                               int span_cap) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ uint8_t span[];
  const int xx0 = blockIdx.x * kThreads;
  const int last = min(xx0 + kThreads, out_w) - 1;
  const int lo = bounds[2 * xx0];
  const int hi = min(bounds[2 * last] + bounds[2 * last + 1], lo + span_cap);
  const int xx = xx0 + threadIdx.x;
  const bool active = xx <= last;
  const int x0 = active ? bounds[2 * xx] - lo : 0;
  const int taps = active ? min(bounds[2 * xx + 1], hi - lo - x0) : 0;
  // this sample's taps stay in registers for all the block's rows
  int kr[KMAX];
#pragma unroll
  for (int x = 0; x < KMAX; ++x) kr[x] = x < taps ? coef[(int64_t)xx * ksize + x] : 0;
  const int r1 = min(rows, (int)(blockIdx.y + 1) * kRowsPerBlock);
  for (int r = blockIdx.y * kRowsPerBlock; r < r1; ++r) {
    const uint8_t* row = in + (int64_t)r * W;
    for (int i = threadIdx.x; i < hi - lo; i += kThreads) span[i] = row[lo + i];
    __syncthreads();
    if (active) {
      int ss = 1 << (kPrecisionBits - 1);
#pragma unroll
      for (int x = 0; x < KMAX; ++x)
        if (x < taps) ss += (int)span[x0 + x] * kr[x];
      out[(int64_t)r * out_w + xx] = clip8(ss);
    }
    __syncthreads();
  }
}

// Vertical pass over in [C, H, out_w] to rows of out_h; MODE 0 writes the
// uint8 image [C, out_h, out_w]; MODE 1 / 2 write (v/255 - mean)/std as fp16 /
// bf16 into the patch layout (merge-block order, frame duplicated over tp).
// grid (out_w / (256 VEC), C*out_h): VEC consecutive samples of one row per
// thread (4-byte loads of each tap row); the 256 normalised values of the
// block's channel are precomputed once per block (same float32 arithmetic,
// so the table holds exactly the values the formula gives).
template <int MODE, int VEC, int KMAX>
__global__ void __launch_bounds__(kThreads) resample_v_kernel(const uint8_t* __restrict__ in, int C, int H,
                                                               int out_h, int out_w, int ksize,
                                                               const int* __restrict__ bounds,
                                                               const int* __restrict__ coef, void* __restrict__ out,
                                                               float3 mean, float3 stdv, int ps, int tp, int ms) {
  pdl_trigger();
  __shared__ uint16_t lut[256];
  const int row_blocks = (out_h + kRowsPerBlock - 1) / kRowsPerBlock;
  const int c = blockIdx.y / row_blocks;
  const int yy0 = (blockIdx.y - c * row_blocks) * kRowsPerBlock, yy1 = min(out_h, yy0 + kRowsPerBlock);
  if (MODE != 0) {
    // the reference's order of operations: (u / 255 - mean) / std in float32
    const float m = c == 0 ? mean.x : (c == 1 ? mean.y : mean.z);
    const float sd = c == 0 ? stdv.x : (c == 1 ? stdv.y : stdv.z);
    const float v = ((float)threadIdx.x / 255.0f - m) / sd;
    if (MODE == 1) lut[threadIdx.x] = __half_as_ushort(__float2half_rn(v));
    else lut[threadIdx.x] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  }
  pdl_wait();
  __syncthreads();
  const int xx = (blockIdx.x * kThreads + threadIdx.x) * VEC;
  if (xx >= out_w) return;
  const int gx = xx / ps, px = xx - gx * ps;
  const int gwm = out_w / ps / ms;
  const int64_t pdim = (int64_t)C * tp * ps * ps;
  for (int yy = yy0; yy < yy1; ++yy) {
    const int y0 = bounds[2 * yy], taps = bounds[2 * yy + 1];
    const uint8_t* src = in + ((int64_t)c * H + y0) * out_w + xx;
    const int* k = coef + yy * ksize;
    int ss[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) ss[e] = 1 << (kPrecisionBits - 1);
#pragma unroll
    for (int y = 0; y < KMAX; ++y) {
      if (y >= taps) break;
      const int ky = k[y];
      if (VEC == 4) {
        const uchar4 q = *reinterpret_cast<const uchar4*>(src + (int64_t)y * out_w);
        ss[0] += (int)q.x * ky;
        ss[1] += (int)q.y * ky;
        ss[2] += (int)q.z * ky;
        ss[3] += (int)q.w * ky;
      } else {
        ss[0] += (int)src[(int64_t)y * out_w] * ky;
      }
    }
    if (MODE == 0) {
      uint8_t* o = static_cast<uint8_t*>(out) + ((int64_t)c * out_h + yy) * out_w + xx;
      if (VEC == 4) *reinterpret_cast<uchar4*>(o) = make_uchar4(clip8(ss[0]), clip8(ss[1]), clip8(ss[2]), clip8(ss[3]));
      else o[0] = clip8(ss[0]);
      continue;
    }
    // patch (gy, gx) in merge-block order, element (c, f, py, px); the VEC
    // samples stay inside one patch row (ps % VEC == 0)
    const int gy = yy / ps, py = yy - gy * ps;
    const int64_t patch = ((int64_t)((gy / ms) * gwm + gx / ms) * ms + gy % ms) * ms + gx % ms;
    uint16_t* o = static_cast<uint16_t*>(out) + patch * pdim + ((int64_t)c * tp * ps + py) * ps + px;
    if (VEC == 4) {
      const uint2 w = make_uint2((uint32_t)lut[clip8(ss[0])] | ((uint32_t)lut[clip8(ss[1])] << 16),
                                 (uint32_t)lut[clip8(ss[2])] | ((uint32_t)lut[clip8(ss[3])] << 16));
      for (int f = 0; f < tp; ++f) *reinterpret_cast<uint2*>(o + (int64_t)f * ps * ps) = w;
    } else {
      const uint16_t w = lut[clip8(ss[0])];
      for (int f = 0; f < tp; ++f) o[(int64_t)f * ps * ps] = w;
    }
  }
}

// ---- Pillow's coefficients for one axis, computed on the device ----
// Every double operation is an explicit round-to-nearest intrinsic, so none
// is fused into an FMA and the values equal the host computation (Pillow's
// precompute_coeffs + normalize_coeffs_8bpc as the reference ports it,
// qwen3vl_preprocess.cpp:38-99) bit for bit.
__device__ __forceinline__ double bicubic_d(double x) {
  const double a = -0.5;
  x = fabs(x);
  if (x < 1.0)  // ((a + 2) x - (a + 3)) x x + 1
    return __dadd_rn(__dmul_rn(__dmul_rn(__dsub_rn(__dmul_rn(__dadd_rn(a, 2.0), x), __dadd_rn(a, 3.0)), x), x), 1.0);
  if (x < 2.0)  // (((x - 5) x + 8) x - 4) a
    return __dmul_rn(__dsub_rn(__dmul_rn(__dadd_rn(__dmul_rn(__dsub_rn(x, 5.0), x), 8.0), x), 4.0), a);
  return 0.0;
}

constexpr int kMaxTaps = 256;  // downscale factors up to 63x per axis

// blockIdx.y = axis (0: vertical, 1: horizontal); one thread per output sample.
// bounds[2*o] = first tap, bounds[2*o+1] = taps; coef[o*ksize + t] in 22-bit
// fixed point.  An axis that keeps its size gets one unit tap per sample.
__global__ void __launch_bounds__(kThreads) coeffs_kernel(int in_v, int out_v, int ks_v, int* bounds_v, int* coef_v,
                                                           int in_h, int out_h, int ks_h, int* bounds_h,
                                                           int* coef_h) {
  pdl_trigger();
  pdl_wait();
  const bool horiz = blockIdx.y == 1;
  const int in = horiz ? in_h : in_v, out = horiz ? out_h : out_v, ks = horiz ? ks_h : ks_v;
  int* bounds = horiz ? bounds_h : bounds_v;
  int* coef = horiz ? coef_h : coef_v;
  if (!bounds || !coef) return;
  for (int o = blockIdx.x * blockDim.x + threadIdx.x; o < out; o += gridDim.x * blockDim.x) {
    int* k = coef + (int64_t)o * ks;
    if (in == out) {
      bounds[2 * o] = o;
      bounds[2 * o + 1] = 1;
      k[0] = 1 << kPrecisionBits;
      continue;
    }
    const double scale = __ddiv_rn((double)in, (double)out);
    const double filterscale = scale < 1.0 ? 1.0 : scale;
    const double support = __dmul_rn(2.0, filterscale);
    const double center = __dmul_rn(__dadd_rn((double)o, 0.5), scale);
    const double rss = __ddiv_rn(1.0, filterscale);
    int xmin = __double2int_rz(__dadd_rn(__dsub_rn(center, support), 0.5));
    if (xmin < 0) xmin = 0;
    int xmax = __double2int_rz(__dadd_rn(__dadd_rn(center, support), 0.5));
    if (xmax > in) xmax = in;
    xmax -= xmin;
    if (xmax > ks) xmax = ks;  // never taken: ks = 2 ceil(support) + 1 covers every window
    double w[kMaxTaps];
    double ww = 0.0;
    for (int x = 0; x < xmax; ++x) {
      w[x] = bicubic_d(__dmul_rn(__dadd_rn(__dsub_rn((double)(x + xmin), center), 0.5), rss));
      ww = __dadd_rn(ww, w[x]);
    }
    for (int x = 0; x < ks; ++x) {
      int q = 0;
      if (x < xmax) {
        const double v = ww != 0.0 ? __ddiv_rn(w[x], ww) : w[x];
        const double f = __dmul_rn(v, (double)(1 << kPrecisionBits));
        q = v < 0 ? __double2int_rz(__dadd_rn(-0.5, f)) : __double2int_rz(__dadd_rn(0.5, f));
      }
      k[x] = q;
    }
    bounds[2 * o] = xmin;
    bounds[2 * o + 1] = xmax;
  }
}

// ---- the resample (+ normalise + patchify) in one launch after the coefficients ----
// Block (x, y, c) produces output columns [256x, 256x + 256) of output rows
// [32y, 32y + 32) of channel c.  It reads its coefficients from the tables
// coeffs_kernel wrote, stages the input tile its windows cover (every row at
// once, so all the loads are in flight together: 16-byte cp.async when the
// rows are 16-byte aligned, batched byte loads otherwise), runs the
// horizontal pass into shared memory (a few halo rows are computed by both
// neighbouring blocks), then the vertical pass from there: the uint8
// intermediate never goes to global memory.  Same integer arithmetic as the
// two-pass kernels, so the same bytes.
constexpr int kFRows = 32;  // output rows per block
constexpr int kFK = 16;     // taps per axis the fused kernel handles (downscale up to ~3.5x)
constexpr int kFusedSmemCap = 96 * 1024;

// Dynamic shared memory: the input tile [rows_cap][tile_w] and the horizontal
// results [rows_cap + K][256].  The tap loops run all K taps without a branch:
// weights past a window are zero, and the K spare rows / the tile's slack
// keep every read in bounds (what they hold is multiplied by zero).
// bh/ch = nullptr: the width does not change (one unit tap per column).
template <int MODE, bool VEC16, int K>
__global__ void __launch_bounds__(kThreads) preprocess_fused_kernel(
    const uint8_t* __restrict__ in, int C, int H, int W, int out_h, int out_w, const int* __restrict__ bv,
    const int* __restrict__ cv, int ksv, const int* __restrict__ bh, const int* __restrict__ ch, int ksh,
    void* __restrict__ out, float3 mean, float3 stdv, int ps, int tp, int ms, int rows_cap, int span_cap, int tile_w,
    unsigned* err) {
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t fsm[];
  uint8_t* tile = fsm;
  uint8_t* hrow = fsm + (int64_t)rows_cap * tile_w;
  __shared__ __align__(16) int vk[kFRows * K];  // vertical taps of the block's output rows
  __shared__ int vb[kFRows * 2];                // first input row, taps
  __shared__ int64_t ro[kFRows];                // output offset of each row's first element
  __shared__ uint16_t lut[256];
  __shared__ int lo_s, hi_s;
  const int c = blockIdx.z;
  const int xx0 = blockIdx.x * kThreads, yy0 = blockIdx.y * kFRows;
  const int nrows = min(kFRows, out_h - yy0);
  const int last = min(xx0 + kThreads, out_w) - 1;
  const int64_t pdim = (int64_t)C * tp * ps * ps;
  if (MODE != 0) {  // (u / 255 - mean) / std in float32, the reference's order of operations
    const float m = c == 0 ? mean.x : (c == 1 ? mean.y : mean.z);
    const float sd = c == 0 ? stdv.x : (c == 1 ? stdv.y : stdv.z);
    const float v = ((float)threadIdx.x / 255.0f - m) / sd;
    if (MODE == 1) lut[threadIdx.x] = __half_as_ushort(__float2half_rn(v));
    else lut[threadIdx.x] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  }
  const int xx = xx0 + threadIdx.x;
  const bool active = xx <= last;
  int64_t col;  // output offset of this column inside a row
  {
    const int gx = xx / ps, px = xx - gx * ps;
    col = MODE == 0 ? (int64_t)xx : ((int64_t)(gx / ms) * ms * ms + gx % ms) * pdim + px;
  }
  if ((int)threadIdx.x < nrows && MODE != 0) {
    // patch ((gy/ms) gw/ms + gx/ms) ms^2 + (gy%ms) ms + gx%ms, element (c, f, py, px): the row part
    const int yy = yy0 + threadIdx.x;
    const int gy = yy / ps, py = yy - gy * ps;
    const int gwm = out_w / ps / ms;
    ro[threadIdx.x] = ((int64_t)(gy / ms) * gwm * ms * ms + (gy % ms) * ms) * pdim + ((int64_t)c * tp * ps + py) * ps;
  } else if ((int)threadIdx.x < nrows) {
    ro[threadIdx.x] = ((int64_t)c * out_h + yy0 + threadIdx.x) * out_w;
  }
  pdl_wait();  // the coefficient tables and the image come from earlier kernels / copies
  if ((int)threadIdx.x < nrows) {
    const int yy = yy0 + threadIdx.x;
#pragma unroll
    for (int y = 0; y < K; ++y) vk[threadIdx.x * K + y] = y < ksv ? cv[(int64_t)yy * ksv + y] : 0;
    vb[2 * threadIdx.x] = bv[2 * yy];
    vb[2 * threadIdx.x + 1] = bv[2 * yy + 1];
  }
  const int sx = active ? xx : last;
  int kr[K], hx0, htaps;
  if (bh) {
    hx0 = bh[2 * sx];
    htaps = bh[2 * sx + 1];
#pragma unroll
    for (int x = 0; x < K; ++x) kr[x] = x < ksh ? ch[(int64_t)sx * ksh + x] : 0;
  } else {
    hx0 = sx;
    htaps = 1;
#pragma unroll
    for (int x = 0; x < K; ++x) kr[x] = x == 0 ? (1 << kPrecisionBits) : 0;
  }
  if (threadIdx.x == 0) lo_s = hx0;
  if (xx == last) hi_s = hx0 + htaps;
  __syncthreads();
  // input columns [lo, hi) (lo rounded down to 16 bytes on the aligned path), rows [ylo, yhi)
  const int lo = VEC16 ? (lo_s & ~15) : lo_s;
  const int hi = min(hi_s, lo_s + span_cap);
  const int ylo = vb[0];
  int yhi = vb[2 * (nrows - 1)] + vb[2 * (nrows - 1) + 1];
  if (yhi - ylo > rows_cap) {  // the host's bound makes this unreachable
    if (threadIdx.x == 0) raise_error(err, DEV_ERR_BAD_INDEX);
    yhi = ylo + rows_cap;
  }
  const int nr = yhi - ylo;
  // this column's window inside the tile; taps past the staged bytes get weight zero
  const int hx = min(hx0 - lo, tile_w - K);
#pragma unroll
  for (int x = 0; x < K; ++x)
    if (hx + x >= hi - lo) kr[x] = 0;
  const uint8_t* src = in + ((int64_t)c * H + ylo) * W + lo;
  if (VEC16) {
    // chunks of 16 bytes: hi - lo rounded up stays inside the row (W % 16 == 0) and inside tile_w
    const int cw = (hi - lo + 15) >> 4;
    for (int i = threadIdx.x; i < nr * cw; i += kThreads) {
      const int r = i / cw, q = i - r * cw;
      cp_async_16(smem_u32(tile + r * tile_w + q * 16), src + (int64_t)r * W + q * 16, true);
    }
    cp_async_commit();
  } else {
    const int sw = hi - lo, total = nr * sw;
    for (int base = threadIdx.x; base < total; base += kThreads * 8) {
      uint8_t v[8];
      int at[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = base + j * kThreads;
        const int r = i / sw, q = i - r * sw;
        at[j] = i < total ? r * tile_w + q : -1;
        v[j] = i < total ? src[(int64_t)r * W + q] : 0;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (at[j] >= 0) tile[at[j]] = v[j];
    }
  }
  // the K spare result rows past nr read as zero-weighted taps: give them defined bytes
#pragma unroll
  for (int y = 0; y < K; ++y) hrow[(nr + y) * kThreads + threadIdx.x] = 0;
  if (VEC16) cp_async_wait<0>();
  __syncthreads();
  // horizontal pass over the staged rows
  const uint8_t* t = tile + hx;
  for (int r = 0; r < nr; ++r, t += tile_w) {
    int ss = 1 << (kPrecisionBits - 1);
#pragma unroll
    for (int x = 0; x < K; ++x) ss += (int)t[x] * kr[x];
    hrow[r * kThreads + threadIdx.x] = clip8(ss);
  }
  __syncthreads();
  if (!active) return;
  for (int i = 0; i < nrows; ++i) {
    const uint8_t* h = hrow + min(vb[2 * i] - ylo, nr) * kThreads + threadIdx.x;  // rows < nr + K
    const int* k = vk + i * K;
    int ss = 1 << (kPrecisionBits - 1);
#pragma unroll
    for (int y = 0; y < K; ++y) ss += (int)h[y * kThreads] * k[y];
    const uint8_t u = clip8(ss);
    if (MODE == 0) {
      static_cast<uint8_t*>(out)[ro[i] + col] = u;
    } else {
      uint16_t* o = static_cast<uint16_t*>(out) + ro[i] + col;
      const uint16_t wv = lut[u];
      for (int f = 0; f < tp; ++f) o[(int64_t)f * ps * ps] = wv;
    }
  }
}

int ksize_of(int in_size, int out_size) {
  const double scale = (double)in_size / out_size;
  const double support = 2.0 * (scale < 1.0 ? 1.0 : scale);
  return (int)ceil(support) * 2 + 1;
}

int64_t align256(int64_t b) { return (b + 255) & ~int64_t(255); }

struct Layout {
  int ksh = 0, ksv = 0;
  int64_t off_bh = 0, off_ch = 0, off_bv = 0, off_cv = 0, off_tmp = 0, total = 0;
};

Layout layout(int C, int H, int W, int oh, int ow) {
  Layout L;
  const bool need_h = ow != W, need_v = oh != H;
  L.ksh = need_h ? ksize_of(W, ow) : 0;
  L.ksv = need_v ? ksize_of(H, oh) : 1;
  int64_t o = 0;
  L.off_bh = o;
  o += align256((int64_t)ow * 2 * 4);
  L.off_ch = o;
  o += align256((int64_t)ow * std::max(L.ksh, 1) * 4);
  L.off_bv = o;
  o += align256((int64_t)oh * 2 * 4);
  L.off_cv = o;
  o += align256((int64_t)oh * L.ksv * 4);
  L.off_tmp = o;
  o += need_h ? align256((int64_t)C * H * ow) : 0;
  L.total = o;
  return L;
}

int cuda_rc(cudaError_t e) { return e == cudaSuccess ? B200_OK : B200_ERROR_CUDA_BASE - (int)e; }

// Resample image [C,H,W] (device) to (oh, ow); MODE as resample_v_kernel.
int run_resample(int mode, const uint8_t* image, int C, int H, int W, int oh, int ow, void* out, float3 mean,
                 float3 stdv, int ps, int tp, int ms, void* ws, int64_t ws_bytes, cudaStream_t st) {
  const Layout L = layout(C, H, W, oh, ow);
  if (!ws || ws_bytes < L.total || (reinterpret_cast<uintptr_t>(ws) & 255)) return B200_ERROR_INVALID_PARAM;
  // coefficients + one fused launch when every window fits its tap budget and a block's tile fits in
  // shared memory; the horizontal intermediate in the workspace serves only the two-pass path below
  {
    const int ksh = ow != W ? ksize_of(W, ow) : 1, ksv = oh != H ? ksize_of(H, oh) : 1;
    const int K = std::max(ksh, ksv) <= 8 ? 8 : kFK;
    // input rows of 32 output rows' windows / input bytes of 256 output columns' windows, with slack
    const int rows_cap = (int)ceil((double)H / oh * kFRows) + ksv + 2;
    const int span_cap = (int)ceil((double)W / ow * kThreads) + ksh + 8;
    const int tile_w = ((span_cap + 15) & ~15) + 32;  // room for the 16-byte round-down and round-up
    const int64_t smem = (int64_t)rows_cap * tile_w + (int64_t)(rows_cap + K) * kThreads;
    const int64_t gy = (oh + kFRows - 1) / kFRows;
    if (ksh <= kFK && ksv <= kFK && smem <= kFusedSmemCap && gy <= 65535 && C <= 65535) {
      const bool vec16 = W % 16 == 0 && (reinterpret_cast<uintptr_t>(image) & 15) == 0;
      int dev = 0;
      cudaGetDevice(&dev);
      static bool attr[64] = {false};
      if (dev >= 0 && dev < 64 && !attr[dev]) {
#define B200_PF_ATTR(V, KK)                                                                                        \
  for (auto f : {preprocess_fused_kernel<0, V, KK>, preprocess_fused_kernel<1, V, KK>,                             \
                 preprocess_fused_kernel<2, V, KK>})                                                                \
    if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kFusedSmemCap) != cudaSuccess) \
      return B200_ERROR_UNSUPPORTED;
        B200_PF_ATTR(true, 8)
        B200_PF_ATTR(false, 8)
        B200_PF_ATTR(true, kFK)
        B200_PF_ATTR(false, kFK)
#undef B200_PF_ATTR
        attr[dev] = true;
      }
      uint8_t* w8 = static_cast<uint8_t*>(ws);
      int* bv = reinterpret_cast<int*>(w8 + L.off_bv);
      int* cv = reinterpret_cast<int*>(w8 + L.off_cv);
      int* bh = ow != W ? reinterpret_cast<int*>(w8 + L.off_bh) : nullptr;
      int* ch = ow != W ? reinterpret_cast<int*>(w8 + L.off_ch) : nullptr;
      launch_kernel(coeffs_kernel, dim3((unsigned)((std::max(oh, ow) + kThreads - 1) / kThreads), 2), kThreads, 0,
                    st, H, oh, L.ksv, bv, cv, W, ow, L.ksh, bh, ch);
      B200_CHECK_LAUNCH();
      const dim3 g((unsigned)((ow + kThreads - 1) / kThreads), (unsigned)gy, (unsigned)C);
      unsigned* err = b200::error_word(dev);
#define B200_PF(M, V, KK)                                                                                     \
  launch_kernel(preprocess_fused_kernel<M, V, KK>, g, kThreads, (size_t)smem, st, image, C, H, W, oh, ow, bv, cv, \
                L.ksv, bh, ch, L.ksh, out, mean, stdv, ps, tp, ms, rows_cap, span_cap, tile_w, err)
#define B200_PF_MODE(V, KK)          \
  if (mode == 0) B200_PF(0, V, KK);  \
  else if (mode == 1) B200_PF(1, V, KK); \
  else B200_PF(2, V, KK);
      if (K == 8) {
        if (vec16) { B200_PF_MODE(true, 8) } else { B200_PF_MODE(false, 8) }
      } else {
        if (vec16) { B200_PF_MODE(true, kFK) } else { B200_PF_MODE(false, kFK) }
      }
#undef B200_PF_MODE
#undef B200_PF
      B200_CHECK_LAUNCH();
      return B200_OK;
    }
  }
  uint8_t* w8 = static_cast<uint8_t*>(ws);
  const bool need_h = ow != W;
  if (L.ksh > kMaxTaps || L.ksv > kMaxTaps) return B200_ERROR_UNSUPPORTED;
  // grid rows: kRowsPerBlock image rows each
  if ((int64_t)C * (std::max(H, oh) / kRowsPerBlock + 1) > 65535) return B200_ERROR_UNSUPPORTED;
  int* bv = reinterpret_cast<int*>(w8 + L.off_bv);
  int* cv = reinterpret_cast<int*>(w8 + L.off_cv);
  int* bh = need_h ? reinterpret_cast<int*>(w8 + L.off_bh) : nullptr;
  int* ch = need_h ? reinterpret_cast<int*>(w8 + L.off_ch) : nullptr;
  const int most = std::max(oh, ow);
  launch_kernel(coeffs_kernel, dim3((unsigned)((most + kThreads - 1) / kThreads), 2), kThreads, 0, st, H, oh, L.ksv,
                bv, cv, W, ow, L.ksh, bh, ch);
  B200_CHECK_LAUNCH();
  const uint8_t* vin = image;
  if (need_h) {
    // bytes the widest block's windows span: 256 samples x the scale + one window
    const int span_cap = (int)ceil((double)W / ow * kThreads) + L.ksh + 8;
    if (span_cap > 160 * 1024) return B200_ERROR_UNSUPPORTED;
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (span_cap > 48 * 1024 && dev >= 0 && dev < 64 && !attr[dev]) {
      for (auto f : {resample_h_kernel<8>, resample_h_kernel<16>, resample_h_kernel<32>, resample_h_kernel<64>})
        if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024) != cudaSuccess)
          return B200_ERROR_UNSUPPORTED;
      attr[dev] = true;
    }
    const dim3 gh((unsigned)((ow + kThreads - 1) / kThreads), (unsigned)((C * H + kRowsPerBlock - 1) / kRowsPerBlock));
#define B200_RH(K) \
  launch_kernel(resample_h_kernel<K>, gh, kThreads, (size_t)span_cap, st, image, C * H, W, ow, L.ksh, bh, ch, \
                w8 + L.off_tmp, span_cap)
    if (L.ksh <= 8) B200_RH(8);
    else if (L.ksh <= 16) B200_RH(16);
    else if (L.ksh <= 32) B200_RH(32);
    else if (L.ksh <= 64) B200_RH(64);
    else return B200_ERROR_UNSUPPORTED;
#undef B200_RH
    B200_CHECK_LAUNCH();
    vin = w8 + L.off_tmp;
  }
  const bool vec = ow % 4 == 0 && (reinterpret_cast<uintptr_t>(vin) & 3) == 0 && (mode == 0 || ps % 4 == 0) &&
                   (reinterpret_cast<uintptr_t>(out) & (mode == 0 ? 3 : 7)) == 0;
  const int per = vec ? 4 : 1;
  const dim3 g((unsigned)((ow + kThreads * per - 1) / (kThreads * per)),
               (unsigned)(C * ((oh + kRowsPerBlock - 1) / kRowsPerBlock)));
  const int ksv = L.ksv;
#define B200_RVK(M, V, K)                                                                                     \
  launch_kernel(resample_v_kernel<M, V, K>, g, kThreads, 0, st, vin, C, H, oh, ow, ksv, bv, cv, out, mean, stdv, ps, \
                tp, ms)
#define B200_RV(M, V) \
  (ksv <= 16 ? B200_RVK(M, V, 16) : ksv <= 64 ? B200_RVK(M, V, 64) : B200_RVK(M, V, 256))
  if (mode == 0) vec ? B200_RV(0, 4) : B200_RV(0, 1);
  else if (mode == 1) vec ? B200_RV(1, 4) : B200_RV(1, 1);
  else vec ? B200_RV(2, 4) : B200_RV(2, 1);
#undef B200_RVK
#undef B200_RV
  B200_CHECK_LAUNCH();
  return B200_OK;
}

}  // namespace

extern "C" int b200_smart_resize(int height, int width, int factor, int min_pixels, int max_pixels, int* new_height,
                                 int* new_width) {
  if (!new_height || !new_width || height <= 0 || width <= 0 || factor <= 0 || min_pixels < 0 ||
      max_pixels < min_pixels)
    return B200_ERROR_INVALID_PARAM;
  // banker's rounding of size / factor evaluated in float32 (as the reference)
  auto bankers = [](float x) {
    const float f = floorf(x);
    const float frac = x - f;
    if (frac < 0.5f) return (int)f;
    if (frac > 0.5f) return (int)(f + 1.0f);
    const int lo = (int)f;
    return lo % 2 == 0 ? lo : lo + 1;
  };
  int h_bar = bankers((float)height / factor) * factor;
  int w_bar = bankers((float)width / factor) * factor;
  const int64_t area = (int64_t)h_bar * w_bar;
  if (area > max_pixels) {
    const double beta = sqrt((double)((int64_t)height * width) / max_pixels);
    h_bar = std::max(factor, (int)floor(height / beta / factor) * factor);
    w_bar = std::max(factor, (int)floor(width / beta / factor) * factor);
  } else if (area < min_pixels) {
    const double beta = sqrt((double)min_pixels / ((double)height * width));
    h_bar = (int)ceil(height * beta / factor) * factor;
    w_bar = (int)ceil(width * beta / factor) * factor;
  }
  *new_height = h_bar;
  *new_width = w_bar;
  return B200_OK;
}

extern "C" int64_t b200_preprocess_workspace_bytes(int channels, int height, int width, int new_height,
                                                   int new_width) {
  if (channels <= 0 || height <= 0 || width <= 0 || new_height <= 0 || new_width <= 0) return 0;
  return layout(channels, height, width, new_height, new_width).total;
}

extern "C" int b200_bicubic_resize_u8(const uint8_t* image, int channels, int height, int width, int out_h, int out_w,
                                      uint8_t* out, void* workspace, int64_t workspace_bytes, b200_stream_t stream) {
  if (!image || !out || channels <= 0 || height <= 0 || width <= 0 || out_h <= 0 || out_w <= 0)
    return B200_ERROR_INVALID_PARAM;
  if ((int64_t)channels * height * width > INT32_MAX || (int64_t)channels * out_h * out_w > INT32_MAX)
    return B200_ERROR_UNSUPPORTED;
  if (out_h == height && out_w == width)
    return cuda_rc(cudaMemcpyAsync(out, image, (size_t)channels * height * width, cudaMemcpyDeviceToDevice, stream));
  return run_resample(0, image, channels, height, width, out_h, out_w, out, make_float3(0, 0, 0),
                      make_float3(1, 1, 1), 1, 1, 1, workspace, workspace_bytes, stream);
}

extern "C" int b200_preprocess_image(const uint8_t* image, int channels, int height, int width, int patch_size,
                                     int temporal_patch_size, int merge_size, int min_pixels, int max_pixels,
                                     const float* mean, const float* stdv, int out_dtype, void* pixel_values,
                                     int64_t pixel_capacity, int64_t* num_patches, int64_t* grid_thw,
                                     void* workspace, int64_t workspace_bytes, b200_stream_t stream) {
  if (!image || !pixel_values || !num_patches || !grid_thw || channels <= 0 || channels > 3 || height <= 0 ||
      width <= 0 || patch_size <= 0 || temporal_patch_size <= 0 || merge_size <= 0 || (out_dtype != 0 && out_dtype != 1))
    return B200_ERROR_INVALID_PARAM;
  int nh = 0, nw = 0;
  int rc = b200_smart_resize(height, width, patch_size * merge_size, min_pixels, max_pixels, &nh, &nw);
  if (rc != B200_OK) return rc;
  if (nh <= 0 || nw <= 0) return B200_ERROR_INVALID_PARAM;
  const int64_t gh = nh / patch_size, gw = nw / patch_size;
  const int64_t n = gh * gw, pdim = (int64_t)channels * temporal_patch_size * patch_size * patch_size;
  *num_patches = n;
  grid_thw[0] = 1;
  grid_thw[1] = gh;
  grid_thw[2] = gw;
  if (pixel_capacity < n * pdim) return B200_ERROR_INVALID_PARAM;
  if ((int64_t)channels * height * width > INT32_MAX || n * pdim > ((int64_t)1 << 40)) return B200_ERROR_UNSUPPORTED;
  float m[3] = {0.5f, 0.5f, 0.5f}, s[3] = {0.5f, 0.5f, 0.5f};
  for (int c = 0; c < channels; ++c) {
    if (mean) m[c] = mean[c];
    if (stdv) s[c] = stdv[c];
  }
  return run_resample(out_dtype == 1 ? 1 : 2, image, channels, height, width, nh, nw, pixel_values,
                      make_float3(m[0], m[1], m[2]), make_float3(s[0], s[1], s[2]), patch_size, temporal_patch_size,
                      merge_size, workspace, workspace_bytes, stream);
}
