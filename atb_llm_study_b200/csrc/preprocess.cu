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
// Work per image: one horizontal-pass kernel (one thread per output sample,
// uint8 intermediate [C, H, out_w]) and one vertical-pass kernel that also
// normalises and scatters each value to its patch positions (frame 0 and the
// duplicated frames).  An axis whose size does not change is not resampled
// (the horizontal pass is skipped; the vertical pass runs with one unit tap,
// which reproduces the input byte exactly).  HBM-bound byte work: no tensor
// cores; grids are sized in whole waves of 256-thread blocks.
#include <cuda_fp16.h>
#include <math.h>

#include <algorithm>
#include <vector>

#include "common.cuh"

using namespace b200;

namespace {

constexpr int kPrecisionBits = 22;
constexpr int kThreads = 256;

__device__ __forceinline__ uint8_t clip8(int v) {
  const int s = v >> kPrecisionBits;  // arithmetic shift
  return (uint8_t)(s < 0 ? 0 : (s > 255 ? 255 : s));
}

// out[c][y][xx] = clip8(2^21 + sum_x in[c][y][xmin + x] * k[xx][x])
__global__ void __launch_bounds__(kThreads) resample_h_kernel(const uint8_t* __restrict__ in, int C, int H, int W,
                                                               int out_w, int ksize, const int* __restrict__ bounds,
                                                               const int* __restrict__ coef, uint8_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int64_t n = (int64_t)C * H * out_w;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int xx = (int)(i % out_w);
    const int64_t row = i / out_w;  // c * H + y
    const int x0 = bounds[2 * xx], taps = bounds[2 * xx + 1];
    const uint8_t* src = in + row * W + x0;
    const int* k = coef + (int64_t)xx * ksize;
    int ss = 1 << (kPrecisionBits - 1);
    for (int x = 0; x < taps; ++x) ss += (int)src[x] * k[x];
    out[i] = clip8(ss);
  }
}

// Vertical pass over in [C, H, out_w] to rows of out_h; MODE 0 writes the
// uint8 image [C, out_h, out_w]; MODE 1 / 2 write (v/255 - mean)/std as fp16 /
// bf16 into the patch layout (merge-block order, frame duplicated over tp).
template <int MODE>
__global__ void __launch_bounds__(kThreads) resample_v_kernel(const uint8_t* __restrict__ in, int C, int H, int out_h,
                                                               int out_w, int ksize, const int* __restrict__ bounds,
                                                               const int* __restrict__ coef, void* __restrict__ out,
                                                               float3 mean, float3 stdv, int ps, int tp, int ms) {
  pdl_trigger();
  pdl_wait();
  const int64_t n = (int64_t)C * out_h * out_w;
  const int gw = out_w / ps;
  const int64_t pdim = (int64_t)C * tp * ps * ps;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int xx = (int)(i % out_w);
    const int64_t r = i / out_w;
    const int yy = (int)(r % out_h);
    const int c = (int)(r / out_h);
    const int y0 = bounds[2 * yy], taps = bounds[2 * yy + 1];
    const uint8_t* src = in + ((int64_t)c * H + y0) * out_w + xx;
    const int* k = coef + (int64_t)yy * ksize;
    int ss = 1 << (kPrecisionBits - 1);
    for (int y = 0; y < taps; ++y) ss += (int)src[(int64_t)y * out_w] * k[y];
    const uint8_t u = clip8(ss);
    if (MODE == 0) {
      static_cast<uint8_t*>(out)[i] = u;
    } else {
      // the reference's order of operations: (u / 255 - mean) / std, float32
      const float m = c == 0 ? mean.x : (c == 1 ? mean.y : mean.z);
      const float s = c == 0 ? stdv.x : (c == 1 ? stdv.y : stdv.z);
      const float v = ((float)u / 255.0f - m) / s;
      // patch (gy, gx) in merge-block order, element (c, f, py, px)
      const int gy = yy / ps, py = yy % ps, gx = xx / ps, px = xx % ps;
      const int64_t patch = (((int64_t)(gy / ms) * (gw / ms) + gx / ms) * ms + gy % ms) * ms + gx % ms;
      const int64_t base = patch * pdim + (int64_t)c * tp * ps * ps + (int64_t)py * ps + px;
      for (int f = 0; f < tp; ++f) {
        if (MODE == 1) static_cast<__half*>(out)[base + (int64_t)f * ps * ps] = __float2half_rn(v);
        else static_cast<__nv_bfloat16*>(out)[base + (int64_t)f * ps * ps] = __float2bfloat16_rn(v);
      }
    }
  }
}

// ---- host: Pillow's coefficient computation for one axis ----
double bicubic(double x) {
  const double a = -0.5;
  x = fabs(x);
  if (x < 1.0) return ((a + 2.0) * x - (a + 3.0)) * x * x + 1.0;
  if (x < 2.0) return (((x - 5.0) * x + 8.0) * x - 4.0) * a;
  return 0.0;
}

int ksize_of(int in_size, int out_size) {
  const double scale = (double)in_size / out_size;
  const double support = 2.0 * (scale < 1.0 ? 1.0 : scale);
  return (int)ceil(support) * 2 + 1;
}

// bounds[2*o] = first tap, bounds[2*o+1] = taps; coef[o*ksize + t] in 22-bit fixed point
int axis_coeffs(int in_size, int out_size, std::vector<int>& bounds, std::vector<int>& coef) {
  const double scale = (double)in_size / out_size;
  const double filterscale = scale < 1.0 ? 1.0 : scale;
  const double support = 2.0 * filterscale;
  const int ksize = (int)ceil(support) * 2 + 1;
  bounds.assign((size_t)out_size * 2, 0);
  coef.assign((size_t)out_size * ksize, 0);
  std::vector<double> w(ksize);
  for (int o = 0; o < out_size; ++o) {
    const double center = (o + 0.5) * scale;
    const double rss = 1.0 / filterscale;
    int xmin = (int)(center - support + 0.5);  // C cast: truncation toward zero
    if (xmin < 0) xmin = 0;
    int xmax = (int)(center + support + 0.5);
    if (xmax > in_size) xmax = in_size;
    xmax -= xmin;
    double ww = 0.0;
    for (int x = 0; x < xmax; ++x) {
      w[x] = bicubic((x + xmin - center + 0.5) * rss);
      ww += w[x];
    }
    for (int x = 0; x < xmax; ++x) {
      const double v = ww != 0.0 ? w[x] / ww : w[x];
      coef[(size_t)o * ksize + x] = v < 0 ? (int)(-0.5 + v * (1 << kPrecisionBits))
                                          : (int)(0.5 + v * (1 << kPrecisionBits));
    }
    bounds[(size_t)o * 2] = xmin;
    bounds[(size_t)o * 2 + 1] = xmax;
  }
  return ksize;
}

// one unit tap per output row: the vertical pass then reproduces its input
int identity_coeffs(int n, std::vector<int>& bounds, std::vector<int>& coef) {
  bounds.resize((size_t)n * 2);
  coef.assign((size_t)n, 1 << kPrecisionBits);
  for (int i = 0; i < n; ++i) {
    bounds[(size_t)i * 2] = i;
    bounds[(size_t)i * 2 + 1] = 1;
  }
  return 1;
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

unsigned grid_for(int64_t n) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = (n + kThreads - 1) / kThreads;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sms * 8));
}

int cuda_rc(cudaError_t e) { return e == cudaSuccess ? B200_OK : B200_ERROR_CUDA_BASE - (int)e; }

// Resample image [C,H,W] (device) to (oh, ow); MODE as resample_v_kernel.
int run_resample(int mode, const uint8_t* image, int C, int H, int W, int oh, int ow, void* out, float3 mean,
                 float3 stdv, int ps, int tp, int ms, void* ws, int64_t ws_bytes, cudaStream_t st) {
  const Layout L = layout(C, H, W, oh, ow);
  if (!ws || ws_bytes < L.total || (reinterpret_cast<uintptr_t>(ws) & 255)) return B200_ERROR_INVALID_PARAM;
  uint8_t* w8 = static_cast<uint8_t*>(ws);
  std::vector<int> bh, ch, bv, cv;
  const bool need_h = ow != W, need_v = oh != H;
  int ksv = need_v ? axis_coeffs(H, oh, bv, cv) : identity_coeffs(oh, bv, cv);
  if (need_h) {
    axis_coeffs(W, ow, bh, ch);
    int rc = cuda_rc(cudaMemcpyAsync(w8 + L.off_bh, bh.data(), bh.size() * 4, cudaMemcpyHostToDevice, st));
    if (rc == B200_OK)
      rc = cuda_rc(cudaMemcpyAsync(w8 + L.off_ch, ch.data(), ch.size() * 4, cudaMemcpyHostToDevice, st));
    if (rc != B200_OK) return rc;
  }
  int rc = cuda_rc(cudaMemcpyAsync(w8 + L.off_bv, bv.data(), bv.size() * 4, cudaMemcpyHostToDevice, st));
  if (rc == B200_OK) rc = cuda_rc(cudaMemcpyAsync(w8 + L.off_cv, cv.data(), cv.size() * 4, cudaMemcpyHostToDevice, st));
  if (rc != B200_OK) return rc;
  const uint8_t* vin = image;
  if (need_h) {
    const int64_t n = (int64_t)C * H * ow;
    launch_kernel(resample_h_kernel, dim3(grid_for(n)), kThreads, 0, st, image, C, H, W, ow, L.ksh,
                  reinterpret_cast<const int*>(w8 + L.off_bh), reinterpret_cast<const int*>(w8 + L.off_ch),
                  w8 + L.off_tmp);
    B200_CHECK_LAUNCH();
    vin = w8 + L.off_tmp;
  }
  const int64_t n = (int64_t)C * oh * ow;
  const dim3 g(grid_for(n));
  const int* vb = reinterpret_cast<const int*>(w8 + L.off_bv);
  const int* vc = reinterpret_cast<const int*>(w8 + L.off_cv);
  if (mode == 0)
    launch_kernel(resample_v_kernel<0>, g, kThreads, 0, st, vin, C, H, oh, ow, ksv, vb, vc, out, mean, stdv, ps, tp,
                  ms);
  else if (mode == 1)
    launch_kernel(resample_v_kernel<1>, g, kThreads, 0, st, vin, C, H, oh, ow, ksv, vb, vc, out, mean, stdv, ps, tp,
                  ms);
  else
    launch_kernel(resample_v_kernel<2>, g, kThreads, 0, st, vin, C, H, oh, ow, ksv, vb, vc, out, mean, stdv, ps, tp,
                  ms);
  B200_CHECK_LAUNCH();
  // the host coefficient vectors were copied from pageable memory: the copies
  // have completed when cudaMemcpyAsync returned, so they may be freed now
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
