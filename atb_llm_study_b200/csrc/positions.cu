// 3-D (t, h, w) position ids of text + image sequences computed on the GPU,
// bit-exact with the host GetRopeIndex (same rules; see engine/positions.cpp,
// which restates atb_cpp_llm/src/components/common/mrope.cpp:234-348).
//
// One CTA walks the rows in order (images are consumed from grid_thw across
// rows).  Per row, block-wide scans turn the attention mask into compacted
// token indices and find, for every compacted position, the next image token;
// one thread then lays out the row's segments (text run, image block, ...),
// a handful per prompt, and all threads fill the three position planes in
// parallel from those segment descriptors.  Integer work on a few thousand
// tokens: the kernel replaces a host round trip (ids and mask stay on the
// device), not a bandwidth problem.
#include <algorithm>

#include "common.cuh"

using namespace b200;

namespace {

constexpr int kThreads = 1024;
constexpr int kMaxSegments = 256;  // images per row handled (two segments each, plus the tail)

struct Segment {
  int start;     // first compacted index
  int end;       // one past the last compacted index
  int64_t pos;   // running position at the segment start
  int image;     // grid_thw index, or -1 for a text run
};

// Block-wide exclusive prefix sum of one int per thread (kThreads threads); returns the total.
__device__ int block_scan(int v, int* warp_sums, int* out_excl) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) warp_sums[w] = inc;
  __syncthreads();
  if (w == 0) {
    int s = lane < kThreads / 32 ? warp_sums[lane] : 0;
    int si = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, si, o);
      if (lane >= o) si += y;
    }
    if (lane < kThreads / 32) warp_sums[lane] = si - s;  // exclusive warp offsets
    if (lane == 31) warp_sums[kThreads / 32] = si;      // total
  }
  __syncthreads();
  *out_excl = warp_sums[w] + inc - v;
  const int total = warp_sums[kThreads / 32];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kThreads) rope_index_kernel(const int64_t* __restrict__ ids, int B, int S,
                                                               const int64_t* __restrict__ mask,
                                                               const int64_t* __restrict__ grid, int num_images,
                                                               int64_t image_token, int64_t vision_start, int merge,
                                                               int64_t* __restrict__ out, int* __restrict__ where,
                                                               int* __restrict__ next_img, unsigned* err) {
  pdl_trigger();
  pdl_wait();
  __shared__ int warp_sums[kThreads / 32 + 1];
  __shared__ Segment seg[2 * kMaxSegments + 1];
  __shared__ int nseg_s, next_image_s;
  const int64_t plane = (int64_t)B * S;
  if (threadIdx.x == 0) next_image_s = 0;
  __syncthreads();
  for (int b = 0; b < B; ++b) {
    const int64_t* row = ids + (int64_t)b * S;
    // 1. compaction: where[i] = i-th unmasked position; masked positions get 1
    int n = 0;
    for (int s0 = 0; s0 < S; s0 += kThreads) {
      const int s = s0 + threadIdx.x;
      const bool keep = s < S && (!mask || mask[(int64_t)b * S + s] != 0);
      if (s < S && !keep)
        for (int p = 0; p < 3; ++p) out[p * plane + (int64_t)b * S + s] = 1;
      int excl;
      const int tot = block_scan(keep ? 1 : 0, warp_sums, &excl);
      if (keep) where[n + excl] = s;
      n += tot;
    }
    __syncthreads();
    // 2. next image token at or after each compacted index (suffix scan, chunked from the end)
    int carry = n;  // "none" = n
    for (int e0 = ((n - 1) / kThreads) * kThreads; e0 >= 0 && n > 0; e0 -= kThreads) {
      const int i = e0 + threadIdx.x;
      int v = (i < n && row[where[i]] == image_token) ? i : n;
      // reverse inclusive min-scan within the chunk: warp level then across warps
      const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_down_sync(0xffffffffu, v, o);
        if (lane + o < 32) v = min(v, y);
      }
      if (lane == 0) warp_sums[w] = v;
      __syncthreads();
      int later = carry;
      for (int w2 = w + 1; w2 < kThreads / 32; ++w2) later = min(later, warp_sums[w2]);
      v = min(v, later);
      if (i < n) next_img[i] = v;
      __syncthreads();
      if (threadIdx.x == 0) warp_sums[0] = v;  // thread 0 holds the chunk's minimum
      __syncthreads();
      carry = warp_sums[0];
      __syncthreads();
    }
    // 3. images announced in this row, then the row's segments (one thread)
    int ann = 0;
    for (int i = threadIdx.x; i + 1 < n; i += kThreads)
      if (row[where[i]] == vision_start && row[where[i + 1]] == image_token) ++ann;
    int excl;
    ann = block_scan(ann, warp_sums, &excl);
    if (threadIdx.x == 0) {
      int images = min(ann, num_images - next_image_s);
      if (num_images == 0) images = 0;
      int st = 0, ns = 0;
      int64_t pos = 0;
      for (int k = 0; k < images; ++k) {
        if (ns + 2 >= 2 * kMaxSegments) {  // more images in one row than segments kept
          raise_error(err, DEV_ERR_BAD_INDEX);
          break;
        }
        const int ed = st < n ? next_img[st] : n;
        if (ed >= n) break;
        seg[ns++] = Segment{st, ed, pos, -1};
        pos += ed - st;
        const int gi = next_image_s++;
        const int64_t gt = grid[3 * gi], gh = grid[3 * gi + 1] / merge, gw = grid[3 * gi + 2] / merge;
        if (gt <= 0 || gh <= 0 || gw <= 0) {  // the host API rejects such grids before any work
          raise_error(err, DEV_ERR_BAD_INDEX);
          break;
        }
        const int64_t len = gt * gh * gw;
        seg[ns++] = Segment{ed, (int)min((int64_t)n, ed + len), pos, gi};
        st = (int)min((int64_t)n, ed + len);
        pos += max(gt, max(gh, gw));
      }
      seg[ns++] = Segment{st, n, pos, -1};
      nseg_s = ns;
    }
    __syncthreads();
    // 4. fill the planes
    const int ns = nseg_s;
    for (int i = threadIdx.x; i < n; i += kThreads) {
      int lo = 0, hi = ns;  // last segment with start <= i
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (seg[mid].start <= i) lo = mid;
        else hi = mid;
      }
      const Segment g = seg[lo];
      int64_t t, h, w;
      if (g.image < 0 || i >= g.end) {
        t = h = w = g.pos + (i - g.start);
      } else {
        const int64_t gh = grid[3 * g.image + 1] / merge, gw = grid[3 * g.image + 2] / merge;
        const int64_t r = i - g.start;
        t = g.pos + r / (gh * gw);
        h = g.pos + (r / gw) % gh;
        w = g.pos + r % gw;
      }
      const int64_t s = (int64_t)b * S + where[i];
      out[s] = t;
      out[plane + s] = h;
      out[2 * plane + s] = w;
    }
    __syncthreads();
  }
}

}  // namespace

extern "C" int64_t b200_rope_index_workspace_bytes(int64_t seq_len) {
  return seq_len > 0 ? 2 * seq_len * (int64_t)sizeof(int) : 0;
}

extern "C" int b200_get_rope_index_device(const int64_t* input_ids, int64_t batch, int64_t seq_len,
                                          const int64_t* attention_mask, const int64_t* image_grid_thw,
                                          int64_t num_images, int64_t image_token_id, int64_t vision_start_token_id,
                                          int64_t spatial_merge_size, int64_t* position_ids, void* workspace,
                                          int64_t workspace_bytes, b200_stream_t stream) {
  if (!input_ids || !position_ids || batch <= 0 || seq_len <= 0 || spatial_merge_size <= 0 || num_images < 0 ||
      (num_images > 0 && !image_grid_thw) || !workspace || workspace_bytes < 2 * seq_len * (int64_t)sizeof(int))
    return B200_ERROR_INVALID_PARAM;
  if (batch > INT32_MAX || seq_len > INT32_MAX / 2 || num_images > INT32_MAX || spatial_merge_size > INT32_MAX)
    return B200_ERROR_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(workspace) & 3) return B200_ERROR_INVALID_PARAM;
  int* where = static_cast<int*>(workspace);
  int* next_img = where + seq_len;
  int dev = 0;
  cudaGetDevice(&dev);
  launch_kernel(rope_index_kernel, dim3(1), kThreads, 0, stream, input_ids, (int)batch, (int)seq_len, attention_mask,
                image_grid_thw, (int)num_images, image_token_id, vision_start_token_id, (int)spatial_merge_size,
                position_ids, where, next_img, b200::error_word(dev));
  B200_CHECK_LAUNCH();
  return B200_OK;
}
