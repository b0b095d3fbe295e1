// Host-side 3-D (t, h, w) position ids of a text + image sequence (integer
// work, bit-exact).  Replaces GetRopeIndex
// (atb_cpp_llm/src/components/common/mrope.cpp:234-348) and, with an
// attention mask, get_rope_index of the Python engine
// (atb_python_qwen3vl_embedding/engine_utils.py:469-590).
//
// Per row: text runs take consecutive positions continuing from the previous
// run; an image (the image tokens that follow a vision-start token) takes its
// merged grid offsets (t, h / merge, w / merge) added to the running position,
// and the next run starts at that position + max(t, h / merge, w / merge).
// Images are consumed from grid_thw in order across rows.  Tokens outside the
// attention mask get position 1 on all three planes, and the remaining tokens
// are processed as one compacted sequence.
#include <algorithm>
#include <vector>

#include "engine/core.h"

namespace b200llm {

Status GetRopeIndex(const int64_t* ids, int64_t B, int64_t S, const int64_t* mask, const int64_t* grid_thw,
                    int64_t num_images, int64_t image_token, int64_t vision_start_token, int64_t merge,
                    int64_t* out) {
  if (!ids || !out || B <= 0 || S <= 0 || merge <= 0 || num_images < 0 || (num_images > 0 && !grid_thw))
    return ERROR_INVALID_PARAM;
  for (int64_t i = 0; i < num_images; ++i)
    if (grid_thw[3 * i] <= 0 || grid_thw[3 * i + 1] <= 0 || grid_thw[3 * i + 2] <= 0) return ERROR_INVALID_PARAM;
  const int64_t plane = B * S;
  int64_t next_image = 0;
  std::vector<int64_t> toks, where;
  for (int64_t b = 0; b < B; ++b) {
    const int64_t* row = ids + b * S;
    toks.clear();
    where.clear();
    for (int64_t s = 0; s < S; ++s) {
      if (mask && mask[b * S + s] == 0) {
        for (int p = 0; p < 3; ++p) out[p * plane + b * S + s] = 1;
        continue;
      }
      toks.push_back(row[s]);
      where.push_back(s);
    }
    const int64_t n = (int64_t)toks.size();
    auto put = [&](int64_t i, int64_t t, int64_t h, int64_t w) {
      const int64_t s = b * S + where[i];
      out[s] = t;
      out[plane + s] = h;
      out[2 * plane + s] = w;
    };
    // images announced in this row: a vision-start token directly followed by an image token
    int64_t images = 0;
    if (num_images > 0)
      for (int64_t i = 0; i + 1 < n; ++i)
        if (toks[i] == vision_start_token && toks[i + 1] == image_token) ++images;
    images = std::min(images, num_images - next_image);
    int64_t st = 0, pos = 0;
    for (int64_t k = 0; k < images; ++k) {
      int64_t ed = st;
      while (ed < n && toks[ed] != image_token) ++ed;
      if (ed >= n) break;
      for (int64_t i = st; i < ed; ++i) put(i, pos + i - st, pos + i - st, pos + i - st);
      pos += ed - st;
      const int64_t* g = grid_thw + 3 * next_image++;
      const int64_t gt = g[0], gh = g[1] / merge, gw = g[2] / merge;
      int64_t i = ed;
      for (int64_t a = 0; a < gt; ++a)
        for (int64_t y = 0; y < gh; ++y)
          for (int64_t x = 0; x < gw; ++x, ++i)
            if (i < n) put(i, pos + a, pos + y, pos + x);
      st = ed + gt * gh * gw;
      pos += std::max(gt, std::max(gh, gw));
    }
    for (int64_t i = st; i < n; ++i) put(i, pos + i - st, pos + i - st, pos + i - st);
  }
  return STATUS_OK;
}

}  // namespace b200llm

extern "C" int b200_get_rope_index(const int64_t* input_ids, int64_t batch, int64_t seq_len,
                                   const int64_t* attention_mask, const int64_t* image_grid_thw, int64_t num_images,
                                   int64_t image_token_id, int64_t vision_start_token_id, int64_t spatial_merge_size,
                                   int64_t* position_ids) {
  return b200llm::GetRopeIndex(input_ids, batch, seq_len, attention_mask, image_grid_thw, num_images, image_token_id,
                               vision_start_token_id, spatial_merge_size, position_ids);
}
