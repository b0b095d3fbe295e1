// extern "C" wrappers around the reference's own CPU position functions,
// compiled from the reference sources in place (oracle/Makefile) into
// oracle/_ref/libref.so.  TEST INFRASTRUCTURE ONLY: the tests use them to pin
// the numpy oracle where the reference's golden files need a checkpoint.
#include <cstdint>
#include <vector>

#include "components/common/mrope.h"
#include "components/vision/pos_embed_interp.h"

using namespace atb_llm::components;

extern "C" {

// ComputePosEmbedInterp (atb_cpp_llm/src/components/vision/pos_embed_interp.cpp:10-90)
void ref_pos_embed_interp(const uint16_t* src_fp16, int32_t hidden, int32_t num_grid, int32_t merge,
                          const int64_t* grid_thw, int64_t num_images, uint16_t* out_fp16) {
  ComputePosEmbedInterp(src_fp16, hidden, num_grid, merge, grid_thw, num_images, out_fp16);
}

// GetRopeIndex (atb_cpp_llm/src/components/common/mrope.cpp:234-348)
void ref_get_rope_index(const int64_t* input_ids, int64_t batch, int64_t seq_len, const int64_t* image_grid_thw,
                        int64_t num_images, int64_t image_token_id, int64_t vision_start_token_id, int64_t merge,
                        int64_t* position_ids_out) {
  GetRopeIndex(input_ids, batch, seq_len, image_grid_thw, num_images, image_token_id, vision_start_token_id, merge,
               position_ids_out);
}

// MRoPE::Compute (atb_cpp_llm/src/components/common/mrope.cpp:16-96)
void ref_mrope_compute(const int64_t* position_ids, int64_t batch, int64_t seq_len, int32_t head_dim, float theta,
                       int32_t s0, int32_t s1, int32_t s2, float* cos_out, float* sin_out) {
  MRoPE m(head_dim, theta, std::vector<int32_t>{s0, s1, s2});
  m.Compute(position_ids, batch, seq_len, cos_out, sin_out);
}

// VisionRotaryEmbedding::ComputeRoPE (atb_cpp_llm/src/components/common/mrope.cpp:155-228)
int64_t ref_vision_rope(const int64_t* grid_thw, int64_t num_images, int32_t dim, int32_t merge, float* cos_out,
                        float* sin_out) {
  VisionRotaryEmbedding v(dim);
  return v.ComputeRoPE(grid_thw, num_images, merge, cos_out, sin_out);
}
}
