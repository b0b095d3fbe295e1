// Qwen3-VL vision tower runner: patch embedding + interpolated position
// embedding, `depth` pre-LN ViT blocks with 2-D rope, deepstack mergers tapped
// after the configured blocks, and the final patch merger.
//
// Replaces the reference's VisionRunner graphs (atb_cpp_llm/src/runners/
// vision_runner.cpp:57-113: first layer = patch embed + pos embed + block 0,
// block graph, merger graph), DeepstackFusion::ExtractFeatures
// (atb_cpp_llm/src/components/common/deepstack_fusion.cpp:55-105) and the
// vision stage of Qwen3VLModel::ForwardWithTiming
// (atb_cpp_llm/src/adapters/qwen3vl_embedding/qwen3vl_model.cpp:384-575).
//
// Token order is the merge-block order produced by the image processor
// (merge x merge patch groups consecutive), so every merger reads its input
// as [N / merge^2, hidden * merge^2] without a permutation.  Attention is
// bidirectional within each temporal frame of each image.
#pragma once

#include <map>
#include <string>
#include <vector>

#include "engine/core.h"
#include "engine/json_config.h"

namespace b200llm {

// "vision_config" of a Qwen3-VL config.json (Qwen3VLConfig vision fields,
// atb_cpp_llm/src/adapters/qwen3vl_embedding/qwen3vl_config.cpp:41-55).
struct VisionConfig {
  int depth = 24, hidden = 1024, heads = 16, intermediate = 4096;
  int in_channels = 3, temporal_patch = 2, patch = 16, merge = 2;
  int out_hidden = 2048, num_position_embeddings = 2304;
  std::vector<int> deepstack;  // block indexes whose outputs feed the deepstack mergers
  float eps = 1e-6f, rope_theta = 10000.f;

  static Status FromJson(const JsonConfig& root, VisionConfig& out);
  int head_dim() const { return hidden / heads; }
  int patch_dim() const { return in_channels * temporal_patch * patch * patch; }
  int merged_dim() const { return hidden * merge * merge; }
  int grid() const;  // side of the square position table
};

class VisionModel {
 public:
  VisionModel() = default;
  ~VisionModel();
  VisionModel(const VisionModel&) = delete;
  VisionModel& operator=(const VisionModel&) = delete;

  // Weights are allocated from `alloc` (shared with the text decoder); all work
  // runs on `ctx`'s stream.
  Status Init(const VisionConfig& cfg, ContextManager* ctx, TensorAllocator* alloc);
  Status InitRandomWeights(uint64_t seed, float std);
  // "model.visual.*" weights by HF name; ERROR_WEIGHT_LOAD for any other name.
  Status SetWeight(const std::string& name, const std::vector<uint16_t>& bf16, int64_t numel);

  // pixels [num_patches, patch_dim] in processor order (bf16 on the device, or
  // bf16/fp16/fp32 on the host); grid_thw [num_images, 3] on the host.  Leaves
  // merged() [N / merge^2, out_hidden] and deepstack(i) of the same shape on
  // the device (valid until the next call).
  Status Forward(const void* pixels, DType dtype, bool on_device, int64_t num_patches, const int64_t* grid_thw,
                 int num_images);

  const VisionConfig& config() const { return cfg_; }
  int64_t MergedTokens() const { return merged_tokens_; }
  const void* Merged() const { return merged_.data; }
  const void* Deepstack(int i) const;
  int NumDeepstack() const { return (int)cfg_.deepstack.size(); }
  size_t WeightBytes() const { return weight_bytes_; }
  int LastLaunches() const { return launches_; }

 private:
  Status Reserve(int64_t patches, int64_t frames);
  Status RunTower(int64_t N, const int64_t* grid_thw, int num_images, int frames, int max_len);
  void DropGraphs();
  Status Gemm(const void* A, int64_t lda, const void* W, void* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int epi,
              const void* bias, const void* R, int64_t ldr);
  // h_ += A W^T + bias (K may split).  When it splits, the reduce and the
  // LayerNorm (gamma, beta) of h_ into normed_ run as one kernel and *normed
  // is set; otherwise the caller normalises.
  Status GemmResidualNorm(const void* A, int64_t lda, const void* W, int64_t M, int64_t K, const void* bias,
                          const void* gamma, const void* beta, bool* normed);
  Status Merger(const void* x, int64_t N, int which, void* out);
  int DeepstackSlot(int block) const;

  VisionConfig cfg_;
  ContextManager* ctx_ = nullptr;
  TensorAllocator* alloc_ = nullptr;
  size_t weight_bytes_ = 0;
  int launches_ = 0;
  int64_t cap_patches_ = 0, cap_frames_ = 0, merged_tokens_ = 0;

  // weights: patch embed, position table, blocks stacked over depth, mergers
  // (index 0 = main merger, 1 + i = deepstack merger i)
  DeviceTensor patch_w_, patch_b_, pos_table_;
  DeviceTensor n1_w_, n1_b_, qkv_w_, qkv_b_, proj_w_, proj_b_, n2_w_, n2_b_, fc1_w_, fc1_b_, fc2_w_, fc2_b_;
  struct MergerWeights {
    DeviceTensor norm_w, norm_b, fc1_w, fc1_b, fc2_w, fc2_b;
    bool postshuffle = false;  // LayerNorm over the grouped width (deepstack) or per token (main)
  };
  std::vector<MergerWeights> mergers_;

  // activations, grown on demand
  DeviceTensor pix_, h_, normed_, qkv_, attn_, act_, cos_, sin_, cu_, merged_, ds_, ws_;
  int64_t ws_bytes_ = 0;

  // tower passes captured per grid list (flattened grid_thw) on its second call
  struct Captured {
    cudaGraphExec_t exec;
    int launches;
  };
  std::map<std::vector<int64_t>, Captured> graphs_;
  std::map<std::vector<int64_t>, int> calls_;
};

}  // namespace b200llm
