// Decoder model runner: GQA or multi-head latent attention, dense or
// mixture-of-experts MLPs (Qwen3, the Qwen3-VL text decoder, Qwen3-MoE,
// Mixtral, DeepSeek-V2), on one GPU or tensor-parallel over a b200_comm_t.
//
// Replaces the reference's per-model layer graph + runner + layer loop
// (TextDecoderLayerGraph::Build, atb_cpp_llm/src/components/text/
// decoder_layer_graph.cpp:13-154; TextRunner, atb_cpp_llm/src/runners/
// text_runner.cpp:12-61; Qwen3VLModel::ForwardWithTiming text stage,
// atb_cpp_llm/src/adapters/qwen3vl_embedding/qwen3vl_model.cpp:685-768) and
// adds what the reference only stubs: a paged KV cache and single-token decode.
//
// All activations live in buffers sized once at Init (no per-layer
// allocation); the decode step is captured in a CUDA graph per batch size.
#pragma once

#include <algorithm>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "engine/core.h"
#include "engine/json_config.h"
#include "engine/safetensors.h"

namespace b200llm {

struct ModelConfig {
  std::string model_type;
  int hidden = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0, intermediate = 0;
  int64_t vocab = 0;
  float eps = 1e-6f, rope_theta = 1e6f;
  bool qk_norm = true, tie_embeddings = false;
  bool mrope = false;
  int mrope_section[3] = {0, 0, 0};
  // Mixture of experts (Mixtral "mixtral", Qwen3-MoE "qwen3_moe"): layers
  // l >= first_dense route each token to top_k of `experts` SwiGLU experts of
  // width moe_intermediate (+ an always-on shared expert of width
  // shared_intermediate); experts == 0 is a dense model.
  int experts = 0, top_k = 0, moe_intermediate = 0, shared_intermediate = 0, first_dense = 0;
  bool norm_topk = true;     // renormalise the chosen weights (else times routed_scale)
  float routed_scale = 1.0f;
  // Multi-head latent attention (DeepSeek-V2 "deepseek_v2"): kv_lora > 0
  // replaces GQA; rope over qk_rope dims with YaRN-scaled frequencies.
  int kv_lora = 0, qk_nope = 0, qk_rope = 0, v_head = 0;
  float yarn_factor = 1.f, yarn_orig_max = 4096.f, yarn_beta_fast = 32.f, yarn_beta_slow = 1.f;
  float yarn_mscale = 1.f, yarn_mscale_all = 1.f;
  float attn_scale = 0.f;  // softmax scale of the MLA heads
  bool mla() const { return kv_lora > 0; }

  // Reads a HF config.json (Qwen3 "qwen3", the "text_config" of "qwen3_vl",
  // Mixtral "mixtral", Qwen3-MoE "qwen3_moe").
  static Status FromJson(const JsonConfig& cfg, ModelConfig& out);
  int qkv_dim() const { return (heads + 2 * kv_heads) * head_dim; }
  bool moe_layer(int l) const { return experts > 0 && l >= first_dense; }
  int dense_layers() const { return experts > 0 ? std::min(first_dense, layers) : layers; }
};

// Weight placement (engine/weight_plan.h): where each Hugging Face weight goes
// in one rank's device tensors.
// The device tensors of a decoder model (DecoderModel's members of the same names).
enum class WTensor : int {
  EMBED, LM_HEAD, FINAL_NORM, WQ, KVNORM, WKVB, WO, WQKV, QNORM, KNORM, ILN, PLN, WGU, WDOWN, ROUTER, EGU, EDOWN,
  SGU, SDOWN
};

// rows x width elements: source row r at src_off + r * src_pitch goes to
// dst_off + r * dst_pitch of tensor `dst` (all in bf16 elements).
struct WeightCopy {
  WTensor dst;
  int64_t dst_off, dst_pitch, src_off, src_pitch, width, rows;
};

// One rank's view of a model: the whole config, the local (sharded) config,
// the group sizes and ranks, and which layers are dense / mixture-of-experts.
struct ShardView {
  ModelConfig whole, local;
  int tp = 1, tp_rank = 0, ep = 1, ep_rank = 0;
  std::vector<int> dense_idx, moe_idx;  // per layer: index into the dense / MoE stacks (-1 = other kind)
};

struct EngineOptions {
  int device = 0;
  int max_batch = 64;          // KV-cache sequence slots
  int max_context = 4096;      // tokens per slot
  int max_prefill_tokens = 16384;
  int block_size = 128;
  uint64_t seed = 0;
  float init_std = 0.02f;
  b200_comm_t comm = nullptr;  // tensor- or expert-parallel group (null: one GPU)
  bool expert_parallel = false;  // comm splits the routed experts (attention data-parallel) instead of every matrix
};

class DecoderModel {
 public:
  DecoderModel() = default;
  ~DecoderModel();

  Status Init(const ModelConfig& cfg, const EngineOptions& opt);
  Status InitRandomWeights(uint64_t seed, float std);
  Status LoadSafetensors(const SafetensorsReader& r, const std::string& prefix);
  // Set one weight from host memory by its HF name (dtype: BF16/FP16/FP32).
  Status SetWeight(const std::string& name, const void* host, DType dtype, int64_t numel);

  // Prefill fresh sequences.  ids: T = sum(seq_lens) token ids (host or
  // device); slots: the KV slot of each sequence; position_ids: optional
  // [3, T] host array (mrope) — default 0..len-1 per sequence.  Writes each
  // sequence's greedy next token to next_tokens (host or device) and, if
  // logits is not null, the last-token logits [num_seqs, vocab] (device, bf16).
  Status Prefill(const int64_t* ids, bool ids_on_device, const int32_t* seq_lens, const int32_t* slots, int num_seqs,
                 const int64_t* position_ids, int64_t* next_tokens, bool next_on_device, void* logits);
  // One decode step for `batch` sequences (one token each).
  Status Decode(const int64_t* ids, bool ids_on_device, const int32_t* slots, int batch, int64_t* next_tokens,
                bool next_on_device, void* logits);

  // Encoder forward of one sequence for a pooled embedding (the text stage of
  // the Qwen3-VL embedding model): causal attention, no KV cache.  Rows
  // vis_rows (host, n_vis) of the input embeddings are replaced by vis_embeds
  // (device bf16 [n_vis, hidden]); deepstack[i] (device bf16 [n_vis, hidden])
  // is added to the same rows after layer i.  position_ids: [3, S] host (null:
  // 0..S-1).  Writes the final-normed row pool_row (L2-normalised when
  // `normalize`) to out (host fp32 [hidden]); hidden_out (device bf16 [S,
  // hidden], optional) receives every final-normed row.
  Status Encode(const int64_t* ids, int64_t S, const int64_t* position_ids, const int32_t* vis_rows, int64_t n_vis,
                const void* vis_embeds, const void* const* deepstack, int n_ds, int64_t pool_row, bool normalize,
                float* out, void* hidden_out);
  int EncodeLaunches() const { return last_encode_launches_; }

  cudaStream_t stream() const { return ctx_ ? ctx_->GetStream() : nullptr; }
  ContextManager* context() const { return ctx_.get(); }
  TensorAllocator* allocator() const { return alloc_.get(); }
  const ModelConfig& config() const { return cfg_; }
  size_t WeightBytes() const { return weight_bytes_; }
  size_t KvBytes() const { return kv_bytes_; }
  int64_t ContextLen(int slot) const { return slot >= 0 && slot < (int)host_ctx_.size() ? host_ctx_[slot] : -1; }
  // Layer l's cache: GQA k / v [num_blocks, kv_heads, block_size, head_dim]
  // (v null for a latent cache [num_blocks * block_size, kv_lora + qk_rope]);
  // slot s owns blocks [s * max_blocks, (s + 1) * max_blocks) in order.
  Status KvCache(int l, void** k, void** v, int64_t* num_blocks, int* block_size, int* max_blocks) const;
  // GPU kernel launches per Decode / Prefill call (for reporting).
  int DecodeLaunches() const;
  int PrefillLaunches() const;
  Status ResetSlots();

 private:
  Status RunLayers(int64_t T, bool decode, int batch);
  Status Head(int64_t rows, bool gather, int64_t* next_tokens, bool next_on_device, void* logits);
  Status DecodeDevice(int batch);
  void* LayerPtr(const DeviceTensor& t, int l, int64_t per_layer_elems) const {
    return static_cast<uint16_t*>(t.data) + (int64_t)l * per_layer_elems;
  }

  ModelConfig cfg_;   // this rank's view (heads, kv heads, intermediate, vocab divided by tp_)
  ModelConfig gcfg_;  // the whole model
  ShardView view_;    // both, with the group sizes / ranks the weight placement plan reads
  DeviceTensor* WeightTensor(WTensor t);
  int tp_ = 1, tp_rank_ = 0;
  void* tp_buf_[2] = {nullptr, nullptr};  // this rank's partial-sum buffers in the group's symmetric memory
  Status TpProject(const void* A, int64_t K, const void* W, int64_t T, bool decode, int parity, const void* norm_w);
  Status TpReduce(int64_t T, bool decode, int parity, const void* norm_w);
  // Expert parallel: ep_ ranks, this rank owns routed experts [ep_rank_*El, (ep_rank_+1)*El);
  // send rows / offsets and expert results live in the group's symmetric buffers
  int ep_ = 1, ep_rank_ = 0;
  int64_t ep_recv_cap_ = 0, ep_send_cap_ = 0;
  int32_t* ep_send_off_ = nullptr;
  void* ep_send_rows_ = nullptr;
  void* ep_results_ = nullptr;
  DeviceTensor ep_recv_, ep_act_, ep_recv_off_, ep_row_base_;
  void* ep_bufs_[2] = {nullptr, nullptr};
  static constexpr int64_t kEpRowsOffset = 64 << 10;  // send rows start after the offsets in buffer 0
  Status MoeBlockEp(int l, int64_t T, const void* next_norm, bool decode);
  Status SharedExpert(int l, int64_t T, const void** out);
  EngineOptions opt_;
  std::unique_ptr<ContextManager> ctx_;
  std::unique_ptr<TensorAllocator> alloc_;
  size_t weight_bytes_ = 0, kv_bytes_ = 0;
  int max_blocks_ = 0;
  int64_t num_blocks_ = 0, max_t_ = 0;
  int cur_num_seqs_ = 0, cur_max_len_ = 0;  // shape of the prefill in flight
  // kernel launches counted while the last decode step / prefill was enqueued
  // (a replayed decode graph launches what its capture counted)
  int launches_ = 0, last_decode_launches_ = 0, last_prefill_launches_ = 0, last_encode_launches_ = 0;
  // set by Encode for the duration of one RunLayers: KV writes off, and the
  // deepstack features added after layers 0..size-1 at rows inject_idx_[:inject_n_]
  bool write_kv_ = true;
  std::vector<const void*> inject_feats_;
  int64_t inject_n_ = 0;

  Status MoeBlock(int l, int64_t T, const void* next_norm, bool decode);
  Status MlaBlock(int l, int64_t T, bool decode, int batch, int* s_o);
  Status MlaAbsorb();
  Status RopeTables(int64_t T);

  // MLA weights per layer: prefill projection [q (nh*192) ; kv_a (576)] x H,
  // decode projection [absorbed q (nh*576) ; kv_a (576)] x H, kv_a RMSNorm,
  // kv_b [nh*256, 512], absorbed output projection [H, nh*512] (wo_ holds the
  // plain one); the latent cache [L][num_blocks*block_size][576]
  DeviceTensor wq_, wqabs_, kvnorm_, wkvb_, woabs_, lat_;
  DeviceTensor ckv_, kpe_, kvb_, kbuf_, mla_ws_;
  int64_t mla_ws_bytes_ = 0;
  bool absorb_dirty_ = true;
  std::vector<float> inv_freq_;  // rope frequencies (YaRN for MLA)
  float rope_mscale_ = 1.f;

  // weights (all layers stacked; dense MLPs over the dense layers only)
  DeviceTensor embed_, lm_head_, final_norm_;
  DeviceTensor wqkv_, wo_, wgu_, wdown_, qnorm_, knorm_, iln_, pln_;
  // MoE layers: router [Lm, E, H], experts gate/up [Lm, E, 2*Im, H] (rows
  // interleaved gate/up), down [Lm, E, H, Im], shared expert gate/up [Lm, 2*Is, H], down [Lm, H, Is]
  DeviceTensor router_, egu_, edown_, sgu_, sdown_;
  std::vector<int> dense_idx_, moe_idx_;  // per layer: index into the dense / MoE stacks (-1 = other kind)
  // MoE activations
  DeviceTensor topk_ids_, topk_w_, rlogits_, xperm_, eact_, ey_, eoff_, ppos_, psrc_, pws_, sact_, sout_;
  int64_t pws_bytes_ = 0;
  // KV cache [layers][2][num_blocks][kv_heads][block_size][head_dim]
  DeviceTensor kv_;
  DeviceTensor block_tables_, ctx_lens_;
  // activations / scratch
  DeviceTensor ids_, hidden_, normed_, qkv_, attn_, act_, cos_, sin_, pos_, slots_, cu_, last_idx_, last_hidden_,
      logits_, next_, seq_slots_, ctx_batch_, bt_batch_, gemm_ws_, attn_ws_, inject_idx_, pooled_, sk_flags_;
  int64_t gemm_ws_bytes_ = 0, attn_ws_bytes_ = 0;
  std::vector<int32_t> host_ctx_;
  // pinned staging for host <-> device copies
  void* pinned_ = nullptr;
  size_t pinned_bytes_ = 0;
  // decode CUDA graphs keyed by batch size; a batch size is captured on its
  // second call (the first runs eagerly and initialises lazy state)
  std::map<int, cudaGraphExec_t> graphs_;
  std::map<int, int> decode_calls_;
  // text encode passes as CUDA graphs, keyed by the shape and the buffers the
  // pass reads (a key is captured on its second call; at most kMaxEncodeGraphs,
  // the least recently replayed one evicted to make room; the once-seen keys
  // waiting for their second call are bounded by the same number)
  struct EncodeGraph {
    cudaGraphExec_t exec = nullptr;
    int launches = 0;
    uint64_t last_use = 0;
  };
  static constexpr size_t kMaxEncodeGraphs = 16;
  std::map<std::string, EncodeGraph> enc_graphs_;
  std::map<std::string, int> enc_calls_;
  uint64_t enc_tick_ = 0;
  Status EncodeDevice(int64_t S, int64_t n_vis, const void* vis_embeds, const void* const* deepstack, int n_ds,
                      bool normalize, void* hidden_out);
  unsigned* err_ = nullptr;
};

}  // namespace b200llm
