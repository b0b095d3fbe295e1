#include "engine/model.h"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <set>

#include "engine/engine_kernels.h"
#include "engine/weight_plan.h"
#include "fused.h"
#include "gemm.h"
#include "mla.h"

namespace b200 {
unsigned* error_word(int device);
void set_pdl(bool on);
}

namespace {
// Long prefill / encode passes launch without programmatic dependent launch:
// their grids fill the GPU on their own, and early-launched successors
// measured slower there (16384-token Qwen3-8B prefill).  Short passes (a few
// hundred tokens: grids of tens of CTAs) keep it, like decode.
constexpr int64_t kPdlMaxTokens = 1024;
struct NoPdlScope {
  explicit NoPdlScope(bool active) : active_(active) {
    if (active_) b200::set_pdl(false);
  }
  ~NoPdlScope() {
    if (active_) b200::set_pdl(true);
  }
  bool active_;
};
}  // namespace

namespace b200llm {

namespace {
constexpr int B200_EPI_NONE_ = B200_EPI_NONE;
// Bytes of the next projection's weights a decode kernel pulls into L2 from its
// tail: about what HBM delivers in the ~8 us a launch boundary leaves idle
// (tuning override: B200_DECODE_PREFETCH_MB=<n>, 0 = off).
const int64_t kPrefetchBytes = [] {
  const char* v = std::getenv("B200_DECODE_PREFETCH_MB");
  return (v ? std::atoll(v) : 48ll) << 20;
}();
// Stream-K flags: one per 128-row weight tile of a decode gate/up projection
// (2 x intermediate / 128 tiles; 1024 covers intermediate sizes up to 65536).
constexpr int64_t kSkFlags = 1024;
bool starts_with(const std::string& s, const std::string& p) { return s.compare(0, p.size(), p) == 0; }
}  // namespace

// ---------------------------------------------------------------- config

Status ModelConfig::FromJson(const JsonConfig& root, ModelConfig& c) {
  if (!root.IsValid()) return ERROR_INVALID_PARAM;
  c = ModelConfig();
  c.model_type = root.GetString("model_type");
  JsonConfig t = root;
  if (root.HasKey("text_config")) t = root.GetSubConfig("text_config");
  c.hidden = t.GetInt("hidden_size");
  c.layers = t.GetInt("num_hidden_layers");
  c.heads = t.GetInt("num_attention_heads");
  c.kv_heads = t.GetInt("num_key_value_heads", c.heads);
  c.head_dim = t.GetInt("head_dim", c.heads > 0 ? c.hidden / c.heads : 0);
  c.intermediate = t.GetInt("intermediate_size");
  c.vocab = t.GetInt64("vocab_size");
  c.eps = t.GetFloat("rms_norm_eps", 1e-6f);
  c.rope_theta = t.GetFloat("rope_theta", 1e6f);
  c.tie_embeddings = root.GetBool("tie_word_embeddings", t.GetBool("tie_word_embeddings", false));
  c.qk_norm = starts_with(c.model_type, "qwen3");
  if (t.HasKey("kv_lora_rank") && t.GetInt("kv_lora_rank", 0) > 0) {  // DeepSeek-V2 multi-head latent attention
    if (t.GetInt("q_lora_rank", 0) > 0) return ERROR_UNSUPPORTED;      // the V2-Lite form (no query LoRA)
    c.kv_lora = t.GetInt("kv_lora_rank");
    c.qk_nope = t.GetInt("qk_nope_head_dim");
    c.qk_rope = t.GetInt("qk_rope_head_dim");
    c.v_head = t.GetInt("v_head_dim");
    if (c.kv_lora != 512 || c.qk_rope != 64 || c.qk_nope != 128 || c.v_head != 128 || c.heads % 16)
      return ERROR_UNSUPPORTED;
    c.head_dim = c.qk_nope + c.qk_rope;
    c.kv_heads = c.heads;
    c.qk_norm = false;
    if (t.HasKey("rope_scaling")) {
      JsonConfig rs = t.GetSubConfig("rope_scaling");
      const std::string type = rs.GetString("type", rs.GetString("rope_type"));
      if (type != "yarn") return ERROR_UNSUPPORTED;
      c.yarn_factor = rs.GetFloat("factor", 1.f);
      c.yarn_orig_max = rs.GetFloat("original_max_position_embeddings", 4096.f);
      c.yarn_beta_fast = rs.GetFloat("beta_fast", 32.f);
      c.yarn_beta_slow = rs.GetFloat("beta_slow", 1.f);
      c.yarn_mscale = rs.GetFloat("mscale", 1.f);
      c.yarn_mscale_all = rs.GetFloat("mscale_all_dim", 0.f);
    }
    auto mscale = [](float s, float m) { return s <= 1.f ? 1.f : 0.1f * m * std::log(s) + 1.f; };
    const float m = mscale(c.yarn_factor, c.yarn_mscale_all);
    c.attn_scale = 1.0f / std::sqrt((float)(c.qk_nope + c.qk_rope)) * m * m;
  }
  if (t.HasKey("n_routed_experts") && t.GetInt("n_routed_experts", 0) > 0) {  // DeepSeek MoE
    c.experts = t.GetInt("n_routed_experts");
    c.top_k = t.GetInt("num_experts_per_tok", 6);
    c.moe_intermediate = t.GetInt("moe_intermediate_size");
    c.shared_intermediate = t.GetInt("n_shared_experts", 0) * c.moe_intermediate;
    c.first_dense = t.GetInt("first_k_dense_replace", 0);
    c.norm_topk = t.GetBool("norm_topk_prob", false);
    if (t.GetInt("moe_layer_freq", 1) != 1) return ERROR_UNSUPPORTED;
    const std::string tm = t.GetString("topk_method", "greedy");
    const std::string sf = t.GetString("scoring_func", "softmax");
    if (tm != "greedy" || sf != "softmax") return ERROR_UNSUPPORTED;
  } else if (t.HasKey("num_local_experts")) {  // Mixtral
    c.experts = t.GetInt("num_local_experts");
    c.top_k = t.GetInt("num_experts_per_tok", 2);
    c.moe_intermediate = c.intermediate;
    c.norm_topk = true;
  } else if (t.HasKey("num_experts") && t.GetInt("num_experts") > 0) {  // Qwen3-MoE
    c.experts = t.GetInt("num_experts");
    c.top_k = t.GetInt("num_experts_per_tok", 8);
    c.moe_intermediate = t.GetInt("moe_intermediate_size");
    c.norm_topk = t.GetBool("norm_topk_prob", true);
    if (t.HasKey("mlp_only_layers") && !t.GetIntArray("mlp_only_layers").empty()) return ERROR_UNSUPPORTED;
    if (t.GetInt("decoder_sparse_step", 1) != 1) return ERROR_UNSUPPORTED;
  }
  if (c.experts > 0) {
    c.routed_scale = t.GetFloat("routed_scaling_factor", 1.0f);
    if (c.top_k <= 0 || c.top_k > 8 || c.top_k > c.experts || c.experts > 128 || c.moe_intermediate <= 0 ||
        c.moe_intermediate % 8)
      return c.experts > 128 ? ERROR_UNSUPPORTED : ERROR_INVALID_PARAM;
  }
  if (t.HasKey("rope_scaling")) {
    JsonConfig rs = t.GetSubConfig("rope_scaling");
    std::vector<int> sec = rs.GetIntArray("mrope_section");
    if (sec.size() == 3) {
      c.mrope = true;
      for (int i = 0; i < 3; ++i) c.mrope_section[i] = sec[i];
    }
  }
  if (c.hidden <= 0 || c.layers <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.heads % c.kv_heads || c.head_dim <= 0 ||
      c.intermediate <= 0 || c.vocab <= 0)
    return ERROR_INVALID_PARAM;
  if (c.hidden % 8 || c.intermediate % 8 || (!c.mla() && c.head_dim != 128)) return ERROR_UNSUPPORTED;
  return STATUS_OK;
}

// ---------------------------------------------------------------- setup

DecoderModel::~DecoderModel() {
  if (ctx_) cudaSetDevice(ctx_->GetDeviceId());
  for (auto& g : graphs_) cudaGraphExecDestroy(g.second);
  graphs_.clear();
  for (auto& g : enc_graphs_) cudaGraphExecDestroy(g.second.exec);
  enc_graphs_.clear();
  if (ctx_) ctx_->Synchronize();
  if (pinned_) cudaFreeHost(pinned_);
  alloc_.reset();
  ctx_.reset();
}

Status DecoderModel::Init(const ModelConfig& whole, const EngineOptions& opt) {
  gcfg_ = whole;
  opt_ = opt;
  if (opt.max_batch <= 0 || opt.max_context <= 0 || opt.max_prefill_tokens <= 0 ||
      (opt.block_size != 64 && opt.block_size != 128))
    return ERROR_INVALID_PARAM;
  if (opt.comm && opt.expert_parallel) {
    // Expert parallel: whole replica of everything but the routed experts, which split into equal blocks
    B200_RETURN_IF(b200_comm_info(opt.comm, &ep_, &ep_rank_, &ep_bufs_[0], &ep_bufs_[1], nullptr));
  } else if (opt.comm) {
    B200_RETURN_IF(b200_comm_info(opt.comm, &tp_, &tp_rank_, &tp_buf_[0], &tp_buf_[1], nullptr));
  }
  // Tensor parallel: this rank keeps nq/P query heads (and the matching kv
  // heads), I/P of the MLP width and V/P of the vocabulary; everything below
  // sizes from that local view.
  B200_RETURN_IF(MakeShardView(whole, tp_, tp_rank_, ep_, ep_rank_, view_));
  const ModelConfig cfg = view_.local;
  cfg_ = cfg;
  B200_RETURN_IF(ContextManager::Create(opt.device, ctx_));
  alloc_.reset(new TensorAllocator(ctx_->GetStream()));
  err_ = b200::error_word(opt.device);
  const int64_t H = cfg.hidden, L = cfg.layers, hd = cfg.head_dim, I = cfg.intermediate, V = cfg.vocab;
  const bool mla = cfg.mla();
  const int64_t nh = cfg.heads;
  // MLA: fused projection widths (prefill q + kv_a, decode absorbed q + kv_a)
  const int64_t NQP = nh * (cfg.qk_nope + cfg.qk_rope) + cfg.kv_lora + cfg.qk_rope;
  const int64_t NQD = nh * (cfg.kv_lora + cfg.qk_rope) + cfg.kv_lora + cfg.qk_rope;
  const int64_t QKV = mla ? std::max(NQP, NQD) : cfg.qkv_dim();
  const int64_t AO = mla ? nh * cfg.v_head : (int64_t)cfg.heads * hd;  // attention output fed to o_proj
  if (mla && opt.block_size % 64) return ERROR_INVALID_PARAM;
  max_t_ = std::max<int64_t>(opt.max_prefill_tokens, opt.max_batch);
  if (tp_ > 1) {  // the partial sums of max_t_ rows must fit one symmetric buffer
    int64_t bb = 0;
    B200_RETURN_IF(b200_comm_info(opt.comm, nullptr, nullptr, nullptr, nullptr, &bb));
    if (bb < max_t_ * H * 2) return ERROR_INVALID_PARAM;
  }
  if (ep_ > 1) {
    // symmetric buffer 0: [E+1 send offsets | 64 KiB][send rows: max_t_*k x H];
    // buffer 1: expert results for up to every rank's rows [P*max_t_*k x H]
    int64_t bb = 0;
    B200_RETURN_IF(b200_comm_info(opt.comm, nullptr, nullptr, nullptr, nullptr, &bb));
    ep_send_cap_ = max_t_ * cfg.top_k;
    ep_recv_cap_ = ep_ * ep_send_cap_;
    if (bb < kEpRowsOffset + ep_send_cap_ * H * 2 || bb < ep_recv_cap_ * H * 2) return ERROR_INVALID_PARAM;
    ep_send_off_ = static_cast<int32_t*>(ep_bufs_[0]);
    ep_send_rows_ = static_cast<uint8_t*>(ep_bufs_[0]) + kEpRowsOffset;
    ep_results_ = ep_bufs_[1];
  }
  max_blocks_ = (opt.max_context + opt.block_size - 1) / opt.block_size;
  num_blocks_ = (int64_t)opt.max_batch * max_blocks_;
  auto A = [&](DeviceTensor& t, DType d, std::vector<int64_t> s) { return alloc_->Alloc(t, d, std::move(s)); };

  B200_RETURN_IF(A(embed_, DType::BF16, {gcfg_.vocab, H}));
  if (!cfg.tie_embeddings) B200_RETURN_IF(A(lm_head_, DType::BF16, {V, H}));
  else lm_head_ = embed_;
  B200_RETURN_IF(A(final_norm_, DType::BF16, {H}));
  if (mla) {
    B200_RETURN_IF(A(wq_, DType::BF16, {L, NQP, H}));
    B200_RETURN_IF(A(wqabs_, DType::BF16, {L, NQD, H}));
    B200_RETURN_IF(A(kvnorm_, DType::BF16, {L, cfg.kv_lora}));
    B200_RETURN_IF(A(wkvb_, DType::BF16, {L, nh * (cfg.qk_nope + cfg.v_head), cfg.kv_lora}));
    B200_RETURN_IF(A(woabs_, DType::BF16, {L, H, nh * cfg.kv_lora}));
    // YaRN frequencies of the rope dims (DeepSeek-V2's yarn_find_correction_range + linear ramp)
    const int d = cfg.qk_rope;
    const double base = cfg.rope_theta;
    auto corr_dim = [&](double rot) {
      return (d * std::log(cfg.yarn_orig_max / (rot * 2 * M_PI))) / (2 * std::log(base));
    };
    double low = std::max(std::floor(corr_dim(cfg.yarn_beta_fast)), 0.0);
    double high = std::min(std::ceil(corr_dim(cfg.yarn_beta_slow)), (double)(d - 1));
    if (low == high) high += 0.001;
    inv_freq_.resize(d / 2);
    for (int i = 0; i < d / 2; ++i) {
      const float e = (float)(2 * i) / (float)d;
      const float extra = 1.0f / std::pow((float)base, e);
      const float inter = 1.0f / ((float)cfg.yarn_factor * std::pow((float)base, e));
      const float ramp = std::min(1.0f, std::max(0.0f, (float)((i - low) / (high - low))));
      const float mask = cfg.yarn_factor > 1.f ? 1.0f - ramp : 1.0f;
      inv_freq_[i] = inter * (1.0f - mask) + extra * mask;
    }
    auto ms = [](float s, float m) { return s <= 1.f ? 1.f : 0.1f * m * std::log(s) + 1.f; };
    rope_mscale_ = ms(cfg.yarn_factor, cfg.yarn_mscale) / ms(cfg.yarn_factor, cfg.yarn_mscale_all);
  } else {
    B200_RETURN_IF(A(wqkv_, DType::BF16, {L, QKV, H}));
  }
  B200_RETURN_IF(A(wo_, DType::BF16, {L, H, AO}));
  dense_idx_.assign(L, -1);
  moe_idx_.assign(L, -1);
  int n_dense = 0, n_moe = 0;
  for (int l = 0; l < L; ++l) {
    if (cfg.moe_layer(l)) moe_idx_[l] = n_moe++;
    else dense_idx_[l] = n_dense++;
  }
  if (n_dense > 0) {
    B200_RETURN_IF(A(wgu_, DType::BF16, {n_dense, 2 * I, H}));
    B200_RETURN_IF(A(wdown_, DType::BF16, {n_dense, H, I}));
  }
  const int64_t E = cfg.experts, Im = cfg.moe_intermediate, Is = cfg.shared_intermediate, El = E / ep_;
  if (n_moe > 0) {
    B200_RETURN_IF(A(router_, DType::BF16, {n_moe, E, H}));
    B200_RETURN_IF(A(egu_, DType::BF16, {n_moe, El, 2 * Im, H}));
    B200_RETURN_IF(A(edown_, DType::BF16, {n_moe, El, H, Im}));
    if (Is > 0) {
      B200_RETURN_IF(A(sgu_, DType::BF16, {n_moe, 2 * Is, H}));
      B200_RETURN_IF(A(sdown_, DType::BF16, {n_moe, H, Is}));
    }
  }
  if (!mla) {
    B200_RETURN_IF(A(qnorm_, DType::BF16, {L, hd}));
    B200_RETURN_IF(A(knorm_, DType::BF16, {L, hd}));
  }
  B200_RETURN_IF(A(iln_, DType::BF16, {L, H}));
  B200_RETURN_IF(A(pln_, DType::BF16, {L, H}));
  weight_bytes_ = alloc_->BytesInUse();

  // finite contents everywhere: tiles past a sequence's end are read (and masked)
  if (mla) {
    B200_RETURN_IF(A(lat_, DType::BF16, {L, num_blocks_ * opt.block_size, cfg.kv_lora + cfg.qk_rope}));
    kv_bytes_ = lat_.bytes();
    B200_RETURN_IF(FromCuda(cudaMemsetAsync(lat_.data, 0, lat_.bytes(), ctx_->GetStream())));
  } else {
    B200_RETURN_IF(A(kv_, DType::BF16, {L, 2, num_blocks_, cfg.kv_heads, opt.block_size, hd}));
    kv_bytes_ = kv_.bytes();
    B200_RETURN_IF(FromCuda(cudaMemsetAsync(kv_.data, 0, kv_.bytes(), ctx_->GetStream())));
  }
  B200_RETURN_IF(A(block_tables_, DType::INT32, {opt.max_batch, max_blocks_}));
  B200_RETURN_IF(A(ctx_lens_, DType::INT32, {opt.max_batch}));
  {
    // slot s owns blocks [s * max_blocks, (s + 1) * max_blocks)
    std::vector<int32_t> bt((size_t)opt.max_batch * max_blocks_);
    for (size_t i = 0; i < bt.size(); ++i) bt[i] = (int32_t)i;
    B200_RETURN_IF(alloc_->CopyToDevice(block_tables_, bt.data(), bt.size() * 4));
  }
  host_ctx_.assign(opt.max_batch, 0);
  B200_RETURN_IF(FromCuda(cudaMemsetAsync(ctx_lens_.data, 0, ctx_lens_.bytes(), ctx_->GetStream())));

  B200_RETURN_IF(A(ids_, DType::INT64, {max_t_}));
  B200_RETURN_IF(A(hidden_, DType::BF16, {max_t_, H}));
  B200_RETURN_IF(A(normed_, DType::BF16, {max_t_, H}));
  B200_RETURN_IF(A(qkv_, DType::BF16, {max_t_, QKV}));
  B200_RETURN_IF(A(attn_, DType::BF16, {max_t_, mla ? std::max(AO, nh * cfg.kv_lora) : AO}));
  if (mla) {
    B200_RETURN_IF(A(ckv_, DType::BF16, {max_t_, cfg.kv_lora}));
    B200_RETURN_IF(A(kpe_, DType::BF16, {max_t_, cfg.qk_rope}));
    B200_RETURN_IF(A(kvb_, DType::BF16, {max_t_, nh * (cfg.qk_nope + cfg.v_head)}));
    B200_RETURN_IF(A(kbuf_, DType::BF16, {max_t_, nh * (cfg.qk_nope + cfg.qk_rope)}));
    mla_ws_bytes_ = b200_mla_decode_workspace_bytes(opt.max_batch, (int)nh, opt.max_context);
    if (mla_ws_bytes_ > 0) B200_RETURN_IF(A(mla_ws_, DType::FP32, {(mla_ws_bytes_ + 3) / 4}));
  }
  B200_RETURN_IF(A(act_, DType::BF16, {max_t_, n_dense > 0 ? I : 8}));
  B200_RETURN_IF(A(cos_, DType::FP32, {max_t_, hd}));
  B200_RETURN_IF(A(sin_, DType::FP32, {max_t_, hd}));
  B200_RETURN_IF(A(pos_, DType::INT64, {3, max_t_}));
  B200_RETURN_IF(A(slots_, DType::INT64, {max_t_}));
  B200_RETURN_IF(A(cu_, DType::INT32, {opt.max_batch + 1}));
  B200_RETURN_IF(A(last_idx_, DType::INT32, {opt.max_batch}));
  B200_RETURN_IF(A(last_hidden_, DType::BF16, {opt.max_batch, H}));
  B200_RETURN_IF(A(logits_, DType::BF16, {opt.max_batch, V}));
  B200_RETURN_IF(A(next_, DType::INT64, {opt.max_batch}));
  B200_RETURN_IF(A(seq_slots_, DType::INT32, {opt.max_batch}));
  B200_RETURN_IF(A(ctx_batch_, DType::INT32, {opt.max_batch}));
  B200_RETURN_IF(A(bt_batch_, DType::INT32, {opt.max_batch, max_blocks_}));
  B200_RETURN_IF(A(inject_idx_, DType::INT32, {max_t_}));
  B200_RETURN_IF(A(pooled_, DType::FP32, {H}));
  if (n_moe > 0) {
    const int64_t R = max_t_ * cfg.top_k;  // (token, choice) rows
    B200_RETURN_IF(A(topk_ids_, DType::INT32, {R}));
    B200_RETURN_IF(A(topk_w_, DType::FP32, {R}));
    B200_RETURN_IF(A(rlogits_, DType::FP32, {max_t_, E}));
    if (ep_ > 1) {  // rows received from every rank for this rank's experts
      B200_RETURN_IF(A(ep_recv_, DType::BF16, {ep_recv_cap_, H}));
      B200_RETURN_IF(A(ep_act_, DType::BF16, {ep_recv_cap_, Im}));
      B200_RETURN_IF(A(ep_recv_off_, DType::INT32, {El + 1}));
      B200_RETURN_IF(A(ep_row_base_, DType::INT32, {E}));
    } else {
      B200_RETURN_IF(A(xperm_, DType::BF16, {R, H}));
      B200_RETURN_IF(A(eact_, DType::BF16, {R, Im}));
      B200_RETURN_IF(A(ey_, DType::BF16, {R, H}));
      B200_RETURN_IF(A(eoff_, DType::INT32, {E + 1}));
    }
    B200_RETURN_IF(A(ppos_, DType::INT32, {R}));
    B200_RETURN_IF(A(psrc_, DType::INT32, {R}));
    pws_bytes_ = b200_moe_permute_workspace_bytes(max_t_, cfg.top_k, cfg.experts);
    B200_RETURN_IF(A(pws_, DType::INT32, {std::max<int64_t>(pws_bytes_ / 4, 1)}));
    if (Is > 0) {
      B200_RETURN_IF(A(sact_, DType::BF16, {max_t_, Is}));
      B200_RETURN_IF(A(sout_, DType::BF16, {max_t_, H}));
    }
  }

  // split-K workspace: the largest any projection asks for at any token count
  // this engine runs (K is split only while the output tiles leave SMs idle,
  // so the need stops growing after a few thousand tokens)
  int64_t ws = 0;
  const int64_t Isx = std::max<int64_t>(Is, 8);
  const int64_t AOx = mla ? nh * cfg.kv_lora : AO;  // decode output projection of MLA reads the latent heads
  const int64_t shapes[8][2] = {{QKV, H}, {H, AO}, {2 * I, H}, {H, I}, {V, H}, {2 * Isx, H}, {H, Isx}, {H, AOx}};
  std::vector<int64_t> ms = {1, (int64_t)opt.max_batch};
  for (int64_t m = 64; m <= std::min<int64_t>(max_t_, 65536); m += 64) ms.push_back(m);
  for (int64_t m : ms)
    for (auto& s : shapes) ws = std::max(ws, b200_gemm_workspace_bytes(m, s[0], s[1], B200_EPI_NONE_));
  gemm_ws_bytes_ = ws;
  if (ws > 0) {
    B200_RETURN_IF(A(gemm_ws_, DType::FP32, {(ws + 3) / 4}));
    // split-K accumulator + tile counters start at zero; every GEMM leaves them zero
    B200_RETURN_IF(FromCuda(cudaMemsetAsync(gemm_ws_.data, 0, gemm_ws_.bytes(), ctx_->GetStream())));
  }
  // stream-K tile flags of the decode gate/up projection: zero, and every launch leaves them zero
  B200_RETURN_IF(A(sk_flags_, DType::INT32, {kSkFlags}));
  B200_RETURN_IF(FromCuda(cudaMemsetAsync(sk_flags_.data, 0, sk_flags_.bytes(), ctx_->GetStream())));
  attn_ws_bytes_ = mla ? 0 : b200_paged_decode_workspace_bytes(opt.max_batch, cfg.heads, (int)hd, opt.max_context);
  if (attn_ws_bytes_ > 0) B200_RETURN_IF(A(attn_ws_, DType::FP32, {(attn_ws_bytes_ + 3) / 4}));

  pinned_bytes_ = (size_t)max_t_ * 8 * 5 + (size_t)(opt.max_batch + 1) * 16 + (size_t)H * 4 + 4096;
  B200_RETURN_IF(FromCuda(cudaMallocHost(&pinned_, pinned_bytes_)));
  return ctx_->Synchronize();
}

Status DecoderModel::InitRandomWeights(uint64_t seed, float std) {
  cudaStream_t st = ctx_->GetStream();
  const uint64_t k0 = seed * 1000003ull;
  // Every matrix is filled as a window of the whole model's matrix (one hash
  // key per matrix kind, values addressed by their index in the whole
  // matrix): with tensor parallelism (rank tp_rank_ of tp_) or expert
  // parallelism (rank ep_rank_ of ep_) each rank's shard holds exactly the
  // values a one-GPU engine built from the same seed holds at those positions.
  auto W = [&](const DeviceTensor& t, int64_t off, int64_t rows, int64_t cols, uint64_t key, int64_t gbase,
               int64_t gstride) -> Status {
    if (FillNormalWindowBf16(static_cast<uint16_t*>(t.data) + off, rows, cols, 0.f, std, k0 + key, gbase, gstride,
                             st))
      return ERROR_INFERENCE;
    return STATUS_OK;
  };
  auto whole = [&](const DeviceTensor& t, uint64_t key) { return t.data ? W(t, 0, 1, t.numel(), key, 0, 0) : STATUS_OK; };
  auto O = [&](DeviceTensor& t) { return FillConstBf16(t.data, t.numel(), 1.f, st); };
  const ModelConfig& g = gcfg_;
  const int64_t H = cfg_.hidden, hd = cfg_.head_dim, L = cfg_.layers, rk = tp_rank_;
  const int64_t n_dense = (int64_t)std::count_if(dense_idx_.begin(), dense_idx_.end(), [](int i) { return i >= 0; });
  const int64_t n_moe = (int64_t)std::count_if(moe_idx_.begin(), moe_idx_.end(), [](int i) { return i >= 0; });
  B200_RETURN_IF(whole(embed_, 1));
  if (!cfg_.tie_embeddings)  // a tied embedding split over tensor-parallel ranks keeps the embedding's values
    B200_RETURN_IF(W(lm_head_, 0, 1, cfg_.vocab * H, g.tie_embeddings ? 1 : 2, rk * cfg_.vocab * H, 0));
  if (!cfg_.mla()) {
    const int64_t ql = (int64_t)cfg_.heads * hd, kl = (int64_t)cfg_.kv_heads * hd;
    const int64_t qg = (int64_t)g.heads * hd, kg = (int64_t)g.kv_heads * hd;
    for (int64_t l = 0; l < L; ++l) {  // fused [q | k | v] rows, each a row block of the whole layer's
      const int64_t lb = l * (ql + 2 * kl) * H, gb = l * (qg + 2 * kg) * H;
      B200_RETURN_IF(W(wqkv_, lb, ql, H, 3, gb + rk * ql * H, H));
      B200_RETURN_IF(W(wqkv_, lb + ql * H, kl, H, 3, gb + qg * H + rk * kl * H, H));
      B200_RETURN_IF(W(wqkv_, lb + (ql + kl) * H, kl, H, 3, gb + (qg + kg) * H + rk * kl * H, H));
    }
  }
  const int64_t AOl = cfg_.mla() ? (int64_t)cfg_.heads * cfg_.v_head : (int64_t)cfg_.heads * hd;
  const int64_t AOg = g.mla() ? (int64_t)g.heads * g.v_head : (int64_t)g.heads * hd;
  B200_RETURN_IF(W(wo_, 0, L * H, AOl, 4, rk * AOl, AOg));  // column block
  const int64_t Il = cfg_.intermediate, Ig = g.intermediate;
  for (int64_t d = 0; d < n_dense; ++d)  // interleaved gate/up rows: a row block per layer
    B200_RETURN_IF(W(wgu_, d * 2 * Il * H, 2 * Il, H, 5, d * 2 * Ig * H + 2 * rk * Il * H, H));
  if (n_dense) B200_RETURN_IF(W(wdown_, 0, n_dense * H, Il, 6, rk * Il, Ig));
  if (n_moe) {
    const int64_t E = g.experts, El = E / ep_, e0 = (int64_t)ep_rank_ * El;
    const int64_t Iml = cfg_.moe_intermediate, Img = g.moe_intermediate;
    const int64_t Isl = cfg_.shared_intermediate, Isg = g.shared_intermediate;
    B200_RETURN_IF(whole(router_, 7));
    for (int64_t m = 0; m < n_moe; ++m) {
      for (int64_t e = 0; e < El; ++e)
        B200_RETURN_IF(W(egu_, (m * El + e) * 2 * Iml * H, 2 * Iml, H, 8, (m * E + e0 + e) * 2 * Img * H +
                         2 * rk * Iml * H, H));
      B200_RETURN_IF(W(edown_, m * El * H * Iml, El * H, Iml, 9, (m * E + e0) * H * Img + rk * Iml, Img));
      if (Isl > 0) B200_RETURN_IF(W(sgu_, m * 2 * Isl * H, 2 * Isl, H, 10, m * 2 * Isg * H + 2 * rk * Isl * H, H));
    }
    if (Isl > 0) B200_RETURN_IF(W(sdown_, 0, n_moe * H, Isl, 11, rk * Isl, Isg));
  }
  B200_RETURN_IF(whole(wq_, 12));
  B200_RETURN_IF(whole(wkvb_, 13));
  if (cfg_.mla()) B200_RETURN_IF(O(kvnorm_));
  absorb_dirty_ = true;
  B200_RETURN_IF(O(final_norm_));
  B200_RETURN_IF(O(qnorm_));
  B200_RETURN_IF(O(knorm_));
  B200_RETURN_IF(O(iln_));
  B200_RETURN_IF(O(pln_));
  return ctx_->Synchronize();
}

Status DecoderModel::SetWeight(const std::string& name, const void* host, DType dtype, int64_t numel) {
  if (!host || numel <= 0) return ERROR_INVALID_PARAM;
  // Tensor parallel: the whole tensor arrives and this rank keeps a block of rows
  // (column-parallel q/k/v, gate/up, lm_head) or of columns (row-parallel o,
  // down); expert parallel: only this rank's experts.  The placement is the
  // host plan the shard query b200_weight_shard also runs.
  std::vector<WeightCopy> ops;
  B200_RETURN_IF(PlanWeight(view_, name, numel, ops));
  if (ops.empty()) return STATUS_OK;
  std::vector<uint16_t> b16;
  const char* dt = dtype == DType::BF16 ? "BF16" : dtype == DType::FP16 ? "F16" : dtype == DType::FP32 ? "F32" : "";
  B200_RETURN_IF(ToBf16(static_cast<const uint8_t*>(host), dt, (size_t)numel, b16));
  cudaStream_t st = ctx_->GetStream();
  for (const WeightCopy& op : ops) {
    DeviceTensor* t = WeightTensor(op.dst);
    if (!t || !t->data) return ERROR_WEIGHT_LOAD;
    if (op.rows <= 0 || op.dst_off + (op.rows - 1) * op.dst_pitch + op.width > t->numel() ||
        op.src_off + (op.rows - 1) * op.src_pitch + op.width > numel)
      return ERROR_INVALID_PARAM;
    B200_RETURN_IF(FromCuda(cudaMemcpy2DAsync(static_cast<uint16_t*>(t->data) + op.dst_off, (size_t)op.dst_pitch * 2,
                                              b16.data() + op.src_off, (size_t)op.src_pitch * 2,
                                              (size_t)op.width * 2, (size_t)op.rows, cudaMemcpyHostToDevice, st)));
    if (cfg_.mla() && (op.dst == WTensor::WQ || op.dst == WTensor::KVNORM || op.dst == WTensor::WKVB ||
                       op.dst == WTensor::WO))
      absorb_dirty_ = true;
  }
  return ctx_->Synchronize();
}

DeviceTensor* DecoderModel::WeightTensor(WTensor t) {
  switch (t) {
    case WTensor::EMBED: return &embed_;
    case WTensor::LM_HEAD: return &lm_head_;
    case WTensor::FINAL_NORM: return &final_norm_;
    case WTensor::WQ: return &wq_;
    case WTensor::KVNORM: return &kvnorm_;
    case WTensor::WKVB: return &wkvb_;
    case WTensor::WO: return &wo_;
    case WTensor::WQKV: return &wqkv_;
    case WTensor::QNORM: return &qnorm_;
    case WTensor::KNORM: return &knorm_;
    case WTensor::ILN: return &iln_;
    case WTensor::PLN: return &pln_;
    case WTensor::WGU: return &wgu_;
    case WTensor::WDOWN: return &wdown_;
    case WTensor::ROUTER: return &router_;
    case WTensor::EGU: return &egu_;
    case WTensor::EDOWN: return &edown_;
    case WTensor::SGU: return &sgu_;
    case WTensor::SDOWN: return &sdown_;
  }
  return nullptr;
}

Status DecoderModel::LoadSafetensors(const SafetensorsReader& r, const std::string& prefix) {
  for (const std::string& key : r.GetAllKeys()) {
    if (!prefix.empty() && !starts_with(key, prefix)) continue;
    WeightInfo w;
    B200_RETURN_IF(r.GetTensor(key, w));
    DType dt;
    if (w.dtype == "BF16") dt = DType::BF16;
    else if (w.dtype == "F16") dt = DType::FP16;
    else if (w.dtype == "F32") dt = DType::FP32;
    else continue;
    int64_t numel = 1;
    for (auto s : w.shape) numel *= s;
    Status s = SetWeight(key, r.GetTensorData(key), dt, numel);
    if (s == ERROR_WEIGHT_LOAD) continue;  // not a decoder weight (e.g. vision tower)
    B200_RETURN_IF(s);
  }
  return STATUS_OK;
}

Status DecoderModel::KvCache(int l, void** k, void** v, int64_t* num_blocks, int* block_size,
                             int* max_blocks) const {
  if (l < 0 || l >= cfg_.layers || !ctx_) return ERROR_INVALID_PARAM;
  if (cfg_.mla()) {
    const int64_t rows = num_blocks_ * opt_.block_size;
    if (k) *k = static_cast<uint16_t*>(lat_.data) + (int64_t)l * rows * (cfg_.kv_lora + cfg_.qk_rope);
    if (v) *v = nullptr;
  } else {
    const int64_t kv_layer = 2 * num_blocks_ * cfg_.kv_heads * opt_.block_size * cfg_.head_dim;
    uint16_t* kc = static_cast<uint16_t*>(kv_.data) + (int64_t)l * kv_layer;
    if (k) *k = kc;
    if (v) *v = kc + kv_layer / 2;
  }
  if (num_blocks) *num_blocks = num_blocks_;
  if (block_size) *block_size = opt_.block_size;
  if (max_blocks) *max_blocks = max_blocks_;
  return STATUS_OK;
}

Status DecoderModel::ResetSlots() {
  std::fill(host_ctx_.begin(), host_ctx_.end(), 0);
  B200_RETURN_IF(FromCuda(cudaMemsetAsync(ctx_lens_.data, 0, ctx_lens_.bytes(), ctx_->GetStream())));
  return ctx_->Synchronize();
}

// ---------------------------------------------------------------- forward

Status DecoderModel::RunLayers(int64_t T, bool decode, int batch) {
  cudaStream_t st = ctx_->GetStream();
  const int64_t H = cfg_.hidden, hd = cfg_.head_dim, I = cfg_.intermediate, QKV = cfg_.qkv_dim();
  const int64_t AO = (int64_t)cfg_.heads * hd;
  const int nq = cfg_.heads, nkv = cfg_.kv_heads, L = cfg_.layers;
  const float scale = 1.0f / std::sqrt((float)hd);
  float* ws = gemm_ws_.as<float>();
  // Projections may split K (decode-sized M): they then leave fp32 partials in
  // ws and the next kernel, which reads the result anyway, finishes the sum.
  // Decode steps stream every weight once: each projection (and the decode
  // attention) pulls the first bytes of the NEXT projection's weights into L2
  // from its tail, so HBM keeps streaming across the launch boundary.
  auto gemm = [&](const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t N, int64_t K,
                  int epi, const void* R, int64_t ldr, int* splits, const void* pf = nullptr, int64_t pf_bytes = 0) {
    ++launches_;
    return b200::gemm_launch(A, lda, B, ldb, C, ldc, T, N, K, epi, nullptr, R, ldr, ws, gemm_ws_bytes_, st, splits,
                             decode && kPrefetchBytes ? pf : nullptr, std::min<int64_t>(pf_bytes, kPrefetchBytes),
                             sk_flags_.as<int>(), (int)kSkFlags);
  };
  auto bf = [](const DeviceTensor& t, int64_t off) { return static_cast<uint16_t*>(t.data) + off; };
  const int64_t kv_layer = 2 * num_blocks_ * nkv * opt_.block_size * hd;
  int s_qkv = 1, s_o = 1, s_gu = 1, s_d = 1;
  for (int l = 0; l < L; ++l) {
    if (l == 0) {
      ++launches_;
      B200_RETURN_IF(b200_rmsnorm(hidden_.data, nullptr, bf(iln_, 0), normed_.data, nullptr, T, H, H, cfg_.eps, st));
    }
    // attention block
    if (cfg_.mla()) {
      B200_RETURN_IF(MlaBlock(l, T, decode, batch, &s_o));
    } else {
    B200_RETURN_IF(gemm(normed_.data, H, bf(wqkv_, (int64_t)l * QKV * H), H, qkv_.data, QKV, QKV, H, B200_EPI_NONE,
                        nullptr, 0, &s_qkv));
    uint16_t* kc = bf(kv_, (int64_t)l * kv_layer);
    uint16_t* vc = kc + kv_layer / 2;
    ++launches_;
    B200_RETURN_IF(b200::qk_norm_rope_launch(
        qkv_.data, T, nq, nkv, (int)hd, QKV, cfg_.qk_norm ? bf(qnorm_, l * hd) : nullptr,
        cfg_.qk_norm ? bf(knorm_, l * hd) : nullptr, cfg_.eps, cos_.as<float>(), sin_.as<float>(),
        write_kv_ ? slots_.as<int64_t>() : nullptr, kc, vc, num_blocks_, opt_.block_size, s_qkv > 1 ? ws : nullptr,
        s_qkv, st));
    uint16_t* q = static_cast<uint16_t*>(qkv_.data);
    if (!decode) {
      ++launches_;
      B200_RETURN_IF(b200_flash_prefill_packed(q, QKV, hd, q + nq * hd, QKV, hd, q + (nq + nkv) * hd, QKV, hd,
                                               attn_.data, AO, hd, cu_.as<int32_t>(), cur_num_seqs_, cur_max_len_, T,
                                               nq, nkv, (int)hd, (int)hd, scale, 1, st));
    } else {
      launches_ += attn_ws_bytes_ > 0 ? 2 : 1;
      B200_RETURN_IF(b200::paged_decode_launch(q, QKV, kc, vc, bt_batch_.as<int32_t>(), max_blocks_,
                                               ctx_batch_.as<int32_t>(), batch, nq, nkv, (int)hd, opt_.block_size,
                                               num_blocks_, scale, attn_.data, AO, attn_ws_.data, attn_ws_bytes_,
                                               opt_.max_context, st,
                                               tp_ > 1 || !kPrefetchBytes ? nullptr : bf(wo_, (int64_t)l * H * AO),
                                               std::min<int64_t>(H * AO * 2, kPrefetchBytes)));
    }
    if (tp_ > 1) {  // row-parallel o: partial sums, all-reduced with the residual and the post-attention norm
      B200_RETURN_IF(TpProject(attn_.data, AO, bf(wo_, (int64_t)l * H * AO), T, decode, 0, bf(pln_, (int64_t)l * H)));
    } else {
    B200_RETURN_IF(gemm(attn_.data, AO, bf(wo_, (int64_t)l * H * AO), AO, hidden_.data, H, H, AO, B200_EPI_RESIDUAL,
                        hidden_.data, H, &s_o, dense_idx_[l] >= 0 ? bf(wgu_, dense_idx_[l] * 2 * I * H) : nullptr,
                        2 * I * H * 2));
    }
    }  // GQA attention
    if (tp_ > 1) {
      if (cfg_.moe_layer(l)) {  // experts split like dense MLPs; the combine's partial sum is all-reduced
        B200_RETURN_IF(MoeBlock(l, T, l + 1 < L ? bf(iln_, (int64_t)(l + 1) * H) : nullptr, decode));
        continue;
      }
      // MLP: column-parallel gate/up, row-parallel down, all-reduce fused with the next input norm
      const int64_t dl = dense_idx_[l];
      B200_RETURN_IF(gemm(normed_.data, H, bf(wgu_, dl * 2 * I * H), H, act_.data, I, 2 * I, H, B200_EPI_SWIGLU,
                          nullptr, 0, &s_gu));
      if (s_gu > 1) {
        ++launches_;
        B200_RETURN_IF(b200::splitk_reduce(ws, s_gu, T, 2 * I, B200_EPI_SWIGLU, nullptr, nullptr, 0, act_.data, I, st));
      }
      B200_RETURN_IF(TpProject(act_.data, I, bf(wdown_, dl * H * I), T, decode, 1,
                               l + 1 < L ? bf(iln_, (int64_t)(l + 1) * H) : nullptr));
      continue;
    }
    ++launches_;
    if (s_o > 1)  // hidden += sum(partials); normed = rmsnorm(hidden)
      B200_RETURN_IF(b200::splitk_residual_rmsnorm(ws, s_o, T, H, hidden_.data, bf(pln_, (int64_t)l * H),
                                                   normed_.data, cfg_.eps, st));
    else
      B200_RETURN_IF(b200_rmsnorm(hidden_.data, nullptr, bf(pln_, (int64_t)l * H), normed_.data, nullptr, T, H, H,
                                  cfg_.eps, st));
    const void* next_norm = l + 1 < L ? bf(iln_, (int64_t)(l + 1) * H) : nullptr;
    if (cfg_.moe_layer(l)) {  // routed experts; the combine adds the residual and applies the next norm
      B200_RETURN_IF(MoeBlock(l, T, next_norm, decode));
      continue;
    }
    // MLP block
    const int64_t dl = dense_idx_[l];
    B200_RETURN_IF(gemm(normed_.data, H, bf(wgu_, dl * 2 * I * H), H, act_.data, I, 2 * I, H, B200_EPI_SWIGLU,
                        nullptr, 0, &s_gu, bf(wdown_, dl * H * I), H * I * 2));
    if (s_gu > 1) {
      ++launches_;
      B200_RETURN_IF(b200::splitk_reduce(ws, s_gu, T, 2 * I, B200_EPI_SWIGLU, nullptr, nullptr, 0, act_.data, I, st));
    }
    const bool next_gqa = l + 1 < L && !cfg_.mla();
    B200_RETURN_IF(gemm(act_.data, I, bf(wdown_, dl * H * I), I, hidden_.data, H, H, I, B200_EPI_RESIDUAL,
                        hidden_.data, H, &s_d,
                        next_gqa ? bf(wqkv_, (int64_t)(l + 1) * QKV * H) : l + 1 == L ? lm_head_.data : nullptr,
                        next_gqa ? QKV * H * 2 : cfg_.vocab * H * 2));
    if (l < (int)inject_feats_.size() && inject_n_ > 0) {
      // deepstack: hidden[rows] += feature[l] between this layer and the next norm
      if (s_d > 1) {
        ++launches_;
        B200_RETURN_IF(b200::splitk_reduce(ws, s_d, T, H, B200_EPI_RESIDUAL, nullptr, hidden_.data, H, hidden_.data,
                                           H, st));
      }
      ++launches_;
      B200_RETURN_IF(b200_scatter_add_rows(hidden_.data, T, H, inject_idx_.as<int32_t>(), inject_feats_[l],
                                           inject_n_, 1.0f, st));
      if (next_norm) {
        ++launches_;
        B200_RETURN_IF(b200_rmsnorm(hidden_.data, nullptr, next_norm, normed_.data, nullptr, T, H, H, cfg_.eps, st));
      }
    } else if (s_d > 1) {
      ++launches_;
      if (next_norm)
        B200_RETURN_IF(b200::splitk_residual_rmsnorm(ws, s_d, T, H, hidden_.data, next_norm, normed_.data, cfg_.eps,
                                                     st));
      else
        B200_RETURN_IF(b200::splitk_reduce(ws, s_d, T, H, B200_EPI_RESIDUAL, nullptr, hidden_.data, H, hidden_.data,
                                           H, st));
    } else if (next_norm) {
      ++launches_;
      B200_RETURN_IF(b200_rmsnorm(hidden_.data, nullptr, next_norm, normed_.data, nullptr, T, H, H, cfg_.eps, st));
    }
  }
  return STATUS_OK;
}

// Row-parallel projection of this rank's K columns: partial = A W^T into the
// group's buffer `parity`, then hidden += (sum over ranks) and normed =
// RMSNorm(hidden) * norm_w (skipped when norm_w is null).  Decode-sized calls
// use the fused peer-memory all-reduce (capturable in the decode graph);
// prefill-sized ones NCCL followed by the residual + RMSNorm kernel.
Status DecoderModel::TpProject(const void* A, int64_t K, const void* W, int64_t T, bool decode, int parity,
                               const void* norm_w) {
  cudaStream_t st = ctx_->GetStream();
  const int64_t H = cfg_.hidden;
  void* buf = tp_buf_[parity];
  float* ws = gemm_ws_.as<float>();
  int s = 1;
  ++launches_;
  B200_RETURN_IF(b200::gemm_launch(A, K, W, K, buf, H, T, H, K, B200_EPI_NONE, nullptr, nullptr, 0, ws, gemm_ws_bytes_,
                                   st, &s));
  if (s > 1) {
    ++launches_;
    B200_RETURN_IF(b200::splitk_reduce(ws, s, T, H, B200_EPI_NONE, nullptr, nullptr, 0, buf, H, st));
  }
  return TpReduce(T, decode, parity, norm_w);
}

// hidden += the group's sum of the partials in buffer `parity`; normed =
// RMSNorm(hidden) * norm_w (skipped when norm_w is null).  Decode-sized calls
// use the fused peer-memory all-reduce (capturable in the decode graph);
// prefill-sized ones NCCL followed by the residual + RMSNorm kernel.
Status DecoderModel::TpReduce(int64_t T, bool decode, int parity, const void* norm_w) {
  cudaStream_t st = ctx_->GetStream();
  const int64_t H = cfg_.hidden;
  void* buf = tp_buf_[parity];
  ++launches_;
  if (decode || T <= 256)
    return (Status)b200_comm_allreduce_rmsnorm(opt_.comm, parity, T, H, hidden_.data, norm_w,
                                               norm_w ? normed_.data : nullptr, cfg_.eps, st);
  B200_RETURN_IF(b200_comm_allreduce_bf16(opt_.comm, buf, T * H, st));
  // hidden = sum + hidden; normed = RMSNorm(hidden) (the final norm's weight stands in when no norm follows:
  // that normed output is then unused)
  return (Status)b200_rmsnorm(buf, hidden_.data, norm_w ? norm_w : final_norm_.data, normed_.data, hidden_.data, T,
                              H, H, cfg_.eps, st);
}

Status DecoderModel::RopeTables(int64_t T) {
  cudaStream_t st = ctx_->GetStream();
  const int hd = cfg_.head_dim;
  if (cfg_.mla())
    return (Status)b200_rope_table_freqs(pos_.as<int64_t>(), T, cfg_.qk_rope, inv_freq_.data(), rope_mscale_,
                                         cos_.as<float>(), sin_.as<float>(), st);
  if (cfg_.mrope)
    return (Status)b200_rope_table_mrope(pos_.as<int64_t>(), T, hd, cfg_.rope_theta, cfg_.mrope_section[0],
                                         cfg_.mrope_section[1], cfg_.mrope_section[2], cos_.as<float>(),
                                         sin_.as<float>(), st);
  return (Status)b200_rope_table_1d(pos_.as<int64_t>(), T, hd, cfg_.rope_theta, cos_.as<float>(), sin_.as<float>(),
                                    st);
}

// Latent attention of layer l on normed_, ending with the output projection
// added into hidden_ (*s_o = its split count, reduced by the caller's norm).
// Prefill decompresses the heads (q_nope|q_pe against k_nope|k_pe, v from
// kv_b) and writes the latent cache; decode runs absorbed over the cache.
Status DecoderModel::MlaBlock(int l, int64_t T, bool decode, int batch, int* s_o) {
  cudaStream_t st = ctx_->GetStream();
  const int64_t H = cfg_.hidden, nh = cfg_.heads, R = cfg_.kv_lora, dr = cfg_.qk_rope, dn = cfg_.qk_nope;
  const int64_t dv = cfg_.v_head;
  const int64_t NQP = nh * (dn + dr) + R + dr, NQD = nh * (R + dr) + R + dr, KVB = nh * (dn + dv);
  const int64_t rows = num_blocks_ * opt_.block_size;
  auto bf = [](const DeviceTensor& t, int64_t off) { return static_cast<uint16_t*>(t.data) + off; };
  uint16_t* lat = bf(lat_, (int64_t)l * rows * (R + dr));
  uint16_t* q = static_cast<uint16_t*>(qkv_.data);
  float* ws = gemm_ws_.as<float>();
  const int64_t* slots = write_kv_ ? slots_.as<int64_t>() : nullptr;
  if (!decode) {
    launches_ += 6;
    B200_RETURN_IF(b200::gemm_launch(normed_.data, H, bf(wq_, (int64_t)l * NQP * H), H, q, NQP, T, NQP, H,
                                     B200_EPI_NONE, nullptr, nullptr, 0, nullptr, 0, st, nullptr));
    B200_RETURN_IF(b200_mla_prep(q, NQP, dn + dr, (int)nh, (int)dn, q + nh * (dn + dr), NQP, bf(kvnorm_, l * R),
                                 cfg_.eps, cos_.as<float>(), sin_.as<float>(), slots, lat, rows, ckv_.data, kpe_.data,
                                 T, st));
    B200_RETURN_IF(b200::gemm_launch(ckv_.data, R, bf(wkvb_, (int64_t)l * KVB * R), R, kvb_.data, KVB, T, KVB, R,
                                     B200_EPI_NONE, nullptr, nullptr, 0, nullptr, 0, st, nullptr));
    B200_RETURN_IF(b200::mla_build_k(kvb_.data, KVB, kpe_.data, kbuf_.data, T, (int)nh, st));
    B200_RETURN_IF(b200_flash_prefill_packed(q, NQP, dn + dr, kbuf_.data, nh * (dn + dr), dn + dr,
                                             static_cast<uint16_t*>(kvb_.data) + dn, KVB, dn + dv, attn_.data,
                                             nh * dv, dv, cu_.as<int32_t>(), cur_num_seqs_, cur_max_len_, T, (int)nh,
                                             (int)nh, (int)(dn + dr), (int)dv, cfg_.attn_scale, 1, st));
    return (Status)b200::gemm_launch(attn_.data, nh * dv, bf(wo_, (int64_t)l * H * nh * dv), nh * dv, hidden_.data,
                                     H, T, H, nh * dv, B200_EPI_RESIDUAL, nullptr, hidden_.data, H, ws,
                                     gemm_ws_bytes_, st, s_o);
  }
  launches_ += 4 + (mla_ws_bytes_ > 0 ? 1 : 0);
  int sq = 1;  // the query projection splits K at decode sizes; reduce before the latent preparation
  B200_RETURN_IF(b200::gemm_launch(normed_.data, H, bf(wqabs_, (int64_t)l * NQD * H), H, q, NQD, T, NQD, H,
                                   B200_EPI_NONE, nullptr, nullptr, 0, ws, gemm_ws_bytes_, st, &sq));
  if (sq > 1) {
    ++launches_;
    B200_RETURN_IF(b200::splitk_reduce(ws, sq, T, NQD, B200_EPI_NONE, nullptr, nullptr, 0, q, NQD, st));
  }
  B200_RETURN_IF(b200_mla_prep(q, NQD, R + dr, (int)nh, (int)R, q + nh * (R + dr), NQD, bf(kvnorm_, l * R), cfg_.eps,
                               cos_.as<float>(), sin_.as<float>(), slots, lat, rows, nullptr, nullptr, T, st));
  B200_RETURN_IF(b200_mla_decode(q, NQD, lat, bt_batch_.as<int32_t>(), max_blocks_, ctx_batch_.as<int32_t>(), batch,
                                 (int)nh, opt_.block_size, num_blocks_, cfg_.attn_scale, attn_.data, nh * R,
                                 mla_ws_.data, mla_ws_bytes_, opt_.max_context, st));
  return (Status)b200::gemm_launch(attn_.data, nh * R, bf(woabs_, (int64_t)l * H * nh * R), nh * R, hidden_.data, H,
                                   T, H, nh * R, B200_EPI_RESIDUAL, nullptr, hidden_.data, H, ws, gemm_ws_bytes_, st,
                                   s_o);
}

// Fold W_UK into the decode query projection and W_UV into the decode output
// projection (once after the weights change):
//   Wqabs[h*576 + c, :] = sum_d Wkvb[h*256 + d, c] Wq[h*192 + d, :]   (c < 512)
//   Wqabs[h*576 + 512 + i, :] = Wq[h*192 + 128 + i, :]                 (rope rows)
//   Woabs[:, h*512 + c] = sum_d Wo[:, h*128 + d] Wkvb[h*256 + 128 + d, c]
Status DecoderModel::MlaAbsorb() {
  if (!cfg_.mla() || !absorb_dirty_) return STATUS_OK;
  cudaStream_t st = ctx_->GetStream();
  const int64_t H = cfg_.hidden, nh = cfg_.heads, R = cfg_.kv_lora, dr = cfg_.qk_rope, dn = cfg_.qk_nope;
  const int64_t dv = cfg_.v_head;
  const int64_t NQP = nh * (dn + dr) + R + dr, NQD = nh * (R + dr) + R + dr, KVB = nh * (dn + dv);
  auto bf = [](const DeviceTensor& t, int64_t off) { return static_cast<uint16_t*>(t.data) + off; };
  for (int l = 0; l < cfg_.layers; ++l) {
    uint16_t* wq = bf(wq_, (int64_t)l * NQP * H);
    uint16_t* wkvb = bf(wkvb_, (int64_t)l * KVB * R);
    uint16_t* wqa = bf(wqabs_, (int64_t)l * NQD * H);
    uint16_t* wo = bf(wo_, (int64_t)l * H * nh * dv);
    uint16_t* woa = bf(woabs_, (int64_t)l * H * nh * R);
    B200_RETURN_IF(b200::mla_absorb(wkvb, 1, R, (dn + dv) * R, wq, H, 1, (dn + dr) * H, wqa, H, 1, (R + dr) * H,
                                    (int)R, (int)H, (int)dn, (int)nh, st));
    B200_RETURN_IF(FromCuda(cudaMemcpy2DAsync(wqa + R * H, (size_t)(R + dr) * H * 2, wq + dn * H,
                                              (size_t)(dn + dr) * H * 2, (size_t)dr * H * 2, (size_t)nh,
                                              cudaMemcpyDeviceToDevice, st)));
    B200_RETURN_IF(FromCuda(cudaMemcpyAsync(wqa + nh * (R + dr) * H, wq + nh * (dn + dr) * H, (size_t)(R + dr) * H * 2,
                                            cudaMemcpyDeviceToDevice, st)));
    B200_RETURN_IF(b200::mla_absorb(wo, nh * dv, 1, dv, wkvb + dn * R, R, 1, (dn + dv) * R, woa, nh * R, 1, R,
                                    (int)H, (int)R, (int)dv, (int)nh, st));
  }
  absorb_dirty_ = false;
  return ctx_->Synchronize();
}

// Routed-expert MLP of layer l on normed_ (the post-attention norm of
// hidden_): router -> permutation -> grouped gate/up (SwiGLU) -> grouped down
// -> weighted combine + shared expert + residual into hidden_, with the next
// layer's input norm fused into the combine.
Status DecoderModel::MoeBlock(int l, int64_t T, const void* next_norm, bool decode) {
  cudaStream_t st = ctx_->GetStream();
  const int64_t H = cfg_.hidden, E = cfg_.experts, Im = cfg_.moe_intermediate, Is = cfg_.shared_intermediate;
  const int k = cfg_.top_k;
  const int64_t mi = moe_idx_[l], R = T * k;
  auto bf = [](const DeviceTensor& t, int64_t off) { return static_cast<uint16_t*>(t.data) + off; };
  // route (logits + selection when few tokens), permutation (count, scan,
  // scatter, gather), 2 grouped GEMMs, combine
  launches_ += T < 1024 ? 2 : 1;
  B200_RETURN_IF(b200_moe_route(normed_.data, H, bf(router_, mi * E * H), T, H, (int)E, k, cfg_.norm_topk ? 1 : 0,
                                cfg_.routed_scale, topk_ids_.as<int32_t>(), topk_w_.as<float>(),
                                rlogits_.as<float>(), st));
  if (ep_ > 1) return MoeBlockEp(l, T, next_norm, decode);
  launches_ += 4 + 2 + 1;
  B200_RETURN_IF(b200_moe_permute(topk_ids_.as<int32_t>(), T, k, (int)E, normed_.data, H, H, xperm_.data,
                                  eoff_.as<int32_t>(), ppos_.as<int32_t>(), psrc_.as<int32_t>(), pws_.data,
                                  pws_bytes_, st));
  B200_RETURN_IF(b200::grouped_gemm_launch(xperm_.data, H, bf(egu_, mi * E * 2 * Im * H), H, eact_.data, Im,
                                           eoff_.as<int32_t>(), (int)E, R, 2 * Im, H, B200_EPI_SWIGLU, st));
  B200_RETURN_IF(b200::grouped_gemm_launch(eact_.data, Im, bf(edown_, mi * E * H * Im), Im, ey_.data, H,
                                           eoff_.as<int32_t>(), (int)E, R, H, Im, B200_EPI_NONE, st));
  const void* shared = nullptr;
  B200_RETURN_IF(SharedExpert(l, T, &shared));
  if (tp_ > 1) {  // this rank's share of every expert (and of the shared expert): all-reduce the combined sum
    B200_RETURN_IF(b200_moe_combine(ey_.data, ppos_.as<int32_t>(), topk_w_.as<float>(), T, k, H, nullptr, shared,
                                    tp_buf_[1], nullptr, nullptr, cfg_.eps, st));
    return TpReduce(T, decode, 1, next_norm);
  }
  return (Status)b200_moe_combine(ey_.data, ppos_.as<int32_t>(), topk_w_.as<float>(), T, k, H, hidden_.data, shared,
                                  hidden_.data, next_norm, next_norm ? normed_.data : nullptr, cfg_.eps, st);
}

// Always-on shared expert of MoE layer l on normed_ into sout_ (*out = null when the model has none).
Status DecoderModel::SharedExpert(int l, int64_t T, const void** out) {
  *out = nullptr;
  const int64_t H = cfg_.hidden, Is = cfg_.shared_intermediate, mi = moe_idx_[l];
  if (Is <= 0) return STATUS_OK;
  cudaStream_t st = ctx_->GetStream();
  auto bf = [](const DeviceTensor& t, int64_t off) { return static_cast<uint16_t*>(t.data) + off; };
  float* ws = gemm_ws_.as<float>();
  int s1 = 1, s2 = 1;
  launches_ += 2;
  B200_RETURN_IF(b200::gemm_launch(normed_.data, H, bf(sgu_, mi * 2 * Is * H), H, sact_.data, Is, T, 2 * Is, H,
                                   B200_EPI_SWIGLU, nullptr, nullptr, 0, ws, gemm_ws_bytes_, st, &s1));
  if (s1 > 1) {
    ++launches_;
    B200_RETURN_IF(b200::splitk_reduce(ws, s1, T, 2 * Is, B200_EPI_SWIGLU, nullptr, nullptr, 0, sact_.data, Is, st));
  }
  B200_RETURN_IF(b200::gemm_launch(sact_.data, Is, bf(sdown_, mi * H * Is), Is, sout_.data, H, T, H, Is,
                                   B200_EPI_NONE, nullptr, nullptr, 0, ws, gemm_ws_bytes_, st, &s2));
  if (s2 > 1) {
    ++launches_;
    B200_RETURN_IF(b200::splitk_reduce(ws, s2, T, H, B200_EPI_NONE, nullptr, nullptr, 0, sout_.data, H, st));
  }
  *out = sout_.data;
  return STATUS_OK;
}

// Expert-parallel MoE layer (routing already done): group this rank's rows by
// expert into the symmetric send area, pull every rank's rows of the local
// experts (dispatch), run the local experts' grouped GEMMs into the symmetric
// result area, then pull this rank's outputs back from the owners and combine
// them with the residual, the shared expert and the next input norm.
Status DecoderModel::MoeBlockEp(int l, int64_t T, const void* next_norm, bool decode) {
  cudaStream_t st = ctx_->GetStream();
  const int64_t H = cfg_.hidden, E = cfg_.experts, Im = cfg_.moe_intermediate, El = E / ep_;
  const int k = cfg_.top_k;
  const int64_t mi = moe_idx_[l];
  auto bf = [](const DeviceTensor& t, int64_t off) { return static_cast<uint16_t*>(t.data) + off; };
  // every rank's batch is at most max_batch rows in decode, max_t_ in prefill
  const int64_t cap = (int64_t)ep_ * (decode ? opt_.max_batch : max_t_) * k;
  launches_ += 4 + 1 + 2 + 1;  // permutation, dispatch, 2 grouped GEMMs, combine
  B200_RETURN_IF(b200_moe_permute(topk_ids_.as<int32_t>(), T, k, (int)E, normed_.data, H, H, ep_send_rows_,
                                  ep_send_off_, ppos_.as<int32_t>(), psrc_.as<int32_t>(), pws_.data, pws_bytes_, st));
  B200_RETURN_IF(b200_ep_dispatch(opt_.comm, ep_send_off_, ep_send_rows_, ep_send_cap_, E, H, ep_recv_.data, cap,
                                  ep_recv_off_.as<int32_t>(), ep_row_base_.as<int32_t>(), st));
  B200_RETURN_IF(b200::grouped_gemm_launch(ep_recv_.data, H, bf(egu_, mi * El * 2 * Im * H), H, ep_act_.data, Im,
                                           ep_recv_off_.as<int32_t>(), (int)El, cap, 2 * Im, H, B200_EPI_SWIGLU, st));
  B200_RETURN_IF(b200::grouped_gemm_launch(ep_act_.data, Im, bf(edown_, mi * El * H * Im), Im, ep_results_, H,
                                           ep_recv_off_.as<int32_t>(), (int)El, cap, H, Im, B200_EPI_NONE, st));
  const void* shared = nullptr;
  B200_RETURN_IF(SharedExpert(l, T, &shared));
  return (Status)b200_ep_combine(opt_.comm, ep_results_, cap, ep_row_base_.as<int32_t>(), ep_send_off_,
                                 topk_ids_.as<int32_t>(), topk_w_.as<float>(), ppos_.as<int32_t>(), T, k, E, H,
                                 hidden_.data, shared, hidden_.data, next_norm, next_norm ? normed_.data : nullptr,
                                 cfg_.eps, st);
}

Status DecoderModel::Head(int64_t rows, bool gather, int64_t* next_tokens, bool next_on_device, void* logits) {
  cudaStream_t st = ctx_->GetStream();
  const int64_t H = cfg_.hidden, V = cfg_.vocab;
  const void* src = hidden_.data;
  if (gather) {
    ++launches_;
    B200_RETURN_IF(GatherRows(hidden_.data, last_idx_.as<int32_t>(), rows, H, last_hidden_.data, st));
    src = last_hidden_.data;
  }
  ++launches_;
  B200_RETURN_IF(b200_rmsnorm(src, nullptr, final_norm_.data, normed_.data, nullptr, rows, H, H, cfg_.eps, st));
  int splits = 1;
  ++launches_;
  B200_RETURN_IF(b200::gemm_launch(normed_.data, H, lm_head_.data, H, logits_.data, V, rows, V, H, B200_EPI_NONE,
                                   nullptr, nullptr, 0, gemm_ws_.data, gemm_ws_bytes_, st, &splits));
  if (splits > 1) {
    ++launches_;
    B200_RETURN_IF(b200::splitk_reduce(gemm_ws_.as<float>(), splits, rows, V, B200_EPI_NONE, nullptr, nullptr, 0,
                                       logits_.data, V, st));
  }
  if (tp_ > 1) {  // vocabulary-parallel: local argmax, exchanged over the group
    launches_ += 2;
    B200_RETURN_IF(b200_comm_argmax(opt_.comm, logits_.data, rows, V, V, next_.as<int64_t>(), st));
  } else {
    ++launches_;
    B200_RETURN_IF(b200_argmax(logits_.data, rows, V, V, next_.as<int64_t>(), st));
  }
  (void)next_tokens;
  (void)next_on_device;
  (void)logits;
  return STATUS_OK;
}

Status DecoderModel::Prefill(const int64_t* ids, bool ids_on_device, const int32_t* seq_lens, const int32_t* slots,
                             int num_seqs, const int64_t* position_ids, int64_t* next_tokens, bool next_on_device,
                             void* logits) {
  if (!ids || !seq_lens || !slots || !next_tokens || num_seqs <= 0 || num_seqs > opt_.max_batch)
    return ERROR_INVALID_PARAM;
  int64_t T = 0;
  int max_len = 0;
  std::set<int> seen;
  for (int i = 0; i < num_seqs; ++i) {
    if (seq_lens[i] <= 0 || seq_lens[i] > opt_.max_context) return ERROR_INVALID_PARAM;
    if (slots[i] < 0 || slots[i] >= opt_.max_batch || !seen.insert(slots[i]).second) return ERROR_INVALID_PARAM;
    T += seq_lens[i];
    max_len = std::max(max_len, seq_lens[i]);
  }
  if (T > max_t_) return ERROR_INVALID_PARAM;
  NoPdlScope no_pdl(T > kPdlMaxTokens);
  cudaStream_t st = ctx_->GetStream();
  // host-side metadata staged in pinned memory
  uint8_t* pin = static_cast<uint8_t*>(pinned_);
  int64_t* h_pos = reinterpret_cast<int64_t*>(pin);
  int64_t* h_slot = h_pos + 3 * T;
  int32_t* h_cu = reinterpret_cast<int32_t*>(h_slot + T);
  int32_t* h_last = h_cu + num_seqs + 1;
  int64_t* h_ids = reinterpret_cast<int64_t*>(pin + ((((uint8_t*)(h_last + num_seqs) - pin) + 15) / 16) * 16);
  int64_t t = 0;
  h_cu[0] = 0;
  for (int i = 0; i < num_seqs; ++i) {
    for (int j = 0; j < seq_lens[i]; ++j, ++t) {
      for (int p = 0; p < 3; ++p) h_pos[p * T + t] = position_ids ? position_ids[p * T + t] : j;
      h_slot[t] = (int64_t)slots[i] * max_blocks_ * opt_.block_size + j;  // block j/bs of slot i's table, offset j%bs
    }
    h_cu[i + 1] = (int32_t)t;
    h_last[i] = (int32_t)(t - 1);
  }
  if (!ids_on_device) std::memcpy(h_ids, ids, (size_t)T * 8);
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(pos_.data, h_pos, (size_t)3 * T * 8, cudaMemcpyHostToDevice, st)));
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(slots_.data, h_slot, (size_t)T * 8, cudaMemcpyHostToDevice, st)));
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(cu_.data, h_cu, (size_t)(num_seqs + 1) * 4, cudaMemcpyHostToDevice, st)));
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(last_idx_.data, h_last, (size_t)num_seqs * 4, cudaMemcpyHostToDevice, st)));
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(ids_.data, ids_on_device ? (const void*)ids : (const void*)h_ids,
                                          (size_t)T * 8, ids_on_device ? cudaMemcpyDeviceToDevice
                                                                       : cudaMemcpyHostToDevice, st)));
  for (int i = 0; i < num_seqs; ++i) host_ctx_[slots[i]] = seq_lens[i];
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(ctx_lens_.data, host_ctx_.data(), host_ctx_.size() * 4,
                                          cudaMemcpyHostToDevice, st)));
  B200_RETURN_IF(ctx_->Synchronize());  // pinned staging is reused by the next call
  cur_num_seqs_ = num_seqs;
  cur_max_len_ = max_len;

  B200_RETURN_IF(RopeTables(T));
  B200_RETURN_IF(b200_embedding(ids_.as<int64_t>(), T, embed_.data, gcfg_.vocab, cfg_.hidden, hidden_.data, st));
  launches_ = 2;  // rope table + embedding
  B200_RETURN_IF(RunLayers(T, false, 0));
  B200_RETURN_IF(Head(num_seqs, true, next_tokens, next_on_device, logits));
  last_prefill_launches_ = launches_;
  if (logits)
    B200_RETURN_IF(FromCuda(cudaMemcpyAsync(logits, logits_.data, (size_t)num_seqs * cfg_.vocab * 2,
                                            cudaMemcpyDeviceToDevice, st)));
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(next_tokens, next_.data, (size_t)num_seqs * 8,
                                          next_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st)));
  if (!next_on_device) B200_RETURN_IF(ctx_->Synchronize());
  return FromCuda(cudaGetLastError());
}

Status DecoderModel::DecodeDevice(int batch) {
  cudaStream_t st = ctx_->GetStream();
  B200_RETURN_IF(DecodePrepare(seq_slots_.as<int32_t>(), batch, ctx_lens_.as<int32_t>(), block_tables_.as<int32_t>(),
                               max_blocks_, opt_.block_size, pos_.as<int64_t>(), slots_.as<int64_t>(),
                               ctx_batch_.as<int32_t>(), bt_batch_.as<int32_t>(), err_, st));
  B200_RETURN_IF(RopeTables(batch));
  B200_RETURN_IF(b200_embedding(ids_.as<int64_t>(), batch, embed_.data, gcfg_.vocab, cfg_.hidden, hidden_.data, st));
  launches_ = 3;  // prepare + rope table + embedding
  B200_RETURN_IF(RunLayers(batch, true, batch));
  B200_RETURN_IF(Head(batch, false, nullptr, true, nullptr));
  last_decode_launches_ = launches_;
  return STATUS_OK;
}

Status DecoderModel::Decode(const int64_t* ids, bool ids_on_device, const int32_t* slots, int batch,
                            int64_t* next_tokens, bool next_on_device, void* logits) {
  if (!ids || !slots || !next_tokens || batch <= 0 || batch > opt_.max_batch) return ERROR_INVALID_PARAM;
  B200_RETURN_IF(MlaAbsorb());  // absorbed projections after a weight change (outside any capture)
  std::set<int> seen;
  for (int i = 0; i < batch; ++i) {
    if (slots[i] < 0 || slots[i] >= opt_.max_batch || !seen.insert(slots[i]).second) return ERROR_INVALID_PARAM;
    if (host_ctx_[slots[i]] <= 0) return ERROR_INVALID_PARAM;  // slot holds no prefilled sequence
    if (host_ctx_[slots[i]] + 1 > opt_.max_context) return ERROR_INVALID_PARAM;
  }
  cudaStream_t st = ctx_->GetStream();
  uint8_t* pin = static_cast<uint8_t*>(pinned_);
  int32_t* h_slots = reinterpret_cast<int32_t*>(pin);
  int64_t* h_ids = reinterpret_cast<int64_t*>(pin + ((batch * 4 + 15) / 16) * 16);
  int64_t* h_next = h_ids + batch;
  std::memcpy(h_slots, slots, (size_t)batch * 4);
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(seq_slots_.data, h_slots, (size_t)batch * 4, cudaMemcpyHostToDevice, st)));
  if (ids_on_device) {
    B200_RETURN_IF(FromCuda(cudaMemcpyAsync(ids_.data, ids, (size_t)batch * 8, cudaMemcpyDeviceToDevice, st)));
  } else {
    std::memcpy(h_ids, ids, (size_t)batch * 8);
    B200_RETURN_IF(FromCuda(cudaMemcpyAsync(ids_.data, h_ids, (size_t)batch * 8, cudaMemcpyHostToDevice, st)));
  }
  static const bool no_graph = EnvInt("B200_DISABLE_GRAPHS", 0) != 0;
  auto it = graphs_.find(batch);
  if (it != graphs_.end()) {
    B200_RETURN_IF(FromCuda(cudaGraphLaunch(it->second, st)));
  } else if (!no_graph && ++decode_calls_[batch] >= 2) {
    B200_RETURN_IF(FromCuda(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed)));
    Status s = DecodeDevice(batch);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (s != STATUS_OK || e != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      return s != STATUS_OK ? s : FromCuda(e);
    }
    cudaGraphExec_t ex = nullptr;
    e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    B200_RETURN_IF(FromCuda(e));
    graphs_[batch] = ex;
    B200_RETURN_IF(FromCuda(cudaGraphLaunch(ex, st)));
  } else {
    B200_RETURN_IF(DecodeDevice(batch));
  }
  for (int i = 0; i < batch; ++i) host_ctx_[slots[i]] += 1;
  if (logits)
    B200_RETURN_IF(FromCuda(cudaMemcpyAsync(logits, logits_.data, (size_t)batch * cfg_.vocab * 2,
                                            cudaMemcpyDeviceToDevice, st)));
  if (next_on_device) {
    B200_RETURN_IF(FromCuda(cudaMemcpyAsync(next_tokens, next_.data, (size_t)batch * 8, cudaMemcpyDeviceToDevice, st)));
    return STATUS_OK;
  }
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(h_next, next_.data, (size_t)batch * 8, cudaMemcpyDeviceToHost, st)));
  B200_RETURN_IF(ctx_->Synchronize());
  std::memcpy(next_tokens, h_next, (size_t)batch * 8);
  return STATUS_OK;
}

Status DecoderModel::Encode(const int64_t* ids, int64_t S, const int64_t* position_ids, const int32_t* vis_rows,
                            int64_t n_vis, const void* vis_embeds, const void* const* deepstack, int n_ds,
                            int64_t pool_row, bool normalize, float* out, void* hidden_out) {
  if (!ids || !out || S <= 0 || S > max_t_ || S > INT32_MAX || pool_row < 0 || pool_row >= S || n_vis < 0 ||
      n_vis > S || n_ds < 0 || n_ds > cfg_.layers)
    return ERROR_INVALID_PARAM;
  if (n_vis > 0 && (!vis_rows || !vis_embeds)) return ERROR_INVALID_PARAM;
  if (n_ds > 0 && (n_vis == 0 || !deepstack)) return ERROR_INVALID_PARAM;
  for (int i = 0; i < n_ds; ++i)
    if (!deepstack[i]) return ERROR_INVALID_PARAM;
  {
    std::vector<char> seen((size_t)S, 0);
    for (int64_t i = 0; i < n_vis; ++i) {
      if (vis_rows[i] < 0 || vis_rows[i] >= S || seen[vis_rows[i]]) return ERROR_INVALID_PARAM;
      seen[vis_rows[i]] = 1;
    }
  }
  NoPdlScope no_pdl(S > kPdlMaxTokens);
  cudaStream_t st = ctx_->GetStream();
  const int64_t H = cfg_.hidden;
  uint8_t* pin = static_cast<uint8_t*>(pinned_);
  int64_t* h_pos = reinterpret_cast<int64_t*>(pin);
  int64_t* h_ids = h_pos + 3 * S;
  int32_t* h_rows = reinterpret_cast<int32_t*>(h_ids + S);
  int32_t* h_cu = h_rows + n_vis;
  for (int64_t t = 0; t < S; ++t)
    for (int p = 0; p < 3; ++p) h_pos[p * S + t] = position_ids ? position_ids[p * S + t] : t;
  std::memcpy(h_ids, ids, (size_t)S * 8);
  if (n_vis) std::memcpy(h_rows, vis_rows, (size_t)n_vis * 4);
  h_cu[0] = 0;
  h_cu[1] = (int32_t)S;
  h_cu[2] = (int32_t)pool_row;
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(pos_.data, h_pos, (size_t)3 * S * 8, cudaMemcpyHostToDevice, st)));
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(ids_.data, h_ids, (size_t)S * 8, cudaMemcpyHostToDevice, st)));
  if (n_vis)
    B200_RETURN_IF(FromCuda(cudaMemcpyAsync(inject_idx_.data, h_rows, (size_t)n_vis * 4, cudaMemcpyHostToDevice, st)));
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(cu_.data, h_cu, 8, cudaMemcpyHostToDevice, st)));
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(last_idx_.data, h_cu + 2, 4, cudaMemcpyHostToDevice, st)));
  B200_RETURN_IF(ctx_->Synchronize());  // pinned staging is reused by the next call
  cur_num_seqs_ = 1;
  cur_max_len_ = (int)S;

  // Every per-call input now sits in the engine's device buffers (ids, positions,
  // image rows, pooled row), so a pass of the same shape over the same feature
  // buffers replays one captured graph.
  std::string key = std::to_string(S) + "/" + std::to_string(n_vis) + "/" +
                    std::to_string(reinterpret_cast<uintptr_t>(vis_embeds)) + "/" + std::to_string(normalize) + "/" +
                    std::to_string(reinterpret_cast<uintptr_t>(hidden_out));
  for (int i = 0; i < n_ds; ++i) key += "/" + std::to_string(reinterpret_cast<uintptr_t>(deepstack[i]));
  static const bool no_graph = EnvInt("B200_DISABLE_GRAPHS", 0) != 0;
  auto it = enc_graphs_.find(key);
  ++enc_tick_;
  // keys seen once and not yet captured: bounded like the graphs (a serving
  // loop whose buffers move would otherwise grow it without end)
  if (it == enc_graphs_.end() && !enc_calls_.count(key) && enc_calls_.size() >= kMaxEncodeGraphs) enc_calls_.clear();
  if (it != enc_graphs_.end()) {
    it->second.last_use = enc_tick_;
    B200_RETURN_IF(FromCuda(cudaGraphLaunch(it->second.exec, st)));
    launches_ = it->second.launches;
  } else if (!no_graph && ++enc_calls_[key] >= 2) {
    if (enc_graphs_.size() >= kMaxEncodeGraphs) {  // evict the least recently replayed graph
      auto lru = enc_graphs_.begin();
      for (auto g = enc_graphs_.begin(); g != enc_graphs_.end(); ++g)
        if (g->second.last_use < lru->second.last_use) lru = g;
      cudaGraphExecDestroy(lru->second.exec);  // an in-flight replay is freed when it completes
      enc_graphs_.erase(lru);
    }
    B200_RETURN_IF(FromCuda(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed)));
    Status s = EncodeDevice(S, n_vis, vis_embeds, deepstack, n_ds, normalize, hidden_out);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &g);
    cudaGraphExec_t ex = nullptr;
    if (s == STATUS_OK && e == cudaSuccess) e = cudaGraphInstantiate(&ex, g, 0);
    if (g) cudaGraphDestroy(g);
    if (s == STATUS_OK && e == cudaSuccess) {
      enc_graphs_[key] = EncodeGraph{ex, launches_, enc_tick_};
      enc_calls_.erase(key);
      B200_RETURN_IF(FromCuda(cudaGraphLaunch(ex, st)));
    } else {
      // nothing of the capture ran: clear its error, never capture this key again, run the pass eagerly
      (void)cudaGetLastError();
      enc_calls_[key] = -(1 << 30);
      B200_RETURN_IF(EncodeDevice(S, n_vis, vis_embeds, deepstack, n_ds, normalize, hidden_out));
    }
  } else {
    B200_RETURN_IF(EncodeDevice(S, n_vis, vis_embeds, deepstack, n_ds, normalize, hidden_out));
  }
  last_encode_launches_ = launches_;
  float* h_out = reinterpret_cast<float*>(pin);
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(h_out, pooled_.data, (size_t)H * 4, cudaMemcpyDeviceToHost, st)));
  B200_RETURN_IF(ctx_->Synchronize());
  std::memcpy(out, h_out, (size_t)H * 4);
  return FromCuda(cudaGetLastError());
}

// The device part of Encode: rope tables, embedding (+ image rows), the
// layers, final RMSNorm of the pooled row and L2 pooling into pooled_.
Status DecoderModel::EncodeDevice(int64_t S, int64_t n_vis, const void* vis_embeds, const void* const* deepstack,
                                  int n_ds, bool normalize, void* hidden_out) {
  cudaStream_t st = ctx_->GetStream();
  const int64_t H = cfg_.hidden;
  B200_RETURN_IF(RopeTables(S));
  B200_RETURN_IF(b200_embedding(ids_.as<int64_t>(), S, embed_.data, gcfg_.vocab, H, hidden_.data, st));
  launches_ = 2;
  if (n_vis) {
    ++launches_;
    B200_RETURN_IF(ScatterRows(hidden_.data, inject_idx_.as<int32_t>(), n_vis, H, vis_embeds, st));
  }
  write_kv_ = false;
  inject_feats_.assign(deepstack, deepstack + n_ds);
  inject_n_ = n_vis;
  Status s = RunLayers(S, false, 0);
  write_kv_ = true;
  inject_feats_.clear();
  inject_n_ = 0;
  B200_RETURN_IF(s);
  // final RMSNorm of the pooled row, then L2 pooling (BaseModel::RunPooling,
  // atb_cpp_llm/src/families/base_model.cpp:137-199)
  launches_ += 3;
  B200_RETURN_IF(GatherRows(hidden_.data, last_idx_.as<int32_t>(), 1, H, last_hidden_.data, st));
  B200_RETURN_IF(b200_rmsnorm(last_hidden_.data, nullptr, final_norm_.data, normed_.data, nullptr, 1, H, H, cfg_.eps,
                              st));
  B200_RETURN_IF(PoolL2(normed_.data, H, normalize ? 1 : 0, pooled_.as<float>(), st));
  if (hidden_out) {
    ++launches_;
    B200_RETURN_IF(b200_rmsnorm(hidden_.data, nullptr, final_norm_.data, hidden_out, nullptr, S, H, H, cfg_.eps, st));
  }
  return STATUS_OK;
}

int DecoderModel::DecodeLaunches() const { return last_decode_launches_; }

int DecoderModel::PrefillLaunches() const { return last_prefill_launches_; }

}  // namespace b200llm
