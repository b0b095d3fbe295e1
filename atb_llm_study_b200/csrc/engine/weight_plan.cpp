#include "engine/weight_plan.h"

#include <cstdlib>
#include <cstring>

#include "engine/json_config.h"
#include "engine/safetensors.h"

namespace b200llm {

namespace {
bool starts_with(const std::string& s, const std::string& p) { return s.compare(0, p.size(), p) == 0; }
}  // namespace

Status MakeShardView(const ModelConfig& whole, int tp, int tp_rank, int ep, int ep_rank, ShardView& v) {
  if (tp < 1 || ep < 1 || tp_rank < 0 || tp_rank >= tp || ep_rank < 0 || ep_rank >= ep || (tp > 1 && ep > 1))
    return ERROR_INVALID_PARAM;
  v = ShardView();
  v.whole = v.local = whole;
  v.tp = tp;
  v.tp_rank = tp_rank;
  v.ep = ep;
  v.ep_rank = ep_rank;
  if (ep > 1 && (whole.experts <= 0 || whole.experts % ep || whole.experts > 256)) return ERROR_UNSUPPORTED;
  if (tp > 1) {
    // GQA attention (dense or mixture-of-experts MLPs; an expert's width is split like a dense MLP's)
    if (whole.mla() || whole.mrope) return ERROR_UNSUPPORTED;
    if (whole.heads % tp || whole.kv_heads % tp || whole.intermediate % tp || whole.vocab % tp ||
        (whole.intermediate / tp) % 8 || (whole.vocab / tp) % 8 || whole.hidden > 8192)
      return ERROR_UNSUPPORTED;
    if (whole.experts > 0 && (whole.moe_intermediate % tp || (whole.moe_intermediate / tp) % 8 ||
                              whole.shared_intermediate % tp || (whole.shared_intermediate / tp) % 8))
      return ERROR_UNSUPPORTED;
    ModelConfig& c = v.local;
    c.heads /= tp;
    c.kv_heads /= tp;
    c.intermediate /= tp;
    c.vocab /= tp;
    c.moe_intermediate /= tp;
    c.shared_intermediate /= tp;
    c.tie_embeddings = false;  // lm_head is this rank's vocabulary rows, the embedding stays whole
  }
  v.dense_idx.assign(whole.layers, -1);
  v.moe_idx.assign(whole.layers, -1);
  int nd = 0, nm = 0;
  for (int l = 0; l < whole.layers; ++l) {
    if (whole.moe_layer(l)) v.moe_idx[l] = nm++;
    else v.dense_idx[l] = nd++;
  }
  return STATUS_OK;
}

Status PlanWeight(const ShardView& v, const std::string& name_in, int64_t numel, std::vector<WeightCopy>& ops) {
  ops.clear();
  const ModelConfig& c = v.local;
  const ModelConfig& g = v.whole;
  std::string name = name_in;
  if (starts_with(name, "model.language_model.")) name = "model." + name.substr(21);
  const int64_t H = c.hidden, hd = c.head_dim, I = c.intermediate, QKV = c.qkv_dim();
  const int64_t AO = (int64_t)c.heads * hd;
  const int64_t P = v.tp, rk = v.tp_rank;
  // the whole tensor, contiguous
  auto whole = [&](WTensor t, int64_t off, int64_t expect) -> Status {
    if (numel != expect) return ERROR_INVALID_PARAM;
    ops.push_back({t, off, numel, 0, numel, numel, 1});
    return STATUS_OK;
  };
  // this rank's block of rows_local rows (column-parallel q/k/v, lm_head)
  auto rows = [&](WTensor t, int64_t off, int64_t expect, int64_t rows_local, int64_t row_len) -> Status {
    if (numel != expect) return ERROR_INVALID_PARAM;
    const int64_t n = rows_local * row_len;
    ops.push_back({t, off, n, rk * n, n, n, 1});
    return STATUS_OK;
  };
  // this rank's block of cols_local columns of a [nrows, cols_local * P] matrix (row-parallel o, down)
  auto cols = [&](WTensor t, int64_t off, int64_t nrows, int64_t cols_local) -> Status {
    if (numel != nrows * cols_local * P) return ERROR_INVALID_PARAM;
    ops.push_back({t, off, cols_local, rk * cols_local, cols_local * P, cols_local, nrows});
    return STATUS_OK;
  };
  // rows 2j / 2j+1 of a fused gate/up matrix hold gate[j] / up[j] (the SwiGLU
  // epilogue's layout); this rank's `inter` rows of the [inter * P, H] source
  auto interleaved = [&](WTensor t, int64_t off, int64_t inter, bool up) -> Status {
    if (numel != inter * P * H) return ERROR_INVALID_PARAM;
    ops.push_back({t, off + (up ? H : 0), 2 * H, rk * inter * H, H, H, inter});
    return STATUS_OK;
  };
  if (name == "model.embed_tokens.weight") {
    B200_RETURN_IF(whole(WTensor::EMBED, 0, g.vocab * H));
    if (g.tie_embeddings && !c.tie_embeddings)  // tensor parallel: lm_head = this rank's embedding rows
      return rows(WTensor::LM_HEAD, 0, g.vocab * H, c.vocab, H);
    return STATUS_OK;
  }
  if (name == "lm_head.weight") {
    if (c.tie_embeddings) return numel == g.vocab * H ? STATUS_OK : ERROR_INVALID_PARAM;
    return rows(WTensor::LM_HEAD, 0, g.vocab * H, c.vocab, H);
  }
  if (name == "model.norm.weight") return whole(WTensor::FINAL_NORM, 0, H);
  const std::string pre = "model.layers.";
  if (!starts_with(name, pre)) return ERROR_WEIGHT_LOAD;
  const size_t dot = name.find('.', pre.size());
  if (dot == std::string::npos) return ERROR_WEIGHT_LOAD;
  const int l = std::atoi(name.substr(pre.size(), dot - pre.size()).c_str());
  if (l < 0 || l >= c.layers) return ERROR_WEIGHT_LOAD;
  const std::string leaf = name.substr(dot + 1);
  if (c.mla() && starts_with(leaf, "self_attn.")) {
    const int64_t nh = c.heads, R = c.kv_lora, dr = c.qk_rope;
    const int64_t NQP = nh * (c.qk_nope + dr) + R + dr, KVB = nh * (c.qk_nope + c.v_head);
    const int64_t AOm = nh * c.v_head;
    if (leaf == "self_attn.q_proj.weight") return whole(WTensor::WQ, (int64_t)l * NQP * H, nh * (c.qk_nope + dr) * H);
    if (leaf == "self_attn.kv_a_proj_with_mqa.weight")
      return whole(WTensor::WQ, (int64_t)l * NQP * H + nh * (c.qk_nope + dr) * H, (R + dr) * H);
    if (leaf == "self_attn.kv_a_layernorm.weight") return whole(WTensor::KVNORM, (int64_t)l * R, R);
    if (leaf == "self_attn.kv_b_proj.weight") return whole(WTensor::WKVB, (int64_t)l * KVB * R, KVB * R);
    if (leaf == "self_attn.o_proj.weight") return whole(WTensor::WO, (int64_t)l * H * AOm, H * AOm);
    return ERROR_WEIGHT_LOAD;
  }
  const int64_t nq = (int64_t)c.heads * hd, nk = (int64_t)c.kv_heads * hd;
  if (leaf == "self_attn.q_proj.weight") return rows(WTensor::WQKV, (int64_t)l * QKV * H, nq * P * H, nq, H);
  if (leaf == "self_attn.k_proj.weight")
    return rows(WTensor::WQKV, (int64_t)l * QKV * H + nq * H, nk * P * H, nk, H);
  if (leaf == "self_attn.v_proj.weight")
    return rows(WTensor::WQKV, (int64_t)l * QKV * H + (nq + nk) * H, nk * P * H, nk, H);
  if (leaf == "self_attn.o_proj.weight") return cols(WTensor::WO, (int64_t)l * H * AO, H, AO);
  if (leaf == "self_attn.q_norm.weight") return whole(WTensor::QNORM, (int64_t)l * hd, hd);
  if (leaf == "self_attn.k_norm.weight") return whole(WTensor::KNORM, (int64_t)l * hd, hd);
  if (leaf == "input_layernorm.weight") return whole(WTensor::ILN, (int64_t)l * H, H);
  if (leaf == "post_attention_layernorm.weight") return whole(WTensor::PLN, (int64_t)l * H, H);
  const int di = v.dense_idx[l], mi = v.moe_idx[l];
  if (di >= 0) {
    if (leaf == "mlp.down_proj.weight") return cols(WTensor::WDOWN, (int64_t)di * H * I, H, I);
    if (leaf == "mlp.gate_proj.weight" || leaf == "mlp.up_proj.weight")
      return interleaved(WTensor::WGU, (int64_t)di * 2 * I * H, I, leaf[4] == 'u');
    return ERROR_WEIGHT_LOAD;
  }
  // MoE layer: Mixtral "block_sparse_moe.{gate, experts.E.w1/w3/w2}", Qwen3-MoE /
  // DeepSeek "mlp.{gate, experts.E.gate_proj/up_proj/down_proj, shared_experts.*}"
  const int64_t E = c.experts, Im = c.moe_intermediate, Is = c.shared_intermediate;
  std::string m;
  if (starts_with(leaf, "block_sparse_moe.")) m = leaf.substr(17);
  else if (starts_with(leaf, "mlp.")) m = leaf.substr(4);
  else return ERROR_WEIGHT_LOAD;
  if (m == "gate.weight") return whole(WTensor::ROUTER, (int64_t)mi * E * H, E * H);
  if (starts_with(m, "shared_experts.") && Is > 0) {
    const std::string s = m.substr(15);
    if (s == "down_proj.weight") return cols(WTensor::SDOWN, (int64_t)mi * H * Is, H, Is);
    if (s == "gate_proj.weight" || s == "up_proj.weight")
      return interleaved(WTensor::SGU, (int64_t)mi * 2 * Is * H, Is, s[0] == 'u');
    return ERROR_WEIGHT_LOAD;
  }
  if (!starts_with(m, "experts.")) return ERROR_WEIGHT_LOAD;
  const size_t d2 = m.find('.', 8);
  if (d2 == std::string::npos) return ERROR_WEIGHT_LOAD;
  const int e = std::atoi(m.substr(8, d2 - 8).c_str());
  if (e < 0 || e >= E) return ERROR_WEIGHT_LOAD;
  const std::string w = m.substr(d2 + 1);
  const int64_t El = E / v.ep, e0 = (int64_t)v.ep_rank * El;
  const bool known = w == "w1.weight" || w == "w2.weight" || w == "w3.weight" || w == "gate_proj.weight" ||
                     w == "up_proj.weight" || w == "down_proj.weight";
  if (!known) return ERROR_WEIGHT_LOAD;
  if (e < e0 || e >= e0 + El) return STATUS_OK;   // another rank's expert (expert parallel)
  const int64_t ge = (int64_t)mi * El + (e - e0);  // expert slot in the MoE stacks
  if (w == "w2.weight" || w == "down_proj.weight") return cols(WTensor::EDOWN, ge * H * Im, H, Im);
  if (w == "w1.weight" || w == "gate_proj.weight") return interleaved(WTensor::EGU, ge * 2 * Im * H, Im, false);
  return interleaved(WTensor::EGU, ge * 2 * Im * H, Im, true);
}

}  // namespace b200llm

// ---------------------------------------------------------------- C ABI (host only)

namespace {

using namespace b200llm;

bool is_vision(const std::string& n) {
  return n.compare(0, 13, "model.visual.") == 0 || n.compare(0, 7, "visual.") == 0;
}

// This rank's part of one whole tensor (bf16) as the dense rows / columns it keeps.
int shard_into(const char* config_json, int tp_world, int tp_rank, int ep_world, int ep_rank, const std::string& name,
               const uint8_t* src, const std::string& dtype, int64_t numel, void* out, int64_t out_capacity,
               int64_t* out_numel) {
  if (!config_json || !src || !out || !out_numel || numel <= 0) return ERROR_INVALID_PARAM;
  *out_numel = 0;
  JsonConfig cfg = JsonConfig::Parse(config_json);
  if (!cfg.IsValid()) return ERROR_INVALID_PARAM;
  ModelConfig mc;
  B200_RETURN_IF(ModelConfig::FromJson(cfg, mc));
  ShardView v;
  B200_RETURN_IF(MakeShardView(mc, tp_world, tp_rank, ep_world, ep_rank, v));
  std::vector<WeightCopy> ops;
  Status s = PlanWeight(v, name, numel, ops);
  const bool replicated_vision = s == ERROR_WEIGHT_LOAD && is_vision(name);  // the vision tower is never split
  if (s != STATUS_OK && !replicated_vision) return s;
  if (replicated_vision) ops.push_back({WTensor::EMBED, 0, numel, 0, numel, numel, 1});
  std::vector<uint16_t> b16;
  B200_RETURN_IF(ToBf16(src, dtype, (size_t)numel, b16));
  int64_t need = 0;
  for (const WeightCopy& op : ops) need += op.rows * op.width;
  if (need > out_capacity) return ERROR_INVALID_PARAM;
  uint16_t* o = static_cast<uint16_t*>(out);
  for (const WeightCopy& op : ops)
    for (int64_t r = 0; r < op.rows; ++r, o += op.width)
      std::memcpy(o, b16.data() + op.src_off + r * op.src_pitch, (size_t)op.width * 2);
  *out_numel = need;
  return STATUS_OK;
}

}  // namespace

extern "C" int b200_weight_shard(const char* config_json, int tp_world, int tp_rank, int ep_world, int ep_rank,
                                 const char* name, const void* host, int dtype, int64_t numel, void* out,
                                 int64_t out_capacity, int64_t* out_numel) {
  if (!name || dtype < 0 || dtype > 2) return ERROR_INVALID_PARAM;
  const char* dt = dtype == 0 ? "BF16" : dtype == 1 ? "F16" : "F32";
  return shard_into(config_json, tp_world, tp_rank, ep_world, ep_rank, name, static_cast<const uint8_t*>(host), dt,
                    numel, out, out_capacity, out_numel);
}

extern "C" int b200_weight_shard_file(const char* config_json, const char* safetensors_path, const char* name,
                                      int tp_world, int tp_rank, int ep_world, int ep_rank, void* out,
                                      int64_t out_capacity, int64_t* out_numel) {
  if (!safetensors_path || !name) return ERROR_INVALID_PARAM;
  SafetensorsReader r;
  B200_RETURN_IF(r.LoadFromFile(safetensors_path));
  WeightInfo w;
  B200_RETURN_IF(r.GetTensor(name, w));
  if (w.dtype != "BF16" && w.dtype != "F16" && w.dtype != "F32") return ERROR_UNSUPPORTED;
  int64_t numel = 1;
  for (int64_t d : w.shape) numel *= d;
  return shard_into(config_json, tp_world, tp_rank, ep_world, ep_rank, name, r.GetTensorData(name), w.dtype, numel,
                    out, out_capacity, out_numel);
}
