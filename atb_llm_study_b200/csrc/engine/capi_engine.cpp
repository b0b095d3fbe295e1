// C ABI of the engine: create a model from a config (HF config.json, model
// directory with safetensors, or inline JSON), prefill, decode, destroy.
// Mirrors LLMEngine::Create/Forward (atb_cpp_llm/include/atb_llm/engine.h:8-24)
// and the model registry (atb_cpp_llm/src/engine/model_registry.cpp:32-121).
#include <sys/stat.h>

#include <cstdio>

#include <functional>
#include <map>
#include <mutex>

#include "engine/model.h"
#include "engine/vision_model.h"

namespace b200llm {

// model_type -> factory, with priority-ordered compatibility fallback
// (exact match first, then the highest-priority entry whose check accepts the
// config), as the reference registry does.
struct RegistryEntry {
  std::string model_type;
  int priority = 0;
  std::function<bool(const JsonConfig&)> compat;
};

class ModelRegistry {
 public:
  static ModelRegistry& Instance() {
    static ModelRegistry r;
    return r;
  }
  void Register(RegistryEntry e) {
    std::lock_guard<std::mutex> g(mu_);
    entries_[e.model_type] = std::move(e);
  }
  // Returns the registered type used for this config ("" = none).
  std::string Resolve(const JsonConfig& cfg) const {
    std::lock_guard<std::mutex> g(mu_);
    const std::string mt = cfg.GetString("model_type");
    if (entries_.count(mt)) return mt;
    const RegistryEntry* best = nullptr;
    for (auto& kv : entries_)
      if (kv.second.compat && kv.second.compat(cfg) && (!best || kv.second.priority > best->priority))
        best = &kv.second;
    return best ? best->model_type : "";
  }

 private:
  ModelRegistry() {
    auto dense = [](const JsonConfig& c) {
      JsonConfig t = c.HasKey("text_config") ? c.GetSubConfig("text_config") : c;
      return t.HasKey("num_key_value_heads") && t.HasKey("intermediate_size") && !t.HasKey("num_local_experts") &&
             !t.HasKey("kv_lora_rank");
    };
    entries_["qwen3"] = {"qwen3", 10, nullptr};
    entries_["qwen3_vl"] = {"qwen3_vl", 10, nullptr};  // text decoder (mrope) + vision tower
    entries_["qwen2"] = {"qwen2", 5, nullptr};
    entries_["mixtral"] = {"mixtral", 10, nullptr};      // GQA + 8 routed SwiGLU experts, top-2
    entries_["qwen3_moe"] = {"qwen3_moe", 10, nullptr};  // GQA + QK-norm + routed experts
    entries_["deepseek_v2"] = {"deepseek_v2", 10, nullptr};  // latent attention + routed & shared experts
    entries_["llama"] = {"llama", 1, dense};
  }
  mutable std::mutex mu_;
  std::map<std::string, RegistryEntry> entries_;
};

}  // namespace b200llm

using namespace b200llm;

namespace b200llm {
Status GetRopeIndex(const int64_t* ids, int64_t B, int64_t S, const int64_t* mask, const int64_t* grid_thw,
                    int64_t num_images, int64_t image_token, int64_t vision_start_token, int64_t merge, int64_t* out);
}

struct b200_engine_s {
  DecoderModel model;
  std::unique_ptr<VisionModel> vision;  // Qwen3-VL configs only
  int64_t image_token_id = 151655, vision_start_token_id = 151652;
};

static bool is_vision_name(const std::string& n) {
  return n.compare(0, 13, "model.visual.") == 0 || n.compare(0, 7, "visual.") == 0;
}

static const char* dtype_name(DType d) {
  return d == DType::BF16 ? "BF16" : d == DType::FP16 ? "F16" : d == DType::FP32 ? "F32" : "";
}

static Status set_vision_weight(b200_engine_s* e, const std::string& name, const void* host, DType dt, int64_t numel) {
  if (!e->vision) return ERROR_WEIGHT_LOAD;
  std::vector<uint16_t> b16;
  B200_RETURN_IF(ToBf16(static_cast<const uint8_t*>(host), dtype_name(dt), (size_t)numel, b16));
  return e->vision->SetWeight(name, b16, numel);
}

static bool file_exists(const std::string& p) {
  struct stat st;
  return stat(p.c_str(), &st) == 0;
}

extern "C" int b200_engine_config_check(const char* config_json, char* model_type, int model_type_len) {
  if (!config_json) return ERROR_INVALID_PARAM;
  JsonConfig cfg = JsonConfig::Parse(config_json);
  if (!cfg.IsValid()) return ERROR_INVALID_PARAM;
  const std::string mt = ModelRegistry::Instance().Resolve(cfg);
  if (model_type && model_type_len > 0) {
    std::snprintf(model_type, (size_t)model_type_len, "%s", mt.c_str());
  }
  if (mt.empty()) return ERROR_UNSUPPORTED;
  ModelConfig mc;
  B200_RETURN_IF(ModelConfig::FromJson(cfg, mc));
  if (cfg.HasKey("vision_config")) {
    VisionConfig vc;
    B200_RETURN_IF(VisionConfig::FromJson(cfg, vc));
  }
  return STATUS_OK;
}

static int create_engine(const b200_engine_config* c, b200_comm_t comm, bool expert_parallel, b200_engine_t* out) {
  if (!c || !out) return ERROR_INVALID_PARAM;
  *out = nullptr;
  JsonConfig cfg;
  std::string dir = c->model_dir ? c->model_dir : "";
  if (!dir.empty()) {
    if (!file_exists(dir + "/config.json")) return ERROR_FILE_NOT_FOUND;
    cfg = JsonConfig::Load(dir + "/config.json");
  } else if (c->config_json) {
    cfg = JsonConfig::Parse(c->config_json);
  } else {
    return ERROR_INVALID_PARAM;
  }
  if (!cfg.IsValid()) return ERROR_INVALID_PARAM;
  if (ModelRegistry::Instance().Resolve(cfg).empty()) return ERROR_UNSUPPORTED;
  ModelConfig mc;
  Status s = ModelConfig::FromJson(cfg, mc);
  if (s != STATUS_OK) return s;
  EngineOptions o;
  o.device = c->device_id;
  o.max_batch = c->max_batch > 0 ? c->max_batch : 64;
  o.max_context = c->max_context > 0 ? c->max_context : 4096;
  o.max_prefill_tokens = c->max_prefill_tokens > 0 ? c->max_prefill_tokens : 16384;
  o.block_size = c->kv_block_size > 0 ? c->kv_block_size : 128;
  o.seed = c->init_seed;
  o.init_std = c->init_std > 0 ? c->init_std : 0.02f;
  o.comm = comm;
  o.expert_parallel = expert_parallel;
  auto* e = new (std::nothrow) b200_engine_s();
  if (!e) return ERROR_DEVICE_MEMORY;
  s = e->model.Init(mc, o);
  if (s == STATUS_OK && cfg.HasKey("vision_config")) {
    VisionConfig vc;
    s = VisionConfig::FromJson(cfg, vc);
    if (s == STATUS_OK) {
      e->vision.reset(new VisionModel());
      s = e->vision->Init(vc, e->model.context(), e->model.allocator());
    }
    e->image_token_id = cfg.GetInt64("image_token_id", 151655);
    e->vision_start_token_id = cfg.GetInt64("vision_start_token_id", 151652);
  }
  if (s == STATUS_OK) {
    const std::string st = dir + "/model.safetensors";
    const bool have_file = !dir.empty() && file_exists(st);
    // random init first: anything a weights file lacks stays initialised
    s = e->model.InitRandomWeights(o.seed, o.init_std);
    if (s == STATUS_OK && e->vision) s = e->vision->InitRandomWeights(o.seed, o.init_std);
    if (s == STATUS_OK && have_file) {
      SafetensorsReader r;
      s = r.LoadFromFile(st);
      if (s == STATUS_OK) s = e->model.LoadSafetensors(r, "");
      if (s == STATUS_OK && e->vision) {
        for (const std::string& key : r.GetAllKeys()) {
          if (!is_vision_name(key)) continue;
          WeightInfo w;
          s = r.GetTensor(key, w);
          if (s != STATUS_OK) break;
          DType dt = w.dtype == "BF16" ? DType::BF16 : w.dtype == "F16" ? DType::FP16 : DType::FP32;
          if (w.dtype != "BF16" && w.dtype != "F16" && w.dtype != "F32") continue;
          int64_t numel = 1;
          for (auto d : w.shape) numel *= d;
          s = set_vision_weight(e, key, r.GetTensorData(key), dt, numel);
          if (s == ERROR_WEIGHT_LOAD) s = STATUS_OK;  // a tensor this runner does not use
          if (s != STATUS_OK) break;
        }
      }
    }
  }
  if (s != STATUS_OK) {
    delete e;
    return s;
  }
  *out = e;
  return STATUS_OK;
}

extern "C" int b200_engine_create(const b200_engine_config* c, b200_engine_t* out) {
  return create_engine(c, nullptr, false, out);
}

extern "C" int b200_engine_create_tp(const b200_engine_config* c, b200_comm_t comm, b200_engine_t* out) {
  if (!comm) return ERROR_INVALID_PARAM;
  return create_engine(c, comm, false, out);
}

extern "C" int b200_engine_create_ep(const b200_engine_config* c, b200_comm_t comm, b200_engine_t* out) {
  if (!comm) return ERROR_INVALID_PARAM;
  return create_engine(c, comm, true, out);
}

extern "C" int b200_engine_destroy(b200_engine_t e) {
  delete e;
  return STATUS_OK;
}

extern "C" int b200_engine_set_weight(b200_engine_t e, const char* name, const void* host, int dtype, int64_t numel) {
  if (!e || !name || dtype < 0 || dtype > 2) return ERROR_INVALID_PARAM;
  if (is_vision_name(name)) {
    if (!host || numel <= 0) return ERROR_INVALID_PARAM;
    return set_vision_weight(e, name, host, (DType)dtype, numel);
  }
  return e->model.SetWeight(name, host, (DType)dtype, numel);
}

extern "C" int b200_engine_prefill(b200_engine_t e, const int64_t* ids, int ids_on_device, const int32_t* seq_lens,
                                   const int32_t* slots, int num_seqs, const int64_t* position_ids,
                                   int64_t* next_tokens, int next_on_device, void* logits) {
  if (!e) return ERROR_INVALID_PARAM;
  return e->model.Prefill(ids, ids_on_device != 0, seq_lens, slots, num_seqs, position_ids, next_tokens,
                          next_on_device != 0, logits);
}

extern "C" int b200_engine_decode(b200_engine_t e, const int64_t* ids, int ids_on_device, const int32_t* slots,
                                  int batch, int64_t* next_tokens, int next_on_device, void* logits) {
  if (!e) return ERROR_INVALID_PARAM;
  return e->model.Decode(ids, ids_on_device != 0, slots, batch, next_tokens, next_on_device != 0, logits);
}

extern "C" int b200_engine_vision(b200_engine_t e, const void* pixels, int pixel_dtype, int pixels_on_device,
                                  int64_t num_patches, const int64_t* grid_thw, int num_images, void* merged_out,
                                  void* deepstack_out, int64_t* merged_tokens) {
  if (!e || pixel_dtype < 0 || pixel_dtype > 2) return ERROR_INVALID_PARAM;
  if (!e->vision) return ERROR_UNSUPPORTED;
  VisionModel& v = *e->vision;
  B200_RETURN_IF(v.Forward(pixels, (DType)pixel_dtype, pixels_on_device != 0, num_patches, grid_thw, num_images));
  cudaStream_t st = e->model.stream();
  const size_t bytes = (size_t)v.MergedTokens() * v.config().out_hidden * 2;
  if (merged_out) B200_RETURN_IF(FromCuda(cudaMemcpyAsync(merged_out, v.Merged(), bytes, cudaMemcpyDeviceToDevice, st)));
  if (deepstack_out)
    for (int i = 0; i < v.NumDeepstack(); ++i)
      B200_RETURN_IF(FromCuda(cudaMemcpyAsync(static_cast<uint8_t*>(deepstack_out) + i * bytes, v.Deepstack(i), bytes,
                                              cudaMemcpyDeviceToDevice, st)));
  if (merged_tokens) *merged_tokens = v.MergedTokens();
  return STATUS_OK;
}

extern "C" int b200_engine_embed(b200_engine_t e, const int64_t* ids, int64_t S, const int64_t* mask,
                                 const void* pixels, int pixel_dtype, int pixels_on_device, int64_t num_patches,
                                 const int64_t* grid_thw, int num_images, int normalize, float* embedding,
                                 void* hidden_out) {
  if (!e || !ids || S <= 0 || !embedding || pixel_dtype < 0 || pixel_dtype > 2) return ERROR_INVALID_PARAM;
  const ModelConfig& mc = e->model.config();
  const bool image = pixels != nullptr;
  if (image && !e->vision) return ERROR_UNSUPPORTED;
  if (image && (!grid_thw || num_images <= 0)) return ERROR_INVALID_PARAM;
  std::vector<int32_t> rows;
  std::vector<const void*> ds;
  if (image) {
    VisionModel& v = *e->vision;
    if (v.config().out_hidden != mc.hidden) return ERROR_INVALID_PARAM;
    B200_RETURN_IF(v.Forward(pixels, (DType)pixel_dtype, pixels_on_device != 0, num_patches, grid_thw, num_images));
    for (int64_t s = 0; s < S; ++s)
      if (ids[s] == e->image_token_id) rows.push_back((int32_t)s);
    if ((int64_t)rows.size() != v.MergedTokens()) return ERROR_INVALID_PARAM;
    for (int i = 0; i < v.NumDeepstack() && i < mc.layers; ++i) ds.push_back(v.Deepstack(i));
  }
  std::vector<int64_t> pos;
  if (mc.mrope) {
    pos.resize((size_t)3 * S);
    const int merge = e->vision ? e->vision->config().merge : 2;
    B200_RETURN_IF(GetRopeIndex(ids, 1, S, mask, image ? grid_thw : nullptr, image ? num_images : 0,
                                e->image_token_id, e->vision_start_token_id, merge, pos.data()));
  }
  int64_t pool = S - 1;
  if (mask) {
    for (int64_t s = S - 1; s >= 0; --s)
      if (mask[s] != 0) {
        pool = s;
        break;
      }
  }
  return e->model.Encode(ids, S, pos.empty() ? nullptr : pos.data(), rows.data(), (int64_t)rows.size(),
                         image ? e->vision->Merged() : nullptr, ds.data(), (int)ds.size(), pool, normalize != 0,
                         embedding, hidden_out);
}

extern "C" int b200_engine_stream(b200_engine_t e, b200_stream_t* out) {
  if (!e || !out) return ERROR_INVALID_PARAM;
  *out = e->model.stream();
  return STATUS_OK;
}

extern "C" int b200_engine_reset(b200_engine_t e) {
  if (!e) return ERROR_INVALID_PARAM;
  return e->model.ResetSlots();
}

extern "C" int b200_engine_query(b200_engine_t e, int what, int64_t* out) {
  if (!e || !out) return ERROR_INVALID_PARAM;
  const ModelConfig& c = e->model.config();
  switch (what) {
    case B200_Q_WEIGHT_BYTES: *out = (int64_t)e->model.WeightBytes(); break;
    case B200_Q_KV_BYTES: *out = (int64_t)e->model.KvBytes(); break;
    case B200_Q_DECODE_LAUNCHES: *out = e->model.DecodeLaunches(); break;
    case B200_Q_PREFILL_LAUNCHES: *out = e->model.PrefillLaunches(); break;
    case B200_Q_HIDDEN: *out = c.hidden; break;
    case B200_Q_LAYERS: *out = c.layers; break;
    case B200_Q_VOCAB: *out = c.vocab; break;
    case B200_Q_HAS_VISION: *out = e->vision ? 1 : 0; break;
    case B200_Q_VISION_WEIGHT_BYTES: *out = e->vision ? (int64_t)e->vision->WeightBytes() : 0; break;
    case B200_Q_VISION_LAUNCHES: *out = e->vision ? e->vision->LastLaunches() : 0; break;
    case B200_Q_ENCODE_LAUNCHES: *out = e->model.EncodeLaunches(); break;
    default: return ERROR_INVALID_PARAM;
  }
  return STATUS_OK;
}

extern "C" int b200_engine_context_len(b200_engine_t e, int slot, int64_t* out) {
  if (!e || !out) return ERROR_INVALID_PARAM;
  *out = e->model.ContextLen(slot);
  return *out < 0 ? ERROR_INVALID_PARAM : STATUS_OK;
}

extern "C" int b200_engine_kv_cache(b200_engine_t e, int layer, void** k_cache, void** v_cache, int64_t* num_blocks,
                                    int* block_size, int* max_blocks_per_seq) {
  if (!e) return ERROR_INVALID_PARAM;
  return e->model.KvCache(layer, k_cache, v_cache, num_blocks, block_size, max_blocks_per_seq);
}
