// C ABI of the engine: create a model from a config (HF config.json, model
// directory with safetensors, or inline JSON), prefill, decode, destroy.
// Mirrors LLMEngine::Create/Forward (atb_cpp_llm/include/atb_llm/engine.h:8-24)
// and the model registry (atb_cpp_llm/src/engine/model_registry.cpp:32-121).
#include <sys/stat.h>

#include <functional>
#include <map>
#include <mutex>

#include "engine/model.h"

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
    entries_["qwen3_vl"] = {"qwen3_vl", 10, nullptr};  // text decoder (mrope); vision tower not in this runner
    entries_["qwen2"] = {"qwen2", 5, nullptr};
    entries_["llama"] = {"llama", 1, dense};
  }
  mutable std::mutex mu_;
  std::map<std::string, RegistryEntry> entries_;
};

}  // namespace b200llm

using namespace b200llm;

struct b200_engine_s {
  DecoderModel model;
};

static bool file_exists(const std::string& p) {
  struct stat st;
  return stat(p.c_str(), &st) == 0;
}

extern "C" int b200_engine_create(const b200_engine_config* c, b200_engine_t* out) {
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
  auto* e = new (std::nothrow) b200_engine_s();
  if (!e) return ERROR_DEVICE_MEMORY;
  s = e->model.Init(mc, o);
  if (s == STATUS_OK) {
    const std::string st = dir + "/model.safetensors";
    if (!dir.empty() && file_exists(st)) {
      SafetensorsReader r;
      s = r.LoadFromFile(st);
      if (s == STATUS_OK) s = e->model.InitRandomWeights(o.seed, o.init_std);  // anything the file lacks
      if (s == STATUS_OK) s = e->model.LoadSafetensors(r, "");
    } else {
      s = e->model.InitRandomWeights(o.seed, o.init_std);
    }
  }
  if (s != STATUS_OK) {
    delete e;
    return s;
  }
  *out = e;
  return STATUS_OK;
}

extern "C" int b200_engine_destroy(b200_engine_t e) {
  delete e;
  return STATUS_OK;
}

extern "C" int b200_engine_set_weight(b200_engine_t e, const char* name, const void* host, int dtype, int64_t numel) {
  if (!e || !name || dtype < 0 || dtype > 2) return ERROR_INVALID_PARAM;
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
    default: return ERROR_INVALID_PARAM;
  }
  return STATUS_OK;
}

extern "C" int b200_engine_context_len(b200_engine_t e, int slot, int64_t* out) {
  if (!e || !out) return ERROR_INVALID_PARAM;
  *out = e->model.ContextLen(slot);
  return *out < 0 ? ERROR_INVALID_PARAM : STATUS_OK;
}
