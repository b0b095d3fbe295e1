// Minimal JSON value + the JsonConfig accessor surface of the reference
// (atb_cpp_llm/src/io/json_config.h:12-49): Load/Parse, GetInt/GetFloat/
// GetString/GetBool/GetIntArray/GetFloatArray, GetSubConfig, HasKey, IsValid.
// Own recursive-descent parser (the reference vendors cJSON; nothing is copied).
#pragma once

#include <stdint.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

namespace b200llm {

struct JsonValue {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<JsonValue> arr;
  std::map<std::string, JsonValue> obj;

  // Parses `text`; returns false (and sets *err) on malformed input.
  static bool Parse(const std::string& text, JsonValue& out, std::string* err = nullptr);
};

class JsonConfig {
 public:
  JsonConfig() = default;
  static JsonConfig Load(const std::string& path);
  static JsonConfig Parse(const std::string& json_str);

  int GetInt(const std::string& key, int default_val = 0) const;
  int64_t GetInt64(const std::string& key, int64_t default_val = 0) const;
  float GetFloat(const std::string& key, float default_val = 0.0f) const;
  std::string GetString(const std::string& key, const std::string& default_val = "") const;
  bool GetBool(const std::string& key, bool default_val = false) const;
  std::vector<int> GetIntArray(const std::string& key) const;
  std::vector<float> GetFloatArray(const std::string& key) const;
  JsonConfig GetSubConfig(const std::string& key) const;
  bool HasKey(const std::string& key) const;
  bool IsValid() const { return root_ && root_->kind == JsonValue::Object; }
  const JsonValue* Root() const { return root_.get(); }

 private:
  explicit JsonConfig(std::shared_ptr<const JsonValue> v) : root_(std::move(v)) {}
  const JsonValue* Find(const std::string& key) const;
  std::shared_ptr<const JsonValue> root_;
};

}  // namespace b200llm
