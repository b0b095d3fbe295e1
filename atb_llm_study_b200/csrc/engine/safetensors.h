// safetensors reader: mmaps the file, parses the JSON header and hands out
// tensor metadata and host pointers.  Same surface as the reference's
// SafetensorsReader (atb_cpp_llm/src/io/safetensors_reader.h:27-55); the file
// format is the published safetensors layout (u64 little-endian header size,
// JSON header, raw little-endian data).
#pragma once

#include <stdint.h>

#include <map>
#include <string>
#include <vector>

#include "engine/core.h"

namespace b200llm {

struct WeightInfo {
  std::string dtype;  // "BF16", "F16", "F32", ...
  std::vector<int64_t> shape;
  size_t offset = 0;  // into the data section
  size_t nbytes = 0;
};

class SafetensorsReader {
 public:
  SafetensorsReader() = default;
  ~SafetensorsReader();
  SafetensorsReader(const SafetensorsReader&) = delete;
  SafetensorsReader& operator=(const SafetensorsReader&) = delete;

  Status LoadFromFile(const std::string& path);
  Status GetTensor(const std::string& key, WeightInfo& info) const;
  const uint8_t* GetTensorData(const std::string& key) const;
  std::vector<std::string> GetKeysByPrefix(const std::string& prefix) const;
  std::vector<std::string> GetAllKeys() const;
  bool HasKey(const std::string& key) const { return tensors_.count(key) != 0; }
  size_t NumTensors() const { return tensors_.size(); }

 private:
  void Close();
  std::map<std::string, WeightInfo> tensors_;
  const uint8_t* map_ = nullptr;
  size_t map_size_ = 0;
  const uint8_t* data_ = nullptr;
};

// Convert one tensor (BF16 / F16 / F32 source) to bf16 on the host.
Status ToBf16(const uint8_t* src, const std::string& dtype, size_t numel, std::vector<uint16_t>& out);

}  // namespace b200llm
