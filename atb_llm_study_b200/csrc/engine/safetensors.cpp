#include "engine/safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

#include "engine/json_config.h"

namespace b200llm {

SafetensorsReader::~SafetensorsReader() { Close(); }

void SafetensorsReader::Close() {
  if (map_) munmap(const_cast<uint8_t*>(map_), map_size_);
  map_ = nullptr;
  map_size_ = 0;
  data_ = nullptr;
  tensors_.clear();
}

static size_t dtype_bytes(const std::string& d) {
  if (d == "BF16" || d == "F16" || d == "I16" || d == "U16") return 2;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  if (d == "I8" || d == "U8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
  return 0;
}

Status SafetensorsReader::LoadFromFile(const std::string& path) {
  Close();
  int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) return ERROR_FILE_NOT_FOUND;
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 8) {
    close(fd);
    return ERROR_WEIGHT_LOAD;
  }
  void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) return ERROR_WEIGHT_LOAD;
  map_ = static_cast<const uint8_t*>(m);
  map_size_ = (size_t)st.st_size;
  uint64_t hlen = 0;
  std::memcpy(&hlen, map_, 8);  // little-endian host assumed (x86-64 / aarch64)
  if (hlen > map_size_ - 8) {
    Close();
    return ERROR_WEIGHT_LOAD;
  }
  std::string header(reinterpret_cast<const char*>(map_ + 8), (size_t)hlen);
  JsonValue root;
  if (!JsonValue::Parse(header, root) || root.kind != JsonValue::Object) {
    Close();
    return ERROR_WEIGHT_LOAD;
  }
  data_ = map_ + 8 + hlen;
  const size_t data_size = map_size_ - 8 - hlen;
  for (auto& kv : root.obj) {
    if (kv.first == "__metadata__") continue;
    const JsonValue& e = kv.second;
    auto dt = e.obj.find("dtype"), sh = e.obj.find("shape"), off = e.obj.find("data_offsets");
    if (dt == e.obj.end() || sh == e.obj.end() || off == e.obj.end() || off->second.arr.size() != 2) {
      Close();
      return ERROR_WEIGHT_LOAD;
    }
    WeightInfo w;
    w.dtype = dt->second.str;
    size_t numel = 1;
    for (auto& d : sh->second.arr) {
      w.shape.push_back((int64_t)d.num);
      numel *= (size_t)d.num;
    }
    const size_t b = (size_t)off->second.arr[0].num, end = (size_t)off->second.arr[1].num;
    if (end < b || end > data_size || dtype_bytes(w.dtype) * numel != end - b) {
      Close();
      return ERROR_WEIGHT_LOAD;
    }
    w.offset = b;
    w.nbytes = end - b;
    tensors_[kv.first] = w;
  }
  return STATUS_OK;
}

Status SafetensorsReader::GetTensor(const std::string& key, WeightInfo& info) const {
  auto it = tensors_.find(key);
  if (it == tensors_.end()) return ERROR_WEIGHT_LOAD;
  info = it->second;
  return STATUS_OK;
}

const uint8_t* SafetensorsReader::GetTensorData(const std::string& key) const {
  auto it = tensors_.find(key);
  return it == tensors_.end() ? nullptr : data_ + it->second.offset;
}

std::vector<std::string> SafetensorsReader::GetKeysByPrefix(const std::string& prefix) const {
  std::vector<std::string> out;
  for (auto& kv : tensors_)
    if (kv.first.compare(0, prefix.size(), prefix) == 0) out.push_back(kv.first);
  return out;
}

std::vector<std::string> SafetensorsReader::GetAllKeys() const {
  std::vector<std::string> out;
  for (auto& kv : tensors_) out.push_back(kv.first);
  return out;
}

static uint16_t f32_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40);  // NaN stays NaN
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static float f16_to_f32(uint16_t h) {
  const uint32_t s = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
  uint32_t u;
  if (e == 0) {
    if (m == 0) {
      u = s;
    } else {  // subnormal: normalise
      e = 127 - 15 + 1;
      while (!(m & 0x400u)) {
        m <<= 1;
        --e;
      }
      m &= 0x3FFu;
      u = s | (e << 23) | (m << 13);
    }
  } else if (e == 31) {
    u = s | 0x7F800000u | (m << 13);
  } else {
    u = s | ((e + 127 - 15) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

Status ToBf16(const uint8_t* src, const std::string& dtype, size_t numel, std::vector<uint16_t>& out) {
  out.resize(numel);
  if (dtype == "BF16") {
    std::memcpy(out.data(), src, numel * 2);
  } else if (dtype == "F16") {
    for (size_t i = 0; i < numel; ++i) {
      uint16_t h;
      std::memcpy(&h, src + 2 * i, 2);
      out[i] = f32_to_bf16(f16_to_f32(h));
    }
  } else if (dtype == "F32") {
    for (size_t i = 0; i < numel; ++i) {
      float f;
      std::memcpy(&f, src + 4 * i, 4);
      out[i] = f32_to_bf16(f);
    }
  } else {
    return ERROR_UNSUPPORTED;
  }
  return STATUS_OK;
}

}  // namespace b200llm
