#include "engine/core.h"

#include <cstdlib>

namespace b200llm {

size_t DTypeSize(DType t) {
  switch (t) {
    case DType::BF16:
    case DType::FP16: return 2;
    case DType::FP32:
    case DType::INT32: return 4;
    case DType::INT64: return 8;
  }
  return 0;
}

Status ContextManager::Create(int device_id, std::unique_ptr<ContextManager>& out) {
  int n = 0;
  B200_RETURN_IF(FromCuda(cudaGetDeviceCount(&n)));
  if (device_id < 0 || device_id >= n) return ERROR_INVALID_PARAM;
  std::unique_ptr<ContextManager> c(new ContextManager(device_id));
  B200_RETURN_IF(FromCuda(cudaSetDevice(device_id)));
  B200_RETURN_IF(FromCuda(cudaDeviceGetAttribute(&c->sms_, cudaDevAttrMultiProcessorCount, device_id)));
  B200_RETURN_IF(FromCuda(cudaStreamCreateWithFlags(&c->stream_, cudaStreamNonBlocking)));
  out = std::move(c);
  return STATUS_OK;
}

ContextManager::~ContextManager() {
  if (stream_) {
    cudaSetDevice(device_id_);
    cudaStreamSynchronize(stream_);
    cudaStreamDestroy(stream_);
  }
}

Status ContextManager::Synchronize() { return FromCuda(cudaStreamSynchronize(stream_)); }

Status TensorAllocator::Alloc(DeviceTensor& t, DType dtype, std::vector<int64_t> shape) {
  t.dtype = dtype;
  t.shape = std::move(shape);
  const size_t bytes = (t.bytes() + 511) / 512 * 512;
  if (bytes == 0) return ERROR_INVALID_PARAM;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    t.data = nullptr;
    return ERROR_DEVICE_MEMORY;
  }
  t.data = p;
  live_[p] = bytes;
  bytes_ += bytes;
  return STATUS_OK;
}

Status TensorAllocator::CopyToDevice(DeviceTensor& t, const void* host, size_t bytes, size_t offset) {
  if (!t.data || !host || offset + bytes > t.bytes()) return ERROR_INVALID_PARAM;
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(static_cast<uint8_t*>(t.data) + offset, host, bytes,
                                          cudaMemcpyHostToDevice, stream_)));
  return FromCuda(cudaStreamSynchronize(stream_));
}

Status TensorAllocator::CopyToHost(void* host, const DeviceTensor& t, size_t bytes, size_t offset) {
  if (!t.data || !host || offset + bytes > t.bytes()) return ERROR_INVALID_PARAM;
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(host, static_cast<const uint8_t*>(t.data) + offset, bytes,
                                          cudaMemcpyDeviceToHost, stream_)));
  return FromCuda(cudaStreamSynchronize(stream_));
}

void TensorAllocator::Free(DeviceTensor& t) {
  auto it = live_.find(t.data);
  if (it != live_.end()) {
    cudaFree(t.data);
    bytes_ -= it->second;
    live_.erase(it);
  }
  t.data = nullptr;
}

void TensorAllocator::Detach(DeviceTensor& t) {
  auto it = live_.find(t.data);
  if (it != live_.end()) {
    bytes_ -= it->second;
    live_.erase(it);
  }
}

void TensorAllocator::FreeAll() {
  for (auto& kv : live_) cudaFree(kv.first);
  live_.clear();
  bytes_ = 0;
}

int EnvInt(const char* name, int dflt) {
  const char* v = std::getenv(name);
  if (!v || !*v) return dflt;
  return std::atoi(v);
}

}  // namespace b200llm
