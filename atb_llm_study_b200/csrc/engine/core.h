// Core runtime of the engine: status codes, device context, tracked device
// allocator.  Same roles and names as the reference's core layer
// (atb_cpp_llm/src/core/context_manager.h, tensor_allocator.h), on CUDA.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "b200_llm.h"

namespace b200llm {

// Mirrors atb_llm::Status (atb_cpp_llm/include/atb_llm/types.h:76-86).
enum Status : int32_t {
  STATUS_OK = 0,
  ERROR_INVALID_PARAM = -1,
  ERROR_FILE_NOT_FOUND = -2,
  ERROR_WEIGHT_LOAD = -3,
  ERROR_GRAPH_BUILD = -4,
  ERROR_DEVICE_MEMORY = -5,
  ERROR_INFERENCE = -6,
  ERROR_UNSUPPORTED = -7,
  ERROR_CUDA_BASE = -1000,
};

inline Status FromCuda(cudaError_t e) { return e == cudaSuccess ? STATUS_OK : (Status)(ERROR_CUDA_BASE - (int)e); }

#define B200_RETURN_IF(expr)              \
  do {                                    \
    int rc__ = (int)(expr);               \
    if (rc__ != 0) return (Status)rc__;   \
  } while (0)

enum class DType : int { BF16 = 0, FP16 = 1, FP32 = 2, INT32 = 3, INT64 = 4 };
size_t DTypeSize(DType t);

// A device buffer with shape; non-owning view (ownership stays with the allocator).
struct DeviceTensor {
  void* data = nullptr;
  DType dtype = DType::BF16;
  std::vector<int64_t> shape;
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return shape.empty() ? 0 : n;
  }
  size_t bytes() const { return (size_t)numel() * DTypeSize(dtype); }
  template <typename T>
  T* as() const { return static_cast<T*>(data); }
};

// One device, one compute stream (the reference binds one stream to its ATB
// context, context_manager.cpp:83-102).
class ContextManager {
 public:
  static Status Create(int device_id, std::unique_ptr<ContextManager>& out);
  ~ContextManager();
  ContextManager(const ContextManager&) = delete;
  ContextManager& operator=(const ContextManager&) = delete;

  cudaStream_t GetStream() const { return stream_; }
  Status Synchronize();
  int GetDeviceId() const { return device_id_; }
  int NumSMs() const { return sms_; }

 private:
  explicit ContextManager(int device_id) : device_id_(device_id) {}
  int device_id_ = 0;
  int sms_ = 0;
  cudaStream_t stream_ = nullptr;
};

// Device allocations, 512-byte aligned (tensor_allocator.cpp:18-204), tracked
// so FreeAll/destructor release everything; Detach hands ownership out.
class TensorAllocator {
 public:
  explicit TensorAllocator(cudaStream_t stream) : stream_(stream) {}
  ~TensorAllocator() { FreeAll(); }
  TensorAllocator(const TensorAllocator&) = delete;
  TensorAllocator& operator=(const TensorAllocator&) = delete;

  Status Alloc(DeviceTensor& t, DType dtype, std::vector<int64_t> shape);
  Status CopyToDevice(DeviceTensor& t, const void* host, size_t bytes, size_t offset = 0);
  Status CopyToHost(void* host, const DeviceTensor& t, size_t bytes, size_t offset = 0);
  void Free(DeviceTensor& t);
  void Detach(DeviceTensor& t);
  void FreeAll();
  size_t BytesInUse() const { return bytes_; }

 private:
  cudaStream_t stream_;
  std::unordered_map<void*, size_t> live_;
  size_t bytes_ = 0;
};

// Environment flag helpers (the reference reads LOG_LEVEL etc. from env / .env,
// atb_cpp_llm/src/utils/dotenv.h:68-190).
int EnvInt(const char* name, int dflt);

}  // namespace b200llm
