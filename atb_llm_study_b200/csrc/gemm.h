// Internal C++ interface of the tcgen05 GEMM (the C ABI wraps gemm_run).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

struct GemmPlan {
  bool swap = false;  // weights on the 128-row MMA side, tokens on the N side
  int bn = 256;       // MMA N tile
  int tiles_m = 0, tiles_n = 0;
  int kb_total = 0, kb_per_split = 0, splits = 1;
  int64_t ws_bytes = 0;  // fp32 split-K workspace needed (0 when splits == 1)
};

GemmPlan plan_gemm(int64_t M, int64_t N, int64_t K, int epilogue, int sms);

int gemm_run(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M, int64_t N,
             int64_t K, int epilogue, const void* bias, const void* R, int64_t ldr, void* ws, int64_t ws_bytes,
             cudaStream_t stream);

}  // namespace b200
