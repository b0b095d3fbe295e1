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

// Launch the GEMM.  When the plan splits K, `ws` holds ws_bytes of the plan and
// splits_out is not null, the kernel only stores fp32 partial tiles
// ws[split][M][N] and *splits_out returns the split count: the caller reduces
// them (splitk_reduce, or a consumer kernel that fuses the reduction).
// Otherwise the epilogue is applied and *splits_out = 1.  prefetch /
// prefetch_bytes (optional, 16-byte aligned): the next projection's weights,
// pulled into L2 from this launch's tail so HBM keeps streaming across the
// launch boundary of a decode chain.  sk_flags (optional): sk_flag_count
// ints, zero, which every launch leaves zero; with them a swapped SwiGLU
// projection of at least as many 128-row weight tiles as SMs runs stream-K
// (ws then holds the cut tiles' fp32 partials) and writes its final output
// (*splits_out = 1).
int gemm_launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M, int64_t N,
                int64_t K, int epilogue, const void* bias, const void* R, int64_t ldr, void* ws, int64_t ws_bytes,
                cudaStream_t stream, int* splits_out, const void* prefetch = nullptr, int64_t prefetch_bytes = 0,
                int* sk_flags = nullptr, int sk_flag_count = 0);

// C[M, N'] = epilogue(sum_s ws[s][M][N]).
int splitk_reduce(const float* ws, int splits, int64_t M, int64_t N, int epilogue, const void* bias, const void* R,
                  int64_t ldr, void* C, int64_t ldc, cudaStream_t stream);

// gemm_launch followed by splitk_reduce when K was split (the C ABI call).
// Grouped (per-expert) GEMM: for each group g, rows [goff[g], goff[g+1]) of A
// (goff on the device, e.g. written by the expert permutation) times the
// weights B[g*N:(g+1)*N, :]^T into the same rows of C.  Epilogue NONE or SWIGLU.
int grouped_gemm_launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                        const int32_t* goff, int groups, int64_t rows, int64_t N, int64_t K, int epilogue,
                        cudaStream_t stream);

int gemm_run(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M, int64_t N,
             int64_t K, int epilogue, const void* bias, const void* R, int64_t ldr, void* ws, int64_t ws_bytes,
             cudaStream_t stream);

}  // namespace b200
