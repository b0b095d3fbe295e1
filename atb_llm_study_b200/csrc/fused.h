// Internal launchers for consumers that finish a split-K projection (the
// projection stored fp32 partial tiles [splits][rows][cols]; see gemm.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

// b200_qk_norm_rope, optionally reading the qkv projection from split-K
// partials [splits][T][row_stride] (and writing every head back to qkv).
int qk_norm_rope_launch(void* qkv, int64_t T, int nq, int nkv, int head_dim, int64_t row_stride, const void* q_norm_w,
                        const void* k_norm_w, float eps, const float* cos_tab, const float* sin_tab,
                        const int64_t* slot_mapping, void* k_cache, void* v_cache, int64_t num_blocks, int block_size,
                        const float* partials, int splits, cudaStream_t stream);

// hidden[rows, dim] += sum_s partials[s]; normed = rmsnorm(hidden) * weight.
int splitk_residual_rmsnorm(const float* partials, int splits, int64_t rows, int64_t dim, void* hidden,
                            const void* weight, void* normed, float eps, cudaStream_t stream);

// hidden[rows, dim] = bf16(sum_s partials[s] + bias + hidden) (the split-K
// reduce of a bias + residual projection, same order of additions);
// normed = layernorm(hidden) * gamma + beta, the arithmetic of b200_layernorm.
// B200_ERROR_UNSUPPORTED for dim > 4096 (the caller reduces and normalises
// separately).
int splitk_bias_residual_layernorm(const float* partials, int splits, int64_t rows, int64_t dim, const void* bias,
                                   void* hidden, const void* gamma, const void* beta, void* normed, float eps,
                                   cudaStream_t stream);

// b200_paged_decode, whose last wave of CTAs also pulls `prefetch_bytes` of
// the next projection's weights into L2 (nullptr: none).
int paged_decode_launch(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                        const int32_t* block_tables, int max_blocks_per_seq, const int32_t* context_lens, int batch,
                        int nq, int nkv, int head_dim, int block_size, int64_t num_blocks, float scale, void* out,
                        int64_t out_stride, void* workspace, int64_t workspace_bytes, int max_context,
                        cudaStream_t stream, const void* prefetch, int64_t prefetch_bytes);

}  // namespace b200
