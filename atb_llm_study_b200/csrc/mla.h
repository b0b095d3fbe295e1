// Internal C++ helpers of the latent-attention path (the C ABI is in b200_llm.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

// C[m, n] = sum_k A(m, k) B(k, n) over strided bf16 views (fp32 accumulation,
// strides in elements), batched over `batch` with per-batch offsets *_z.
int mla_absorb(const void* A, int64_t a_sm, int64_t a_sk, int64_t a_z, const void* B, int64_t b_sk, int64_t b_sn,
               int64_t b_z, void* C, int64_t c_sm, int64_t c_sn, int64_t c_z, int M, int N, int K, int batch,
               cudaStream_t st);

// Decompressed keys for prefill: kbuf[t, h, :128] = kvb[t, h*256 : h*256+128]
// (k_nope), kbuf[t, h, 128:192] = kpe[t, :] (the shared roped key dims).
int mla_build_k(const void* kvb, int64_t kvb_stride, const void* kpe, void* kbuf, int64_t T, int nh, cudaStream_t st);

}  // namespace b200
