// Small device helpers used by the model runner (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200llm {

// x[i] = mean + std * N(0,1) from a counter-based hash of (seed, i); bf16.
int FillNormalBf16(void* x, int64_t n, float mean, float std, uint64_t seed, cudaStream_t st);
// x[r * cols + c] = the value FillNormalBf16(seed) gives global element
// gbase + r * gstride + c: fills a shard (row block / column block) of a
// matrix with exactly the whole matrix's values at those positions.
int FillNormalWindowBf16(void* x, int64_t rows, int64_t cols, float mean, float std, uint64_t seed, int64_t gbase,
                         int64_t gstride, cudaStream_t st);
// x[i] = value; bf16.
int FillConstBf16(void* x, int64_t n, float value, cudaStream_t st);
// out[i, :] = src[idx[i], :]; bf16 rows of width dim (dim % 8 == 0).
int GatherRows(const void* src, const int32_t* idx, int64_t n, int64_t dim, void* out, cudaStream_t st);
// dst[idx[i], :] = src[i, :]; bf16 rows of width dim (dim % 8 == 0), unique idx.
int ScatterRows(void* dst, const int32_t* idx, int64_t n, int64_t dim, const void* src, cudaStream_t st);
// out[:dim] (fp32) = x / sqrt(sum(x^2) + 1e-12) when normalize, else x; one bf16 row.
int PoolL2(const void* x, int64_t dim, int normalize, float* out, cudaStream_t st);

// Per decode row b with cache slot s = seq_slots[b] and p = ctx_lens[s]:
//   positions[plane*B + b] = p (three planes), slots[b] = paged slot of p,
//   ctx_batch[b] = p + 1, bt_batch[b, :] = block_tables[s, :], ctx_lens[s] = p + 1.
// A context that would exceed max_blocks * block_size sets the device error
// word and writes slot -1 (the token is not cached).
int DecodePrepare(const int32_t* seq_slots, int B, int32_t* ctx_lens, const int32_t* block_tables, int max_blocks,
                  int block_size, int64_t* positions, int64_t* slots, int32_t* ctx_batch, int32_t* bt_batch,
                  unsigned* err, cudaStream_t st);

}  // namespace b200llm
