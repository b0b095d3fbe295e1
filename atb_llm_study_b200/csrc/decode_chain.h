// Internal interface of the decode chain: one persistent launch that runs the
// projections of a dense GQA decoder between two decode attentions.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

// Which phases one chain launch runs (bit set):
//   CHAIN_O   o projection of the attention output, hidden += it, normed =
//             RMSNorm(hidden) * post_norm
//   CHAIN_MLP gate/up projection, SwiGLU, down projection, hidden += it,
//             normed = RMSNorm(hidden) * next_norm (or only the residual add
//             when next_norm is null: the last layer)
//   CHAIN_QKV q/k/v projection of normed, per-head QK RMSNorm + rope, k / v
//             into the paged cache at slot[t], q (and k, v) into qkv rows
enum ChainFlags { CHAIN_O = 1, CHAIN_MLP = 2, CHAIN_QKV = 4 };

struct ChainArgs {
  int flags;
  int64_t T, H, I;  // tokens (<= 64), hidden, intermediate
  int nq, nkv, hd;  // heads (hd 128)
  float eps;
  // weights of this launch's projections (bf16, [out, in] row-major)
  const void* w_o;     // [H, nq*hd]
  const void* w_gu;    // [2I, H], rows 2j / 2j+1 = gate j / up j
  const void* w_down;  // [H, I]
  const void* w_qkv;   // [(nq+2nkv)*hd, H] of the NEXT layer
  const void* post_norm;  // [H]
  const void* next_norm;  // [H] or null
  const void* q_norm;     // [hd] or null (no QK norm)
  const void* k_norm;
  // activations
  const void* attn;  // [T, nq*hd]
  void* hidden;      // [T, H] residual stream
  void* normed;      // [T, H]
  void* act;         // [T, I]
  void* qkv;         // [T, (nq+2nkv)*hd]
  const float* cos_tab;  // [T, hd]
  const float* sin_tab;
  const int64_t* slots;  // [T] (negative = not cached)
  void* k_cache;         // [num_blocks, nkv, block, hd] of the next layer
  void* v_cache;
  int64_t num_blocks;
  int block_size;
  // fp32 split-K partials of each projection and the chain's grid-barrier
  // counters (two uint32 + an abort word, zero before the first launch)
  void* workspace;
  int64_t workspace_bytes;
  unsigned* sync;
};

// Bytes of fp32 partials the chain needs at this shape (0 = unsupported shape).
int64_t chain_workspace_bytes(int64_t T, int64_t H, int64_t I, int nq, int nkv, int hd);

// Launch one chain on `stream` (programmatic dependent launch like every
// kernel here).  Returns a b200_status.
int chain_launch(const ChainArgs& a, cudaStream_t stream);

}  // namespace b200
