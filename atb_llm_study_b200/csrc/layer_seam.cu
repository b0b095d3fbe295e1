// Whole-layer entry points with the reference's variant-pack input order: the
// drop-in for a caller that builds one decoder layer / one vision block per
// call (TextDecoderLayerGraph::Build + ExecuteOperation,
// atb_cpp_llm/src/components/text/decoder_layer_graph.cpp:13-154 and
// atb_cpp_llm/src/families/base_model.h:91-148; VisionBlockGraph::Build,
// atb_cpp_llm/src/components/vision/vision_block_graph.cpp:12-79).
//
// Each layer is the engine's kernel chain on the caller's stream, with every
// intermediate in the caller's workspace (sized by the *_workspace_bytes
// query, as ExecuteOperation sizes its workspace with Setup first):
//   decoder layer: RMSNorm -> q / k / v projections into one packed row
//     [q | k | v] (three GEMMs writing column ranges, so the caller's separate
//     weights need no concatenation) -> per-head QK RMSNorm + rope -> flash
//     attention over the packed sequences -> o projection with the residual
//     add in its epilogue -> RMSNorm -> gate and up projections -> SiLU(gate)
//     * up -> down projection with the residual add in its epilogue;
//   vision block: LayerNorm -> qkv projection (+bias) -> 2-D rope on the q and
//     k heads -> bidirectional flash attention per sequence -> proj (+bias,
//     +residual) -> LayerNorm -> fc1 (+bias, GELU-tanh) -> fc2 (+bias,
//     +residual).
#include <math.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "gemm.h"

using namespace b200;

#define B200_RETURN_IF_RC(x)      \
  do {                            \
    const int rc_ = (x);          \
    if (rc_ != B200_OK) return rc_; \
  } while (0)

namespace {

// g[t, j] = silu(g[t, j]) * u[t, j] (bf16, 8 per thread, fp32 arithmetic).
__global__ void silu_mul_kernel(__nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ u, int64_t n8) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float a[8], b[8];
  unpack8(reinterpret_cast<const uint4*>(g)[i], a);
  unpack8(reinterpret_cast<const uint4*>(u)[i], b);
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = a[k] / (1.f + __expf(-a[k])) * b[k];
  reinterpret_cast<uint4*>(g)[i] = pack8(a);
}

constexpr int64_t kAlign = 256;
int64_t up(int64_t b) { return (b + kAlign - 1) / kAlign * kAlign; }

// Carves consecutive 256-byte-aligned buffers out of a workspace.
struct Carve {
  uint8_t* base;
  int64_t used = 0;
  void* take(int64_t bytes) {
    void* p = base ? base + used : nullptr;
    used += up(bytes);
    return p;
  }
};

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// cu_seqlens [num_seqs + 1] from host lengths; false when a length is not
// positive or they do not sum to T.
bool prefix(const int32_t* lens, int num_seqs, int64_t T, std::vector<int32_t>& cu, int& max_len) {
  cu.assign(num_seqs + 1, 0);
  max_len = 0;
  int64_t acc = 0;
  for (int i = 0; i < num_seqs; ++i) {
    if (lens[i] <= 0) return false;
    acc += lens[i];
    if (acc > T) return false;
    cu[i + 1] = (int32_t)acc;
    max_len = std::max(max_len, (int)lens[i]);
  }
  return acc == T;
}

int64_t gemm_ws(int64_t M, int64_t N, int64_t K, int epi) { return b200_gemm_workspace_bytes(M, N, K, epi); }

int64_t text_layer_ws(int64_t T, int H, int nq, int nkv, int hd, int I) {
  const int64_t qkv = (int64_t)(nq + 2 * nkv) * hd;
  int64_t g = 0;
  for (int64_t v : {gemm_ws(T, (int64_t)nq * hd, H, 0), gemm_ws(T, (int64_t)nkv * hd, H, 0),
                    gemm_ws(T, H, (int64_t)nq * hd, B200_EPI_RESIDUAL), gemm_ws(T, I, H, 0),
                    gemm_ws(T, H, I, B200_EPI_RESIDUAL)})
    g = std::max(g, v);
  return up((T + 1) * 4) + up(T * H * 2) + up(T * qkv * 2) + up(T * (int64_t)nq * hd * 2) + 2 * up(T * (int64_t)I * 2) +
         up(g);
}

int64_t vision_block_ws(int64_t N, int H, int I) {
  int64_t g = 0;
  for (int64_t v : {gemm_ws(N, 3 * (int64_t)H, H, B200_EPI_BIAS), gemm_ws(N, H, H, B200_EPI_BIAS_RESIDUAL),
                    gemm_ws(N, I, H, B200_EPI_BIAS_GELU), gemm_ws(N, H, I, B200_EPI_BIAS_RESIDUAL)})
    g = std::max(g, v);
  return up((N + 1) * 4) + up(N * H * 2) + up(N * 3 * (int64_t)H * 2) + up(N * (int64_t)H * 2) +
         up(N * (int64_t)I * 2) + up(g);
}

}  // namespace

extern "C" int64_t b200_text_decoder_layer_workspace_bytes(int64_t T, int hidden, int num_heads, int num_kv_heads,
                                                           int head_dim, int intermediate) {
  if (T <= 0 || hidden <= 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || intermediate <= 0) return 0;
  return text_layer_ws(T, hidden, num_heads, num_kv_heads, head_dim, intermediate);
}

extern "C" int b200_text_decoder_layer(const void* const* inputs, int num_inputs, void* output, int64_t T,
                                       int num_seqs, int hidden, int num_heads, int num_kv_heads, int head_dim,
                                       int intermediate, float epsilon, int use_qk_norm, int use_mask,
                                       void* workspace, int64_t workspace_bytes, b200_stream_t stream) {
  if (!inputs || !output || T <= 0 || num_seqs <= 0 || hidden <= 0 || num_heads <= 0 || num_kv_heads <= 0 ||
      num_heads % num_kv_heads || head_dim <= 0 || intermediate <= 0)
    return B200_ERROR_INVALID_PARAM;
  // hidden, q, k, v, o, [qn, kn], gate, up, down, iln, pln, cos, sin, [mask], seqlen
  const int expect = 13 + (use_qk_norm ? 2 : 0) + (use_mask ? 1 : 0);
  if (num_inputs != expect) return B200_ERROR_INVALID_PARAM;
  int i = 0;
  const void* hid = inputs[i++];
  const void* qw = inputs[i++];
  const void* kw = inputs[i++];
  const void* vw = inputs[i++];
  const void* ow = inputs[i++];
  const void* qn = use_qk_norm ? inputs[i++] : nullptr;
  const void* kn = use_qk_norm ? inputs[i++] : nullptr;
  const void* gw = inputs[i++];
  const void* uw = inputs[i++];
  const void* dw = inputs[i++];
  const void* iln = inputs[i++];
  const void* pln = inputs[i++];
  const float* cos_t = static_cast<const float*>(inputs[i++]);
  const float* sin_t = static_cast<const float*>(inputs[i++]);
  if (use_mask) ++i;  // the causal mask: applied as the in-kernel rule (key j masked for query i when j > i)
  const int32_t* seqlen = static_cast<const int32_t*>(inputs[i++]);
  for (const void* p : {hid, qw, kw, vw, ow, gw, uw, dw, iln, pln, (const void*)cos_t, (const void*)sin_t,
                        (const void*)seqlen})
    if (!p) return B200_ERROR_INVALID_PARAM;
  if (use_qk_norm && (!qn || !kn)) return B200_ERROR_INVALID_PARAM;
  if (hidden % 8 || intermediate % 8 || head_dim % 8 || !al16(output) || !al16(workspace))
    return B200_ERROR_INVALID_PARAM;
  if (T > INT32_MAX) return B200_ERROR_UNSUPPORTED;
  std::vector<int32_t> cu;
  int max_len = 0;
  if (!prefix(seqlen, num_seqs, T, cu, max_len)) return B200_ERROR_INVALID_PARAM;
  const int64_t H = hidden, I = intermediate, hd = head_dim, nq = num_heads, nkv = num_kv_heads;
  const int64_t QKV = (nq + 2 * nkv) * hd, AO = nq * hd;
  if (!workspace || workspace_bytes < text_layer_ws(T, hidden, num_heads, num_kv_heads, head_dim, intermediate))
    return B200_ERROR_INVALID_PARAM;
  Carve c{static_cast<uint8_t*>(workspace)};
  int32_t* d_cu = static_cast<int32_t*>(c.take((T + 1) * 4));
  __nv_bfloat16* normed = static_cast<__nv_bfloat16*>(c.take(T * H * 2));
  __nv_bfloat16* qkv = static_cast<__nv_bfloat16*>(c.take(T * QKV * 2));
  __nv_bfloat16* attn = static_cast<__nv_bfloat16*>(c.take(T * AO * 2));
  __nv_bfloat16* g = static_cast<__nv_bfloat16*>(c.take(T * I * 2));
  __nv_bfloat16* u = static_cast<__nv_bfloat16*>(c.take(T * I * 2));
  void* ws = c.take(0);
  const int64_t wsb = workspace_bytes - c.used;
  cudaStream_t st = stream;
  // pageable source: the copy is staged before cudaMemcpyAsync returns
  const cudaError_t ce = cudaMemcpyAsync(d_cu, cu.data(), cu.size() * 4, cudaMemcpyHostToDevice, st);
  if (ce != cudaSuccess) return B200_ERROR_CUDA_BASE - (int)ce;
  B200_RETURN_IF_RC(b200_rmsnorm(hid, nullptr, iln, normed, nullptr, T, H, H, epsilon, st));
  B200_RETURN_IF_RC(gemm_run(normed, H, qw, H, qkv, QKV, T, AO, H, B200_EPI_NONE, nullptr, nullptr, 0, ws, wsb, st));
  B200_RETURN_IF_RC(
      gemm_run(normed, H, kw, H, qkv + AO, QKV, T, nkv * hd, H, B200_EPI_NONE, nullptr, nullptr, 0, ws, wsb, st));
  B200_RETURN_IF_RC(gemm_run(normed, H, vw, H, qkv + AO + nkv * hd, QKV, T, nkv * hd, H, B200_EPI_NONE, nullptr,
                             nullptr, 0, ws, wsb, st));
  B200_RETURN_IF_RC(b200_qk_norm_rope(qkv, T, (int)nq, (int)nkv, (int)hd, QKV, qn, kn, epsilon, cos_t, sin_t, nullptr,
                                      nullptr, nullptr, 0, 0, st));
  B200_RETURN_IF_RC(b200_flash_prefill_packed(qkv, QKV, hd, qkv + AO, QKV, hd, qkv + AO + nkv * hd, QKV, hd, attn, AO,
                                              hd, d_cu, num_seqs, max_len, T, (int)nq, (int)nkv, (int)hd, (int)hd,
                                              1.0f / sqrtf((float)hd), use_mask ? 1 : 0, st));
  // h1 = hidden + o(attn), written to the output (which may alias hidden)
  B200_RETURN_IF_RC(gemm_run(attn, AO, ow, AO, output, H, T, H, AO, B200_EPI_RESIDUAL, nullptr, hid, H, ws, wsb, st));
  B200_RETURN_IF_RC(b200_rmsnorm(output, nullptr, pln, normed, nullptr, T, H, H, epsilon, st));
  B200_RETURN_IF_RC(gemm_run(normed, H, gw, H, g, I, T, I, H, B200_EPI_NONE, nullptr, nullptr, 0, ws, wsb, st));
  B200_RETURN_IF_RC(gemm_run(normed, H, uw, H, u, I, T, I, H, B200_EPI_NONE, nullptr, nullptr, 0, ws, wsb, st));
  const int64_t n8 = T * I / 8;
  launch_kernel(silu_mul_kernel, dim3((unsigned)((n8 + 255) / 256)), 256, 0, st, g, u, n8);
  B200_CHECK_LAUNCH();
  return gemm_run(g, I, dw, I, output, H, T, H, I, B200_EPI_RESIDUAL, nullptr, output, H, ws, wsb, st);
}

extern "C" int64_t b200_vision_block_workspace_bytes(int64_t N, int hidden, int intermediate) {
  if (N <= 0 || hidden <= 0 || intermediate <= 0) return 0;
  return vision_block_ws(N, hidden, intermediate);
}

extern "C" int b200_vision_block(const void* const* inputs, int num_inputs, void* output, int64_t N, int num_seqs,
                                 int hidden, int num_heads, int head_dim, int intermediate, float epsilon,
                                 void* workspace, int64_t workspace_bytes, b200_stream_t stream) {
  if (!inputs || !output || num_inputs != 16 || N <= 0 || num_seqs <= 0 || hidden <= 0 || num_heads <= 0 ||
      head_dim <= 0 || (int64_t)num_heads * head_dim != hidden || intermediate <= 0)
    return B200_ERROR_INVALID_PARAM;
  // hidden, qkv_w, qkv_b, proj_w, proj_b, fc1_w, fc1_b, fc2_w, fc2_b, n1_w, n1_b, n2_w, n2_b, c, s, seq
  for (int i = 0; i < 16; ++i)
    if (!inputs[i]) return B200_ERROR_INVALID_PARAM;
  const void* hid = inputs[0];
  const void *qkv_w = inputs[1], *qkv_b = inputs[2], *proj_w = inputs[3], *proj_b = inputs[4];
  const void *fc1_w = inputs[5], *fc1_b = inputs[6], *fc2_w = inputs[7], *fc2_b = inputs[8];
  const void *n1_w = inputs[9], *n1_b = inputs[10], *n2_w = inputs[11], *n2_b = inputs[12];
  const float* cos_t = static_cast<const float*>(inputs[13]);
  const float* sin_t = static_cast<const float*>(inputs[14]);
  const int32_t* seqlen = static_cast<const int32_t*>(inputs[15]);
  if (hidden % 8 || intermediate % 8 || head_dim % 2 || !al16(output) || !al16(workspace))
    return B200_ERROR_INVALID_PARAM;
  if (N > INT32_MAX) return B200_ERROR_UNSUPPORTED;
  std::vector<int32_t> cu;
  int max_len = 0;
  if (!prefix(seqlen, num_seqs, N, cu, max_len)) return B200_ERROR_INVALID_PARAM;
  const int64_t H = hidden, I = intermediate;
  if (!workspace || workspace_bytes < vision_block_ws(N, hidden, intermediate)) return B200_ERROR_INVALID_PARAM;
  Carve c{static_cast<uint8_t*>(workspace)};
  int32_t* d_cu = static_cast<int32_t*>(c.take((N + 1) * 4));
  __nv_bfloat16* normed = static_cast<__nv_bfloat16*>(c.take(N * H * 2));
  __nv_bfloat16* qkv = static_cast<__nv_bfloat16*>(c.take(N * 3 * H * 2));
  __nv_bfloat16* attn = static_cast<__nv_bfloat16*>(c.take(N * H * 2));
  __nv_bfloat16* f1 = static_cast<__nv_bfloat16*>(c.take(N * I * 2));
  void* ws = c.take(0);
  const int64_t wsb = workspace_bytes - c.used;
  cudaStream_t st = stream;
  const cudaError_t ce = cudaMemcpyAsync(d_cu, cu.data(), cu.size() * 4, cudaMemcpyHostToDevice, st);
  if (ce != cudaSuccess) return B200_ERROR_CUDA_BASE - (int)ce;
  B200_RETURN_IF_RC(b200_layernorm(hid, n1_w, n1_b, normed, N, H, epsilon, st));
  B200_RETURN_IF_RC(gemm_run(normed, H, qkv_w, H, qkv, 3 * H, N, 3 * H, H, B200_EPI_BIAS, qkv_b, nullptr, 0, ws, wsb,
                             st));
  // q heads then k heads: the first 2 * num_heads heads of each qkv row
  B200_RETURN_IF_RC(b200_rope_apply(qkv, N, 2 * num_heads, head_dim, 3 * H, cos_t, sin_t, st));
  B200_RETURN_IF_RC(b200_flash_prefill_packed(qkv, 3 * H, head_dim, qkv + H, 3 * H, head_dim, qkv + 2 * H, 3 * H,
                                              head_dim, attn, H, head_dim, d_cu, num_seqs, max_len, N, num_heads,
                                              num_heads, head_dim, head_dim, 1.0f / sqrtf((float)head_dim), 0, st));
  B200_RETURN_IF_RC(gemm_run(attn, H, proj_w, H, output, H, N, H, H, B200_EPI_BIAS_RESIDUAL, proj_b, hid, H, ws, wsb,
                             st));
  B200_RETURN_IF_RC(b200_layernorm(output, n2_w, n2_b, normed, N, H, epsilon, st));
  B200_RETURN_IF_RC(gemm_run(normed, H, fc1_w, H, f1, I, N, I, H, B200_EPI_BIAS_GELU, fc1_b, nullptr, 0, ws, wsb, st));
  return gemm_run(f1, I, fc2_w, I, output, H, N, H, I, B200_EPI_BIAS_RESIDUAL, fc2_b, output, H, ws, wsb, st);
}
