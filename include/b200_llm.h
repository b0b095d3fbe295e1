/*
 * b200_llm.h — C ABI of the B200 (sm_100a) transformer-layer library.
 *
 * Every entry point takes raw device pointers, int64 sizes/strides and a CUDA
 * stream, launches asynchronously on that stream and returns an int status
 * (B200_OK or a negative code; shape / alignment violations return
 * B200_ERROR_INVALID_PARAM and launch nothing).  No C++ or torch types cross
 * this boundary and no exception escapes it.
 *
 * Storage type is bf16 (passed as void*); accumulation is fp32.  Each
 * declaration names the reference interface it replaces: the reference
 * (atb_cpp_llm) builds these steps from closed ATB operators created in
 * atb_cpp_llm/src/ops/*.cpp and wired by the graph builders in
 * atb_cpp_llm/src/components/.
 */
#ifndef B200_LLM_H_
#define B200_LLM_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define B200_API __attribute__((visibility("default")))
#else
#define B200_API
#endif

typedef struct CUstream_st* b200_stream_t; /* == cudaStream_t */

/* Status codes mirror atb_llm::Status (atb_cpp_llm/include/atb_llm/types.h:76-86);
 * a CUDA error e is reported as B200_ERROR_CUDA_BASE - e, the way the reference
 * adds the backend's code to ERROR_ATB_BASE (atb_cpp_llm/src/core/context_manager.cpp:97). */
enum b200_status {
  B200_OK = 0,
  B200_ERROR_INVALID_PARAM = -1,
  B200_ERROR_FILE_NOT_FOUND = -2,
  B200_ERROR_WEIGHT_LOAD = -3,
  B200_ERROR_GRAPH_BUILD = -4,
  B200_ERROR_DEVICE_MEMORY = -5,
  B200_ERROR_INFERENCE = -6,
  B200_ERROR_UNSUPPORTED = -7,
  B200_ERROR_CUDA_BASE = -1000
};

/* ---------------------------------------------------------------- library */

/* ABI version of this header (major*100 + minor). */
B200_API int b200_abi_version(void);

/* Read (and optionally clear) the device error word of the current device:
 * bit 0 = a bounded device wait timed out, bit 1 = a device-side index check
 * failed.  Synchronises `stream`.  No reference counterpart: the reference
 * relies on ATB's own status codes (atb_cpp_llm/include/atb_llm/types.h:76-86). */
B200_API int b200_device_error_read(unsigned* out_bits, int clear, b200_stream_t stream);

/* ------------------------------------------------------------ norms / rope */

/* RMSNorm over the last dim, optionally fused with a residual add.
 *   residual == NULL : out = rmsnorm(x) * w                       (NORM)
 *   residual != NULL : h = x + residual; out = rmsnorm(h) * w;
 *                      residual_out (if not NULL) = h              (PRENORM / POSTNORM)
 * x / residual / residual_out / out are [rows, dim] with row stride `stride`
 * (elements); residual_out may alias residual.  dim % 8 == 0.
 * Replaces RmsNormOp::Create (atb_cpp_llm/src/ops/rms_norm_op.cpp:7-19) and
 * RmsNormGraph::Build (atb_cpp_llm/src/components/common/rms_norm_graph.cpp:59-84). */
B200_API int b200_rmsnorm(const void* x, const void* residual, const void* weight, void* out, void* residual_out,
                 int64_t rows, int64_t dim, int64_t stride, float eps, b200_stream_t stream);

/* LayerNorm with gamma/beta over the last dim ([rows, dim], contiguous, dim % 8 == 0).
 * Replaces LayerNormOp::Create (atb_cpp_llm/src/ops/layer_norm_op.cpp:7-22). */
B200_API int b200_layernorm(const void* x, const void* gamma, const void* beta, void* out, int64_t rows, int64_t dim,
                   float eps, b200_stream_t stream);

/* cos/sin tables [T, head_dim] (fp32) for interleaved 3-section mrope from
 * position ids [3, T] (int64, planes t, h, w).
 * Replaces MRoPE::Compute (atb_cpp_llm/src/components/common/mrope.cpp:27-96). */
B200_API int b200_rope_table_mrope(const int64_t* position_ids, int64_t T, int head_dim, float theta, int section_t,
                          int section_h, int section_w, float* cos_out, float* sin_out, b200_stream_t stream);

/* Host function (no GPU): 3-D position ids [3, batch, seq_len] (int64,
 * bit-exact) of text + image sequences.  Text runs are consecutive; the image
 * tokens after a vision-start token take their merged (t, h, w) grid offsets
 * from the running position, and the next run starts max(t, h/merge, w/merge)
 * later.  Images are taken from image_grid_thw [num_images, 3] in order;
 * tokens outside attention_mask (optional [batch, seq_len]) get 1.
 * Replaces GetRopeIndex (atb_cpp_llm/src/components/common/mrope.cpp:234-348). */
B200_API int b200_get_rope_index(const int64_t* input_ids, int64_t batch, int64_t seq_len,
                                 const int64_t* attention_mask, const int64_t* image_grid_thw, int64_t num_images,
                                 int64_t image_token_id, int64_t vision_start_token_id, int64_t spatial_merge_size,
                                 int64_t* position_ids);

/* b200_get_rope_index on the GPU: input_ids, attention_mask (or NULL),
 * image_grid_thw and position_ids are device arrays; the same positions,
 * bit for bit (one CTA walks the rows; block scans compact the mask and find
 * the image runs).  workspace: b200_rope_index_workspace_bytes(seq_len).
 * Grids with a zero or negative dimension (which the host call rejects) set
 * the device error word and end that row's image layout. */
B200_API int64_t b200_rope_index_workspace_bytes(int64_t seq_len);
B200_API int b200_get_rope_index_device(const int64_t* input_ids, int64_t batch, int64_t seq_len,
                                        const int64_t* attention_mask, const int64_t* image_grid_thw,
                                        int64_t num_images, int64_t image_token_id, int64_t vision_start_token_id,
                                        int64_t spatial_merge_size, int64_t* position_ids, void* workspace,
                                        int64_t workspace_bytes, b200_stream_t stream);

/* cos/sin tables [T, head_dim] (fp32) for standard 1-D rope from positions [T].
 * Replaces Rope1D::Compute (atb_cpp_llm/src/components/common/rope_1d.h:23-167). */
B200_API int b200_rope_table_1d(const int64_t* positions, int64_t T, int head_dim, float theta, float* cos_out,
                       float* sin_out, b200_stream_t stream);

/* cos/sin tables [T, head_dim] (fp32) of the 2-D vision rope for num_images
 * grids grid_thw [num_images, 3] (host, t/h/w in patches; h, w multiples of
 * merge_size; at most 64 images), tokens in merge-block order:
 * freq = cat(row * inv_freq, col * inv_freq), inv_freq over head_dim/2 with
 * step 2, emb = cat(freq, freq).  Replaces ComputeVisionRotPosEmb
 * (atb_cpp_llm/src/components/common/mrope.cpp:155-228) and VisRopeGraph
 * (atb_cpp_llm/src/components/vision/vis_rope_npu_graph.cpp:18-139). */
B200_API int b200_rope_table_vision(const int64_t* grid_thw, int num_images, int merge_size, int head_dim,
                                    float theta, float* cos_out, float* sin_out, b200_stream_t stream);

/* In place half rotation x*cos + cat(-x2, x1)*sin on `nheads` consecutive
 * heads of each row of x [T, stride] (any even head_dim), cos/sin [T, head_dim].
 * Replaces RopeOp::Create(rotaryCoeff=2) where no per-head norm precedes it
 * (atb_cpp_llm/src/components/vision/vision_attention_graph.cpp:71). */
B200_API int b200_rope_apply(void* x, int64_t T, int nheads, int head_dim, int64_t stride, const float* cos_tab,
                             const float* sin_tab, b200_stream_t stream);

/* out[t] (+)= bilinear interpolation of the learned [num_grid^2, dim] position
 * table at token t's patch position (tokens of grid_thw in merge-block order;
 * accumulate != 0 adds onto out, e.g. the patch embeddings).  Replaces
 * ComputePosEmbedInterp / PosEmbedInterpGraph
 * (atb_cpp_llm/src/components/vision/pos_embed_interp.cpp:10-90,
 * atb_cpp_llm/src/components/vision/pos_embed_npu_graph.cpp:19-211). */
B200_API int b200_pos_embed_interp(const void* table, int num_grid, int64_t dim, const int64_t* grid_thw,
                                   int num_images, int merge_size, void* out, int accumulate, b200_stream_t stream);

/* In place on the fused projection output qkv [T, row_stride] laid out as
 * [q heads | k heads | v heads] x head_dim: per-head RMSNorm of q and k
 * (skipped when the norm weight is NULL), then the half rotation
 * x*cos + cat(-x2, x1)*sin with cos/sin [T, head_dim] fp32.  When
 * slot_mapping is not NULL, the rotated k and the untouched v of token t are
 * also written to k_cache / v_cache ([num_blocks, nkv, block_size, head_dim])
 * at slot slot_mapping[t] (negative slot = skip).
 * Replaces the RmsNorm -> Rope steps of GqaAttentionBuilder::Build
 * (atb_cpp_llm/src/components/common/gqa_attention_builder.cpp:60-130) and
 * RopeOp::Create(rotaryCoeff=2) (atb_cpp_llm/src/ops/rope_op.cpp:7-18). */
B200_API int b200_qk_norm_rope(void* qkv, int64_t T, int nq, int nkv, int head_dim, int64_t row_stride,
                      const void* q_norm_w, const void* k_norm_w, float eps, const float* cos_tab,
                      const float* sin_tab, const int64_t* slot_mapping, void* k_cache, void* v_cache,
                      int64_t num_blocks, int block_size, b200_stream_t stream);

/* ------------------------------------------------------------------- GEMM */

enum b200_epilogue {
  B200_EPI_NONE = 0,          /* C = A B^T                                   */
  B200_EPI_BIAS = 1,          /* C = A B^T + bias[n]                         */
  B200_EPI_RESIDUAL = 2,      /* C = A B^T + R[m, n]   (R may alias C)       */
  B200_EPI_SWIGLU = 3,        /* rows of B interleave gate/up: C[m, j] = silu(G[m,2j]) * G[m,2j+1], C is [M, N/2] */
  B200_EPI_BIAS_GELU = 4,     /* C = gelu_tanh(A B^T + bias[n])              */
  B200_EPI_BIAS_RESIDUAL = 5  /* C = A B^T + bias[n] + R[m, n]               */
};

/* C[M, N] = epilogue(A[M, K] * B[N, K]^T), bf16 in / fp32 accumulate / bf16 out,
 * on tcgen05 tensor cores with TMEM accumulators and TMA-fed shared memory.
 * Row strides lda/ldb/ldc/ldr in elements; K, lda, ldb, ldc, ldr multiples of 8;
 * 16-byte aligned base pointers.  `workspace` (may be NULL) enables split-K
 * for skinny problems; b200_gemm_workspace_bytes() gives the size it can use.
 * With split-K each K slice stores its fp32 partial tile in the workspace and
 * a second kernel sums them and applies the epilogue; calls that overlap on
 * the GPU must not share a workspace.
 * Replaces LinearOp::Create(transB=true) (atb_cpp_llm/src/ops/linear_op.cpp:7-20)
 * and the SiLU/Mul/Add ops fused into its consumers
 * (atb_cpp_llm/src/components/common/mlp_builder.cpp:12-56). */
B200_API int b200_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, int64_t M,
                   int64_t N, int64_t K, int epilogue, const void* bias, const void* residual, int64_t ldr,
                   void* workspace, int64_t workspace_bytes, b200_stream_t stream);

/* Bytes of workspace b200_gemm_bf16 uses for split-K at this shape (0 = none). */
B200_API int64_t b200_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int epilogue);

/* ---------------------------------------------------------------- experts */

/* Grouped expert GEMM: for each group g < groups (<= 256), the rows
 * [group_offsets[g], group_offsets[g+1]) of A ([rows, K], the tokens routed to
 * expert g) times B[g*N:(g+1)*N, :]^T into the same rows of C.  group_offsets
 * ([groups + 1], int32) is read on the device, so it can come straight from
 * b200_moe_permute.  Epilogue NONE or SWIGLU (gate/up rows interleaved as in
 * b200_gemm_bf16; C then has N/2 columns).  Fills the grouped expert GEMMs the
 * reference leaves to its MoE stubs (MoeBuilder,
 * atb_cpp_llm/src/components/common/mlp_builder.h:73-82; MoEMlpGraph,
 * atb_cpp_llm/src/components/moe/moe_mlp_graph.h:22-29). */
B200_API int b200_grouped_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                                    const int32_t* group_offsets, int groups, int64_t rows, int64_t N, int64_t K,
                                    int epilogue, b200_stream_t stream);

/* Router: logits = x [T, H] (bf16, row stride ldx) . gate_weight [E, H]^T in
 * fp32, softmax over the E (<= 128) experts, the top_k (<= 8) largest logits
 * (ties to the lower expert index) -> topk_ids [T, top_k] (int32, in
 * descending order) and topk_weights [T, top_k] (fp32): the chosen softmax
 * probabilities renormalised to sum 1 when `renormalize` (Mixtral), else
 * multiplied by `scale` (DeepSeek routed_scaling_factor).  logits [T, E] (fp32)
 * is written when not NULL.  Fills MlpConfig.num_experts / top_k
 * (atb_cpp_llm/include/atb_llm/layer_desc.h:59-60), which the reference never
 * routes. */
B200_API int b200_moe_route(const void* x, int64_t ldx, const void* gate_weight, int64_t T, int64_t H,
                            int num_experts, int top_k, int renormalize, float scale, int32_t* topk_ids,
                            float* topk_weights, float* logits, b200_stream_t stream);

/* The selection of b200_moe_route from given fp32 logits [T, E]. */
B200_API int b200_moe_topk(const float* logits, int64_t T, int num_experts, int top_k, int renormalize, float scale,
                           int32_t* topk_ids, float* topk_weights, b200_stream_t stream);

/* Expert permutation of the T*top_k (token, choice) entries: entry i = t*top_k
 * + j goes to slot perm_pos[i] = expert_offsets[e] + (entries of expert e
 * before i), so each expert's slots hold its tokens in token order
 * (deterministic, bit-exact); perm_src[slot] = t; expert_offsets [E + 1].
 * When x_perm is not NULL, x_perm[slot, :] = x[t, :] (bf16, H columns).
 * Workspace: b200_moe_permute_workspace_bytes().  Out-of-range expert ids set
 * the device error word and get perm_pos = -1. */
B200_API int64_t b200_moe_permute_workspace_bytes(int64_t T, int top_k, int num_experts);
B200_API int b200_moe_permute(const int32_t* topk_ids, int64_t T, int top_k, int num_experts, const void* x,
                              int64_t ldx, int64_t H, void* x_perm, int32_t* expert_offsets, int32_t* perm_pos,
                              int32_t* perm_src, void* workspace, int64_t workspace_bytes, b200_stream_t stream);

/* out[t] = residual[t] + shared[t] + sum_j topk_weights[t, j] * y_perm[perm_pos[t*top_k + j]]
 * (fp32, one rounding to bf16; residual / shared optional, out may alias
 * residual); when norm_weight is not NULL also normed[t] = RMSNorm(out[t]) *
 * norm_weight (the next layer's input norm).  H <= 8192. */
B200_API int b200_moe_combine(const void* y_perm, const int32_t* perm_pos, const float* topk_weights, int64_t T,
                              int top_k, int64_t H, const void* residual, const void* shared, void* out,
                              const void* norm_weight, void* normed, float eps, b200_stream_t stream);

/* -------------------------------------------------------------- attention */

/* Prefill attention over packed sequences: softmax(q k^T * scale [+ causal]) v,
 * GQA with nq % nkv == 0.  Sequence i owns rows cu_seqlens[i]..cu_seqlens[i+1]
 * of q [T, q_stride], k/v [T, kv_stride] (head h at column h*head_dim) and of
 * out [T, out_stride].  head_dim in {16, 32, 64, 128}.  The causal rule (key j
 * masked for query i when j > i) is applied in-kernel; no S x S mask exists.
 * Replaces SelfAttentionOp::Create (PA_ENCODER, BSND, MASK_TYPE_NORM)
 * (atb_cpp_llm/src/ops/self_attention_op.cpp:8-30) fed by
 * MakeCausalMaskFp16 (atb_cpp_llm/src/runners/text_runner.cpp:74-85). */
B200_API int b200_flash_prefill(const void* q, int64_t q_stride, const void* k, const void* v, int64_t kv_stride,
                       void* out, int64_t out_stride, const int32_t* cu_seqlens, int num_seqs, int max_seqlen,
                       int nq, int nkv, int head_dim, float scale, int causal, b200_stream_t stream);

/* b200_flash_prefill with a row and a head stride per operand (elements) and
 * separate query/key and value head widths: (qk, v) in {(16,16), (32,32),
 * (64,64), (128,128), (192,128)} — the last is a decompressed MLA head
 * (128 no-rope + 64 rope dims against 128 value dims).  Same causal rule. */
B200_API int b200_flash_prefill_ex(const void* q, int64_t q_stride, int64_t q_head_stride, const void* k,
                                   int64_t k_stride, int64_t k_head_stride, const void* v, int64_t v_stride,
                                   int64_t v_head_stride, void* out, int64_t out_stride, int64_t out_head_stride,
                                   const int32_t* cu_seqlens, int num_seqs, int max_seqlen, int nq, int nkv,
                                   int head_dim_qk, int head_dim_v, float scale, int causal, b200_stream_t stream);

/* b200_flash_prefill_ex for callers that know the packed row count on the
 * host (total_tokens = cu_seqlens[num_seqs]).  64- and 128-wide heads and
 * latent attention's decompressed heads (192-wide query / key, 128-wide value)
 * run on the tcgen05 tensor cores: 128 query rows per CTA, K/V tiles of 128 keys by TMA
 * (tile reads stop at total_tokens and at each operand's last head), scores
 * and the output accumulator in TMEM, the running max moved only when it grows
 * by more than 2^8 (exact rescaling, rarely needed).  Other head widths, or
 * total_tokens <= 0, run b200_flash_prefill_ex.  Same causal rule. */
B200_API int b200_flash_prefill_packed(const void* q, int64_t q_stride, int64_t q_head_stride, const void* k,
                                       int64_t k_stride, int64_t k_head_stride, const void* v, int64_t v_stride,
                                       int64_t v_head_stride, void* out, int64_t out_stride, int64_t out_head_stride,
                                       const int32_t* cu_seqlens, int num_seqs, int max_seqlen, int64_t total_tokens,
                                       int nq, int nkv, int head_dim_qk, int head_dim_v, float scale, int causal,
                                       b200_stream_t stream);

/* ---- multi-head latent attention (DeepSeek-V2): fills the reference's stubs
 * MlaAttentionBuilder (atb_cpp_llm/src/components/common/attention_builder.h:60-69)
 * and AttnConfig.kv_lora_rank / q_lora_rank (atb_cpp_llm/include/atb_llm/layer_desc.h:47-49).
 * Latent cache: [num_blocks * block_size, 576] bf16 — per token the 512
 * normalised compressed-KV values, then the 64 roped key dims shared by all
 * heads. */

/* Per token t < T: c = RMSNorm(kv_a[t, :512]) * kv_norm_weight and k_pe =
 * rope(kv_a[t, 512:576]) into latent-cache row slot_mapping[t] (skipped when
 * slot_mapping is NULL or the slot is -1) and into ckv_out [T, 512] /
 * kpe_out [T, 64] when not NULL; the 64 rope dims at q_rope_offset of each
 * of the num_heads query heads (head stride q_head_stride) are rotated in
 * place.  Rope pairs are the interleaved (2i, 2i+1) of the projection, stored
 * de-interleaved (DeepSeek-V2's layout); cos/sin [T, 64] from
 * b200_rope_table_freqs. */
B200_API int b200_mla_prep(void* q, int64_t q_stride, int64_t q_head_stride, int num_heads, int q_rope_offset,
                           const void* kv_a, int64_t kv_a_stride, const void* kv_norm_weight, float eps,
                           const float* cos_tab, const float* sin_tab, const int64_t* slot_mapping,
                           void* latent_cache, int64_t num_slots, void* ckv_out, void* kpe_out, int64_t T,
                           b200_stream_t stream);

/* Absorbed-latent decode attention: q [batch, q_stride] holds per head (576
 * wide) the query projected into the latent space (512) then its roped dims
 * (64); out [batch, out_stride] receives per head (512 wide) sum_t softmax_t
 * (q . cache_t * scale) cache_t[:512].  num_heads % 16 == 0, block_size % 64
 * == 0; workspace (b200_mla_decode_workspace_bytes) enables splitting the
 * context across CTAs. */
B200_API int b200_mla_decode(const void* q, int64_t q_stride, const void* latent_cache, const int32_t* block_tables,
                             int max_blocks_per_seq, const int32_t* context_lens, int batch, int num_heads,
                             int block_size, int64_t num_blocks, float scale, void* out, int64_t out_stride,
                             void* workspace, int64_t workspace_bytes, int max_context, b200_stream_t stream);
B200_API int64_t b200_mla_decode_workspace_bytes(int batch, int num_heads, int max_context);

/* cos/sin tables [T, rot_dim] (fp32) = cos/sin(positions[t] * inv_freq[i]) *
 * mscale, i = d mod rot_dim/2, for a host array of rot_dim/2 (<= 128)
 * frequencies — e.g. DeepSeek-V2's YaRN-scaled ones. */
B200_API int b200_rope_table_freqs(const int64_t* positions, int64_t T, int rot_dim, const float* inv_freq,
                                   float mscale, float* cos_out, float* sin_out, b200_stream_t stream);

/* Single-token decode attention over a paged KV cache
 * (k_cache/v_cache [num_blocks, nkv, block_size, head_dim], block_size 128 or 64):
 * sequence b attends to its first context_lens[b] cached positions through
 * block_tables[b, 0..max_blocks_per_seq).  q [batch, q_stride] (head h at h*head_dim),
 * out [batch, out_stride].  head_dim == 128.  Uses split-KV with `workspace`
 * (size from b200_paged_decode_workspace_bytes; NULL disables splitting).
 * No reference counterpart: the reference's KV cache is a stub
 * (atb_cpp_llm/include/atb_llm/kv_cache.h:23-35, atb_cpp_llm/src/core/kv_cache_manager.h:25-76). */
B200_API int b200_paged_decode(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                      const int32_t* block_tables, int max_blocks_per_seq, const int32_t* context_lens, int batch,
                      int nq, int nkv, int head_dim, int block_size, int64_t num_blocks, float scale, void* out,
                      int64_t out_stride, void* workspace, int64_t workspace_bytes, int max_context,
                      b200_stream_t stream);

B200_API int64_t b200_paged_decode_workspace_bytes(int batch, int nq, int head_dim, int max_context);

/* b200_paged_decode for callers that cannot allocate device memory — for
 * example code running as an operator inside another framework whose memory
 * pool owns the GPU and forbids raw cudaMalloc, or a serving loop that froze
 * its memory plan at start-up.  It takes no workspace and allocates nothing:
 * the split-KV scratch is a fixed 8 MiB array compiled into this library,
 * held on every GPU that loads it until the process exits
 * (b200_paged_decode_noalloc_max_scratch_bytes()).  Inputs and outputs are
 * the caller's, with the same meaning and limits as b200_paged_decode.  The
 * scratch a call needs is batch x nq x splits x (head_dim + 1) x 4 bytes,
 * where splits is the KV split count the kernel picks (1 = no scratch, e.g.
 * batch 64 x 8 kv heads; 5 for batch 8 x 8 kv heads at context 2048, i.e.
 * 660 KB); a call that would need more than 8 MiB is rejected with
 * B200_ERROR_INVALID_PARAM before anything is launched.
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  All calls share the one array and it keeps the
 * last call's contents (nothing in it needs to start at zero: each call
 * writes every scratch entry it reads), so calls whose executions overlap on
 * the GPU — on different streams, or on several host threads — race and must
 * be serialised by the caller.
 * This entry point has no counterpart in the reference. */
B200_API int b200_paged_decode_noalloc(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                                       const int32_t* block_tables, int max_blocks_per_seq,
                                       const int32_t* context_lens, int batch, int nq, int nkv, int head_dim,
                                       int block_size, int64_t num_blocks, float scale, void* out,
                                       int64_t out_stride, int max_context, b200_stream_t stream);
B200_API int64_t b200_paged_decode_noalloc_max_scratch_bytes(void);

/* slots[t] = block_tables[seq_ids[t], positions[t] / block_size] * block_size
 *            + positions[t] % block_size   (int64, bit-exact).
 * No reference counterpart (the reference has no paged KV cache,
 * atb_cpp_llm/include/atb_llm/kv_cache.h:23-35). */
B200_API int b200_slot_mapping(const int32_t* block_tables, int max_blocks_per_seq, const int32_t* seq_ids,
                      const int64_t* positions, int64_t T, int block_size, int64_t* slots, b200_stream_t stream);

/* ------------------------------------------------------------ elementwise */

/* out[t] = table[ids[t]] ([vocab, dim] bf16); ids outside [0, vocab) give zeros.
 * Replaces BaseModel::EmbeddingLookup (atb_cpp_llm/src/families/base_model.cpp:99-116),
 * which the reference runs on the host. */
B200_API int b200_embedding(const int64_t* ids, int64_t T, const void* table, int64_t vocab, int64_t dim, void* out,
                   b200_stream_t stream);

/* hidden[idx[i], :] += alpha * feat[i, :] for i < n (hidden [rows, dim]); indices
 * must be unique.  Replaces IndexAddOp (atb_cpp_llm/src/ops/index_add_op.cpp:7-19)
 * as used by DeepstackFusion::InjectFeatures
 * (atb_cpp_llm/src/components/common/deepstack_fusion.cpp:188-195). */
B200_API int b200_scatter_add_rows(void* hidden, int64_t rows, int64_t dim, const int32_t* idx, const void* feat, int64_t n,
                          float alpha, b200_stream_t stream);

/* out[r] = argmax_j logits[r, j] (lowest index on ties), logits [rows, vocab] bf16. */
B200_API int b200_argmax(const void* logits, int64_t rows, int64_t vocab, int64_t ld, int64_t* out, b200_stream_t stream);

/* -------------------------------------------------------- image preprocess */

/* Qwen3-VL SmartResize (host, no GPU): the nearest multiple of factor per
 * side (size / factor rounded half to even in float32), scaled down to
 * max_pixels or up to min_pixels when outside (factor = patch * merge).
 * Same result as SmartResize (atb_cpp_llm/src/adapters/qwen3vl_embedding/
 * qwen3vl_preprocess.cpp:219-243). */
B200_API int b200_smart_resize(int height, int width, int factor, int min_pixels, int max_pixels, int* new_height,
                               int* new_width);
/* Device scratch for one resize of a [C, H, W] image to (new_h, new_w):
 * both axes' fixed-point coefficients and the horizontal-pass image. */
B200_API int64_t b200_preprocess_workspace_bytes(int channels, int height, int width, int new_height,
                                                 int new_width);
/* Pillow's BICUBIC Image.resize on 8-bit planes, bit-exact: image [C, H, W]
 * uint8 (device) -> out [C, out_h, out_w] uint8 (device).  Antialiased
 * (support 2 x max(1, in/out)), coefficients quantised to 22 fractional bits,
 * horizontal then vertical pass each clipped to [0, 255], an unchanged axis
 * not resampled.  Replaces BicubicResize / ResampleCore8bpc
 * (qwen3vl_preprocess.cpp:52-207) and the device path of PreprocessImageNpu
 * (qwen3vl_preprocess.cpp:369-824). */
B200_API int b200_bicubic_resize_u8(const uint8_t* image, int channels, int height, int width, int out_h, int out_w,
                                    uint8_t* out, void* workspace, int64_t workspace_bytes, b200_stream_t stream);
/* The whole Qwen3-VL processor on the GPU: SmartResize, the bicubic resample,
 * (v/255 - mean[c]) / std[c] in float32 (mean / std NULL: 0.5), and the
 * patchify in merge-block order with the frame duplicated over the temporal
 * patch, written as pixel_values [num_patches, C*tp*ps*ps] (out_dtype 1:
 * fp16 as the reference, 0: bf16) on the device.  num_patches and grid_thw
 * [3] = (1, new_h/ps, new_w/ps) are host outputs, known before the kernels
 * run.  Replaces PreprocessImage (qwen3vl_preprocess.cpp:245-366); fp16
 * output equals the reference's bit for bit.  workspace: at least
 * b200_preprocess_workspace_bytes(C, H, W, new_h, new_w) (256-byte aligned). */
B200_API int b200_preprocess_image(const uint8_t* image, int channels, int height, int width, int patch_size,
                                   int temporal_patch_size, int merge_size, int min_pixels, int max_pixels,
                                   const float* mean, const float* stdv, int out_dtype, void* pixel_values,
                                   int64_t pixel_capacity, int64_t* num_patches, int64_t* grid_thw, void* workspace,
                                   int64_t workspace_bytes, b200_stream_t stream);

/* --------------------------------------------------------- tensor parallel */

/* A tensor-parallel group of `world` (<= 8) processes, one GPU each: an NCCL
 * communicator for large all-reduces and a symmetric device buffer that every
 * rank maps over NVLink (CUDA IPC) for the fused decode-sized ones.
 * Bootstrap: rank 0 calls b200_comm_unique_id and shares the 128 bytes;
 * every rank calls b200_comm_create (collective), shares its 64-byte
 * b200_comm_ipc_handle, then calls b200_comm_connect with all ranks' handles
 * concatenated in rank order.  No reference counterpart: the reference runs
 * on one device (tensor and expert parallelism are new here). */
typedef struct b200_comm_s* b200_comm_t;
B200_API int b200_comm_unique_id(void* nccl_id_out);
B200_API int b200_comm_create(int world, int rank, int device, const void* nccl_id, int64_t symmetric_bytes,
                              b200_comm_t* out);
B200_API int b200_comm_ipc_handle(b200_comm_t comm, void* handle_out);
B200_API int b200_comm_connect(b200_comm_t comm, const void* all_handles);
B200_API int b200_comm_destroy(b200_comm_t comm);
/* world, rank, and this rank's two partial-sum buffers (parity 0 / 1) of buffer_bytes each. */
B200_API int b200_comm_info(b200_comm_t comm, int* world, int* rank, void** buffer0, void** buffer1,
                            int64_t* buffer_bytes);
/* In-place sum over the group (NCCL, bf16). */
B200_API int b200_comm_allreduce_bf16(b200_comm_t comm, void* buf, int64_t count, b200_stream_t stream);
/* recv [world * count] = every rank's send [count] in rank order (NCCL, bf16). */
B200_API int b200_comm_allgather_bf16(b200_comm_t comm, const void* send, void* recv, int64_t count,
                                      b200_stream_t stream);
/* Fused decode all-reduce: each rank's partial rows [T, H] already sit in its
 * buffer `parity`; every rank computes hidden[t] += sum over ranks (rank order,
 * fp32, identical on all ranks) and, when norm_weight is not NULL, normed[t] =
 * RMSNorm(hidden[t]) * norm_weight — reading the peers' partials over NVLink,
 * with a bounded wait on the peers' epoch flags (timeouts set the device error
 * word).  Consecutive calls must alternate parity. */
B200_API int b200_comm_allreduce_rmsnorm(b200_comm_t comm, int parity, int64_t T, int64_t H, void* hidden,
                                         const void* norm_weight, void* normed, float eps, b200_stream_t stream);
/* Vocabulary-parallel greedy token: logits [rows, vocab_local] (row stride ld)
 * are this rank's shard (rank r holds global ids r*vocab_local ..); out[rows]
 * = the global argmax (lowest id on ties), identical on every rank. */
B200_API int b200_comm_argmax(b200_comm_t comm, const void* logits, int64_t rows, int64_t vocab_local, int64_t ld,
                              int64_t* out, b200_stream_t stream);

/* ---------------------------------------------------------- expert parallel */

/* Expert-parallel token exchange over a connected b200_comm_t (experts split
 * into equal blocks: rank d owns experts [d*E/P, (d+1)*E/P)).  Collective:
 * every rank calls dispatch, then combine, once per MoE layer, in the same
 * order, even with no tokens of its own.  No reference counterpart (the
 * reference declares EP but runs one device: layer_desc.h:59-60).
 *
 * Dispatch: send_offsets [E+1] (int32) and send_rows [send_cap, H] (bf16) are
 * this rank's rows grouped by expert (b200_moe_permute's output); both must
 * lie in the communicator's symmetric buffers (b200_comm_info), at the same
 * offsets on every rank.  After a bounded wait for every rank's rows, this
 * rank copies the rows of its own experts from every source over NVLink into
 * recv_rows [recv_cap, H] — expert-major, then source rank, then the source's
 * row order — and writes recv_offsets [E/P + 1] (the grouped GEMM's group
 * offsets) and row_base [E] (where this rank's first row of expert e sits in
 * the owner's receive buffer; read by the combine).  recv_cap must cover the
 * worst case (P * tokens * top_k) or rows are dropped and the device error
 * word is set. */
B200_API int b200_ep_dispatch(b200_comm_t comm, const int32_t* send_offsets, const void* send_rows, int64_t send_cap,
                              int64_t experts, int64_t H, void* recv_rows, int64_t recv_cap, int32_t* recv_offsets,
                              int32_t* row_base, b200_stream_t stream);
/* Combine: results [recv_cap, H] (bf16, in the symmetric buffers) are this
 * rank's expert outputs for its received rows; top_k <= 8.  After a bounded wait for every
 * rank's results, out[t] = residual[t] + shared[t] + sum_j w[t,j] *
 * y(t, j) (fp32, choices in order, one rounding), y read from the owner of
 * expert topk_ids[t,j] at row row_base[e] + perm_pos[t*k+j] - send_offsets[e];
 * normed[t] = RMSNorm(out[t]) * norm_weight when norm_weight is not NULL.
 * residual / shared may be NULL; out may alias residual. */
B200_API int b200_ep_combine(b200_comm_t comm, const void* results, int64_t recv_cap, const int32_t* row_base,
                             const int32_t* send_offsets, const int32_t* topk_ids, const float* topk_weights,
                             const int32_t* perm_pos, int64_t T, int top_k, int64_t experts, int64_t H,
                             const void* residual, const void* shared, void* out, const void* norm_weight,
                             void* normed, float eps, b200_stream_t stream);

/* -------------------------------------------------------- layer-graph seam */

/* One pre-norm decoder layer, inputs in the reference's variant-pack order:
 *   inputs[] = hidden [T, H], q_w [nq*hd, H], k_w [nkv*hd, H], v_w [nkv*hd, H],
 *              o_w [H, nq*hd], (q_norm_w [hd], k_norm_w [hd] when use_qk_norm),
 *              gate_w [I, H], up_w [I, H], down_w [H, I], input_ln_w [H],
 *              post_ln_w [H]                    (bf16, device),
 *              cos, sin [T, hd]                 (fp32, device; rotation over the whole head),
 *              (mask when use_mask; never read),
 *              seqlen [num_seqs]                (int32, HOST; lengths of the packed sequences, sum T)
 * num_inputs = 13 + 2 * use_qk_norm + use_mask (15 / 16 with QK norm, as
 * the reference's graph).  use_mask != 0 gives causal attention (key j masked
 * for query i when j > i, the only mask the reference builds,
 * MakeCausalMaskFp16, atb_cpp_llm/src/runners/text_runner.cpp:74-85; its
 * tensor is not read); use_mask == 0 attends over the whole sequence.
 * output [T, H] bf16 (may alias hidden).  out = h1 + down(silu(gate n2) * up n2),
 * h1 = hidden + o(attn(rope(qknorm(qkv(n1))))), n1 / n2 the RMSNorms.
 * workspace >= b200_text_decoder_layer_workspace_bytes (256-byte aligned);
 * calls sharing a workspace must not overlap on the GPU.
 * Replaces TextDecoderLayerGraph::Build + ExecuteOperation
 * (atb_cpp_llm/src/components/text/decoder_layer_graph.cpp:13-154,
 * atb_cpp_llm/src/families/base_model.h:91-148). */
B200_API int64_t b200_text_decoder_layer_workspace_bytes(int64_t T, int hidden, int num_heads, int num_kv_heads,
                                                         int head_dim, int intermediate);
B200_API int b200_text_decoder_layer(const void* const* inputs, int num_inputs, void* output, int64_t T,
                                     int num_seqs, int hidden, int num_heads, int num_kv_heads, int head_dim,
                                     int intermediate, float epsilon, int use_qk_norm, int use_mask,
                                     void* workspace, int64_t workspace_bytes, b200_stream_t stream);

/* One vision (ViT) block, inputs in the reference's variant-pack order:
 *   inputs[] = hidden [N, H], qkv_w [3H, H], qkv_b [3H], proj_w [H, H], proj_b [H],
 *              fc1_w [I, H], fc1_b [I], fc2_w [H, I], fc2_b [H],
 *              n1_w, n1_b, n2_w, n2_b [H]      (bf16, device),
 *              c, s [N, head_dim]               (fp32, device; the 2-D vision rope tables),
 *              seq [num_seqs]                   (int32, HOST; attention stays within each sequence)
 * num_inputs = 16, H = num_heads * head_dim.  out = r1 + fc2(gelu_tanh(fc1(LN2(r1)))),
 * r1 = hidden + proj(attn(rope(qkv(LN1(hidden))))) (bidirectional).
 * output [N, H] bf16 (may alias hidden); workspace >= b200_vision_block_workspace_bytes.
 * Replaces VisionBlockGraph::Build (atb_cpp_llm/src/components/vision/vision_block_graph.cpp:12-79)
 * + ExecuteOperation. */
B200_API int64_t b200_vision_block_workspace_bytes(int64_t N, int hidden, int intermediate);
B200_API int b200_vision_block(const void* const* inputs, int num_inputs, void* output, int64_t N, int num_seqs,
                               int hidden, int num_heads, int head_dim, int intermediate, float epsilon,
                               void* workspace, int64_t workspace_bytes, b200_stream_t stream);

/* ----------------------------------------------------------------- engine */

/* A decoder model on one GPU: weights, a paged KV cache of max_batch slots x
 * max_context tokens, activation buffers sized once, and the layer loop.
 * Replaces LLMEngine::Create / Forward (atb_cpp_llm/include/atb_llm/engine.h:8-24,
 * atb_cpp_llm/src/engine/llm_engine.cpp:22-108) with EngineConfig
 * (atb_cpp_llm/include/atb_llm/types.h:70-74) extended by the KV-cache sizes
 * the reference leaves unimplemented (atb_cpp_llm/include/atb_llm/runtime.h:45-54).
 * Not thread-safe: one engine per thread, as the reference's models
 * (atb_cpp_llm/include/atb_llm/model.h:33-36). */
typedef struct b200_engine_s* b200_engine_t;

typedef struct b200_engine_config {
  const char* model_dir;   /* directory with config.json (+ model.safetensors), or NULL */
  const char* config_json; /* inline config.json text when model_dir is NULL */
  int device_id;
  int max_batch;          /* KV-cache sequence slots (default 64) */
  int max_context;        /* tokens per slot (default 4096) */
  int max_prefill_tokens; /* packed tokens per prefill call (default 16384) */
  int kv_block_size;      /* 64 or 128 (default 128) */
  uint64_t init_seed;     /* seed of the N(0, init_std) init used when no weights file is given */
  float init_std;         /* default 0.02 */
} b200_engine_config;

enum b200_engine_query_key {
  B200_Q_WEIGHT_BYTES = 0,
  B200_Q_KV_BYTES = 1,
  B200_Q_DECODE_LAUNCHES = 2,  /* kernels one b200_engine_decode step launches at max_batch */
  B200_Q_PREFILL_LAUNCHES = 3, /* kernels one b200_engine_prefill call launches */
  B200_Q_HIDDEN = 4,
  B200_Q_LAYERS = 5,
  B200_Q_VOCAB = 6,
  B200_Q_HAS_VISION = 7,           /* 1 when the config carried a vision tower */
  B200_Q_VISION_WEIGHT_BYTES = 8,
  B200_Q_VISION_LAUNCHES = 9,      /* kernels the last b200_engine_vision / embed vision stage launched */
  B200_Q_ENCODE_LAUNCHES = 10      /* kernels the last b200_engine_embed text stage launched */
};

/* Model type is resolved from config.json "model_type" through a registry with
 * exact match first, then priority-ordered compatibility checks
 * (atb_cpp_llm/src/engine/model_registry.cpp:90-121). */
B200_API int b200_engine_create(const b200_engine_config* config, b200_engine_t* out);

/* Tensor-parallel engine over `comm` (GQA models, dense or mixture-of-experts):
 * rank r holds heads [r*nq/P, (r+1)*nq/P) (and the matching kv heads), rows
 * r*I/P.. of gate/up, the matching columns of o/down (of every expert and the
 * shared expert too; the router is replicated), vocabulary rows r*V/P.. of
 * lm_head; two all-reduces per layer (fused with residual + RMSNorm for
 * decode-sized batches, NCCL for prefill), a vocabulary-parallel argmax.
 * Weights are given whole through b200_engine_set_weight and sliced on the
 * host.  Every rank must make the same prefill/decode calls in the same
 * order; `logits` outputs receive this rank's vocabulary shard [rows, V/P]. */
B200_API int b200_engine_create_tp(const b200_engine_config* config, b200_comm_t comm, b200_engine_t* out);

/* Expert-parallel engine over `comm` (mixture-of-experts models, GQA or MLA):
 * every rank is a whole replica of the attention, dense and shared-expert
 * weights serving its OWN sequences (data-parallel attention, its own KV
 * cache); rank r holds routed experts [r*E/P, (r+1)*E/P) and every MoE layer
 * exchanges tokens with b200_ep_dispatch / b200_ep_combine.  Expert weights of
 * other ranks given to b200_engine_set_weight are skipped.  Every rank must
 * make the same sequence of prefill/decode calls (each with its own
 * sequences, at least one); `logits` are whole rows. */
B200_API int b200_engine_create_ep(const b200_engine_config* config, b200_comm_t comm, b200_engine_t* out);

/* Host function (no GPU): resolve and validate a config.json text the way
 * b200_engine_create does, without allocating anything; the registry entry it
 * resolves to is written to model_type (when not NULL).  Returns the status
 * b200_engine_create would return for the config. */
B200_API int b200_engine_config_check(const char* config_json, char* model_type, int model_type_len);
B200_API int b200_engine_destroy(b200_engine_t engine);

/* Load one weight by its HF name from host memory (dtype 0 = bf16, 1 = fp16,
 * 2 = fp32), e.g. "model.layers.3.self_attn.q_proj.weight".  Replaces
 * LoadQwen3VLWeights / CopyWeightToFp16NPU
 * (atb_cpp_llm/src/adapters/qwen3vl_embedding/qwen3vl_weights.cpp:79-264,
 * atb_cpp_llm/src/io/weight_helpers.cpp:16-76) with a direct bf16 upload. */
B200_API int b200_engine_set_weight(b200_engine_t engine, const char* name, const void* host, int dtype,
                                    int64_t numel);

/* Host functions (no GPU): the part of one whole weight that a rank of a
 * tensor-parallel group (tp_rank of tp_world; ep_world = 1) or of an
 * expert-parallel group (ep_rank of ep_world; tp_world = 1) keeps, exactly as
 * its b200_engine_create_tp / _create_ep engine places it: the dense bf16 rows
 * (q / k / v heads, gate / up / lm_head rows) or columns (o / down) of its
 * block, the whole tensor when replicated (norms, router, MLA, the vision
 * tower), nothing (*out_numel = 0) for another rank's expert.  The weight
 * comes from host memory (dtype 0 bf16, 1 fp16, 2 fp32) or from one tensor of
 * a safetensors file; out holds out_capacity bf16 values.  Returns the status
 * b200_engine_set_weight would (ERROR_WEIGHT_LOAD: a name the model does not
 * use).  Replaces the per-rank placement the reference lacks
 * (LoadQwen3VLWeights loads one device, qwen3vl_weights.cpp:79-264). */
B200_API int b200_weight_shard(const char* config_json, int tp_world, int tp_rank, int ep_world, int ep_rank,
                               const char* name, const void* host, int dtype, int64_t numel, void* out,
                               int64_t out_capacity, int64_t* out_numel);
B200_API int b200_weight_shard_file(const char* config_json, const char* safetensors_path, const char* name,
                                    int tp_world, int tp_rank, int ep_world, int ep_rank, void* out,
                                    int64_t out_capacity, int64_t* out_numel);

/* Prefill fresh sequences packed back to back: ids [sum(seq_lens)] (host or
 * device), seq_lens / slots [num_seqs] (host), optional position_ids [3, T]
 * (host, mrope; NULL = 0..len-1 per sequence).  Fills the KV cache of each
 * slot and writes each sequence's greedy next token to next_tokens (host or
 * device); logits (device, bf16 [num_seqs, vocab]) when not NULL.
 * Replaces Qwen3VLModel::ForwardWithTiming's text stage
 * (atb_cpp_llm/src/adapters/qwen3vl_embedding/qwen3vl_model.cpp:685-768). */
B200_API int b200_engine_prefill(b200_engine_t engine, const int64_t* ids, int ids_on_device,
                                 const int32_t* seq_lens, const int32_t* slots, int num_seqs,
                                 const int64_t* position_ids, int64_t* next_tokens, int next_on_device,
                                 void* logits);

/* One decode step: one token per listed slot (ids host or device, slots host).
 * No reference counterpart (the reference has no decode, IsGenerative() is
 * false for its only model, atb_cpp_llm/include/atb_llm/model.h:47-50). */
B200_API int b200_engine_decode(b200_engine_t engine, const int64_t* ids, int ids_on_device, const int32_t* slots,
                                int batch, int64_t* next_tokens, int next_on_device, void* logits);

/* Vision tower of a Qwen3-VL engine: pixels [num_patches, C*tp*p*p] in the
 * image processor's merge-block order (host bf16/fp16/fp32 by pixel_dtype
 * 0/1/2, or device bf16), grid_thw [num_images, 3] (host).  Writes the merged
 * embeddings [num_patches / merge^2, out_hidden] (device bf16) to merged_out
 * and the deepstack features [num_deepstack, num_patches / merge^2,
 * out_hidden] to deepstack_out when not NULL; *merged_tokens when not NULL.
 * Replaces the vision stage of Qwen3VLModel::ForwardWithTiming
 * (atb_cpp_llm/src/adapters/qwen3vl_embedding/qwen3vl_model.cpp:384-575) and
 * VisionRunner (atb_cpp_llm/src/runners/vision_runner.cpp:57-113). */
B200_API int b200_engine_vision(b200_engine_t engine, const void* pixels, int pixel_dtype, int pixels_on_device,
                                int64_t num_patches, const int64_t* grid_thw, int num_images, void* merged_out,
                                void* deepstack_out, int64_t* merged_tokens);

/* Qwen3-VL embedding forward of one request: input_ids [seq_len] (host),
 * optional attention_mask [seq_len] (host; pools the last unmasked token),
 * optional image (pixels as for b200_engine_vision; NULL = text only).  The
 * merged vision embeddings replace the rows of the image tokens, deepstack
 * feature i is added to them after text layer i, position ids follow
 * b200_get_rope_index, attention is causal.  Writes the final-normed pooled
 * token, L2-normalised when `normalize`, to embedding (host fp32 [hidden]);
 * hidden_out (device bf16 [seq_len, hidden]) receives every final-normed row
 * when not NULL.  An image-token count that differs from the merged vision
 * token count is ERROR_INVALID_PARAM.  Replaces Qwen3VLModel::Forward /
 * ForwardWithTiming (atb_cpp_llm/src/adapters/qwen3vl_embedding/qwen3vl_model.cpp:262-802)
 * with BaseModel::RunPooling (atb_cpp_llm/src/families/base_model.cpp:137-199). */
B200_API int b200_engine_embed(b200_engine_t engine, const int64_t* input_ids, int64_t seq_len,
                               const int64_t* attention_mask, const void* pixels, int pixel_dtype,
                               int pixels_on_device, int64_t num_patches, const int64_t* grid_thw, int num_images,
                               int normalize, float* embedding, void* hidden_out);

/* The engine's CUDA stream (device-side results are ordered on it). */
B200_API int b200_engine_stream(b200_engine_t engine, b200_stream_t* out);
/* Forget every slot's context (the KV cache contents stay, unreferenced). */
B200_API int b200_engine_reset(b200_engine_t engine);
B200_API int b200_engine_query(b200_engine_t engine, int what, int64_t* out);
B200_API int b200_engine_context_len(b200_engine_t engine, int slot, int64_t* out);

/* Device addresses of layer `layer`'s KV cache (ordered on the engine's
 * stream; valid until b200_engine_destroy).  GQA models: k_cache / v_cache
 * [num_blocks, kv_heads, block_size, head_dim] bf16.  Latent-attention models:
 * k_cache is the latent cache [num_blocks * block_size, kv_lora + qk_rope]
 * (per token the normalised compressed KV, then the roped key dims) and
 * *v_cache is NULL.  Slot s owns blocks [s * max_blocks_per_seq, (s + 1) *
 * max_blocks_per_seq) in order: its position p sits in block
 * s * max_blocks_per_seq + p / block_size at offset p % block_size.  Output
 * pointers may be NULL.  Replaces KVCacheManager::GetCachePtr
 * (atb_cpp_llm/src/core/kv_cache_manager.h:58-66), which the reference only
 * declares. */
B200_API int b200_engine_kv_cache(b200_engine_t engine, int layer, void** k_cache, void** v_cache,
                                  int64_t* num_blocks, int* block_size, int* max_blocks_per_seq);

#ifdef __cplusplus
}
#endif

#endif /* B200_LLM_H_ */
