#include "engine/vision_model.h"

#include <cmath>
#include <cstring>

#include "engine/engine_kernels.h"
#include "engine/safetensors.h"
#include "fused.h"
#include "gemm.h"

namespace b200llm {

namespace {
bool starts_with(const std::string& s, const std::string& p) { return s.compare(0, p.size(), p) == 0; }
}  // namespace

// ---------------------------------------------------------------- config

int VisionConfig::grid() const {
  const int g = (int)std::lround(std::sqrt((double)num_position_embeddings));
  return g * g == num_position_embeddings ? g : 0;
}

Status VisionConfig::FromJson(const JsonConfig& root, VisionConfig& c) {
  if (!root.IsValid() || !root.HasKey("vision_config")) return ERROR_INVALID_PARAM;
  const JsonConfig v = root.GetSubConfig("vision_config");
  c = VisionConfig();
  c.hidden = v.GetInt("hidden_size", 1024);
  c.heads = v.GetInt("num_heads", 16);
  c.intermediate = v.GetInt("intermediate_size", 4096);
  c.depth = v.GetInt("depth", 24);
  c.in_channels = v.GetInt("in_channels", 3);
  c.temporal_patch = v.GetInt("temporal_patch_size", 2);
  c.patch = v.GetInt("patch_size", 16);
  c.merge = v.GetInt("spatial_merge_size", 2);
  c.num_position_embeddings = v.GetInt("num_position_embeddings", 2304);
  c.out_hidden = v.GetInt("out_hidden_size", 2048);
  c.deepstack = v.GetIntArray("deepstack_visual_indexes");
  c.eps = v.GetFloat("layer_norm_eps", 1e-6f);
  if (c.hidden <= 0 || c.heads <= 0 || c.hidden % c.heads || c.depth <= 0 || c.intermediate <= 0 || c.merge <= 0 ||
      c.out_hidden <= 0 || c.patch <= 0 || c.in_channels <= 0 || c.temporal_patch <= 0 || c.grid() < 2)
    return ERROR_INVALID_PARAM;
  for (int d : c.deepstack)
    if (d < 0 || d >= c.depth) return ERROR_INVALID_PARAM;
  const int hd = c.head_dim();
  if (hd != 16 && hd != 32 && hd != 64 && hd != 128) return ERROR_UNSUPPORTED;
  if (c.hidden % 8 || c.intermediate % 8 || c.out_hidden % 8 || c.patch_dim() % 8) return ERROR_UNSUPPORTED;
  return STATUS_OK;
}

// ---------------------------------------------------------------- setup

VisionModel::~VisionModel() { DropGraphs(); }

void VisionModel::DropGraphs() {
  for (auto& g : graphs_) cudaGraphExecDestroy(g.second.exec);
  graphs_.clear();
  calls_.clear();
}

Status VisionModel::Init(const VisionConfig& cfg, ContextManager* ctx, TensorAllocator* alloc) {
  if (!ctx || !alloc) return ERROR_INVALID_PARAM;
  cfg_ = cfg;
  ctx_ = ctx;
  alloc_ = alloc;
  const int64_t H = cfg.hidden, L = cfg.depth, I = cfg.intermediate, P = cfg.patch_dim(), D = cfg.merged_dim();
  const int64_t O = cfg.out_hidden;
  const size_t before = alloc->BytesInUse();
  auto A = [&](DeviceTensor& t, std::vector<int64_t> s) { return alloc_->Alloc(t, DType::BF16, std::move(s)); };
  B200_RETURN_IF(A(patch_w_, {H, P}));
  B200_RETURN_IF(A(patch_b_, {H}));
  B200_RETURN_IF(A(pos_table_, {cfg.num_position_embeddings, H}));
  B200_RETURN_IF(A(n1_w_, {L, H}));
  B200_RETURN_IF(A(n1_b_, {L, H}));
  B200_RETURN_IF(A(qkv_w_, {L, 3 * H, H}));
  B200_RETURN_IF(A(qkv_b_, {L, 3 * H}));
  B200_RETURN_IF(A(proj_w_, {L, H, H}));
  B200_RETURN_IF(A(proj_b_, {L, H}));
  B200_RETURN_IF(A(n2_w_, {L, H}));
  B200_RETURN_IF(A(n2_b_, {L, H}));
  B200_RETURN_IF(A(fc1_w_, {L, I, H}));
  B200_RETURN_IF(A(fc1_b_, {L, I}));
  B200_RETURN_IF(A(fc2_w_, {L, H, I}));
  B200_RETURN_IF(A(fc2_b_, {L, H}));
  mergers_.resize(1 + cfg.deepstack.size());
  for (size_t i = 0; i < mergers_.size(); ++i) {
    MergerWeights& m = mergers_[i];
    m.postshuffle = i > 0;
    const int64_t nd = m.postshuffle ? D : H;
    B200_RETURN_IF(A(m.norm_w, {nd}));
    B200_RETURN_IF(A(m.norm_b, {nd}));
    B200_RETURN_IF(A(m.fc1_w, {D, D}));
    B200_RETURN_IF(A(m.fc1_b, {D}));
    B200_RETURN_IF(A(m.fc2_w, {O, D}));
    B200_RETURN_IF(A(m.fc2_b, {O}));
  }
  weight_bytes_ = alloc->BytesInUse() - before;
  return STATUS_OK;
}

Status VisionModel::InitRandomWeights(uint64_t seed, float std) {
  cudaStream_t st = ctx_->GetStream();
  uint64_t k = seed * 7919ull + 17;
  auto N = [&](DeviceTensor& t) { return FillNormalBf16(t.data, t.numel(), 0.f, std, ++k, st); };
  auto C = [&](DeviceTensor& t, float v) { return FillConstBf16(t.data, t.numel(), v, st); };
  for (DeviceTensor* t : {&patch_w_, &patch_b_, &pos_table_, &qkv_w_, &qkv_b_, &proj_w_, &proj_b_, &fc1_w_, &fc1_b_,
                          &fc2_w_, &fc2_b_})
    B200_RETURN_IF(N(*t));
  for (DeviceTensor* t : {&n1_w_, &n2_w_}) B200_RETURN_IF(C(*t, 1.f));
  for (DeviceTensor* t : {&n1_b_, &n2_b_}) B200_RETURN_IF(C(*t, 0.f));
  for (MergerWeights& m : mergers_) {
    for (DeviceTensor* t : {&m.fc1_w, &m.fc1_b, &m.fc2_w, &m.fc2_b}) B200_RETURN_IF(N(*t));
    B200_RETURN_IF(C(m.norm_w, 1.f));
    B200_RETURN_IF(C(m.norm_b, 0.f));
  }
  return ctx_->Synchronize();
}

Status VisionModel::SetWeight(const std::string& full, const std::vector<uint16_t>& b16, int64_t numel) {
  std::string name;
  if (starts_with(full, "model.visual.")) name = full.substr(13);
  else if (starts_with(full, "visual.")) name = full.substr(7);
  else return ERROR_WEIGHT_LOAD;
  const int64_t H = cfg_.hidden, I = cfg_.intermediate, P = cfg_.patch_dim(), D = cfg_.merged_dim();
  const int64_t O = cfg_.out_hidden;
  cudaStream_t st = ctx_->GetStream();
  auto put = [&](const DeviceTensor& t, int64_t elem_off, int64_t expect) -> Status {
    if (numel != expect) return ERROR_INVALID_PARAM;
    B200_RETURN_IF(FromCuda(cudaMemcpyAsync(static_cast<uint16_t*>(t.data) + elem_off, b16.data(),
                                            (size_t)numel * 2, cudaMemcpyHostToDevice, st)));
    return ctx_->Synchronize();
  };
  if (name == "patch_embed.proj.weight") return put(patch_w_, 0, H * P);  // Conv3d [H, C, tp, p, p] = [H, P]
  if (name == "patch_embed.proj.bias") return put(patch_b_, 0, H);
  if (name == "pos_embed.weight") return put(pos_table_, 0, (int64_t)cfg_.num_position_embeddings * H);
  if (starts_with(name, "blocks.")) {
    const size_t dot = name.find('.', 7);
    if (dot == std::string::npos) return ERROR_WEIGHT_LOAD;
    const int l = std::atoi(name.substr(7, dot - 7).c_str());
    if (l < 0 || l >= cfg_.depth) return ERROR_WEIGHT_LOAD;
    const std::string leaf = name.substr(dot + 1);
    if (leaf == "norm1.weight") return put(n1_w_, l * H, H);
    if (leaf == "norm1.bias") return put(n1_b_, l * H, H);
    if (leaf == "norm2.weight") return put(n2_w_, l * H, H);
    if (leaf == "norm2.bias") return put(n2_b_, l * H, H);
    if (leaf == "attn.qkv.weight") return put(qkv_w_, l * 3 * H * H, 3 * H * H);
    if (leaf == "attn.qkv.bias") return put(qkv_b_, l * 3 * H, 3 * H);
    if (leaf == "attn.proj.weight") return put(proj_w_, l * H * H, H * H);
    if (leaf == "attn.proj.bias") return put(proj_b_, l * H, H);
    if (leaf == "mlp.linear_fc1.weight") return put(fc1_w_, l * I * H, I * H);
    if (leaf == "mlp.linear_fc1.bias") return put(fc1_b_, l * I, I);
    if (leaf == "mlp.linear_fc2.weight") return put(fc2_w_, l * H * I, H * I);
    if (leaf == "mlp.linear_fc2.bias") return put(fc2_b_, l * H, H);
    return ERROR_WEIGHT_LOAD;
  }
  int mi = -1;
  std::string leaf;
  if (starts_with(name, "merger.")) {
    mi = 0;
    leaf = name.substr(7);
  } else if (starts_with(name, "deepstack_merger_list.")) {
    const size_t dot = name.find('.', 22);
    if (dot == std::string::npos) return ERROR_WEIGHT_LOAD;
    const int i = std::atoi(name.substr(22, dot - 22).c_str());
    if (i < 0 || i >= (int)cfg_.deepstack.size()) return ERROR_WEIGHT_LOAD;
    mi = 1 + i;
    leaf = name.substr(dot + 1);
  } else {
    return ERROR_WEIGHT_LOAD;
  }
  MergerWeights& m = mergers_[mi];
  const int64_t nd = m.postshuffle ? D : H;
  if (leaf == "norm.weight") return put(m.norm_w, 0, nd);
  if (leaf == "norm.bias") return put(m.norm_b, 0, nd);
  if (leaf == "linear_fc1.weight") return put(m.fc1_w, 0, D * D);
  if (leaf == "linear_fc1.bias") return put(m.fc1_b, 0, D);
  if (leaf == "linear_fc2.weight") return put(m.fc2_w, 0, O * D);
  if (leaf == "linear_fc2.bias") return put(m.fc2_b, 0, O);
  return ERROR_WEIGHT_LOAD;
}

const void* VisionModel::Deepstack(int i) const {
  if (i < 0 || i >= NumDeepstack() || !ds_.data) return nullptr;
  return static_cast<const uint16_t*>(ds_.data) + (int64_t)i * merged_tokens_ * cfg_.out_hidden;
}

int VisionModel::DeepstackSlot(int block) const {
  for (size_t i = 0; i < cfg_.deepstack.size(); ++i)
    if (cfg_.deepstack[i] == block) return (int)i;
  return -1;
}

// Activation buffers sized for `patches` tokens in `frames` attention groups;
// grown (never shrunk) when a larger request arrives.
Status VisionModel::Reserve(int64_t N, int64_t frames) {
  if (N <= cap_patches_ && frames <= cap_frames_) return STATUS_OK;
  B200_RETURN_IF(ctx_->Synchronize());
  DropGraphs();  // captured passes point at the buffers freed below
  N = std::max(N, cap_patches_);
  frames = std::max(frames, cap_frames_);
  for (DeviceTensor* t : {&pix_, &h_, &normed_, &qkv_, &attn_, &act_, &cos_, &sin_, &cu_, &merged_, &ds_, &ws_})
    if (t->data) alloc_->Free(*t);
  const int64_t H = cfg_.hidden, I = cfg_.intermediate, P = cfg_.patch_dim(), D = cfg_.merged_dim();
  const int64_t O = cfg_.out_hidden, hd = cfg_.head_dim(), g = (int64_t)cfg_.merge * cfg_.merge;
  const int64_t Nm = N / g;
  auto A = [&](DeviceTensor& t, DType d, std::vector<int64_t> s) { return alloc_->Alloc(t, d, std::move(s)); };
  B200_RETURN_IF(A(pix_, DType::BF16, {N, P}));
  B200_RETURN_IF(A(h_, DType::BF16, {N, H}));
  B200_RETURN_IF(A(normed_, DType::BF16, {N, H}));
  B200_RETURN_IF(A(qkv_, DType::BF16, {N, 3 * H}));
  B200_RETURN_IF(A(attn_, DType::BF16, {N, H}));
  B200_RETURN_IF(A(act_, DType::BF16, {N, std::max(I, H)}));
  B200_RETURN_IF(A(cos_, DType::FP32, {N, hd}));
  B200_RETURN_IF(A(sin_, DType::FP32, {N, hd}));
  B200_RETURN_IF(A(cu_, DType::INT32, {frames + 1}));
  B200_RETURN_IF(A(merged_, DType::BF16, {std::max<int64_t>(Nm, 1), O}));
  B200_RETURN_IF(A(ds_, DType::BF16, {std::max<int64_t>((int64_t)cfg_.deepstack.size(), 1), std::max<int64_t>(Nm, 1), O}));
  int64_t ws = 0;
  const int64_t shapes[5][2] = {{3 * H, H}, {H, H}, {I, H}, {H, I}, {H, P}};
  for (auto& s : shapes) ws = std::max(ws, b200_gemm_workspace_bytes(N, s[0], s[1], B200_EPI_BIAS));
  ws = std::max(ws, b200_gemm_workspace_bytes(Nm, D, D, B200_EPI_BIAS));
  ws = std::max(ws, b200_gemm_workspace_bytes(Nm, O, D, B200_EPI_BIAS));
  ws_bytes_ = ws;
  if (ws > 0) B200_RETURN_IF(A(ws_, DType::FP32, {(ws + 3) / 4}));
  cap_patches_ = N;
  cap_frames_ = frames;
  return STATUS_OK;
}

// ---------------------------------------------------------------- forward

Status VisionModel::Gemm(const void* A, int64_t lda, const void* W, void* C, int64_t ldc, int64_t M, int64_t N,
                         int64_t K, int epi, const void* bias, const void* R, int64_t ldr) {
  cudaStream_t st = ctx_->GetStream();
  int splits = 1;
  ++launches_;
  B200_RETURN_IF(b200::gemm_launch(A, lda, W, K, C, ldc, M, N, K, epi, bias, R, ldr, ws_.data, ws_bytes_, st, &splits));
  if (splits > 1) {
    ++launches_;
    B200_RETURN_IF(b200::splitk_reduce(ws_.as<float>(), splits, M, N, epi, bias, R, ldr, C, ldc, st));
  }
  return STATUS_OK;
}

Status VisionModel::GemmResidualNorm(const void* A, int64_t lda, const void* W, int64_t M, int64_t K,
                                     const void* bias, const void* gamma, const void* beta, bool* normed) {
  cudaStream_t st = ctx_->GetStream();
  const int64_t H = cfg_.hidden;
  int splits = 1;
  *normed = false;
  ++launches_;
  B200_RETURN_IF(b200::gemm_launch(A, lda, W, K, h_.data, H, M, H, K, B200_EPI_BIAS_RESIDUAL, bias, h_.data, H,
                                   ws_.data, ws_bytes_, st, &splits));
  if (splits <= 1) return STATUS_OK;
  ++launches_;
  const int rc = b200::splitk_bias_residual_layernorm(ws_.as<float>(), splits, M, H, bias, h_.data, gamma, beta,
                                                      normed_.data, cfg_.eps, st);
  if (rc == B200_OK) {
    *normed = true;
    return STATUS_OK;
  }
  if (rc != B200_ERROR_UNSUPPORTED) return (Status)rc;
  return (Status)b200::splitk_reduce(ws_.as<float>(), splits, M, H, B200_EPI_BIAS_RESIDUAL, bias, h_.data, H,
                                     h_.data, H, st);
}

// LayerNorm -> fc1 (+bias, GELU-tanh) -> fc2 (+bias).  The main merger
// normalises each token over `hidden` before grouping; a deepstack merger
// groups merge^2 tokens first and normalises over the grouped width
// (VisionMergerGraph::Build, atb_cpp_llm/src/components/vision/vision_merger_graph.cpp:11-87).
Status VisionModel::Merger(const void* x, int64_t N, int which, void* out) {
  cudaStream_t st = ctx_->GetStream();
  const MergerWeights& m = mergers_[which];
  const int64_t H = cfg_.hidden, D = cfg_.merged_dim(), O = cfg_.out_hidden;
  const int64_t Nm = N / ((int64_t)cfg_.merge * cfg_.merge);
  ++launches_;
  if (m.postshuffle)
    B200_RETURN_IF(b200_layernorm(x, m.norm_w.data, m.norm_b.data, normed_.data, Nm, D, cfg_.eps, st));
  else
    B200_RETURN_IF(b200_layernorm(x, m.norm_w.data, m.norm_b.data, normed_.data, N, H, cfg_.eps, st));
  B200_RETURN_IF(Gemm(normed_.data, D, m.fc1_w.data, act_.data, D, Nm, D, D, B200_EPI_BIAS_GELU, m.fc1_b.data, nullptr,
                      0));
  return Gemm(act_.data, D, m.fc2_w.data, out, O, Nm, O, D, B200_EPI_BIAS, m.fc2_b.data, nullptr, 0);
}

Status VisionModel::Forward(const void* pixels, DType dtype, bool on_device, int64_t N, const int64_t* grid_thw,
                            int num_images) {
  if (!pixels || !grid_thw || num_images <= 0 || num_images > 64 || N <= 0) return ERROR_INVALID_PARAM;
  const int m = cfg_.merge;
  int64_t total = 0, frames = 0;
  int max_len = 0;
  std::vector<int32_t> cu(1, 0);
  for (int i = 0; i < num_images; ++i) {
    const int64_t t = grid_thw[3 * i], h = grid_thw[3 * i + 1], w = grid_thw[3 * i + 2];
    if (t <= 0 || h <= 0 || w <= 0 || h % m || w % m || h * w > INT32_MAX / 2) return ERROR_INVALID_PARAM;
    total += t * h * w;
    frames += t;
    if (total > INT32_MAX / 2) return ERROR_INVALID_PARAM;
    max_len = std::max<int>(max_len, (int)(h * w));
    for (int64_t f = 0; f < t; ++f) cu.push_back(cu.back() + (int32_t)(h * w));
  }
  if (total != N) return ERROR_INVALID_PARAM;
  if (on_device && dtype != DType::BF16) return ERROR_UNSUPPORTED;
  B200_RETURN_IF(Reserve(N, frames));
  cudaStream_t st = ctx_->GetStream();
  const int64_t P = cfg_.patch_dim();
  const void* pix = pixels;
  if (!on_device) {
    std::vector<uint16_t> b16;
    const char* dt = dtype == DType::BF16 ? "BF16" : dtype == DType::FP16 ? "F16" : dtype == DType::FP32 ? "F32" : "";
    B200_RETURN_IF(ToBf16(static_cast<const uint8_t*>(pixels), dt, (size_t)(N * P), b16));
    B200_RETURN_IF(FromCuda(cudaMemcpyAsync(pix_.data, b16.data(), b16.size() * 2, cudaMemcpyHostToDevice, st)));
    B200_RETURN_IF(FromCuda(cudaStreamSynchronize(st)));  // b16 goes out of scope
    pix = pix_.data;
  } else if (reinterpret_cast<uintptr_t>(pixels) & 15) {
    return ERROR_INVALID_PARAM;
  }
  B200_RETURN_IF(FromCuda(cudaMemcpyAsync(cu_.data, cu.data(), cu.size() * 4, cudaMemcpyHostToDevice, st)));
  if (pix != pix_.data)  // the tower always reads pix_, so a captured graph serves any caller buffer
    B200_RETURN_IF(FromCuda(cudaMemcpyAsync(pix_.data, pix, (size_t)(N * P) * 2, cudaMemcpyDeviceToDevice, st)));
  B200_RETURN_IF(FromCuda(cudaStreamSynchronize(st)));
  merged_tokens_ = N / ((int64_t)m * m);

  // The kernel sequence depends only on the image grids: it is captured in a
  // CUDA graph the second time a grid list is seen and replayed afterwards.
  static const bool no_graph = EnvInt("B200_DISABLE_GRAPHS", 0) != 0;
  std::vector<int64_t> key(grid_thw, grid_thw + 3 * num_images);
  auto it = graphs_.find(key);
  if (it != graphs_.end()) {
    launches_ = it->second.launches;
    return FromCuda(cudaGraphLaunch(it->second.exec, st));
  }
  if (no_graph || ++calls_[key] < 2) return RunTower(N, grid_thw, num_images, (int)frames, max_len);
  B200_RETURN_IF(FromCuda(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed)));
  Status s = RunTower(N, grid_thw, num_images, (int)frames, max_len);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(st, &g);
  if (s != STATUS_OK || e != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return s != STATUS_OK ? s : FromCuda(e);
  }
  cudaGraphExec_t ex = nullptr;
  e = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  B200_RETURN_IF(FromCuda(e));
  graphs_[key] = {ex, launches_};
  return FromCuda(cudaGraphLaunch(ex, st));
}

// Patch embed + position embedding, the blocks with their deepstack taps, the
// main merger: every kernel of one tower pass, enqueued on the stream.
Status VisionModel::RunTower(int64_t N, const int64_t* grid_thw, int num_images, int frames, int max_len) {
  cudaStream_t st = ctx_->GetStream();
  const int m = cfg_.merge;
  const int64_t H = cfg_.hidden, I = cfg_.intermediate, P = cfg_.patch_dim(), hd = cfg_.head_dim();
  const int nh = cfg_.heads;
  launches_ = 0;

  // patch embedding (Conv3d with stride = kernel is a linear map of the flattened patch)
  B200_RETURN_IF(Gemm(pix_.data, P, patch_w_.data, h_.data, H, N, H, P, B200_EPI_BIAS, patch_b_.data, nullptr, 0));
  launches_ += 2;
  B200_RETURN_IF(b200_pos_embed_interp(pos_table_.data, cfg_.grid(), H, grid_thw, num_images, m, h_.data, 1, st));
  B200_RETURN_IF(b200_rope_table_vision(grid_thw, num_images, m, (int)hd, cfg_.rope_theta, cos_.as<float>(),
                                        sin_.as<float>(), st));
  const float scale = 1.0f / std::sqrt((float)hd);
  auto bf = [](const DeviceTensor& t, int64_t off) { return static_cast<const uint16_t*>(t.data) + off; };
  uint16_t* qkv = qkv_.as<uint16_t>();
  bool n1_ready = false;  // normed_ already holds this block's first LayerNorm (fused into fc2's reduce)
  for (int l = 0; l < cfg_.depth; ++l) {
    if (!n1_ready) {
      ++launches_;
      B200_RETURN_IF(b200_layernorm(h_.data, bf(n1_w_, l * H), bf(n1_b_, l * H), normed_.data, N, H, cfg_.eps, st));
    }
    B200_RETURN_IF(Gemm(normed_.data, H, bf(qkv_w_, l * 3 * H * H), qkv, 3 * H, N, 3 * H, H, B200_EPI_BIAS,
                        bf(qkv_b_, l * 3 * H), nullptr, 0));
    launches_ += 2;
    B200_RETURN_IF(b200_rope_apply(qkv, N, 2 * nh, (int)hd, 3 * H, cos_.as<float>(), sin_.as<float>(), st));
    B200_RETURN_IF(b200_flash_prefill_packed(qkv, 3 * H, hd, qkv + H, 3 * H, hd, qkv + 2 * H, 3 * H, hd, attn_.data,
                                             H, hd, cu_.as<int32_t>(), (int)frames, max_len, N, nh, nh, (int)hd,
                                             (int)hd, scale, 0, st));
    bool n2_ready = false;
    B200_RETURN_IF(GemmResidualNorm(attn_.data, H, bf(proj_w_, l * H * H), N, H, bf(proj_b_, l * H),
                                    bf(n2_w_, l * H), bf(n2_b_, l * H), &n2_ready));
    if (!n2_ready) {
      ++launches_;
      B200_RETURN_IF(b200_layernorm(h_.data, bf(n2_w_, l * H), bf(n2_b_, l * H), normed_.data, N, H, cfg_.eps, st));
    }
    B200_RETURN_IF(Gemm(normed_.data, H, bf(fc1_w_, l * I * H), act_.data, I, N, I, H, B200_EPI_BIAS_GELU,
                        bf(fc1_b_, l * I), nullptr, 0));
    const int ds = DeepstackSlot(l);
    if (ds < 0 && l + 1 < cfg_.depth) {
      // the next block's first LayerNorm rides on fc2's split-K reduce (a merger
      // after this block would use normed_ itself, so those blocks normalise later)
      B200_RETURN_IF(GemmResidualNorm(act_.data, I, bf(fc2_w_, l * H * I), N, I, bf(fc2_b_, l * H),
                                      bf(n1_w_, (l + 1) * H), bf(n1_b_, (l + 1) * H), &n1_ready));
    } else {
      B200_RETURN_IF(Gemm(act_.data, I, bf(fc2_w_, l * H * I), h_.data, H, N, H, I, B200_EPI_BIAS_RESIDUAL,
                          bf(fc2_b_, l * H), h_.data, H));
      n1_ready = false;
    }
    if (ds >= 0)
      B200_RETURN_IF(Merger(h_.data, N, 1 + ds,
                            static_cast<uint16_t*>(ds_.data) + (int64_t)ds * merged_tokens_ * cfg_.out_hidden));
  }
  B200_RETURN_IF(Merger(h_.data, N, 0, merged_.data));
  return FromCuda(cudaGetLastError());
}

}  // namespace b200llm
