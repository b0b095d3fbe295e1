// Where each Hugging Face weight goes in one rank's device tensors: the
// tensor-parallel and expert-parallel slicing as a host-only plan of strided
// copies, shared by the engine's weight upload (DecoderModel::SetWeight) and
// the host query b200_weight_shard / b200_weight_shard_file, so the slicing a
// rank applies can be checked without a GPU.
//
// Replaces the per-tensor placement of LoadQwen3VLWeights
// (atb_cpp_llm/src/adapters/qwen3vl_embedding/qwen3vl_weights.cpp:79-264),
// which the reference runs for one device only.
#pragma once

#include <stdint.h>

#include <string>
#include <vector>

#include "engine/model.h"

namespace b200llm {

// WTensor, WeightCopy and ShardView are declared beside ModelConfig (engine/model.h).

// The local config of rank tp_rank of tp tensor-parallel ranks (tp = 1: the
// whole model) or of ep_rank of ep expert-parallel ranks (routed experts
// split E/ep, everything else whole).  ERROR_UNSUPPORTED for a model that
// does not split that way.
Status MakeShardView(const ModelConfig& whole, int tp, int tp_rank, int ep, int ep_rank, ShardView& v);

// The copies that place weight `name` (the whole HF tensor, numel elements)
// into this rank's tensors.  OK with no copies: a weight this rank does not
// keep (another rank's expert, lm_head of a tied embedding).  ERROR_WEIGHT_LOAD
// for a name the model does not use; ERROR_INVALID_PARAM for a wrong size.
Status PlanWeight(const ShardView& v, const std::string& name, int64_t numel, std::vector<WeightCopy>& ops);

}  // namespace b200llm
