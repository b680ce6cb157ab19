// The reference's C++ host interface (src/MatVec.h:13, src/RmsNorm.h:13, src/Rope.h:14,
// src/Swiglu.h:13, src/ElementwiseAdd.h:14, src/SoftMax.h:13, src/Argmax.h:13, src/GetRows.h:13,
// src/Attention.h:15, src/KvCache.h:16, src/TransformerLayer.h:20, src/FullModel.h:34), with the same
// names, options and return codes, backed by the B200 kernels through include/muyo_cuda.h.
//
// Each Run<Op>() runs the reference's own known-answer check for that op (the same inputs and
// tolerance) on the GPU and compares it with a CPU loop: 0 when it matches, 1 otherwise.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace muyo_llm
{
/// Sampling controls of src/Sampler.h:14-22, passed to the device sampler (MuyoSamplerParams).
/// The whole-vocabulary top-k (topK <= 0 with temperature > 0) is limited to 4096 candidates.
struct SamplerParams
{
    float temperature = 0.0F;
    int32_t topK = 40;
    float topP = 0.95F;
    float repeatPenalty = 1.0F;
    int32_t repeatLastN = 64;
    uint64_t seed = 0;
};

/// src/FullModel.h:12-21. Text prompts, chat framing and interactive turns need the tokenizer,
/// which is outside this build: RunFullModel takes token ids.
struct ForwardOptions
{
    std::vector<int32_t> tokens;
    std::string prompt;
    uint32_t nPredict = 32;
    SamplerParams sampler;
    bool chat = false;
    bool interactive = false;
    std::string system;
};

int RunElementwiseAdd();
int RunMatVec();
int RunRmsNorm();
int RunRope();
int RunSwiglu();
int RunGetRows();
int RunArgmax();
int RunSoftMax();
int RunAttention();
int RunKvCache();
int RunTransformerLayer();

/// Loads a Qwen2 GGUF (F16/F32 tensors), feeds options.tokens one position at a time and greedily
/// generates options.nPredict ids, printed to stdout as a comma-separated list.
/// @return 0 on success, 1 on a load or device failure, 2 for options this build does not support.
int RunFullModel(const std::string& ggufPath, const ForwardOptions& options);
}  // namespace muyo_llm
