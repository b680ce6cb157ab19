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

/// src/FullModel.h:12-21: a text prompt (run through the GGUF's tokenizer) or ids, the generation
/// budget, the sampler and the chat controls (--chat frames the prompt as a ChatML turn; interactive
/// reads further user turns from stdin).
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

/// Loads a Qwen2 GGUF (F16/F32 tensors and its tokenizer), feeds the prompt and generates up to
/// options.nPredict ids, stopping after tokenizer.ggml.eos_token_id: the reply's text goes to stdout,
/// its ids to stderr ("[forward] generated N tokens: ...").
/// @return 0 on success, 1 on a load, tokenizer or device failure.
int RunFullModel(const std::string& ggufPath, const ForwardOptions& options);

/// src/Tokenize.cpp:12-48: prints the ids of `text`, checks that they decode back to it exactly and,
/// when token 0 is "!", that "!" encodes to {0}. No device. @return 0 when both hold, else 1.
int RunTokenize(const std::string& ggufPath, const std::string& text);
}  // namespace muyo_llm
