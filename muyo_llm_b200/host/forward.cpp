// RunFullModel (src/FullModel.cpp:487-1291) on the B200 decode engine: the GGUF's weights go to the
// device once, the prompt ids are fed one position at a time and the generated ids (greedy, or drawn
// by the device sampler with --temp / --top-k / --top-p / --repeat-penalty / --seed) come back in one
// call (muyo_model_generate). The cache is F32, as the reference's (src/FullModel.cpp:622-625).
#include <cstdio>
#include <string>
#include <vector>

#include "host.h"
#include "muyo_cuda.h"

namespace muyo_llm
{
namespace
{
constexpr uint32_t K_MAX_SEQ = 2048;  // cache capacity (the reference's default context)

int Fail(const char* what)
{
    std::fprintf(stderr, "[forward] %s: %s\n", what, muyo_cuda_last_error());
    return 1;
}
}  // namespace

int RunFullModel(const std::string& ggufPath, const ForwardOptions& options)
{
    if (options.tokens.empty()) {
        std::fprintf(stderr, "[forward] text prompts need the tokenizer, which this build does not include: "
                             "pass the prompt as --tokens id,id,...\n");
        return 2;
    }
    if (options.chat || options.interactive) {
        std::fprintf(stderr, "[forward] --chat and --interactive need the tokenizer and chat template, which this "
                             "build does not include\n");
        return 2;
    }
    if (options.tokens.size() + options.nPredict > K_MAX_SEQ) {
        std::fprintf(stderr, "[forward] %zu prompt + %u generated positions exceed the %u-position cache\n",
                     options.tokens.size(), options.nPredict, K_MAX_SEQ);
        return 2;
    }
    MuyoQwen2Config cfg{};
    if (muyo_gguf_read_qwen2_config(ggufPath.c_str(), K_MAX_SEQ, MUYO_KV_F32, &cfg) != MUYO_OK)
        return Fail("config");
    std::fprintf(stderr, "[forward] qwen2: %u layers, hidden %u, ffn %u, heads %u/%u, vocab %u\n", cfg.layers,
                 cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.vocab);
    if (muyo_cuda_init(0) != MUYO_OK)
        return Fail("init");
    MuyoModel* m = nullptr;
    if (muyo_model_create(&cfg, 0, &m) != MUYO_OK)
        return Fail("create");
    // One Sampler per run (src/FullModel.cpp:1058): the device engine draws once per generated id.
    const SamplerParams& o = options.sampler;
    const MuyoSamplerParams sp{o.temperature, o.topK, o.topP, o.repeatPenalty, o.repeatLastN, 0, o.seed};
    int rc = 0;
    std::vector<int32_t> out(options.nPredict > 0 ? options.nPredict : 1);
    if (muyo_model_load_gguf(m, ggufPath.c_str()) != MUYO_OK)
        rc = Fail("load");
    else if (muyo_model_finalize(m, nullptr) != MUYO_OK)
        rc = Fail("finalize");
    else if (muyo_model_set_sampler(m, &sp, nullptr) != MUYO_OK)
        rc = Fail("sampler");
    else if (muyo_model_generate(m, options.tokens.data(), (int)options.tokens.size(), (int)options.nPredict,
                                 out.data(), nullptr) != MUYO_OK)
        rc = Fail("generate");
    if (rc == 0) {
        for (uint32_t i = 0; i < options.nPredict; ++i)
            std::printf(i + 1 < options.nPredict ? "%d," : "%d\n", out[i]);
        if (options.nPredict == 0)
            std::printf("\n");
    }
    muyo_model_destroy(m);
    return rc;
}
}  // namespace muyo_llm
