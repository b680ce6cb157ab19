// TEST INFRASTRUCTURE - a C entry point over the reference's own sampler (src/Sampler.cpp, compiled
// unmodified from the reference tree by oracle/Makefile into oracle/_ref/). Used only by tests, to
// pin oracle.c's restatement of Sampler::Sample; never by the product.
#include "Sampler.h"

extern "C" void* ref_sampler_create(float temperature, int top_k, float top_p, float repeat_penalty,
                                    int repeat_last_n, unsigned long long seed)
{
    muyo_llm::SamplerParams p;
    p.temperature = temperature;
    p.topK = top_k;
    p.topP = top_p;
    p.repeatPenalty = repeat_penalty;
    p.repeatLastN = repeat_last_n;
    p.seed = seed;
    return new muyo_llm::Sampler(p);
}

extern "C" int ref_sampler_sample(void* s, float* logits, int vocab, const int* history, int hist_len)
{
    std::vector<int32_t> h(history, history + hist_len);
    return static_cast<muyo_llm::Sampler*>(s)->Sample(logits, vocab, h);
}

extern "C" void ref_sampler_destroy(void* s) { delete static_cast<muyo_llm::Sampler*>(s); }
