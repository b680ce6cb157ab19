// RunFullModel (src/FullModel.cpp:487-1291) on the B200 decode engine: the GGUF's weights go to the
// device once; the prompt (a text run through the GGUF's tokenizer, ids given with --tokens, or a
// ChatML turn with --chat) is fed one position at a time; the reply streams to stdout as text and its
// ids go to stderr. A generated id is fed back like the reference's feedToken, the end-of-sequence id
// included, and generation stops there.
//
// A single turn is one muyo_model_generate call (greedy, or drawn by the device sampler in the step
// graph) whose ids are cut after the first end-of-sequence id; nothing follows it, so the output is
// the reference's. An interactive session must leave the cache ending exactly at that id for the
// next turn, so it steps one position per call (muyo_model_step) and draws with muyo_cuda_sample on
// the step's logits, as the reference's feedToken / sampleNext loop does. The cache is F32, as the
// reference's (src/FullModel.cpp:622-625).
#include <chrono>
#include <cstdio>
#include <iostream>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "host.h"
#include "muyo_cuda.h"
#include "tokenizer.h"

namespace muyo_llm
{
namespace
{
constexpr uint32_t K_MAX_SEQ = 2048;  // cache positions the reference's context holds

int Fail(const char* what)
{
    std::fprintf(stderr, "[fail] %s: %s\n", what, muyo_cuda_last_error());
    return 1;
}

// Bytes of generated text held back until their UTF-8 character completes
// (src/FullModel.cpp:1068-1091).
struct TextStream
{
    std::string pending;
    void Flush(bool final)
    {
        size_t done = 0;
        while (done < pending.size()) {
            const auto lead = static_cast<unsigned char>(pending[done]);
            const size_t len = (lead & 0xE0) == 0xC0 ? 2 : (lead & 0xF0) == 0xE0 ? 3 : (lead & 0xF8) == 0xF0 ? 4 : 1;
            if (!final && done + len > pending.size())
                break;
            done += len;
        }
        std::fwrite(pending.data(), 1, done < pending.size() ? done : pending.size(), stdout);
        pending.erase(0, done);
        std::fflush(stdout);
    }
};

// The device session: the model and, for an interactive run, the per-step sampler's buffers.
class Session
{
public:
    Session(MuyoModel* m, const MuyoSamplerParams& sp, bool stepwise, int vocab)
        : m_(m), sp_(sp), stepwise_(stepwise), vocab_(vocab)
    {
    }
    ~Session()
    {
        cudaFree(history_);
        cudaFree(state_);
        cudaFree(token_);
    }
    int Init()
    {
        sampling_ = sp_.temperature > 0.0F || sp_.repeat_penalty != 1.0F;
        if (!stepwise_)
            return muyo_model_set_sampler(m_, &sp_, nullptr) != MUYO_OK ? Fail("sampler") : 0;
        if (!sampling_)
            return 0;
        if (cudaMalloc(&history_, sizeof(int32_t) * (K_MAX_SEQ + 1)) != cudaSuccess ||
            cudaMalloc(&state_, muyo_sampler_state_bytes()) != cudaSuccess ||
            cudaMalloc(&token_, sizeof(int32_t)) != cudaSuccess) {
            std::fprintf(stderr, "[fail] device buffers for the sampler\n");
            return 1;
        }
        void* logits = nullptr;
        size_t bytes = 0;
        if (muyo_model_buffer(m_, "logits", &logits, &bytes) != MUYO_OK)
            return Fail("logits buffer");
        logits_ = static_cast<float*>(logits);
        return muyo_sampler_seed(state_, sp_.seed, nullptr) != MUYO_OK ? Fail("sampler seed") : 0;
    }

    // Feed `ids` and generate up to `budget` ids, stopping after `eos` (src/FullModel.cpp:1173-1208).
    // Returns 0, or 1 on a device error; `full` reports a cache that filled up.
    int Turn(const std::vector<int32_t>& ids, uint32_t budget, int32_t eos, const Tokenizer& tok, TextStream& text,
             std::vector<int32_t>& generated, bool& full)
    {
        generated.clear();
        full = false;
        if (ids.empty())
            return 0;
        if (fed_.size() + ids.size() > K_MAX_SEQ) {
            std::fprintf(stderr, "[forward] the context is full (%u tokens)\n", K_MAX_SEQ);
            full = true;
            return 0;
        }
        if (!stepwise_) {
            // The reference's last id is sampled after the cache filled and is not fed; the engine
            // holds one position more so that it can feed it.
            const uint32_t room = K_MAX_SEQ + 1 - (uint32_t)(fed_.size() + ids.size());
            const uint32_t n = budget < room ? budget : room;
            std::vector<int32_t> out(n > 0 ? n : 1);
            if (muyo_model_generate(m_, ids.data(), (int)ids.size(), (int)n, out.data(), nullptr) != MUYO_OK)
                return Fail("generate");
            fed_.insert(fed_.end(), ids.begin(), ids.end());
            for (uint32_t i = 0; i < n; ++i) {
                Emit(out[i], tok, text, generated);
                fed_.push_back(out[i]);
                if (out[i] == eos)
                    break;
            }
            if (generated.size() == room) {  // the last id found the cache full (even an end id)
                std::fprintf(stderr, "[forward] the context is full (%u tokens)\n", K_MAX_SEQ);
                full = true;
            }
            return 0;
        }
        int32_t next = 0;
        for (int32_t id : ids)
            if (Feed(id, next))
                return 1;
        for (uint32_t k = 0; k < budget; ++k) {
            if (sampling_ && Draw(next))
                return 1;
            Emit(next, tok, text, generated);
            if (fed_.size() >= K_MAX_SEQ) {
                std::fprintf(stderr, "[forward] the context is full (%u tokens)\n", K_MAX_SEQ);
                full = true;
                break;
            }
            const int32_t id = next;
            if (Feed(id, next))
                return 1;
            if (id == eos)
                break;
        }
        return 0;
    }

    // Feed ids without generating (the system turn of an interactive session).
    int Prime(const std::vector<int32_t>& ids)
    {
        int32_t next = 0;
        for (int32_t id : ids) {
            if (fed_.size() >= K_MAX_SEQ)
                break;
            if (Feed(id, next))
                return 1;
        }
        return 0;
    }

private:
    static void Emit(int32_t id, const Tokenizer& tok, TextStream& text, std::vector<int32_t>& generated)
    {
        generated.push_back(id);
        if (!tok.IsSpecial(id)) {
            text.pending += tok.TokenBytes(id);
            text.Flush(false);
        }
    }
    int Feed(int32_t id, int32_t& greedy)
    {
        if (muyo_model_step(m_, id, nullptr, &greedy, nullptr) != MUYO_OK)
            return Fail("step");
        fed_.push_back(id);
        return 0;
    }
    // The device sampler on the step's logits, with every id in the cache as its history.
    int Draw(int32_t& next)
    {
        if (cudaMemcpy(history_, fed_.data(), sizeof(int32_t) * fed_.size(), cudaMemcpyHostToDevice) != cudaSuccess)
            return Fail("history copy");
        if (muyo_cuda_sample(&sp_, logits_, (uint32_t)vocab_, history_, (uint32_t)fed_.size(), state_, token_,
                             nullptr) != MUYO_OK)
            return Fail("sample");
        if (cudaMemcpy(&next, token_, sizeof(int32_t), cudaMemcpyDeviceToHost) != cudaSuccess)
            return Fail("token copy");
        return 0;
    }

    MuyoModel* m_;
    MuyoSamplerParams sp_;
    bool stepwise_;
    int vocab_;
    bool sampling_ = false;
    std::vector<int32_t> fed_;  // every id in the cache, in order
    int32_t* history_ = nullptr;
    void* state_ = nullptr;
    int32_t* token_ = nullptr;
    float* logits_ = nullptr;
};

void PrintIds(const char* label, const std::vector<int32_t>& ids)
{
    std::fprintf(stderr, "[forward] %s", label);
    for (int32_t id : ids)
        std::fprintf(stderr, " %d", id);
    std::fprintf(stderr, "\n");
}

int Run(const std::string& ggufPath, const ForwardOptions& options)
{
    const GgufMeta meta(ggufPath);
    const Tokenizer tokenizer(meta);
    // In chat mode the prompt is the user's raw text, framed later.
    const std::vector<int32_t> prompt =
        options.chat ? std::vector<int32_t>{}
                     : (options.prompt.empty() ? options.tokens : tokenizer.Encode(options.prompt));
    if (prompt.size() >= K_MAX_SEQ) {
        std::fprintf(stderr, "[fail] prompt is %zu tokens, the cache holds %u\n", prompt.size(), K_MAX_SEQ);
        return 1;
    }
    MuyoQwen2Config cfg{};
    if (muyo_gguf_read_qwen2_config(ggufPath.c_str(), K_MAX_SEQ + 1, MUYO_KV_F32, &cfg) != MUYO_OK)
        return Fail("config");
    for (int32_t id : prompt)
        if (id < 0 || (uint32_t)id >= cfg.vocab) {
            std::fprintf(stderr, "[fail] prompt id %d outside the %u-token vocabulary\n", id, cfg.vocab);
            return 1;
        }
    std::fprintf(stderr, "[forward] %s\n[forward] layers=%u hidden=%u ffn=%u heads=%u kv_heads=%u vocab=%u\n",
                 ggufPath.c_str(), cfg.layers, cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.vocab);
    if (muyo_cuda_init(0) != MUYO_OK)
        return Fail("init");
    MuyoModel* m = nullptr;
    if (muyo_model_create(&cfg, 0, &m) != MUYO_OK)
        return Fail("create");
    struct Guard
    {
        MuyoModel* m;
        ~Guard() { muyo_model_destroy(m); }
    } guard{m};
    if (muyo_model_load_gguf(m, ggufPath.c_str()) != MUYO_OK)
        return Fail("load");
    if (muyo_model_finalize(m, nullptr) != MUYO_OK)
        return Fail("finalize");

    const uint64_t eosKey = meta.UintOr("tokenizer.ggml.eos_token_id", UINT64_MAX);
    const int32_t eos = eosKey == UINT64_MAX ? -1 : static_cast<int32_t>(eosKey);
    const SamplerParams& o = options.sampler;
    const MuyoSamplerParams sp{o.temperature, o.topK, o.topP, o.repeatPenalty, o.repeatLastN, 0, o.seed};
    Session session(m, sp, options.interactive, (int)cfg.vocab);
    if (int rc = session.Init())
        return rc;

    const auto start = std::chrono::steady_clock::now();
    TextStream text;
    std::vector<int32_t> generated;
    bool full = false;
    if (options.chat) {
        const std::string system = options.system.empty() ? chat_template::QWEN2_DEFAULT_SYSTEM : options.system;
        bool firstUserTurn = true;
        if (!options.prompt.empty() || !options.interactive) {
            const std::string user = options.prompt.empty() ? "Hello" : options.prompt;
            if (session.Turn(tokenizer.Encode(chat_template::Qwen2ChatStart(system, user), true), options.nPredict,
                             eos, tokenizer, text, generated, full))
                return 1;
            firstUserTurn = false;
        } else if (session.Prime(tokenizer.Encode(chat_template::Qwen2SystemStart(system), true))) {
            return 1;
        }
        while (options.interactive && !full) {
            std::fprintf(stderr, "\n[chat] you> ");
            std::fflush(stderr);
            std::string line;
            if (!std::getline(std::cin, line))
                break;
            if (line.empty())
                continue;
            if (line == "/exit" || line == "/quit")
                break;
            // Every turn after the assistant's <|im_end|> starts with a newline.
            const std::string prefix = firstUserTurn ? "" : "\n";
            firstUserTurn = false;
            std::printf("\n");
            if (session.Turn(tokenizer.Encode(prefix + chat_template::Qwen2UserTurn(line), true), options.nPredict,
                             eos, tokenizer, text, generated, full))
                return 1;
        }
    } else {
        std::vector<int32_t> ids = prompt;
        if (ids.empty())
            ids.push_back(static_cast<int32_t>(meta.UintOr("tokenizer.ggml.bos_token_id", 0)));
        PrintIds("prompt tokens:", ids);
        if (session.Turn(ids, options.nPredict, eos, tokenizer, text, generated, full))
            return 1;
    }
    text.Flush(true);
    std::printf("\n");
    std::fflush(stdout);
    const double seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
    std::fprintf(stderr, "[forward] generated %zu tokens:", generated.size());
    for (int32_t id : generated)
        std::fprintf(stderr, " %d", id);
    std::fprintf(stderr, "\n");
    if (seconds > 0.0)
        std::fprintf(stderr, "[forward] %.2f tok/s (%.0f ms total)\n", generated.size() / seconds, seconds * 1000.0);
    return 0;
}
}  // namespace

int RunFullModel(const std::string& ggufPath, const ForwardOptions& options)
{
    try {
        return Run(ggufPath, options);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "[fail] %s\n", e.what());
        return 1;
    }
}

int RunTokenize(const std::string& path, const std::string& text)
{
    const GgufMeta meta(path);
    const Tokenizer tokenizer(meta);
    std::printf("[tokenize] vocab %zu, model %s\n", tokenizer.VocabSize(),
                meta.StringOr("tokenizer.ggml.model", "(none)").c_str());
    const std::vector<int32_t> ids = tokenizer.Encode(text);
    std::printf("[tokenize] \"%s\" ->", text.c_str());
    for (int32_t id : ids)
        std::printf(" %d", id);
    std::printf("\n");
    const std::string back = tokenizer.Decode(ids);
    if (back != text) {
        std::fprintf(stderr, "[fail] round-trip differs: '%s' != '%s'\n", back.c_str(), text.c_str());
        return 1;
    }
    // The Qwen2/GPT-2 vocabularies have token 0 = "!", which byte-encodes to itself and is a piece
    // of its own, so it must encode to exactly {0} (src/Tokenize.cpp:35-45).
    if (tokenizer.TokenFor(0) == "!") {
        const std::vector<int32_t> bang = tokenizer.Encode("!");
        if (bang.size() != 1 || bang[0] != 0) {
            std::fprintf(stderr, "[fail] Encode(\"!\") is not {0}\n");
            return 1;
        }
        std::printf("[tokenize] anchor OK: Encode(\"!\") == {0}\n");
    }
    std::printf("[tokenize] OK: %zu tokens, round-trip exact\n", ids.size());
    return 0;
}
}  // namespace muyo_llm
