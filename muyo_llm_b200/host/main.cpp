// muyo-llm command line (src/main.cpp:186-431): the same mode flags and exit codes (0 ok, 1 check
// failed or error, 2 usage) for the decode-step modes and --tokenize, run on the B200 kernels. The
// modes of the reference that are not part of the decode step (--smoke, --gguf, --model, --embed)
// exit with 2 and say so.
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <vector>

#include "host.h"

namespace
{
std::vector<int32_t> ParseTokens(const std::string& s)
{
    std::vector<int32_t> ids;
    size_t i = 0;
    while (i < s.size()) {
        size_t j = s.find(',', i);
        if (j == std::string::npos)
            j = s.size();
        if (j > i)
            ids.push_back((int32_t)std::stol(s.substr(i, j - i)));
        i = j + 1;
    }
    return ids;
}

void Usage(const char* argv0)
{
    std::fprintf(stderr,
                 "usage: %s --add | --matvec | --rmsnorm | --rope | --swiglu | --getrows | --argmax | --softmax |\n"
                 "       --attention | --kvcache | --layer | --tokenize <gguf> <text> |\n"
                 "       --forward <gguf> [-p TEXT | --tokens id,id] [--chat] [-i] [--system TEXT] [-n N] [--temp T]\n"
                 "       [--top-k K] [--top-p P] [--repeat-penalty R] [--repeat-last-n N] [--seed S]\n",
                 argv0);
}
}  // namespace

int main(int argc, char** argv)
{
    const std::string mode = argc > 1 ? argv[1] : "";
    for (const char* other : {"--smoke", "--gguf", "--model", "--embed"})
        if (mode == other) {
            std::fprintf(stderr, "%s is not part of this build (the decode-step kernels only)\n", other);
            return 2;
        }
    // --tokenize reads the GGUF's tokenizer; it needs no device (src/main.cpp:209-226).
    if (mode == "--tokenize") {
        if (argc < 4) {
            std::fprintf(stderr, "usage: %s --tokenize <gguf> <text>\n", argv[0]);
            return 2;
        }
        try {
            return muyo_llm::RunTokenize(argv[2], argv[3]);
        } catch (const std::exception& e) {
            std::fprintf(stderr, "[fail] %s\n", e.what());
            return 1;
        }
    }
    try {
        if (mode == "--add")
            return muyo_llm::RunElementwiseAdd();
        if (mode == "--matvec")
            return muyo_llm::RunMatVec();
        if (mode == "--rmsnorm")
            return muyo_llm::RunRmsNorm();
        if (mode == "--rope")
            return muyo_llm::RunRope();
        if (mode == "--swiglu")
            return muyo_llm::RunSwiglu();
        if (mode == "--getrows")
            return muyo_llm::RunGetRows();
        if (mode == "--argmax")
            return muyo_llm::RunArgmax();
        if (mode == "--softmax")
            return muyo_llm::RunSoftMax();
        if (mode == "--attention")
            return muyo_llm::RunAttention();
        if (mode == "--kvcache")
            return muyo_llm::RunKvCache();
        if (mode == "--layer")
            return muyo_llm::RunTransformerLayer();
        if (mode == "--forward") {
            if (argc < 3) {
                Usage(argv[0]);
                return 2;
            }
            muyo_llm::ForwardOptions options;
            bool chosePrompt = false;
            for (int i = 3; i < argc; ++i) {
                const std::string arg = argv[i];
                auto value = [&](const char* name) -> std::string {
                    if (i + 1 >= argc)
                        throw std::invalid_argument(std::string(name) + " needs a value");
                    return argv[++i];
                };
                if (arg == "-p" || arg == "--prompt") {
                    options.prompt = value("--prompt");
                    options.tokens.clear();
                    chosePrompt = true;
                } else if (arg == "--tokens") {
                    options.tokens = ParseTokens(value("--tokens"));
                    options.prompt.clear();
                    chosePrompt = true;
                }
                else if (arg == "-n" || arg == "--n-predict")
                    options.nPredict = (uint32_t)std::stoul(value("--n-predict"));
                else if (arg == "--temp" || arg == "--temperature")
                    options.sampler.temperature = std::stof(value("--temp"));
                else if (arg == "--top-k")
                    options.sampler.topK = std::stoi(value("--top-k"));
                else if (arg == "--top-p")
                    options.sampler.topP = std::stof(value("--top-p"));
                else if (arg == "--repeat-penalty")
                    options.sampler.repeatPenalty = std::stof(value("--repeat-penalty"));
                else if (arg == "--repeat-last-n")
                    options.sampler.repeatLastN = std::stoi(value("--repeat-last-n"));
                else if (arg == "--seed")
                    options.sampler.seed = std::stoull(value("--seed"));
                else if (arg == "--chat")
                    options.chat = true;
                else if (arg == "-i" || arg == "--interactive")
                    options.chat = options.interactive = true;
                else if (arg == "--system")
                    options.system = value("--system");
                else {
                    std::fprintf(stderr, "unknown --forward option: %s\n", arg.c_str());
                    return 2;
                }
            }
            if (!chosePrompt && !options.chat) {
                // A completion needs a prompt; in chat mode an empty prompt means "no initial turn".
                options.prompt = "Hello world";
                std::fprintf(stderr, "[forward] no -p/--tokens given, using -p \"%s\"\n", options.prompt.c_str());
            }
            return muyo_llm::RunFullModel(argv[2], options);
        }
    } catch (const std::invalid_argument& e) {
        std::fprintf(stderr, "%s\n", e.what());
        return 2;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
    Usage(argv[0]);
    return 2;
}
