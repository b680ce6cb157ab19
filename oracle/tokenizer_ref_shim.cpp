// TEST INFRASTRUCTURE - a C entry point over the reference's own tokenizer (src/Tokenizer.cpp with
// src/Gguf.cpp and its vendored llama.cpp unicode tables, compiled unmodified from the reference tree
// by oracle/Makefile into oracle/_ref/). Used only by tests and by the script that writes the
// tokenizer golden fixtures, to pin the product tokenizer (muyo_llm_b200/host/tokenizer.cpp); never
// by the product.
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "Gguf.h"
#include "Tokenizer.h"
#include "llama/unicode.h"

namespace
{
struct RefTok
{
    muyo_llm::GgufReader reader;
    muyo_llm::Tokenizer tok;
    explicit RefTok(const char* path) : reader(path), tok(reader) {}
};
}  // namespace

extern "C" void* ref_tok_open(const char* path)
{
    try {
        return new RefTok(path);
    } catch (const std::exception&) {
        return nullptr;
    }
}

extern "C" void ref_tok_close(void* t) { delete static_cast<RefTok*>(t); }

// Encode text[0..len); writes up to cap ids, returns the full count.
extern "C" long ref_tok_encode(void* t, const char* text, long len, int parse_special, int* out, long cap)
{
    const std::vector<int32_t> ids = static_cast<RefTok*>(t)->tok.Encode(std::string(text, len), parse_special != 0);
    for (long i = 0; i < (long)ids.size() && i < cap; ++i)
        out[i] = ids[i];
    return (long)ids.size();
}

// Decode ids into out (up to cap bytes); returns the full byte count.
extern "C" long ref_tok_decode(void* t, const int* ids, long n, char* out, long cap)
{
    const std::string s = static_cast<RefTok*>(t)->tok.Decode(std::vector<int32_t>(ids, ids + n));
    std::memcpy(out, s.data(), s.size() < (size_t)cap ? s.size() : (size_t)cap);
    return (long)s.size();
}

extern "C" int ref_tok_is_special(void* t, int id) { return static_cast<RefTok*>(t)->tok.IsSpecial(id) ? 1 : 0; }

// llama.cpp's code-point flags (unicode_cpt_flags, 16 bits) for `n` code points from `first`.
extern "C" void ref_unicode_flags(unsigned first, unsigned n, unsigned short* out)
{
    for (unsigned i = 0; i < n; ++i)
        out[i] = unicode_cpt_flags_from_cpt(first + i).as_uint();
}
