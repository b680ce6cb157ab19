// Byte-level BPE tokenizer and Qwen2 chat framing read from a GGUF's tokenizer.ggml.* metadata: the
// reference's Tokenizer (src/Tokenizer.h:1-89) and chat_template (src/ChatTemplate.h:1-31), with the
// same method names, arguments and results. Host-only: the decode kernels consume and produce ids.
#pragma once

#include <cstdint>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "gguf_meta.h"

namespace muyo_llm
{
class Tokenizer
{
public:
    /// Reads tokenizer.ggml.tokens / merges / token_type / pre from `meta`.
    /// @throws std::runtime_error when the file has no tokenizer.ggml.tokens.
    explicit Tokenizer(const GgufMeta& meta);

    /// Text -> ids. With parseSpecial, the longest special token (token type 3 CONTROL or 4
    /// USER_DEFINED) starting at each position is emitted as its id; the text between special
    /// tokens is split by the pre-tokenizer and each piece byte-encoded and merged.
    /// @throws std::runtime_error on a decoded code point above U+10FFFF (a 4-byte sequence led by
    /// 0xF4 above U+10FFFF or by 0xF5..0xF7), which the reference's split also rejects.
    std::vector<int32_t> Encode(const std::string& text, bool parseSpecial = true) const;
    /// Ids -> bytes (ids out of range are skipped).
    std::string Decode(const std::vector<int32_t>& ids) const;
    /// The bytes of one token ("" for an id out of range).
    std::string TokenBytes(int32_t id) const;
    bool IsSpecial(int32_t id) const;
    size_t VocabSize() const { return m_tokens.size(); }
    /// The token's vocabulary string as stored (byte-encoded), "" out of range.
    const std::string& TokenFor(size_t id) const;

    /// The pre-tokenizer's split of `text` into UTF-8 pieces (exposed for tests).
    std::vector<std::string> PreTokenize(const std::string& text) const;

private:
    void MergePiece(const std::string& encoded, std::vector<int32_t>& out) const;

    std::vector<std::string> m_tokens;        // id -> vocabulary string
    std::vector<std::string> m_bytes;         // id -> decoded bytes
    std::unordered_map<std::string, int32_t> m_ids;
    std::unordered_map<std::string, int32_t> m_mergeRank;  // "left right" -> rank (first one wins)
    std::vector<uint8_t> m_special;           // id -> 1 for token types 3 and 4
    // Special tokens by first byte, longest text first (then lowest id).
    std::vector<std::vector<std::pair<std::string, int32_t>>> m_specialByByte;
    bool m_qwen2Split = false;                // tokenizer.ggml.pre selects the Qwen2 split, else GPT-2's
    // Ids of pieces already merged (a word recurs often in a text); bounded, emptied when full.
    mutable std::mutex m_cacheMutex;
    mutable std::unordered_map<std::string, std::vector<int32_t>> m_pieceCache;
};

/// Qwen2.5's ChatML framing (src/ChatTemplate.h:14-30).
namespace chat_template
{
inline constexpr char QWEN2_DEFAULT_SYSTEM[] = "You are Qwen, created by Alibaba Cloud. You are a helpful assistant.";
/// `<|im_start|>system\n{system}<|im_end|>\n`
std::string Qwen2SystemStart(const std::string& system);
/// `<|im_start|>user\n{user}<|im_end|>\n<|im_start|>assistant\n`
std::string Qwen2UserTurn(const std::string& user);
/// Qwen2SystemStart(system) + Qwen2UserTurn(user).
std::string Qwen2ChatStart(const std::string& system, const std::string& user);
}  // namespace chat_template
}  // namespace muyo_llm
