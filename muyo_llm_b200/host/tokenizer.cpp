// Byte-level BPE over a GGUF vocabulary (src/Tokenizer.cpp:88-345 for the behaviour it reproduces):
//
//   text --special-token scan--> runs of plain text and special ids
//   run  --code points (UTF-8, invalid bytes -> U+FFFD)--> pre-tokenizer pieces (Qwen2 or GPT-2 rules)
//   piece --GPT-2 byte map--> one symbol per byte --lowest-rank merges--> vocabulary ids
//
// The pre-tokenizers are hand-written scanners over four code-point classes (letter, number, white
// space, other; unicode_classes.inc), one per split rule of llama.cpp's pre-types "qwen2" and
// "gpt2" (the regexes in the comments), with llama.cpp's segment-boundary behaviour: a white-space
// run followed by more text gives its last character to the next piece. Merging keeps a min-heap of
// adjacent pairs keyed (rank, position), which applies the same merge as rescanning for the lowest
// rank, leftmost on ties, at every step.
#include "tokenizer.h"

#include <algorithm>
#include <queue>
#include <stdexcept>

namespace muyo_llm
{
namespace
{
#include "unicode_classes.inc"

enum : uint8_t
{
    C_OTHER = 0,
    C_LETTER = 1,
    C_NUMBER = 2,
    C_SPACE = 3,
    C_END = 4  // past the end of the text: no code point
};

constexpr uint32_t kReplacement = 0xFFFD;
constexpr uint32_t kMaxCodePoint = 0x10FFFF;

uint8_t ClassOf(uint32_t cp)
{
    if (cp > kMaxCodePoint)
        return C_OTHER;  // decodable from 0xF4..0xF7 leads; llama.cpp flags it undefined
    const uint32_t* it = std::upper_bound(kUniStart, kUniStart + sizeof(kUniStart) / sizeof(kUniStart[0]), cp);
    return kUniClass[(it - kUniStart) - 1];
}

bool IsCont(unsigned char b) { return (b & 0xC0) == 0x80; }

// Strict UTF-8 to code points as llama.cpp's unicode_cpts_from_utf8 decodes (src/llama/unicode.cpp:
// 30-66, 1130-1145): a lead byte needs all its continuation bytes, else it becomes U+FFFD and only
// that byte is consumed. Overlong forms are accepted as their value.
std::vector<uint32_t> CodePoints(const char* s, size_t n)
{
    std::vector<uint32_t> cps;
    cps.reserve(n);
    size_t i = 0;
    while (i < n) {
        const auto b = static_cast<unsigned char>(s[i]);
        size_t len = 0;
        uint32_t cp = 0;
        if (b < 0x80) {
            len = 1, cp = b;
        } else if (b >= 0xC0 && b < 0xE0) {
            len = 2, cp = b & 0x1F;
        } else if (b >= 0xE0 && b < 0xF0) {
            len = 3, cp = b & 0x0F;
        } else if (b >= 0xF0 && b < 0xF8) {
            len = 4, cp = b & 0x07;
        }
        bool ok = len > 0 && i + len <= n;
        for (size_t k = 1; ok && k < len; ++k) {
            const auto c = static_cast<unsigned char>(s[i + k]);
            ok = IsCont(c);
            cp = (cp << 6) | (c & 0x3F);
        }
        if (ok) {
            cps.push_back(cp);
            i += len;
        } else {
            cps.push_back(kReplacement);
            i += 1;
        }
    }
    return cps;
}

void AppendUtf8(std::string& out, uint32_t cp)
{
    if (cp < 0x80) {
        out.push_back(static_cast<char>(cp));
    } else if (cp < 0x800) {
        out.push_back(static_cast<char>(0xC0 | (cp >> 6)));
        out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
        out.push_back(static_cast<char>(0xE0 | (cp >> 12)));
        out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
        out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else if (cp <= kMaxCodePoint) {
        out.push_back(static_cast<char>(0xF0 | (cp >> 18)));
        out.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
        out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
        out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else {
        throw std::runtime_error("tokenizer: code point above U+10FFFF in the input");
    }
}

// The tolerant decode the reference applies to vocabulary strings (src/Tokenizer.cpp:43-67): the
// lead byte alone fixes the length, continuation bytes are taken as they are, a truncated sequence
// ends the string.
std::vector<uint32_t> LooseCodePoints(const std::string& s)
{
    std::vector<uint32_t> cps;
    size_t i = 0;
    while (i < s.size()) {
        const auto b = static_cast<unsigned char>(s[i]);
        size_t len = b >= 0xF0 ? 4 : b >= 0xE0 ? 3 : b >= 0xC0 ? 2 : 1;
        uint32_t cp = len == 4 ? b & 0x07u : len == 3 ? b & 0x0Fu : len == 2 ? b & 0x1Fu : b;
        for (size_t k = 1; k < len && i + k < s.size(); ++k)
            cp = (cp << 6) | (static_cast<unsigned char>(s[i + k]) & 0x3Fu);
        cps.push_back(cp);
        i += len;
    }
    return cps;
}

// Byte-length of each code point of a well-formed UTF-8 string, in order.
size_t Utf8Len(unsigned char lead) { return lead >= 0xF0 ? 4 : lead >= 0xE0 ? 3 : lead >= 0xC0 ? 2 : 1; }

// GPT-2's reversible byte -> code point map: the printable bytes '!'..'~', 0xA1..0xAC and 0xAE..0xFF
// stand for themselves; the other 68 bytes take U+0100.. in byte order.
struct ByteMap
{
    std::string encoded[256];  // byte -> UTF-8 of its code point
    int16_t decode[324];       // code point -> byte, -1 when none
    ByteMap()
    {
        std::fill(decode, decode + 324, int16_t(-1));
        uint32_t next = 256;
        for (int b = 0; b < 256; ++b) {
            const bool self = (b >= '!' && b <= '~') || (b >= 0xA1 && b <= 0xAC) || b >= 0xAE;
            const uint32_t cp = self ? uint32_t(b) : next++;
            AppendUtf8(encoded[b], cp);
            decode[cp] = int16_t(b);
        }
    }
};

const ByteMap& Bytes()
{
    static const ByteMap map;
    return map;
}

// A piece is [begin, end) in code-point indices.
using Pieces = std::vector<std::pair<size_t, size_t>>;

uint32_t LowerAscii(uint32_t c) { return c >= 'A' && c <= 'Z' ? c + 32 : c; }

// Length of a contraction starting at p ('s 't 'm 'd 're 've 'll), 0 if none. `fold` lowercases
// the letters (Qwen2's case-insensitive form).
size_t Contraction(const std::vector<uint32_t>& cp, size_t p, bool fold)
{
    const size_t n = cp.size();
    if (cp[p] != '\'' || p + 1 >= n)
        return 0;
    const uint32_t a = fold ? LowerAscii(cp[p + 1]) : cp[p + 1];
    if (a == 's' || a == 't' || a == 'm' || a == 'd')
        return 2;
    if (p + 2 >= n)
        return 0;
    const uint32_t b = fold ? LowerAscii(cp[p + 2]) : cp[p + 2];
    if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l'))
        return 3;
    return 0;
}

// (?:'[sS]|'[tT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD])|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}|
//  ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+
Pieces SplitQwen2(const std::vector<uint32_t>& cp, const std::vector<uint8_t>& cls)
{
    const size_t n = cp.size();
    auto C = [&](size_t p) { return p < n ? cls[p] : uint8_t(C_END); };
    auto nl = [&](size_t p) { return p < n && (cp[p] == '\r' || cp[p] == '\n'); };
    Pieces out;
    size_t p = 0;
    while (p < n) {
        size_t e = 0;
        if (size_t c = Contraction(cp, p, true)) {
            e = p + c;
        } else if (!nl(p) && C(p) != C_NUMBER && (C(p) == C_LETTER || C(p + 1) == C_LETTER)) {
            e = p + 1;  // an optional non-letter lead, then the letter run
            while (C(e) == C_LETTER)
                ++e;
        } else if (C(p) == C_NUMBER) {
            e = p + 1;  // one digit per piece
        } else if ((cp[p] == ' ' ? C(p + 1) : C(p)) == C_OTHER) {
            e = p + (cp[p] == ' ');
            while (C(e) == C_OTHER)
                ++e;
            while (nl(e))
                ++e;
        } else {
            size_t run = p, lastNl = 0;
            while (C(run) == C_SPACE) {
                if (nl(run))
                    lastNl = run + 1;
                ++run;
            }
            if (lastNl != 0)
                e = lastNl;  // up to the last line break of the run
            else if (run - p > 1 && run < n)
                e = run - 1;  // leave the last blank to the text that follows
            else
                e = std::max(run, p + 1);
        }
        out.emplace_back(p, e);
        p = e;
    }
    return out;
}

// 's|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+
Pieces SplitGpt2(const std::vector<uint32_t>& cp, const std::vector<uint8_t>& cls)
{
    const size_t n = cp.size();
    auto C = [&](size_t p) { return p < n ? cls[p] : uint8_t(C_END); };
    Pieces out;
    size_t p = 0;
    while (p < n) {
        size_t e = 0;
        const uint8_t lead = cp[p] == ' ' ? C(p + 1) : C(p);
        if (size_t c = Contraction(cp, p, false)) {
            e = p + c;
        } else if (lead == C_LETTER || lead == C_NUMBER || lead == C_OTHER) {
            e = p + (cp[p] == ' ');  // an optional space, then a run of one class
            while (C(e) == lead)
                ++e;
        } else {
            size_t run = p;
            while (C(run) == C_SPACE)
                ++run;
            if (run - p > 1 && run < n)
                e = run - 1;
            else
                e = std::max(run, p + 1);
        }
        out.emplace_back(p, e);
        p = e;
    }
    return out;
}

struct PairEntry
{
    int32_t rank;
    uint32_t pos;  // byte offset of the left symbol in the encoded piece
    int32_t left, right;
    uint32_t leftLen, rightLen;
    bool operator>(const PairEntry& o) const { return rank != o.rank ? rank > o.rank : pos > o.pos; }
};
}  // namespace

Tokenizer::Tokenizer(const GgufMeta& meta)
{
    const GgufMetaValue* tokens = meta.Find("tokenizer.ggml.tokens");
    if (!tokens || tokens->strings.empty())
        throw std::runtime_error("Tokenizer: GGUF has no tokenizer.ggml.tokens");
    m_tokens = tokens->strings;
    m_ids.reserve(m_tokens.size() * 2);
    m_bytes.resize(m_tokens.size());
    const ByteMap& bm = Bytes();
    for (size_t i = 0; i < m_tokens.size(); ++i) {
        m_ids.emplace(m_tokens[i], static_cast<int32_t>(i));  // a repeated string keeps its first id
        for (uint32_t c : LooseCodePoints(m_tokens[i]))
            if (c < 324 && bm.decode[c] >= 0)
                m_bytes[i].push_back(static_cast<char>(bm.decode[c]));
    }
    if (const GgufMetaValue* merges = meta.Find("tokenizer.ggml.merges")) {
        m_mergeRank.reserve(merges->strings.size() * 2);
        for (size_t r = 0; r < merges->strings.size(); ++r) {
            // The first space separates the pair: no byte maps to a raw space (0x20 -> U+0120).
            const std::string& s = merges->strings[r];
            const size_t sp = s.find(' ');
            if (sp != std::string::npos && s.find(' ', sp + 1) == std::string::npos)
                m_mergeRank.emplace(s, static_cast<int32_t>(r));
        }
    }
    const std::string pre = meta.StringOr("tokenizer.ggml.pre", "gpt2");
    m_qwen2Split = pre == "qwen2" || pre == "stablelm2" || pre == "hunyuan" || pre == "solar-open";

    m_specialByByte.resize(256);
    const GgufMetaValue* types = meta.Find("tokenizer.ggml.token_type");
    if (types && types->type == 9 && types->elemType == 5) {  // an array of int32, as the reference reads it
        m_special.assign(m_tokens.size(), 0);
        for (size_t i = 0; i < types->ints.size() && i < m_tokens.size(); ++i) {
            if (types->ints[i] != 3 && types->ints[i] != 4)
                continue;
            m_special[i] = 1;
            // An empty special text can never be matched usefully; the reference would emit it
            // forever at one position, so it is left out of the scan.
            if (!m_tokens[i].empty())
                m_specialByByte[static_cast<unsigned char>(m_tokens[i][0])].emplace_back(m_tokens[i],
                                                                                          static_cast<int32_t>(i));
        }
        for (auto& list : m_specialByByte)
            std::stable_sort(list.begin(), list.end(),
                             [](const auto& a, const auto& b) { return a.first.size() > b.first.size(); });
    }
}

std::vector<std::string> Tokenizer::PreTokenize(const std::string& text) const
{
    const std::vector<uint32_t> cps = CodePoints(text.data(), text.size());
    std::vector<uint8_t> cls(cps.size());
    for (size_t i = 0; i < cps.size(); ++i)
        cls[i] = cps[i] < 128 ? (cps[i] >= 'a' && cps[i] <= 'z') || (cps[i] >= 'A' && cps[i] <= 'Z') ? C_LETTER
                                : cps[i] >= '0' && cps[i] <= '9'                                    ? C_NUMBER
                                : (cps[i] >= 9 && cps[i] <= 13) || cps[i] == ' '                    ? C_SPACE
                                                                                                    : C_OTHER
                                : ClassOf(cps[i]);
    const Pieces pieces = m_qwen2Split ? SplitQwen2(cps, cls) : SplitGpt2(cps, cls);
    std::vector<std::string> out;
    out.reserve(pieces.size());
    for (const auto& [b, e] : pieces) {
        out.emplace_back();
        for (size_t i = b; i < e; ++i)
            AppendUtf8(out.back(), cps[i]);
    }
    return out;
}

void Tokenizer::MergePiece(const std::string& enc, std::vector<int32_t>& out) const
{
    // Symbols: one per code point of the byte-encoded piece, linked left to right.
    std::vector<uint32_t> start, len;
    std::vector<int32_t> next, prev;
    for (size_t i = 0; i < enc.size();) {
        const size_t l = Utf8Len(static_cast<unsigned char>(enc[i]));
        start.push_back(uint32_t(i));
        len.push_back(uint32_t(l));
        i += l;
    }
    const int32_t n = static_cast<int32_t>(start.size());
    for (int32_t i = 0; i < n; ++i) {
        prev.push_back(i - 1);
        next.push_back(i + 1 < n ? i + 1 : -1);
    }
    std::string key;
    std::priority_queue<PairEntry, std::vector<PairEntry>, std::greater<PairEntry>> heap;
    auto push = [&](int32_t a, int32_t b) {
        if (a < 0 || b < 0)
            return;
        key.assign(enc, start[a], len[a]);
        key.push_back(' ');
        key.append(enc, start[b], len[b]);
        const auto it = m_mergeRank.find(key);
        if (it != m_mergeRank.end())
            heap.push(PairEntry{it->second, start[a], a, b, len[a], len[b]});
    };
    for (int32_t i = 0; i + 1 < n; ++i)
        push(i, i + 1);
    while (!heap.empty()) {
        const PairEntry top = heap.top();
        heap.pop();
        // Stale when either side has merged since the pair was pushed.
        if (len[top.left] != top.leftLen || len[top.right] != top.rightLen || next[top.left] != top.right)
            continue;
        len[top.left] += len[top.right];
        len[top.right] = 0;  // dead
        next[top.left] = next[top.right];
        if (next[top.left] >= 0)
            prev[next[top.left]] = top.left;
        push(prev[top.left], top.left);
        push(top.left, next[top.left]);
    }
    for (int32_t i = n > 0 ? 0 : -1; i >= 0; i = next[i]) {
        key.assign(enc, start[i], len[i]);
        const auto it = m_ids.find(key);
        if (it != m_ids.end()) {
            out.push_back(it->second);
            continue;
        }
        // Not in the vocabulary: one id per code point, skipping any that are missing too.
        for (size_t j = 0; j < key.size();) {
            const size_t l = Utf8Len(static_cast<unsigned char>(key[j]));
            const auto single = m_ids.find(key.substr(j, l));
            if (single != m_ids.end())
                out.push_back(single->second);
            j += l;
        }
    }
}

std::vector<int32_t> Tokenizer::Encode(const std::string& text, bool parseSpecial) const
{
    std::vector<int32_t> ids;
    const ByteMap& bm = Bytes();
    constexpr size_t kCacheEntries = 1 << 16;
    auto plain = [&](size_t b, size_t e) {
        if (e <= b)
            return;
        std::string enc;
        std::vector<int32_t> merged;
        for (const std::string& piece : PreTokenize(text.substr(b, e - b))) {
            {
                std::lock_guard<std::mutex> lock(m_cacheMutex);
                const auto it = m_pieceCache.find(piece);
                if (it != m_pieceCache.end()) {
                    ids.insert(ids.end(), it->second.begin(), it->second.end());
                    continue;
                }
            }
            enc.clear();
            for (unsigned char c : piece)
                enc += bm.encoded[c];
            merged.clear();
            MergePiece(enc, merged);
            ids.insert(ids.end(), merged.begin(), merged.end());
            std::lock_guard<std::mutex> lock(m_cacheMutex);
            if (m_pieceCache.size() >= kCacheEntries)
                m_pieceCache.clear();
            m_pieceCache.emplace(piece, merged);
        }
    };
    size_t runStart = 0, i = 0;
    while (i < text.size()) {
        const std::pair<std::string, int32_t>* hit = nullptr;
        if (parseSpecial)
            for (const auto& sp : m_specialByByte[static_cast<unsigned char>(text[i])])
                if (text.compare(i, sp.first.size(), sp.first) == 0) {
                    hit = &sp;  // longest first
                    break;
                }
        if (!hit) {
            ++i;
            continue;
        }
        plain(runStart, i);
        ids.push_back(hit->second);
        i += hit->first.size();
        runStart = i;
    }
    plain(runStart, text.size());
    return ids;
}

std::string Tokenizer::TokenBytes(int32_t id) const
{
    return id >= 0 && static_cast<size_t>(id) < m_bytes.size() ? m_bytes[static_cast<size_t>(id)] : std::string();
}

bool Tokenizer::IsSpecial(int32_t id) const
{
    return id >= 0 && static_cast<size_t>(id) < m_special.size() && m_special[static_cast<size_t>(id)] != 0;
}

std::string Tokenizer::Decode(const std::vector<int32_t>& ids) const
{
    std::string text;
    for (int32_t id : ids)
        text += TokenBytes(id);
    return text;
}

const std::string& Tokenizer::TokenFor(size_t id) const
{
    static const std::string empty;
    return id < m_tokens.size() ? m_tokens[id] : empty;
}

namespace chat_template
{
std::string Qwen2SystemStart(const std::string& system) { return "<|im_start|>system\n" + system + "<|im_end|>\n"; }

std::string Qwen2UserTurn(const std::string& user)
{
    return "<|im_start|>user\n" + user + "<|im_end|>\n<|im_start|>assistant\n";
}

std::string Qwen2ChatStart(const std::string& system, const std::string& user)
{
    return Qwen2SystemStart(system) + Qwen2UserTurn(user);
}
}  // namespace chat_template
}  // namespace muyo_llm
