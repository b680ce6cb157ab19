// The metadata half of a GGUF file (src/Gguf.h:53-105, GgufReader): the key/value section only, for
// the tokenizer and the run's special ids. Tensor data is the device loader's (muyo_model_load_gguf).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace muyo_llm
{
/// One metadata value. Scalars keep their numeric value in `u` (unsigned types, bool), `i` (signed
/// types) or `f` (floats); arrays of strings fill `strings`, arrays of integers `ints`.
struct GgufMetaValue
{
    uint32_t type = 0;       // GGUF value type (0 u8 ... 12 f64; 8 string, 9 array)
    uint32_t elemType = 0;   // for arrays
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0.0;
    std::string str;
    std::vector<std::string> strings;
    std::vector<int64_t> ints;
};

class GgufMeta
{
public:
    /// Parses the header and metadata of the file at `path` (versions 2 and 3).
    /// @throws std::runtime_error on a missing file, a bad magic, an unknown type or a short read.
    explicit GgufMeta(const std::string& path);

    bool Has(const std::string& key) const { return m_values.count(key) != 0; }
    /// @return The value for `key`, or nullptr when absent.
    const GgufMetaValue* Find(const std::string& key) const;
    /// Same contracts as GgufReader::StringOr / UintOr / StringArraySize (src/Gguf.h:86-95).
    std::string StringOr(const std::string& key, const std::string& fallback) const;
    uint64_t UintOr(const std::string& key, uint64_t fallback) const;
    size_t StringArraySize(const std::string& key) const;

private:
    std::map<std::string, GgufMetaValue> m_values;
};
}  // namespace muyo_llm
