// GGUF header + key/value parse (the format of src/Gguf.cpp:161-336: magic "GGUF", version, tensor
// count, key/value count, then typed values; strings are a u64 length and bytes, arrays a u32
// element type, a u64 count and the elements). Reads through one buffered stream and stops before
// the tensor table.
#include "gguf_meta.h"

#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>

namespace muyo_llm
{
namespace
{
enum : uint32_t
{
    T_U8 = 0, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STRING, T_ARRAY, T_U64, T_I64, T_F64
};

class Stream
{
public:
    explicit Stream(const std::string& path) : m_f(std::fopen(path.c_str(), "rb"), &std::fclose)
    {
        if (!m_f)
            throw std::runtime_error("GGUF: cannot open " + path);
    }
    void Read(void* dst, size_t n)
    {
        if (n != 0 && std::fread(dst, 1, n, m_f.get()) != n)
            throw std::runtime_error("GGUF: truncated metadata");
    }
    template <typename T> T Get()
    {
        T v;
        Read(&v, sizeof v);
        return v;
    }
    std::string String()
    {
        const uint64_t n = Get<uint64_t>();
        if (n > (uint64_t(1) << 32))
            throw std::runtime_error("GGUF: implausible string length");
        std::string s(n, '\0');
        Read(s.data(), n);
        return s;
    }

private:
    std::unique_ptr<FILE, int (*)(FILE*)> m_f;
};

size_t ScalarBytes(uint32_t t)
{
    switch (t) {
    case T_U8: case T_I8: case T_BOOL: return 1;
    case T_U16: case T_I16: return 2;
    case T_U32: case T_I32: case T_F32: return 4;
    case T_U64: case T_I64: case T_F64: return 8;
    default: throw std::runtime_error("GGUF: unknown value type " + std::to_string(t));
    }
}

// One scalar of type t into (u, i, f).
void Scalar(Stream& s, uint32_t t, uint64_t& u, int64_t& i, double& f)
{
    unsigned char b[8] = {};
    s.Read(b, ScalarBytes(t));
    auto as = [&b](auto v) {
        std::memcpy(&v, b, sizeof v);
        return v;
    };
    switch (t) {
    case T_U8: case T_BOOL: u = as(uint8_t{}); i = (int64_t)u; break;
    case T_U16: u = as(uint16_t{}); i = (int64_t)u; break;
    case T_U32: u = as(uint32_t{}); i = (int64_t)u; break;
    case T_U64: u = as(uint64_t{}); i = (int64_t)u; break;
    case T_I8: i = as(int8_t{}); u = (uint64_t)i; break;
    case T_I16: i = as(int16_t{}); u = (uint64_t)i; break;
    case T_I32: i = as(int32_t{}); u = (uint64_t)i; break;
    case T_I64: i = as(int64_t{}); u = (uint64_t)i; break;
    case T_F32: f = as(float{}); break;
    case T_F64: f = as(double{}); break;
    }
    if (t != T_F32 && t != T_F64)
        f = (double)i;
}
}  // namespace

GgufMeta::GgufMeta(const std::string& path)
{
    Stream s(path);
    char magic[4];
    s.Read(magic, 4);
    if (std::memcmp(magic, "GGUF", 4) != 0)
        throw std::runtime_error("GGUF: bad magic in " + path);
    const uint32_t version = s.Get<uint32_t>();
    if (version < 2 || version > 3)
        throw std::runtime_error("GGUF: unsupported version " + std::to_string(version));
    (void)s.Get<uint64_t>();  // tensor count: the tensor table is not read here
    const uint64_t nkv = s.Get<uint64_t>();
    for (uint64_t k = 0; k < nkv; ++k) {
        std::string key = s.String();
        GgufMetaValue v;
        v.type = s.Get<uint32_t>();
        if (v.type == T_STRING) {
            v.str = s.String();
        } else if (v.type == T_ARRAY) {
            v.elemType = s.Get<uint32_t>();
            const uint64_t n = s.Get<uint64_t>();
            if (v.elemType == T_STRING) {
                v.strings.reserve(n);
                for (uint64_t j = 0; j < n; ++j)
                    v.strings.push_back(s.String());
            } else if (v.elemType == T_ARRAY) {
                throw std::runtime_error("GGUF: nested arrays are not supported (key " + key + ")");
            } else {
                v.ints.reserve(n);
                for (uint64_t j = 0; j < n; ++j) {
                    uint64_t u;
                    int64_t i;
                    double f;
                    Scalar(s, v.elemType, u, i, f);
                    v.ints.push_back(v.elemType == T_F32 || v.elemType == T_F64 ? (int64_t)f : i);
                }
            }
        } else {
            Scalar(s, v.type, v.u, v.i, v.f);
        }
        m_values.emplace(std::move(key), std::move(v));  // a repeated key keeps its first value
    }
}

const GgufMetaValue* GgufMeta::Find(const std::string& key) const
{
    const auto it = m_values.find(key);
    return it == m_values.end() ? nullptr : &it->second;
}

std::string GgufMeta::StringOr(const std::string& key, const std::string& fallback) const
{
    const GgufMetaValue* v = Find(key);
    return v && v->type == T_STRING ? v->str : fallback;
}

uint64_t GgufMeta::UintOr(const std::string& key, uint64_t fallback) const
{
    const GgufMetaValue* v = Find(key);
    if (!v || v->type == T_STRING || v->type == T_ARRAY)
        return fallback;
    return v->type == T_F32 || v->type == T_F64 ? (uint64_t)v->f : v->u;
}

size_t GgufMeta::StringArraySize(const std::string& key) const
{
    const GgufMetaValue* v = Find(key);
    return v && v->type == T_ARRAY && v->elemType == T_STRING ? v->strings.size() : 0;
}
}  // namespace muyo_llm
