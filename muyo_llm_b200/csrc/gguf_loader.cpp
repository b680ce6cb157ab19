// muyo_model_load_gguf: reads a Qwen2 GGUF (F32/F16 tensors) and uploads every tensor the decode
// step reads through muyo_model_set_tensor. The parse follows the GGUF v2/v3 layout the reference's
// GgufReader walks (src/Gguf.cpp:161-373): magic, version, tensor count, KV count, KV pairs (values
// skipped here; the caller's MuyoQwen2Config carries the shape), tensor infos, aligned data section.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "muyo_cuda.h"

namespace muyo {
void set_error(const char* fmt, ...);
void clear_error();
}  // namespace muyo

namespace {

struct Reader {
    FILE* f = nullptr;
    bool ok = true;
    explicit Reader(const char* path) : f(std::fopen(path, "rb")) { ok = f != nullptr; }
    ~Reader()
    {
        if (f)
            std::fclose(f);
    }
    void bytes(void* p, size_t n)
    {
        if (ok && std::fread(p, 1, n, f) != n)
            ok = false;
    }
    uint32_t u32()
    {
        uint32_t v = 0;
        bytes(&v, 4);
        return v;
    }
    uint64_t u64()
    {
        uint64_t v = 0;
        bytes(&v, 8);
        return v;
    }
    std::string str()
    {
        const uint64_t n = u64();
        if (!ok || n > (1u << 24)) {
            ok = false;
            return {};
        }
        std::string s(n, '\0');
        bytes(s.data(), n);
        return s;
    }
    void skip_value(uint32_t type, int depth = 0)
    {
        static const int sizes[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (!ok || type > 12 || depth > 2) {
            ok = false;
            return;
        }
        if (type == 8) {
            str();
        } else if (type == 9) {
            const uint32_t et = u32();
            const uint64_t n = u64();
            if (et == 8 || et == 9) {
                for (uint64_t i = 0; i < n && ok; ++i)
                    skip_value(et, depth + 1);
            } else if (et <= 12) {
                ok = ok && std::fseek(f, (long)(n * sizes[et]), SEEK_CUR) == 0;
            } else {
                ok = false;
            }
        } else {
            ok = ok && std::fseek(f, sizes[type], SEEK_CUR) == 0;
        }
    }
};

struct TensorInfo {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type;
    uint64_t offset;
};

}  // namespace

extern "C" int muyo_model_load_gguf(MuyoModel* m, const char* path)
{
    muyo::clear_error();
    if (!m || !path) {
        muyo::set_error("load_gguf: null argument");
        return MUYO_EINVAL;
    }
    Reader r(path);
    if (!r.ok) {
        muyo::set_error("load_gguf: cannot open %s", path);
        return MUYO_EINVAL;
    }
    char magic[4] = {};
    r.bytes(magic, 4);
    if (!r.ok || std::memcmp(magic, "GGUF", 4) != 0) {
        muyo::set_error("load_gguf: %s is not a GGUF file", path);
        return MUYO_EINVAL;
    }
    const uint32_t version = r.u32();
    const uint64_t n_tensors = r.u64(), n_kv = r.u64();
    if (!r.ok || version < 2 || n_tensors > (1u << 20) || n_kv > (1u << 20)) {
        muyo::set_error("load_gguf: unsupported header (version %u)", version);
        return MUYO_EINVAL;
    }
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        const std::string key = r.str();
        const uint32_t type = r.u32();
        if (key == "general.alignment" && type == 4)
            alignment = r.u32();
        else
            r.skip_value(type);
    }
    std::vector<TensorInfo> infos;
    for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
        TensorInfo t;
        t.name = r.str();
        const uint32_t nd = r.u32();
        if (nd > 4) {
            r.ok = false;
            break;
        }
        for (uint32_t d = 0; d < nd; ++d)
            t.dims.push_back(r.u64());
        t.type = r.u32();
        t.offset = r.u64();
        infos.push_back(t);
    }
    if (!r.ok || alignment == 0) {
        muyo::set_error("load_gguf: truncated or malformed header in %s", path);
        return MUYO_EINVAL;
    }
    const long here = std::ftell(r.f);
    const uint64_t data = ((uint64_t)here + alignment - 1) / alignment * alignment;
    std::vector<char> buf;
    for (const TensorInfo& t : infos) {
        if (t.type != 0 && t.type != 1) {
            muyo::set_error("load_gguf: tensor %s has type %u; only F32 (0) and F16 (1) are supported",
                            t.name.c_str(), t.type);
            return MUYO_EUNSUPPORTED;
        }
        uint64_t n = 1;
        for (uint64_t d : t.dims)
            n *= d;
        const uint64_t bytes = n * (t.type == 1 ? 2 : 4);
        buf.resize(bytes);
        if (std::fseek(r.f, (long)(data + t.offset), SEEK_SET) != 0 || std::fread(buf.data(), 1, bytes, r.f) != bytes) {
            muyo::set_error("load_gguf: tensor %s runs past the end of %s", t.name.c_str(), path);
            return MUYO_EINVAL;
        }
        const int rc = muyo_model_set_tensor(m, t.name.c_str(), buf.data(), bytes);
        if (rc != MUYO_OK)
            return rc;
    }
    return MUYO_OK;
}

// Scalar metadata value of GGUF type `type` as a double (integers and floats), or false.
static bool read_number(Reader& r, uint32_t type, double& out)
{
    switch (type) {
        case 0: { uint8_t v = 0; r.bytes(&v, 1); out = v; return r.ok; }
        case 1: { int8_t v = 0; r.bytes(&v, 1); out = v; return r.ok; }
        case 2: { uint16_t v = 0; r.bytes(&v, 2); out = v; return r.ok; }
        case 3: { int16_t v = 0; r.bytes(&v, 2); out = v; return r.ok; }
        case 4: { out = r.u32(); return r.ok; }
        case 5: { int32_t v = 0; r.bytes(&v, 4); out = v; return r.ok; }
        case 6: { float v = 0; r.bytes(&v, 4); out = v; return r.ok; }
        case 10: { out = (double)r.u64(); return r.ok; }
        case 11: { int64_t v = 0; r.bytes(&v, 8); out = (double)v; return r.ok; }
        case 12: { double v = 0; r.bytes(&v, 8); out = v; return r.ok; }
        default: return false;
    }
}

extern "C" int muyo_gguf_read_qwen2_config(const char* path, uint32_t max_seq, uint32_t kv_dtype,
                                           MuyoQwen2Config* out)
{
    muyo::clear_error();
    if (!path || !out) {
        muyo::set_error("read_qwen2_config: null argument");
        return MUYO_EINVAL;
    }
    Reader r(path);
    char magic[4] = {};
    if (r.ok)
        r.bytes(magic, 4);
    if (!r.ok || std::memcmp(magic, "GGUF", 4) != 0) {
        muyo::set_error("read_qwen2_config: %s is not a readable GGUF file", path);
        return MUYO_EINVAL;
    }
    const uint32_t version = r.u32();
    r.u64();  // tensor count
    const uint64_t n_kv = r.u64();
    if (!r.ok || version < 2 || n_kv > (1u << 20)) {
        muyo::set_error("read_qwen2_config: unsupported header (version %u)", version);
        return MUYO_EINVAL;
    }
    double layers = 0, hidden = 0, ffn = 0, heads = 0, kv_heads = 0, eps = 0, base = 10000.0;
    uint64_t vocab = 0;
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        const std::string key = r.str();
        const uint32_t type = r.u32();
        double* num = key == "qwen2.block_count"                        ? &layers
                      : key == "qwen2.embedding_length"                 ? &hidden
                      : key == "qwen2.feed_forward_length"              ? &ffn
                      : key == "qwen2.attention.head_count"             ? &heads
                      : key == "qwen2.attention.head_count_kv"          ? &kv_heads
                      : key == "qwen2.attention.layer_norm_rms_epsilon" ? &eps
                      : key == "qwen2.rope.freq_base"                   ? &base
                                                                        : nullptr;
        if (num && type != 8 && type != 9) {
            if (!read_number(r, type, *num))
                r.ok = false;
        } else if (key == "tokenizer.ggml.tokens" && type == 9) {
            const uint32_t et = r.u32();
            const uint64_t n = r.u64();
            vocab = n;
            for (uint64_t k = 0; k < n && r.ok; ++k)
                r.skip_value(et, 1);
        } else {
            r.skip_value(type);
        }
    }
    if (!r.ok) {
        muyo::set_error("read_qwen2_config: %s: truncated or malformed metadata", path);
        return MUYO_EINVAL;
    }
    if (hidden <= 0 || heads <= 0 || kv_heads <= 0 || vocab == 0 || layers <= 0 || ffn <= 0) {
        muyo::set_error("read_qwen2_config: %s is missing the qwen2 dimensions or the token list", path);
        return MUYO_EINVAL;
    }
    out->layers = (uint32_t)layers;
    out->hidden = (uint32_t)hidden;
    out->ffn = (uint32_t)ffn;
    out->heads = (uint32_t)heads;
    out->kv_heads = (uint32_t)kv_heads;
    out->vocab = (uint32_t)vocab;
    out->max_seq = max_seq;
    out->rms_eps = (float)eps;
    out->rope_base = (float)base;
    out->kv_dtype = kv_dtype;
    return MUYO_OK;
}
