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
