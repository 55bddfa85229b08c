// gguf_file.cu -- read-only GGUF v2/v3 container parser (host code).
//
// The part of gguf_init_from_file (the gguf API behind src/models/gguf_loader.cpp:9-162) that the BitVLA
// engine needs: the file is memory-mapped, the key/value metadata is parsed into typed scalars, strings
// and arrays, and every tensor's name, shape (ggml order, ne[0] innermost), ggml type and data pointer is
// indexed. Layout: "GGUF" magic, u32 version, u64 tensor count, u64 kv count, the kv pairs, the tensor
// infos (name, u32 n_dims, u64 ne[n_dims], u32 type, u64 offset), padding to general.alignment (default
// 32), then the tensor data, each tensor at its offset from the data start. Tensor byte sizes follow the
// ggml type: F32 4 bytes per element, I2_S (type 36, the BitNet fork's 2-bit ternary) n/4 codes plus a
// 32-byte trailer holding the fp32 scale.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <vector>

#include "b2s_internal.h"

namespace b2s {

namespace {
enum : uint32_t {
    kU8 = 0, kI8, kU16, kI16, kU32, kI32, kF32, kBool, kString, kArray, kU64, kI64, kF64
};
size_t scalar_size(uint32_t t) {
    switch (t) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}
}  // namespace

struct GgufReader {
    const uint8_t* p;
    const uint8_t* end;
    bool ok = true;
    template <typename T>
    T get() {
        T v{};
        if (end - p < (ptrdiff_t)sizeof(T)) { ok = false; return v; }
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || (uint64_t)(end - p) < n) { ok = false; return {}; }
        std::string s(reinterpret_cast<const char*>(p), (size_t)n);
        p += n;
        return s;
    }
};

GgufFile::~GgufFile() { close(); }

void GgufFile::close() {
    if (map_ && map_ != MAP_FAILED) munmap(const_cast<void*>(map_), size_);
    map_ = nullptr;
    size_ = 0;
    kv_.clear();
    tensors_.clear();
}

bool GgufFile::open(const char* path, std::string* err) {
    close();
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) { *err = std::string("cannot open GGUF file: ") + path; return false; }
    struct stat st{};
    if (fstat(fd, &st) != 0 || st.st_size < 24) { ::close(fd); *err = "GGUF file too small"; return false; }
    size_ = (size_t)st.st_size;
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) { map_ = nullptr; *err = "mmap of the GGUF file failed"; return false; }
    map_ = m;
    GgufReader r{static_cast<const uint8_t*>(map_), static_cast<const uint8_t*>(map_) + size_};
    if (r.get<uint32_t>() != 0x46554747u) { *err = "not a GGUF file (bad magic)"; return false; }
    const uint32_t version = r.get<uint32_t>();
    if (version < 2 || version > 3) { *err = "unsupported GGUF version " + std::to_string(version); return false; }
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    if (!r.ok || n_tensors > (1u << 24) || n_kv > (1u << 24)) { *err = "corrupt GGUF header"; return false; }
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        GgufValue v;
        const std::string key = r.str();
        v.type = r.get<uint32_t>();
        if (v.type == kString) {
            v.s = r.str();
        } else if (v.type == kArray) {
            v.arr_type = r.get<uint32_t>();
            const uint64_t n = r.get<uint64_t>();
            v.arr_n = n;
            if (v.arr_type == kString) {
                for (uint64_t j = 0; j < n && r.ok; ++j) (void)r.str();
            } else {
                const size_t es = scalar_size(v.arr_type);
                if (!es || (uint64_t)(r.end - r.p) / es < n) { r.ok = false; break; }
                v.arr = r.p;
                r.p += es * n;
            }
        } else {
            const size_t es = scalar_size(v.type);
            if (!es || r.end - r.p < (ptrdiff_t)es) { r.ok = false; break; }
            memcpy(v.raw, r.p, es);
            r.p += es;
        }
        kv_[key] = v;
    }
    if (!r.ok) { *err = "corrupt GGUF metadata"; return false; }
    std::vector<std::pair<std::string, GgufTensor>> infos;
    for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
        GgufTensor t;
        const std::string name = r.str();
        const uint32_t nd = r.get<uint32_t>();
        if (nd == 0 || nd > 4) { r.ok = false; break; }
        for (uint32_t d = 0; d < nd; ++d) t.ne[d] = (int64_t)r.get<uint64_t>();
        for (uint32_t d = nd; d < 4; ++d) t.ne[d] = 1;
        t.type = r.get<uint32_t>();
        t.offset = r.get<uint64_t>();
        infos.emplace_back(name, t);
    }
    if (!r.ok) { *err = "corrupt GGUF tensor infos"; return false; }
    uint64_t align = 32;
    auto it = kv_.find("general.alignment");
    if (it != kv_.end() && it->second.type == kU32) {
        uint32_t a;
        memcpy(&a, it->second.raw, 4);
        if (a) align = a;
    }
    const size_t header = (size_t)(r.p - static_cast<const uint8_t*>(map_));
    const size_t data0 = (header + align - 1) / align * align;
    for (auto& [name, t] : infos) {
        const int64_t n = t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3];
        if (t.type == 0) t.nbytes = (size_t)n * 4;
        else if (t.type == 36) t.nbytes = (size_t)(n / 4) + 32;
        else t.nbytes = 0;  // other ggml types are not read by this library
        if (t.offset > size_ || t.nbytes > size_ || data0 + t.offset + t.nbytes > size_) { *err = "tensor '" + name + "' extends past the end of the file"; return false; }
        t.data = static_cast<const uint8_t*>(map_) + data0 + t.offset;
        tensors_[name] = t;
    }
    return true;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

bool GgufFile::u32(const std::string& key, uint32_t* out) const {
    auto it = kv_.find(key);
    if (it == kv_.end()) return false;
    const GgufValue& v = it->second;
    if (v.type == kU32 || v.type == kI32) { memcpy(out, v.raw, 4); return true; }
    if (v.type == kU64 || v.type == kI64) { uint64_t x; memcpy(&x, v.raw, 8); *out = (uint32_t)x; return true; }
    return false;
}

bool GgufFile::f32(const std::string& key, float* out) const {
    auto it = kv_.find(key);
    if (it == kv_.end()) return false;
    const GgufValue& v = it->second;
    if (v.type == kF32) { memcpy(out, v.raw, 4); return true; }
    if (v.type == kF64) { double x; memcpy(&x, v.raw, 8); *out = (float)x; return true; }
    return false;
}

bool GgufFile::str(const std::string& key, std::string* out) const {
    auto it = kv_.find(key);
    if (it == kv_.end() || it->second.type != kString) return false;
    *out = it->second.s;
    return true;
}

}  // namespace b2s
