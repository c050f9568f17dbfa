// af_gguf.cpp — minimal mmap GGUF v2/v3 reader for the engine's own loader
// (af_engine_load_gguf).  Same parse as GgufReader::parse
// (src/loader/gguf_loader.cpp:84-163) and the exact block byte sizes of
// gguf_tensor_nbytes (include/axonforge/dtype.hpp:136-155).
#include "af_gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>

namespace af {

static size_t pod_size(int t) {
    switch (t) {
        case 0: case 1: case 7: return 1;
        case 2: case 3: return 2;
        case 4: case 5: case 6: return 4;
        case 10: case 11: case 12: return 8;
        default: return 0;
    }
}

size_t ggml_nbytes(int type, int64_t numel) {
    const size_t n = (size_t)numel;
    switch (type) {
        case 0: return n * 4;
        case 1: case 30: return n * 2;
        case 8: return (n + 31) / 32 * 34;
        case 12: return (n + 255) / 256 * 144;
        case 14: return (n + 255) / 256 * 210;
        default: return 0;
    }
}

GgufFile::~GgufFile() {
    if (base_) munmap(const_cast<uint8_t*>(base_), size_);
}

void GgufFile::need(size_t n) const {
    if (cur_ + n > size_) throw std::runtime_error("GGUF: unexpected end of file (truncated)");
}

std::string GgufFile::str() {
    uint64_t n;
    need(8);
    std::memcpy(&n, base_ + cur_, 8);
    cur_ += 8;
    need(n);
    std::string s(reinterpret_cast<const char*>(base_ + cur_), n);
    cur_ += n;
    return s;
}

void GgufFile::open(const std::string& path) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("GGUF: cannot open " + path);
    struct stat st;
    fstat(fd, &st);
    size_ = (size_t)st.st_size;
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) throw std::runtime_error("GGUF: mmap failed");
    base_ = static_cast<const uint8_t*>(m);
    cur_ = 0;
    need(4);
    if (std::memcmp(base_, "GGUF", 4) != 0) throw std::runtime_error("GGUF: invalid magic (not a GGUF file)");
    cur_ = 4;
    const uint32_t ver = pod<uint32_t>();
    if (ver < 2 || ver > 3) throw std::runtime_error("GGUF: unsupported version");
    const int64_t nt = pod<int64_t>(), nkv = pod<int64_t>();
    if (nt < 0 || nkv < 0) throw std::runtime_error("GGUF: negative counts");
    for (int64_t i = 0; i < nkv; ++i) {
        const std::string key = str();
        const int32_t tag = pod<int32_t>();
        GgufValue v;
        v.type = tag;
        if (tag == 8) {
            v.s = str();
        } else if (tag == 9) {
            v.arr_type = pod<int32_t>();
            v.arr_count = pod<uint64_t>();
            if (v.arr_type == 8) {
                for (uint64_t j = 0; j < v.arr_count; ++j) str();
            } else {
                const size_t es = pod_size(v.arr_type);
                if (!es) throw std::runtime_error("GGUF: nested ARRAY or unknown type in array");
                need(es * v.arr_count);
                cur_ += es * v.arr_count;
            }
        } else {
            const size_t es = pod_size(tag);
            if (!es) throw std::runtime_error("GGUF: unknown KV type");
            need(es);
            std::memcpy(&v.u, base_ + cur_, es);
            if (tag == 1) v.i = (int8_t)v.u;
            else if (tag == 3) v.i = (int16_t)v.u;
            else if (tag == 5) v.i = (int32_t)v.u;
            else if (tag == 11) v.i = (int64_t)v.u;
            else v.i = (int64_t)v.u;
            if (tag == 6) { float f; std::memcpy(&f, base_ + cur_, 4); v.f = f; }
            if (tag == 12) { double d; std::memcpy(&d, base_ + cur_, 8); v.f = d; }
            cur_ += es;
        }
        kv_[key] = v;
    }
    uint64_t align = 32;
    auto it = kv_.find("general.alignment");
    if (it != kv_.end() && it->second.type == 4) align = it->second.u;
    for (int64_t i = 0; i < nt; ++i) {
        GgufTensor t;
        t.name = str();
        const uint32_t nd = pod<uint32_t>();
        if (nd > 4) throw std::runtime_error("GGUF: tensor with more than 4 dimensions");
        int64_t numel = 1;
        for (uint32_t d = 0; d < nd; ++d) {
            t.dims.push_back(pod<int64_t>());
            numel *= t.dims.back();
        }
        t.type = pod<int32_t>();
        t.offset = pod<uint64_t>();
        t.nbytes = ggml_nbytes(t.type, numel);
        tensors_.push_back(t);
    }
    const size_t data = (cur_ + align - 1) / align * align;
    for (auto& t : tensors_) {
        t.offset += data;
        if (t.offset + t.nbytes > size_) throw std::runtime_error("GGUF: tensor extends past end of file: " + t.name);
    }
}

const GgufValue* GgufFile::find(const std::string& k) const {
    auto it = kv_.find(k);
    return it == kv_.end() ? nullptr : &it->second;
}

int64_t GgufFile::get_int(const std::string& k, int64_t def) const {
    const GgufValue* v = find(k);
    if (!v || v->type == 8 || v->type == 9 || v->type == 6 || v->type == 12) return def;
    return v->i;
}

double GgufFile::get_float(const std::string& k, double def) const {
    const GgufValue* v = find(k);
    if (!v || (v->type != 6 && v->type != 12)) return def;
    return v->f;
}

std::string GgufFile::get_str(const std::string& k, const std::string& def) const {
    const GgufValue* v = find(k);
    return (v && v->type == 8) ? v->s : def;
}

uint64_t GgufFile::array_count(const std::string& k) const {
    const GgufValue* v = find(k);
    return (v && v->type == 9) ? v->arr_count : 0;
}

}  // namespace af
