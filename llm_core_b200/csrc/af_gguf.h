// af_gguf.h — minimal mmap GGUF reader (host side of the engine's loader).
#pragma once
#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace af {

struct GgufValue {
    int type = -1;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0;
    std::string s;
    int arr_type = -1;
    uint64_t arr_count = 0;
};

struct GgufTensor {
    std::string name;
    std::vector<int64_t> dims;
    int type = 0;
    uint64_t offset = 0;  // absolute file offset
    size_t nbytes = 0;
};

size_t ggml_nbytes(int type, int64_t numel);

class GgufFile {
public:
    ~GgufFile();
    void open(const std::string& path);
    const GgufValue* find(const std::string& k) const;
    int64_t get_int(const std::string& k, int64_t def) const;
    double get_float(const std::string& k, double def) const;
    std::string get_str(const std::string& k, const std::string& def) const;
    uint64_t array_count(const std::string& k) const;
    const std::vector<GgufTensor>& tensors() const { return tensors_; }
    const uint8_t* data(const GgufTensor& t) const { return base_ + t.offset; }

private:
    template <class T>
    T pod() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, base_ + cur_, sizeof(T));
        cur_ += sizeof(T);
        return v;
    }
    std::string str();
    void need(size_t n) const;

    const uint8_t* base_ = nullptr;
    size_t size_ = 0, cur_ = 0;
    std::map<std::string, GgufValue> kv_;
    std::vector<GgufTensor> tensors_;
};

}  // namespace af
