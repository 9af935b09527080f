// gguf.h — read-only GGUF v2/v3 container reader for the B200 engine.
//
// Parses the header, metadata table and tensor directory with bounds checks on
// every field and maps the file read-only (the reference reader's contract,
// model/fish/include/fish/gguf.h:1-15). Tensor bytes are only touched by the
// device upload.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

namespace fb {

size_t ggml_block_elems(int type);
size_t ggml_block_bytes(int type);
uint64_t ggml_row_bytes(int type, uint64_t n);
const char* ggml_type_name(int type);

struct MetaValue {
    enum Kind : uint8_t { UINT, INT, FLOAT, BOOL, STRING, ARRAY } kind = UINT;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0;
    bool b = false;
    std::string s;
    std::vector<std::string> sarr;
    std::vector<int32_t> iarr;
    std::vector<float> farr;
    uint64_t count = 0;   // array length
};

struct Tensor {
    std::string name;
    int type = 0;
    std::vector<uint64_t> ne;
    uint64_t offset = 0;
    uint64_t nbytes = 0;
    const uint8_t* data = nullptr;
    uint64_t rows() const {
        uint64_t r = 1;
        for (size_t d = 1; d < ne.size(); ++d) r *= ne[d];
        return r;
    }
    uint64_t n_elements() const { return ne.empty() ? 0 : ne[0] * rows(); }
};

class Gguf {
public:
    static std::unique_ptr<Gguf> open(const std::string& path, std::string* err);
    ~Gguf();
    const Tensor* find(const std::string& name) const;
    const MetaValue* meta(const std::string& key) const;
    uint64_t u64(const std::string& key, uint64_t def) const;
    int64_t i64(const std::string& key, int64_t def) const;
    double f64(const std::string& key, double def) const;
    bool flag(const std::string& key, bool def) const;
    std::string str(const std::string& key, const std::string& def) const;
    const std::vector<Tensor>& tensors() const { return tensors_; }
    const std::string& path() const { return path_; }
    size_t file_size() const { return size_; }
    const uint8_t* map_base() const { return map_; }   // the file's first byte in the mapping

private:
    Gguf() = default;
    bool parse(std::string* err);
    std::string path_;
    const uint8_t* map_ = nullptr;
    size_t size_ = 0;
    std::vector<Tensor> tensors_;
    std::unordered_map<std::string, size_t> tindex_;
    std::unordered_map<std::string, MetaValue> kv_;
};

}  // namespace fb
