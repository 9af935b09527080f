// gguf.cpp — GGUF reader (see gguf.h). Value type ids, alignment rule and
// tensor-table layout follow the GGUF specification as the reference reads it
// (model/fish/src/gguf.cpp:75-170 values, 380-421 header/tensors/alignment).
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace fb {

size_t ggml_block_elems(int t) {
    switch (t) {
        case 0: case 1: case 30: return 1;
        case 10: case 11: case 12: case 13: case 14: case 15: return 256;
        case 2: case 3: case 6: case 7: case 8: case 9: return 32;
        default: return 0;
    }
}

size_t ggml_block_bytes(int t) {
    switch (t) {
        case 0: return 4;
        case 1: case 30: return 2;
        case 2: return 18;
        case 3: return 20;
        case 6: return 22;
        case 7: return 24;
        case 8: return 34;
        case 9: return 36;
        case 10: return 84;
        case 11: return 110;
        case 12: return 144;
        case 13: return 176;
        case 14: return 210;
        case 15: return 292;
        default: return 0;
    }
}

uint64_t ggml_row_bytes(int t, uint64_t n) {
    const size_t be = ggml_block_elems(t), bb = ggml_block_bytes(t);
    if (!be || !bb) return 0;
    return n / be * bb;
}

const char* ggml_type_name(int t) {
    switch (t) {
        case 0: return "F32"; case 1: return "F16"; case 2: return "Q4_0"; case 3: return "Q4_1";
        case 6: return "Q5_0"; case 7: return "Q5_1"; case 8: return "Q8_0"; case 9: return "Q8_1";
        case 10: return "Q2_K"; case 11: return "Q3_K"; case 12: return "Q4_K"; case 13: return "Q5_K";
        case 14: return "Q6_K"; case 15: return "Q8_K"; case 30: return "BF16";
        default: return "UNSUPPORTED";
    }
}

namespace {

struct Reader {
    const uint8_t* p;
    size_t n, off = 0;
    bool ok = true;
    bool need(size_t k) {
        if (!ok || k > n || off > n - k) { ok = false; return false; }
        return true;
    }
    template <class T> T get() {
        T v{};
        if (!need(sizeof(T))) return v;
        std::memcpy(&v, p + off, sizeof(T));
        off += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t len = get<uint64_t>();
        if (!ok || len > (64ull << 20) || !need(static_cast<size_t>(len))) { ok = false; return {}; }
        std::string s(reinterpret_cast<const char*>(p + off), static_cast<size_t>(len));
        off += static_cast<size_t>(len);
        return s;
    }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;
        case 2: case 3: return 2;
        case 4: case 5: case 6: return 4;
        case 10: case 11: case 12: return 8;
        default: return 0;
    }
}

bool read_value(Reader& r, uint32_t t, MetaValue& v, int depth) {
    if (depth > 8) return false;
    switch (t) {
        case 0: v.kind = MetaValue::UINT; v.u = r.get<uint8_t>(); break;
        case 2: v.kind = MetaValue::UINT; v.u = r.get<uint16_t>(); break;
        case 4: v.kind = MetaValue::UINT; v.u = r.get<uint32_t>(); break;
        case 10: v.kind = MetaValue::UINT; v.u = r.get<uint64_t>(); break;
        case 1: v.kind = MetaValue::INT; v.i = r.get<int8_t>(); break;
        case 3: v.kind = MetaValue::INT; v.i = r.get<int16_t>(); break;
        case 5: v.kind = MetaValue::INT; v.i = r.get<int32_t>(); break;
        case 11: v.kind = MetaValue::INT; v.i = r.get<int64_t>(); break;
        case 6: v.kind = MetaValue::FLOAT; v.f = r.get<float>(); break;
        case 12: v.kind = MetaValue::FLOAT; v.f = r.get<double>(); break;
        case 7: v.kind = MetaValue::BOOL; v.b = r.get<uint8_t>() != 0; break;
        case 8: v.kind = MetaValue::STRING; v.s = r.str(); break;
        case 9: {
            const uint32_t et = r.get<uint32_t>();
            const uint64_t cnt = r.get<uint64_t>();
            if (!r.ok || cnt > (1ull << 26)) return false;
            v.kind = MetaValue::ARRAY;
            v.count = cnt;
            if (et == 8) {
                v.sarr.reserve(static_cast<size_t>(cnt));
                for (uint64_t i = 0; i < cnt && r.ok; ++i) v.sarr.push_back(r.str());
            } else if (et == 4 || et == 5) {
                v.iarr.resize(static_cast<size_t>(cnt));
                for (uint64_t i = 0; i < cnt && r.ok; ++i) v.iarr[i] = static_cast<int32_t>(r.get<uint32_t>());
            } else if (et == 6) {
                v.farr.resize(static_cast<size_t>(cnt));
                for (uint64_t i = 0; i < cnt && r.ok; ++i) v.farr[i] = r.get<float>();
            } else if (et == 12) {
                v.farr.resize(static_cast<size_t>(cnt));
                for (uint64_t i = 0; i < cnt && r.ok; ++i) v.farr[i] = static_cast<float>(r.get<double>());
            } else if (scalar_size(et)) {
                if (!r.need(static_cast<size_t>(cnt * scalar_size(et)))) return false;
                r.off += static_cast<size_t>(cnt * scalar_size(et));
            } else {
                for (uint64_t i = 0; i < cnt && r.ok; ++i) {
                    MetaValue sub;
                    if (!read_value(r, et, sub, depth + 1)) return false;
                }
            }
            break;
        }
        default: return false;
    }
    return r.ok;
}

}  // namespace

std::unique_ptr<Gguf> Gguf::open(const std::string& path, std::string* err) {
    auto fail = [&](const std::string& why) -> std::unique_ptr<Gguf> { if (err) *err = why; return nullptr; };
    std::unique_ptr<Gguf> g(new Gguf());
    g->path_ = path;
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return fail("cannot open " + path);
    struct stat st{};
    if (fstat(fd, &st) != 0 || st.st_size <= 0) { ::close(fd); return fail("cannot size " + path); }
    void* base = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (base == MAP_FAILED) return fail("cannot map " + path);
    g->map_ = static_cast<const uint8_t*>(base);
    g->size_ = static_cast<size_t>(st.st_size);
    if (!g->parse(err)) return nullptr;
    return g;
}

Gguf::~Gguf() {
    if (map_) munmap(const_cast<uint8_t*>(map_), size_);
}

bool Gguf::parse(std::string* err) {
    auto fail = [&](const std::string& why) { if (err) *err = why; return false; };
    Reader r{map_, size_};
    if (r.get<uint32_t>() != 0x46554747u) return fail("not a GGUF file");
    const uint32_t ver = r.get<uint32_t>();
    if (ver < 2 || ver > 3) return fail("unsupported GGUF version " + std::to_string(ver));
    const uint64_t nt = r.get<uint64_t>(), nkv = r.get<uint64_t>();
    if (!r.ok || nt > (1ull << 20) || nkv > (1ull << 20)) return fail("bad GGUF header");
    for (uint64_t i = 0; i < nkv; ++i) {
        std::string key = r.str();
        const uint32_t t = r.get<uint32_t>();
        MetaValue v;
        if (!r.ok || !read_value(r, t, v, 0)) return fail("bad metadata value for " + key);
        kv_.emplace(std::move(key), std::move(v));
    }
    uint64_t align = 32;
    if (const MetaValue* a = meta("general.alignment")) {
        const uint64_t v = a->kind == MetaValue::UINT ? a->u : static_cast<uint64_t>(a->i);
        if (v >= 1 && v <= (1u << 20) && (v & (v - 1)) == 0) align = v;
    }
    tensors_.reserve(static_cast<size_t>(nt));
    for (uint64_t i = 0; i < nt; ++i) {
        Tensor t;
        t.name = r.str();
        const uint32_t nd = r.get<uint32_t>();
        if (!r.ok || nd == 0 || nd > 4) return fail("bad tensor rank for " + t.name);
        t.ne.resize(nd);
        for (uint32_t d = 0; d < nd; ++d) {
            t.ne[d] = r.get<uint64_t>();
            if (!r.ok || t.ne[d] == 0 || t.ne[d] > (1ull << 40)) return fail("bad tensor dim for " + t.name);
        }
        t.type = static_cast<int>(r.get<uint32_t>());
        t.offset = r.get<uint64_t>();
        if (!r.ok) return fail("truncated tensor info for " + t.name);
        const size_t be = ggml_block_elems(t.type);
        if (!be || !ggml_block_bytes(t.type)) return fail(std::string("unsupported tensor type for ") + t.name);
        if (t.ne[0] % be) return fail("tensor " + t.name + " row is not a whole number of blocks");
        t.nbytes = ggml_row_bytes(t.type, t.ne[0]) * t.rows();
        tensors_.push_back(std::move(t));
    }
    const uint64_t data_off = (r.off + align - 1) / align * align;
    if (data_off > size_) return fail("data section beyond end of file");
    for (size_t i = 0; i < tensors_.size(); ++i) {
        Tensor& t = tensors_[i];
        if (t.offset > size_ - data_off || t.nbytes > size_ - data_off - t.offset)
            return fail("tensor " + t.name + " extends past end of file");
        t.data = map_ + data_off + t.offset;
        tindex_[t.name] = i;
    }
    return true;
}

const Tensor* Gguf::find(const std::string& name) const {
    auto it = tindex_.find(name);
    return it == tindex_.end() ? nullptr : &tensors_[it->second];
}

const MetaValue* Gguf::meta(const std::string& key) const {
    auto it = kv_.find(key);
    return it == kv_.end() ? nullptr : &it->second;
}

uint64_t Gguf::u64(const std::string& key, uint64_t def) const {
    const MetaValue* v = meta(key);
    if (!v) return def;
    switch (v->kind) {
        case MetaValue::UINT: return v->u;
        case MetaValue::INT: return v->i < 0 ? def : static_cast<uint64_t>(v->i);
        case MetaValue::FLOAT: return v->f < 0 ? def : static_cast<uint64_t>(v->f);
        case MetaValue::BOOL: return v->b ? 1 : 0;
        default: return def;
    }
}

int64_t Gguf::i64(const std::string& key, int64_t def) const {
    const MetaValue* v = meta(key);
    if (!v) return def;
    switch (v->kind) {
        case MetaValue::UINT: return static_cast<int64_t>(v->u);
        case MetaValue::INT: return v->i;
        case MetaValue::FLOAT: return static_cast<int64_t>(v->f);
        case MetaValue::BOOL: return v->b ? 1 : 0;
        default: return def;
    }
}

double Gguf::f64(const std::string& key, double def) const {
    const MetaValue* v = meta(key);
    if (!v) return def;
    switch (v->kind) {
        case MetaValue::UINT: return static_cast<double>(v->u);
        case MetaValue::INT: return static_cast<double>(v->i);
        case MetaValue::FLOAT: return v->f;
        case MetaValue::BOOL: return v->b ? 1.0 : 0.0;
        default: return def;
    }
}

bool Gguf::flag(const std::string& key, bool def) const {
    const MetaValue* v = meta(key);
    if (!v) return def;
    switch (v->kind) {
        case MetaValue::BOOL: return v->b;
        case MetaValue::UINT: return v->u != 0;
        case MetaValue::INT: return v->i != 0;
        case MetaValue::FLOAT: return v->f != 0;
        default: return def;
    }
}

std::string Gguf::str(const std::string& key, const std::string& def) const {
    const MetaValue* v = meta(key);
    return v && v->kind == MetaValue::STRING ? v->s : def;
}

}  // namespace fb
