// GgufModel / GgufTensor (reference src/gguf.cpp:9-19), re-implemented over a
// read-only memory map instead of a full in-memory copy of the file. Parse
// rules follow the reference loader: little-endian fields, metadata types
// 0..12, tensor data at the next multiple of general.alignment (default 32,
// values 0 or > 4096 fall back to 32), every tensor bounds-checked.
#include "laic/gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <limits>
#include <stdexcept>

namespace laic {
namespace {

float half_bits_to_float(uint16_t h) {
    const uint32_t sign = uint32_t(h & 0x8000u) << 16;
    int exp = (h >> 10) & 0x1f;
    uint32_t mant = h & 0x3ffu, out;
    if (exp == 0x1f) out = sign | 0x7f800000u | (mant << 13);
    else if (exp) out = sign | (uint32_t(exp + 112) << 23) | (mant << 13);
    else if (!mant) out = sign;
    else {  // subnormal: normalise
        int e = 113;
        while (!(mant & 0x400u)) { mant <<= 1; --e; }
        out = sign | (uint32_t(e) << 23) | ((mant & 0x3ffu) << 13);
    }
    float f;
    std::memcpy(&f, &out, 4);
    return f;
}

size_t type_block_bytes(GgmlType t) {
    switch (t) {
    case GgmlType::F32: return 4;
    case GgmlType::F16: return 2;
    case GgmlType::Q4_0: return 18;
    case GgmlType::Q4_1: return 20;
    case GgmlType::Q5_0: return 22;
    case GgmlType::Q5_1: return 24;
    case GgmlType::Q8_0: return 34;
    case GgmlType::Q2_K: return 84;
    case GgmlType::Q3_K: return 110;
    case GgmlType::Q4_K: return 144;
    case GgmlType::Q5_K: return 176;
    case GgmlType::Q6_K: return 210;
    }
    throw std::runtime_error("unsupported GGML type");
}

class Cursor {
public:
    Cursor(const uint8_t* p, size_t n) : p_(p), end_(p + n), base_(p) {}
    template <class T> T get() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, p_, sizeof(T));  // the format and the host are little-endian
        p_ += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (n > uint64_t(end_ - p_)) throw std::runtime_error("invalid GGUF string");
        std::string s(reinterpret_cast<const char*>(p_), size_t(n));
        p_ += n;
        return s;
    }
    size_t offset() const { return size_t(p_ - base_); }

private:
    void need(size_t n) {
        if (n > size_t(end_ - p_)) throw std::runtime_error("invalid/truncated GGUF");
    }
    const uint8_t* p_;
    const uint8_t* end_;
    const uint8_t* base_;
};

GgufValue read_value(Cursor& c, uint32_t type) {
    switch (type) {
    case 0: return uint64_t(c.get<uint8_t>());
    case 1: return int64_t(c.get<int8_t>());
    case 2: return uint64_t(c.get<uint16_t>());
    case 3: return int64_t(c.get<int16_t>());
    case 4: return uint64_t(c.get<uint32_t>());
    case 5: return int64_t(c.get<int32_t>());
    case 6: return double(c.get<float>());
    case 7: return c.get<uint8_t>() != 0;
    case 8: return c.str();
    case 10: return c.get<uint64_t>();
    case 11: return c.get<int64_t>();
    case 12: return c.get<double>();
    case 9: {
        const uint32_t et = c.get<uint32_t>();
        const uint64_t n = c.get<uint64_t>();
        if (n > 100000000ull) throw std::runtime_error("GGUF array too large");
        if (et == 8) {
            std::vector<std::string> v;
            v.reserve(size_t(n));
            for (uint64_t i = 0; i < n; ++i) v.push_back(c.str());
            return v;
        }
        std::vector<uint64_t> v;
        v.reserve(size_t(n));
        for (uint64_t i = 0; i < n; ++i) {
            GgufValue e = read_value(c, et);
            if (auto* u = std::get_if<uint64_t>(&e)) v.push_back(*u);
            else if (auto* s = std::get_if<int64_t>(&e)) v.push_back(uint64_t(*s));
            else throw std::runtime_error("unsupported GGUF array type");
        }
        return v;
    }
    }
    throw std::runtime_error("unsupported GGUF metadata type");
}

}  // namespace

size_t GgufTensor::elements() const noexcept {
    size_t n = 1;
    for (uint64_t d : shape) {
        if (d && n > std::numeric_limits<size_t>::max() / size_t(d)) return 0;
        n *= size_t(d);
    }
    return n;
}

size_t GgufTensor::bytes() const noexcept {
    const size_t n = elements();
    if (type == GgmlType::F32) return n * 4;
    if (type == GgmlType::F16) return n * 2;
    size_t bb = 0;
    try { bb = type_block_bytes(type); } catch (...) { return 0; }
    return (n + 31) / 32 * bb;
}

float GgufTensor::value(size_t i) const {
    if (!data || i >= elements()) throw std::out_of_range("GGUF tensor index");
    switch (type) {
    case GgmlType::F32: { float v; std::memcpy(&v, data + 4 * i, 4); return v; }
    case GgmlType::F16: return half_bits_to_float(uint16_t(data[2 * i] | (data[2 * i + 1] << 8)));
    case GgmlType::Q8_0: {
        const uint8_t* b = data + (i / 32) * 34;
        return half_bits_to_float(uint16_t(b[0] | (b[1] << 8))) * float(int8_t(b[2 + i % 32]));
    }
    case GgmlType::Q4_0: {
        // element o of a block: byte o/2, low nibble for even o, high for odd (src/quant_v2.cpp:10)
        const uint8_t* b = data + (i / 32) * 18;
        const size_t o = i % 32;
        const int q = (o & 1) ? (b[2 + o / 2] >> 4) : (b[2 + o / 2] & 15);
        return half_bits_to_float(uint16_t(b[0] | (b[1] << 8))) * float(q - 8);
    }
    default: break;
    }
    throw std::runtime_error("unsupported GGUF tensor type");
}

GgufModel::~GgufModel() { unmap(); }

void GgufModel::unmap() noexcept {
    if (map_) munmap(const_cast<uint8_t*>(map_), map_size_);
    map_ = nullptr;
    map_size_ = 0;
}

void GgufModel::load(const std::string& path) {
    unmap();
    meta_.clear();
    tensors_.clear();
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("cannot open GGUF: " + path);
    struct stat st {};
    if (fstat(fd, &st) != 0 || st.st_size < 0) { ::close(fd); throw std::runtime_error("cannot size GGUF"); }
    map_size_ = size_t(st.st_size);
    void* m = map_size_ ? mmap(nullptr, map_size_, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
    ::close(fd);
    if (m == MAP_FAILED) { map_size_ = 0; throw std::runtime_error("cannot read GGUF"); }
    map_ = static_cast<const uint8_t*>(m);
    path_ = path;

    Cursor c(map_, map_size_);
    if (c.get<uint32_t>() != 0x46554747u) throw std::runtime_error("bad GGUF magic");
    const uint32_t ver = c.get<uint32_t>();
    if (ver < 2 || ver > 3) throw std::runtime_error("unsupported GGUF version");
    const uint64_t nt = c.get<uint64_t>(), nm = c.get<uint64_t>();
    if (nt > 1000000 || nm > 1000000) throw std::runtime_error("unreasonable GGUF counts");
    for (uint64_t i = 0; i < nm; ++i) {
        std::string k = c.str();
        const uint32_t t = c.get<uint32_t>();
        meta_.emplace(std::move(k), read_value(c, t));
    }
    std::vector<GgufTensor> infos;
    infos.reserve(size_t(nt));
    for (uint64_t i = 0; i < nt; ++i) {
        GgufTensor t;
        t.name = c.str();
        const uint32_t nd = c.get<uint32_t>();
        if (nd > 8) throw std::runtime_error("invalid GGUF rank");
        t.shape.resize(nd);
        for (auto& d : t.shape) d = c.get<uint64_t>();
        t.type = GgmlType(c.get<uint32_t>());
        t.offset = c.get<uint64_t>();
        (void)type_block_bytes(t.type);
        infos.push_back(std::move(t));
    }
    uint64_t align = u64("general.alignment", 32);
    if (!align || align > 4096) align = 32;
    const size_t start = (c.offset() + size_t(align) - 1) / size_t(align) * size_t(align);
    if (start > map_size_) throw std::runtime_error("tensor data starts past end");
    for (auto& t : infos) {
        if (t.offset > uint64_t(map_size_ - start)) throw std::runtime_error("tensor offset out of range");
        const size_t base = start + size_t(t.offset);
        t.data = map_ + base;
        if (t.bytes() > map_size_ - base) throw std::runtime_error("tensor data out of range");
        std::string key = t.name;
        tensors_.emplace(std::move(key), std::move(t));
    }
}

const GgufTensor& GgufModel::tensor(const std::string& n) const {
    auto it = tensors_.find(n);
    if (it == tensors_.end()) throw std::runtime_error("missing tensor: " + n);
    return it->second;
}

bool GgufModel::has_tensor(const std::string& n) const noexcept { return tensors_.count(n) != 0; }

const GgufValue* GgufModel::metadata(const std::string& k) const noexcept {
    auto it = meta_.find(k);
    return it == meta_.end() ? nullptr : &it->second;
}

uint64_t GgufModel::u64(const std::string& k, uint64_t fb) const {
    const GgufValue* v = metadata(k);
    if (!v) return fb;
    if (auto* p = std::get_if<uint64_t>(v)) return *p;
    if (auto* p = std::get_if<int64_t>(v)) return uint64_t(*p);
    if (auto* p = std::get_if<bool>(v)) return *p ? 1 : 0;
    return fb;
}

double GgufModel::f64(const std::string& k, double fb) const {
    const GgufValue* v = metadata(k);
    if (!v) return fb;
    if (auto* p = std::get_if<double>(v)) return *p;
    if (auto* p = std::get_if<uint64_t>(v)) return double(*p);
    return fb;
}

std::string GgufModel::str(const std::string& k, const std::string& fb) const {
    const GgufValue* v = metadata(k);
    if (!v) return fb;
    if (auto* p = std::get_if<std::string>(v)) return *p;
    return fb;
}

const std::vector<std::string>& GgufModel::strings(const std::string& k) const {
    const GgufValue* v = metadata(k);
    if (!v) return empty_strings_;
    if (auto* p = std::get_if<std::vector<std::string>>(v)) return *p;
    return empty_strings_;
}

}  // namespace laic
