// GGUF header parsing and the POSIX tensor store (interfaces in
// include/arcllm/v1/gguf.h).
#include "arcllm/v1/gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <memory>
#include <sstream>
#include <stdexcept>

namespace {

enum : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
    kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12
};

// Sequential little-endian reader over a FILE*, failing loudly on truncation.
class Cursor {
public:
    explicit Cursor(const std::string& path) : f_(std::fopen(path.c_str(), "rb"), &std::fclose) {
        if (!f_) throw std::runtime_error("cannot open GGUF: " + path);
    }
    void bytes(void* dst, size_t n) {
        if (n && std::fread(dst, 1, n, f_.get()) != n) throw std::runtime_error("unexpected EOF");
        pos_ += n;
    }
    template <typename T> T pod() { T v{}; bytes(&v, sizeof(T)); return v; }
    std::string str() {
        const uint64_t n = pod<uint64_t>();
        if (n > (1ull << 31)) throw std::runtime_error("GGUF string too large");
        std::string s(size_t(n), '\0');
        bytes(s.data(), size_t(n));
        return s;
    }
    void skip(uint64_t n) {
        if (std::fseek(f_.get(), long(n), SEEK_CUR) != 0) throw std::runtime_error("unexpected EOF");
        pos_ += n;
    }
    uint64_t pos() const { return pos_; }

private:
    std::unique_ptr<FILE, int (*)(FILE*)> f_;
    uint64_t pos_ = 0;
};

template <typename T> std::string num(T v) {
    std::ostringstream o;
    o << v;
    return o.str();
}

uint64_t scalar_size(uint32_t type) {
    switch (type) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}

std::string value_string(Cursor& c, uint32_t type, uint64_t* array_len) {
    switch (type) {
        case kU8: return num(uint32_t(c.pod<uint8_t>()));
        case kI8: return num(int32_t(c.pod<int8_t>()));
        case kU16: return num(c.pod<uint16_t>());
        case kI16: return num(c.pod<int16_t>());
        case kU32: return num(c.pod<uint32_t>());
        case kI32: return num(c.pod<int32_t>());
        case kF32: return num(c.pod<float>());
        case kBool: return c.pod<uint8_t>() ? "true" : "false";
        case kString: return c.str();
        case kU64: return num(c.pod<uint64_t>());
        case kI64: return num(c.pod<int64_t>());
        case kF64: return num(c.pod<double>());
        case kArray: {
            const uint32_t et = c.pod<uint32_t>();
            const uint64_t n = c.pod<uint64_t>();
            if (array_len) *array_len = n;
            if (et == kString) {
                for (uint64_t i = 0; i < n; ++i) c.skip(c.pod<uint64_t>());
            } else if (et == kArray) {
                throw std::runtime_error("unsupported GGUF nested array");
            } else {
                const uint64_t sz = scalar_size(et);
                if (!sz) throw std::runtime_error("unsupported GGUF metadata type: " + std::to_string(et));
                if (n > (1ull << 40) / sz) throw std::runtime_error("GGUF array too large");
                c.skip(n * sz);
            }
            return "<array type=" + std::to_string(et) + " len=" + std::to_string(n) + ">";
        }
        default: throw std::runtime_error("unsupported GGUF metadata type: " + std::to_string(type));
    }
}

uint64_t align_up(uint64_t x, uint64_t a) { return a ? (x + a - 1) / a * a : x; }

}  // namespace

GgufReader::GgufReader(const std::string& path) : path_(path) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) throw std::runtime_error("cannot open GGUF: " + path);
    std::fclose(f);
}

GgufInfo GgufReader::read() {
    Cursor c(path_);
    char magic[4]{};
    c.bytes(magic, 4);
    if (std::memcmp(magic, "GGUF", 4) != 0) throw std::runtime_error("not a GGUF file");
    GgufInfo out;
    out.version = c.pod<uint32_t>();
    if (out.version < 2 || out.version > 3)
        throw std::runtime_error("unsupported GGUF version: " + std::to_string(out.version));
    out.tensor_count = c.pod<uint64_t>();
    out.metadata_count = c.pod<uint64_t>();
    if (out.tensor_count > (1ull << 24) || out.metadata_count > (1ull << 24))
        throw std::runtime_error("GGUF header counts out of range");
    for (uint64_t i = 0; i < out.metadata_count; ++i) {
        std::string key = c.str();
        const uint32_t type = c.pod<uint32_t>();
        uint64_t n = 0;
        std::string v = value_string(c, type, &n);
        if (type == kArray) out.array_lengths[key] = n;
        if (key == "general.alignment") {
            try { out.alignment = std::stoull(v); } catch (...) {}
        }
        out.scalars[key] = std::move(v);
    }
    out.tensors.reserve(size_t(out.tensor_count));
    for (uint64_t i = 0; i < out.tensor_count; ++i) {
        GgufTensorInfo t;
        t.name = c.str();
        t.n_dims = c.pod<uint32_t>();
        if (t.n_dims > 8) throw std::runtime_error("unexpected tensor ndim > 8");
        for (uint32_t d = 0; d < t.n_dims; ++d) t.dims.push_back(c.pod<uint64_t>());
        t.ggml_type = c.pod<uint32_t>();
        t.offset = c.pod<uint64_t>();
        out.tensor_type_counts[t.ggml_type]++;
        out.tensors.push_back(std::move(t));
    }
    out.data_offset = align_up(c.pos(), out.alignment);
    return out;
}

namespace arcllm::v1::gguf {

uint64_t row_bytes(uint32_t type, uint64_t n) {
    switch (type) {
        case F32: return n * 4;
        case F16: return n * 2;
        case Q4_K:
            if (n % 256) throw std::runtime_error("Q4_K row length not a multiple of 256");
            return n / 256 * 144;
        case Q6_K:
            if (n % 256) throw std::runtime_error("Q6_K row length not a multiple of 256");
            return n / 256 * 210;
        default: throw std::runtime_error("unsupported ggml type " + std::to_string(type));
    }
}

uint64_t tensor_rows(const GgufTensorInfo& t) {
    if (t.dims.empty()) throw std::runtime_error("tensor has no dims: " + t.name);
    uint64_t r = 1;
    for (size_t i = 1; i < t.dims.size(); ++i) r *= t.dims[i];
    return r;
}

uint64_t tensor_nbytes(const GgufTensorInfo& t) {
    if (t.dims.empty()) throw std::runtime_error("tensor has no dims: " + t.name);
    return row_bytes(t.ggml_type, t.dims[0]) * tensor_rows(t);
}

const GgufTensorInfo* find_tensor(const GgufInfo& g, const std::string& name) {
    for (const auto& t : g.tensors)
        if (t.name == name) return &t;
    return nullptr;
}

TensorStore::~TensorStore() { close(); }

void TensorStore::close() {
    if (base_) munmap(const_cast<uint8_t*>(base_), size_t(size_));
    if (fd_ >= 0) ::close(fd_);
    base_ = nullptr;
    size_ = 0;
    fd_ = -1;
}

TensorStoreReport TensorStore::inspect(const std::string& path, const GgufInfo& g) {
    close();
    TensorStoreReport r;
    fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd_ < 0) { r.error = "cannot open " + path; return r; }
    struct stat st{};
    if (fstat(fd_, &st) != 0 || st.st_size <= 0) { r.error = "cannot stat " + path; close(); return r; }
    size_ = uint64_t(st.st_size);
    void* p = mmap(nullptr, size_t(size_), PROT_READ, MAP_SHARED, fd_, 0);
    if (p == MAP_FAILED) { r.error = "mmap failed"; size_ = 0; close(); return r; }
    base_ = static_cast<const uint8_t*>(p);
    r.mapped = true;
    r.file_size = size_;
    r.data_offset = g.data_offset;

    struct Span { uint64_t s, e; };
    std::vector<Span> spans;
    r.all_bounds_valid = g.data_offset <= size_;
    r.supported_types_only = true;
    for (const auto& t : g.tensors) {
        uint64_t nb = 0;
        try {
            nb = tensor_nbytes(t);
        } catch (...) {
            r.supported_types_only = false;
            continue;
        }
        const uint64_t s = g.data_offset + t.offset;
        if (t.offset > size_ || s < g.data_offset || s > size_ || nb > size_ - s) r.all_bounds_valid = false;
        spans.push_back({s, s + nb});
        r.tensor_bytes_total += nb;
        if (t.ggml_type == Q4_K) ++r.q4_k_tensor_count;
        if (t.ggml_type == Q6_K) ++r.q6_k_tensor_count;
        if (t.ggml_type == F32) ++r.f32_tensor_count;
        if (t.ggml_type == F16) ++r.f16_tensor_count;
    }
    std::sort(spans.begin(), spans.end(), [](const Span& a, const Span& b) { return a.s < b.s; });
    r.no_overlap = true;
    for (size_t i = 1; i < spans.size(); ++i)
        if (spans[i].s < spans[i - 1].e) r.no_overlap = false;
    // Q4_K direct access: the first super-block of the first Q4_K tensor is
    // readable in place (its fp16 scale is touched through the mapping).
    r.q4_k_direct_access = false;
    if (r.all_bounds_valid)
        for (const auto& t : g.tensors)
            if (t.ggml_type == Q4_K) {
                volatile uint8_t probe = base_[g.data_offset + t.offset];
                (void)probe;
                r.q4_k_direct_access = true;
                break;
            }
    return r;
}

const uint8_t* TensorStore::tensor_data(const GgufInfo& g, const GgufTensorInfo& t) const {
    if (!base_) throw std::runtime_error("tensor store not mapped");
    const uint64_t s = g.data_offset + t.offset, nb = tensor_nbytes(t);
    if (s > size_ || nb > size_ - s) throw std::runtime_error("tensor out of bounds: " + t.name);
    return base_ + s;
}

}  // namespace arcllm::v1::gguf
