// GGUF container access for the ArcLLM CUDA runtime.
//
// GgufInfo / GgufTensorInfo / GgufReader keep the field names and meaning of
// the reference's src/gguf.h:8-48 (metadata values are kept as strings,
// numbers formatted like an ostream with default precision, src/gguf.cpp:26-31,
// so std::stof/std::stoul on them give the same values), because the runtime's
// model checks are written against those names.  TensorStore replaces the
// reference's Win32 file mapping (src/tensor_store.h:37-58) with POSIX mmap and
// keeps its TensorStoreReport invariants.  GgufWriter is new: it writes the
// synthetic GGUF files the tests and benchmarks run generate() on.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

struct GgufTensorInfo {
    std::string name;
    uint32_t n_dims = 0;
    std::vector<uint64_t> dims;  // dims[0] is the contiguous (row) dimension
    uint32_t ggml_type = 0;
    uint64_t offset = 0;         // relative to GgufInfo::data_offset
};

struct GgufInfo {
    uint32_t version = 0;
    uint64_t tensor_count = 0;
    uint64_t metadata_count = 0;
    uint64_t alignment = 32;
    uint64_t data_offset = 0;

    std::map<std::string, std::string> scalars;
    std::map<std::string, uint64_t> array_lengths;
    std::map<uint32_t, uint64_t> tensor_type_counts;
    std::vector<GgufTensorInfo> tensors;
};

class GgufReader {
public:
    explicit GgufReader(const std::string& path);  // throws std::runtime_error if unreadable
    GgufInfo read();                                 // throws on malformed input

private:
    std::string path_;
};

namespace arcllm::v1::gguf {

enum GgmlType : uint32_t { F32 = 0, F16 = 1, Q4_K = 12, Q6_K = 14 };

// Bytes of one row of `n` elements; throws for types the runtime does not run.
uint64_t row_bytes(uint32_t ggml_type, uint64_t n);
// Bytes of the whole tensor (rows = product of dims[1..]).
uint64_t tensor_nbytes(const GgufTensorInfo& t);
uint64_t tensor_rows(const GgufTensorInfo& t);
const GgufTensorInfo* find_tensor(const GgufInfo& g, const std::string& name);

// A read-only POSIX mapping of a GGUF file with the reference's invariants:
// every tensor inside the file, no two tensors overlapping, only F32/F16/Q4_K/Q6_K,
// and at least one Q4_K tensor readable in place.
struct TensorStoreReport {
    bool mapped = false;
    bool all_bounds_valid = false;
    bool no_overlap = false;
    bool supported_types_only = false;
    bool q4_k_direct_access = false;
    uint64_t file_size = 0;
    uint64_t data_offset = 0;
    uint64_t tensor_bytes_total = 0;
    uint64_t q4_k_tensor_count = 0;
    uint64_t q6_k_tensor_count = 0;
    uint64_t f32_tensor_count = 0;
    uint64_t f16_tensor_count = 0;
    std::string error;
};

class TensorStore {
public:
    TensorStore() = default;
    ~TensorStore();
    TensorStore(const TensorStore&) = delete;
    TensorStore& operator=(const TensorStore&) = delete;

    TensorStoreReport inspect(const std::string& path, const GgufInfo& gguf);
    const uint8_t* mapped_base() const { return base_; }
    uint64_t mapped_size() const { return size_; }
    // Pointer to a tensor's bytes inside the mapping (after a successful inspect).
    const uint8_t* tensor_data(const GgufInfo& g, const GgufTensorInfo& t) const;

private:
    void close();
    const uint8_t* base_ = nullptr;
    uint64_t size_ = 0;
    int fd_ = -1;
};

}  // namespace arcllm::v1::gguf
