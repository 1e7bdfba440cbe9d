// Q4CudaBackend (include/arcllm/v1/q4_cuda_backend.h).
#include "arcllm/v1/q4_cuda_backend.h"

#include <sys/stat.h>

#include <cstdio>
#include <memory>
#include <stdexcept>
#include <vector>

#include "arcllm_cuda.h"

namespace arcllm::v1::cuda {

using binding_v4::BackendStatus;

namespace {

void check(int st, const char* what) {
    if (st != ARC_OK) throw std::runtime_error(std::string(what) + ": " + arcllm_cuda_last_error_message());
}

// src/p8c_segmented_access_correctness.cpp:531-540
void scale_min(const std::uint8_t* s, std::uint32_t j, std::uint8_t& sc, std::uint8_t& mn) {
    if (j < 4) {
        sc = s[j] & 63u;
        mn = s[j + 4] & 63u;
    } else {
        sc = std::uint8_t((s[j + 4] & 15u) | ((s[j - 4] >> 6) << 4));
        mn = std::uint8_t((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

// One Q4_K super-block (144 B) -> EXEC148 block (148 B): d, dmin; 8 x (sc, mn);
// codes as nibble pairs in element order (src/q4_down_exec148_materializer.h:14).
void materialize_block(const std::uint8_t* src, std::uint8_t* dst) {
    for (int i = 0; i < 4; ++i) dst[i] = src[i];
    for (std::uint32_t j = 0; j < 8; ++j) scale_min(src + 4, j, dst[4 + 2 * j], dst[5 + 2 * j]);
    auto code = [&](std::uint32_t k) {
        const std::uint32_t x = k & 63u;
        const std::uint8_t b = src[16u + (k >> 6) * 32u + (x & 31u)];
        return std::uint8_t(x < 32u ? (b & 15u) : (b >> 4));
    };
    for (std::uint32_t p = 0; p < 128; ++p) dst[20 + p] = std::uint8_t(code(2 * p) | (code(2 * p + 1) << 4));
}

}  // namespace

Q4CudaBackend::Q4CudaBackend(std::vector<Source> sources, std::uint32_t rows, std::uint32_t k,
                             std::string sidecar)
    : sources_(std::move(sources)), rows_(rows), k_(k), sidecar_(std::move(sidecar)) {}

Q4CudaBackend::~Q4CudaBackend() { free_image(); }

void Q4CudaBackend::free_image() noexcept {
    if (image_) arcllm_cuda_free(image_);
    image_ = nullptr;
}

std::uint64_t Q4CudaBackend::exec_family_bytes() const noexcept { return std::uint64_t(sources_.size()) * layer_bytes(); }

bool Q4CudaBackend::p3_available() const noexcept {
    struct stat st{};
    return !sidecar_.empty() && ::stat(sidecar_.c_str(), &st) == 0 &&
           std::uint64_t(st.st_size) == exec_family_bytes();
}

const Q4CudaBackend::Source* Q4CudaBackend::find(std::uint32_t layer) const noexcept {
    for (const auto& s : sources_)
        if (s.layer == layer) return &s;
    return nullptr;
}

const void* Q4CudaBackend::exec_image(std::uint32_t layer) const noexcept {
    if (!resident_ || !image_) return nullptr;
    for (std::size_t i = 0; i < sources_.size(); ++i)
        if (sources_[i].layer == layer) return static_cast<const std::uint8_t*>(image_) + i * layer_bytes();
    return nullptr;
}

BackendStatus Q4CudaBackend::acquire(registry::AcquisitionPathId path, registry::PrimitiveId target,
                                     std::uint64_t residency_bytes,
                                     binding_v4::RepresentationHandle& out) noexcept {
    out = {};
    // Same precondition order as the Vulkan backend: wrong target or size, or
    // already resident, is a binding-state error; a missing or wrong-size
    // sidecar makes P3 unavailable; unknown paths are unavailable.
    if (target != kPrimitiveB || residency_bytes != exec_family_bytes()) return BackendStatus::INVALID_BINDING_STATE;
    if (resident_) return BackendStatus::INVALID_BINDING_STATE;
    if (path == kAcquireSecondary && !p3_available()) return BackendStatus::UNAVAILABLE;
    if (path != kAcquirePrimary && path != kAcquireSecondary && path != kAcquireTertiary)
        return BackendStatus::UNAVAILABLE;
    try {
        const std::uint64_t lb = layer_bytes(), nblk = std::uint64_t(rows_) * (k_ / 256u);
        check(arcllm_cuda_malloc(exec_family_bytes(), &image_), "EXEC148 image allocation");
        ++counters_.b_allocations;
        auto* img = static_cast<std::uint8_t*>(image_);
        if (path == kAcquirePrimary) {  // P1: materialise on the GPU from the resident Q4_K weights
            ++counters_.p1_calls;
            for (std::size_t i = 0; i < sources_.size(); ++i)
                check(arcllm_cuda_exec148_materialize(sources_[i].device, nblk, img + i * lb, nullptr),
                      "P1 materialisation");
            check(arcllm_cuda_stream_synchronize(nullptr), "P1 materialisation");
        } else if (path == kAcquireSecondary) {  // P3: the pre-materialised image from the sidecar
            ++counters_.p3_calls;
            std::unique_ptr<FILE, int (*)(FILE*)> f(std::fopen(sidecar_.c_str(), "rb"), &std::fclose);
            if (!f) throw std::runtime_error("P3: cannot open sidecar");
            constexpr std::uint64_t kChunk = 4ull << 20;  // the reference's 4 MiB transfers (:96)
            std::vector<std::uint8_t> buf(kChunk);
            for (std::uint64_t off = 0; off < exec_family_bytes(); off += kChunk) {
                const std::uint64_t n = std::min(kChunk, exec_family_bytes() - off);
                if (std::fread(buf.data(), 1, n, f.get()) != n) throw std::runtime_error("P3 short read");
                check(arcllm_cuda_memcpy_h2d(img + off, buf.data(), n, nullptr), "P3 upload");
            }
        } else {  // P0: materialise on the CPU from the mapped Q4_K weights
            ++counters_.p0_calls;
            std::vector<std::uint8_t> buf(lb);
            for (std::size_t i = 0; i < sources_.size(); ++i) {
                if (!sources_[i].host) throw std::runtime_error("P0: no host copy of the Q4_K weights");
                for (std::uint64_t b = 0; b < nblk; ++b) materialize_block(sources_[i].host + b * 144u, &buf[b * 148u]);
                check(arcllm_cuda_memcpy_h2d(img + i * lb, buf.data(), lb, nullptr), "P0 upload");
            }
        }
        ++counters_.b_materializations;
        resident_ = true;
        validated_ = false;
        out = {1ull};
        return BackendStatus::OK;
    } catch (const std::exception& e) {
        last_error_ = e.what();
    } catch (...) {
        last_error_ = "unknown acquisition failure";
    }
    free_image();
    resident_ = false;
    validated_ = false;
    return BackendStatus::ACQUISITION_FAILED;
}

BackendStatus Q4CudaBackend::validate(binding_v4::RepresentationHandle representation,
                                      registry::CapabilityId capability, registry::PrimitiveId target) noexcept {
    if (representation.opaque != 1ull || capability != kCapability || target != kPrimitiveB || !resident_)
        return BackendStatus::INVALID_BINDING_STATE;
    try {
        ++counters_.b_validations;
        const std::uint64_t nblk = std::uint64_t(rows_) * (k_ / 256u);
        std::uint64_t bad = 0;
        for (std::size_t i = 0; i < sources_.size(); ++i) {
            std::uint64_t mm = 0;
            check(arcllm_cuda_exec148_validate(sources_[i].device,
                                               static_cast<const std::uint8_t*>(image_) + i * layer_bytes(), nblk,
                                               &mm, nullptr),
                  "EXEC148 validation");
            bad += mm;
        }
        validated_ = bad == 0;
        if (!validated_) last_error_ = "EXEC148 image differs from its Q4_K source in " + std::to_string(bad) + " blocks";
        return validated_ ? BackendStatus::OK : BackendStatus::VALIDATION_FAILED;
    } catch (const std::exception& e) {
        last_error_ = e.what();
    } catch (...) {
        last_error_ = "unknown validation failure";
    }
    validated_ = false;
    return BackendStatus::VALIDATION_FAILED;
}

BackendStatus Q4CudaBackend::release(registry::PrimitiveId target,
                                     binding_v4::RepresentationHandle representation) noexcept {
    if (target != kPrimitiveB || representation.opaque != 1ull || !resident_)
        return BackendStatus::INVALID_BINDING_STATE;
    free_image();
    resident_ = false;
    validated_ = false;
    ++counters_.b_releases;
    return BackendStatus::OK;
}

BackendStatus Q4CudaBackend::resolve_primitive(registry::PrimitiveId primitive,
                                               binding_v4::PrimitiveHandle& out) noexcept {
    out = {};
    int n = 0;
    const bool device = arcllm_cuda_abi_version() != 0 && arcllm_cuda_device_count(&n) == ARC_OK && n > 0;
    if (primitive == kPrimitiveA) {
        ++counters_.resolve_a;
        // Route A needs the CUDA library and a device; the Vulkan backend
        // checks for its shader file at this point instead.
        if (!device) return BackendStatus::PRIMITIVE_UNAVAILABLE;
        out = {primitive.value};
        return BackendStatus::OK;
    }
    if (primitive == kPrimitiveB) {
        ++counters_.resolve_b;
        if (!resident_ || !validated_ || !device) return BackendStatus::PRIMITIVE_UNAVAILABLE;
        out = {primitive.value};
        return BackendStatus::OK;
    }
    return BackendStatus::PRIMITIVE_UNAVAILABLE;
}

int Q4CudaBackend::launch_ffn_down(binding_v4::PrimitiveHandle handle, std::uint32_t layer, const float* s,
                                   const float* residual, float* y, void* stream) const noexcept {
    const Source* src = find(layer);
    if (!src) return ARC_E_INVALID_ARGUMENT;
    if (handle.opaque == kPrimitiveA.value)
        return arcllm_cuda_matvec(ARC_GGML_Q4_K, src->device, rows_, k_, s, nullptr, 0.0f, nullptr, residual, y,
                                  stream);
    if (handle.opaque == kPrimitiveB.value && resident_ && validated_)
        return arcllm_cuda_matvec(ARC_TYPE_EXEC148, exec_image(layer), rows_, k_, s, nullptr, 0.0f, nullptr, residual,
                                  y, stream);
    return ARC_E_INVALID_ARGUMENT;
}

}  // namespace arcllm::v1::cuda
