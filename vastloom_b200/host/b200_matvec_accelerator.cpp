// B200MatvecAccelerator implementation (see the header for the contract it keeps).
#include "b200_matvec_accelerator.hpp"

#include <algorithm>
#include <chrono>
#include <new>

#include "vastloom/inference/ggml_quantization.hpp"

namespace vastloom::b200 {
namespace {

constexpr std::uint32_t kTypeQ8_0 = 8U;
constexpr std::uint32_t kTypeIq2Xxs = 16U;
constexpr std::uint32_t kTypeIq3Xxs = 18U;
constexpr std::uint32_t kTypeIq1S = 19U;

struct Layout {
    std::size_t block_elements;
    std::size_t block_bytes;
};

// The storage types the sm_100a kernels take (ggml_quantization.hpp:12-31 layouts).
bool layout_for(std::uint32_t type, Layout* l) {
    switch (type) {
        case kTypeQ8_0: *l = {32U, 34U}; return true;
        case kTypeIq2Xxs: *l = {256U, 66U}; return true;
        case kTypeIq3Xxs: *l = {256U, 98U}; return true;
        case kTypeIq1S: *l = {256U, 50U}; return true;
        case inference::kGgmlTypeQ4K: *l = {256U, 144U}; return true;
        case inference::kGgmlTypeQ5K: *l = {256U, 176U}; return true;
        case inference::kGgmlTypeQ6K: *l = {256U, 210U}; return true;
        case inference::kGgmlTypeIq2S: *l = {256U, 82U}; return true;
        case inference::kGgmlTypeMxfp4: *l = {32U, 17U}; return true;
        default: return false;
    }
}

ErrorCode error_code_for(int status) {
    // VLB_ERR_* = ErrorCode + 1 (include/vlb200.h)
    if (status >= 1 && status <= 10) return static_cast<ErrorCode>(status - 1);
    return ErrorCode::internal_error;
}

}  // namespace

const VlbApi& default_vlb_api() noexcept {
    static const VlbApi api{&vlb_open,          &vlb_close,          &vlb_last_error,
                            &vlb_set_codebook,  &vlb_upload_matrix,  &vlb_release_matrix,
                            &vlb_matvec};
    return api;
}

B200MatvecAccelerator::B200MatvecAccelerator(safety::ResourceGovernor& governor,
                                             B200MatvecAcceleratorOptions options,
                                             const VlbApi& api)
    : governor_(&governor), options_(options), api_(api) {
    hooks_.ctx = this;
    hooks_.reserve = &B200MatvecAccelerator::reserve_hook;
    hooks_.release = &B200MatvecAccelerator::release_hook;
}

B200MatvecAccelerator::~B200MatvecAccelerator() {
    if (handle_ != nullptr) api_.close(handle_);  // frees every allocation, releasing through the hooks
    // Anything still reserved here had a release the device refused: keep it charged.
    for (auto& entry : reservations_) entry.second.abandon_accounting_on_external_release_failure();
}

int B200MatvecAccelerator::reserve_hook(void* ctx, uint64_t bytes, const char* tag) {
    auto* self = static_cast<B200MatvecAccelerator*>(ctx);
    try {
        auto reserved = self->governor_->try_reserve(safety::ResourceKind::vram, bytes,
                                                     tag != nullptr ? tag : "b200");
        if (!reserved) return 1;
        self->reservations_.emplace(std::make_pair(ByteCount{bytes}, std::string(tag ? tag : "b200")),
                                    reserved.take_value());
        return 0;
    } catch (...) {
        return 1;
    }
}

void B200MatvecAccelerator::release_hook(void* ctx, uint64_t bytes, const char* tag) {
    auto* self = static_cast<B200MatvecAccelerator*>(ctx);
    auto found = self->reservations_.find(std::make_pair(ByteCount{bytes}, std::string(tag ? tag : "b200")));
    if (found != self->reservations_.end()) {
        found->second.release();
        self->reservations_.erase(found);
    }
}

ByteCount B200MatvecAccelerator::reserved_bytes() const noexcept {
    ByteCount total = 0U;
    for (const auto& entry : reservations_) total += entry.second.bytes();
    return total;
}

Error B200MatvecAccelerator::api_error(int status, std::string_view operation) const {
    char buffer[512] = {0};
    if (handle_ != nullptr) api_.last_error(handle_, buffer, sizeof(buffer));
    return make_error(error_code_for(status), std::string("vlb200 call failed: ") + std::string(operation),
                      buffer);
}

Result<std::unique_ptr<B200MatvecAccelerator>> B200MatvecAccelerator::create(
    safety::ResourceGovernor& governor, const B200MatvecAcceleratorOptions& options,
    const VlbApi& api) {
    if (options.device_ordinal < 0 || options.maximum_resident_bytes == 0U ||
        options.maximum_matrices == 0U) {
        return make_error(ErrorCode::invalid_argument, "B200 matvec accelerator options are invalid");
    }
    std::unique_ptr<B200MatvecAccelerator> self;
    try {
        self.reset(new B200MatvecAccelerator(governor, options, api));
    } catch (const std::bad_alloc&) {
        return make_error(ErrorCode::resource_exhausted, "Unable to allocate the B200 matvec accelerator");
    }
    const int opened = api.open(options.device_ordinal, &self->hooks_,
                                options.minimum_free_vram_after, &self->handle_);
    if (opened != VLB_OK) {
        self->handle_ = nullptr;
        return make_error(error_code_for(opened), "Unable to open the B200 device");
    }
    // The codebooks come from the reference's own tables; the ABI verifies their fingerprints.
    const auto install = [&](std::uint32_t type, std::span<const std::byte> table) -> Result<void> {
        const int st = api.set_codebook(self->handle_, type, table.data(), table.size());
        if (st != VLB_OK) return self->api_error(st, "set_codebook");
        return {};
    };
    if (auto s = install(kTypeIq1S, std::as_bytes(inference::iq1_s_grid_table())); !s) return s.error();
    if (auto s = install(kTypeIq2Xxs, std::as_bytes(inference::iq2_xxs_grid_table())); !s) return s.error();
    if (auto s = install(kTypeIq3Xxs, std::as_bytes(inference::iq3_xxs_grid_table())); !s) return s.error();
    if (auto s = install(inference::kGgmlTypeIq2S, std::as_bytes(inference::iq2_s_grid_table())); !s) return s.error();
    return self;
}

Result<B200MatvecAccelerator::Resident*> B200MatvecAccelerator::ensure_resident(
    const inference::DeepseekV4PackedMatrix& matrix) {
    if (options_.experts_only && matrix.recurring) {
        ++stats_.declined_recurring;
        return nullptr;
    }
    Layout layout{};
    if (!layout_for(matrix.ggml_type, &layout)) {
        try {
            ++stats_.declined_by_type[matrix.ggml_type];
        } catch (const std::bad_alloc&) {
        }
        return nullptr;
    }
    if (matrix.rows == 0U || matrix.storage_columns == 0U ||
        matrix.storage_columns % layout.block_elements != 0U || matrix.storage_columns % 32U != 0U) {
        return nullptr;
    }
    if (matrix.cache_identity == 0U) return nullptr;

    auto entry = resident_.find(matrix.cache_identity);
    if (entry != resident_.end()) {
        entry->second.last_used = ++clock_;
        return &entry->second;
    }
    auto payload = inference::deepseek_v4_packed_matrix_payload(matrix, "b200-matvec");
    if (!payload) return payload.error();
    const ByteCount matrix_bytes =
        static_cast<ByteCount>(matrix.rows) * (matrix.storage_columns / layout.block_elements) *
        layout.block_bytes;
    if (payload.value().size() != matrix_bytes) return nullptr;
    if (matrix_bytes > options_.maximum_resident_bytes) return nullptr;

    // Room first: non-recurring matrices go before recurring ones, then least recently used.
    while ((stats_.resident_bytes + matrix_bytes > options_.maximum_resident_bytes ||
            resident_.size() >= options_.maximum_matrices) &&
           !resident_.empty()) {
        auto victim = std::min_element(resident_.begin(), resident_.end(),
                                       [](const auto& left, const auto& right) {
                                           if (left.second.recurring != right.second.recurring)
                                               return !left.second.recurring;
                                           return left.second.last_used < right.second.last_used;
                                       });
        const int released = api_.release_matrix(handle_, victim->second.matrix);
        if (released != VLB_OK) return api_error(released, "release_matrix");
        stats_.resident_bytes -= std::min(victim->second.bytes, stats_.resident_bytes);
        resident_.erase(victim);
        ++stats_.evicted;
    }
    if (matrix_bytes > options_.maximum_resident_bytes - stats_.resident_bytes) return nullptr;

    vlb_matrix* uploaded = nullptr;
    const auto started = std::chrono::steady_clock::now();
    const int st = api_.upload_matrix(handle_, matrix.cache_identity, matrix.ggml_type, matrix.rows,
                                      matrix.storage_columns, payload.value().data(),
                                      payload.value().size(), &uploaded);
    stats_.upload_ms += std::chrono::duration<double, std::milli>(
                            std::chrono::steady_clock::now() - started).count();
    // Out of device memory (or a governor refusal) is a reason to stop offering, not a failure.
    if (st == VLB_ERR_RESOURCE_EXHAUSTED || st == VLB_ERR_UNSUPPORTED) return nullptr;
    if (st != VLB_OK) return api_error(st, "upload_matrix");
    Resident resident{uploaded, matrix_bytes, ++clock_, matrix.recurring};
    try {
        entry = resident_.emplace(matrix.cache_identity, resident).first;
    } catch (const std::bad_alloc&) {
        api_.release_matrix(handle_, uploaded);
        return make_error(ErrorCode::resource_exhausted, "Unable to record a resident B200 matrix");
    }
    stats_.uploaded_bytes += matrix_bytes;
    stats_.resident_bytes += matrix_bytes;
    stats_.resident_matrices = resident_.size();
    return &entry->second;
}

Result<bool> B200MatvecAccelerator::matvec(const inference::DeepseekV4PackedMatrix& matrix,
                                           std::span<const float> input,
                                           std::span<float> output) {
    ++stats_.offered;
    if (input.size() != matrix.storage_columns || output.size() != matrix.rows) {
        ++stats_.declined;
        return false;
    }
    auto made = ensure_resident(matrix);
    if (!made) return made.error();
    if (made.value() == nullptr) {
        ++stats_.declined;
        return false;
    }
    const auto started = std::chrono::steady_clock::now();
    const int st = api_.matvec(handle_, made.value()->matrix, input.data(), output.data());
    if (st != VLB_OK) return api_error(st, "matvec");
    stats_.kernel_ms += std::chrono::duration<double, std::milli>(
                            std::chrono::steady_clock::now() - started).count();
    ++stats_.accelerated;
    stats_.resident_matrices = resident_.size();
    return true;
}

}  // namespace vastloom::b200
