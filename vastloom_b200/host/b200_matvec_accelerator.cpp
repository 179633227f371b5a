// B200MatvecAccelerator implementation (see the header for the contract it keeps).
#include "b200_matvec_accelerator.hpp"

#include <algorithm>
#include <chrono>
#include <fstream>
#include <new>

#include "vastloom/inference/ggml_quantization.hpp"
#include "vastloom/util/sha256.hpp"

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
                            &vlb_matvec,        &vlb_upload_record_async, &vlb_upload_finish,
                            &vlb_host_alloc,    &vlb_host_free};
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
    for (auto& pending : pending_) abandon_record(pending, "the accelerator was destroyed");
    pending_.clear();
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

    // a record upload in flight holds these weights: finish it rather than upload them twice
    for (std::size_t i = 0; i < pending_.size(); ++i) {
        const auto& ids = pending_[i].group->identities;
        if (std::find(ids.begin(), ids.end(), matrix.cache_identity) != ids.end()) {
            if (auto finished = finish_record(i); !finished) return finished.error();
            break;
        }
    }
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

    if (auto room = make_room(matrix_bytes, 1U); !room) return room.error();
    if (matrix_bytes + stats_.resident_bytes + pending_bytes_ > options_.maximum_resident_bytes) return nullptr;

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
    Resident resident{uploaded, matrix_bytes, ++clock_, matrix.recurring, nullptr};
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

std::uint64_t B200MatvecAccelerator::expert_matrix_identity(std::uint32_t layer, std::uint32_t expert,
                                                            std::uint64_t catalog_tensor_index) noexcept {
    std::uint64_t identity = UINT64_C(14695981039346656037);
    for (const std::uint64_t part : {static_cast<std::uint64_t>(layer), static_cast<std::uint64_t>(expert),
                                     catalog_tensor_index}) {
        for (unsigned shift = 0U; shift < 64U; shift += 8U) {
            identity ^= (part >> shift) & 0xffU;
            identity *= UINT64_C(1099511628211);
        }
    }
    return identity | 1ULL;
}

Result<void> B200MatvecAccelerator::evict(std::map<std::uint64_t, Resident>::iterator victim) {
    std::shared_ptr<RecordGroup> group = victim->second.group;
    if (!group) {
        const int released = api_.release_matrix(handle_, victim->second.matrix);
        if (released != VLB_OK) return api_error(released, "release_matrix");
        stats_.resident_bytes -= std::min(victim->second.bytes, stats_.resident_bytes);
        resident_.erase(victim);
        ++stats_.evicted;
        return {};
    }
    // a record's matrices share one VRAM reservation: they leave together
    for (const std::uint64_t identity : group->identities) {
        auto found = resident_.find(identity);
        if (found == resident_.end() || found->second.group != group) continue;
        const int released = api_.release_matrix(handle_, found->second.matrix);
        if (released != VLB_OK) return api_error(released, "release_matrix");
        stats_.resident_bytes -= std::min(found->second.bytes, stats_.resident_bytes);
        resident_.erase(found);
        ++stats_.evicted;
    }
    auto record = records_.find({group->layer, group->expert});
    if (record != records_.end() && record->second == group) records_.erase(record);
    if (auto evicted = group->object.evict_vram(); !evicted) return evicted.error();
    return {};
}

Result<void> B200MatvecAccelerator::make_room(ByteCount bytes, std::size_t count) {
    // Non-recurring matrices go before recurring ones, then least recently used.
    while ((stats_.resident_bytes + pending_bytes_ + bytes > options_.maximum_resident_bytes ||
            resident_.size() + pending_matrices_ + count > options_.maximum_matrices) &&
           !resident_.empty()) {
        auto victim = std::min_element(resident_.begin(), resident_.end(),
                                       [](const auto& left, const auto& right) {
                                           if (left.second.recurring != right.second.recurring)
                                               return !left.second.recurring;
                                           return left.second.last_used < right.second.last_used;
                                       });
        if (auto evicted = evict(victim); !evicted) return evicted.error();
    }
    stats_.resident_matrices = resident_.size();
    return {};
}

namespace {

// One contiguous span of the pack payload in one read (the record is the H2D unit).
Result<void> read_span(const std::filesystem::path& path, ByteCount offset, ByteCount bytes, void* out) {
    std::ifstream file(path, std::ios::binary);
    if (!file) return make_error(ErrorCode::io_error, "Unable to open the expert pack payload", path.string());
    file.seekg(static_cast<std::streamoff>(offset));
    file.read(static_cast<char*>(out), static_cast<std::streamsize>(bytes));
    if (!file || static_cast<ByteCount>(file.gcount()) != bytes)
        return make_error(ErrorCode::io_error, "Expert pack record read was short", path.string());
    return {};
}

bool refused(const Error& error) { return error.code == ErrorCode::resource_exhausted; }

}  // namespace

Result<bool> B200MatvecAccelerator::begin_expert_pack_record(const inference::DeepseekV4ExpertPack& pack,
                                                             const inference::DeepseekV4ExpertPackRecord& record,
                                                             std::span<const std::uint64_t> identities) {
    const std::size_t n = record.tensors.size();
    const std::string where = "layer " + std::to_string(pack.layer) + " expert " + std::to_string(record.expert);
    if (n == 0U || n > 64U || identities.size() != n || record.bytes == 0U)
        return make_error(ErrorCode::invalid_argument, "Expert pack record identities do not match its tensors", where);
    std::vector<vlb_record_tensor> tensors(n);
    std::vector<ByteCount> tensor_bytes(n);
    for (std::size_t i = 0; i < n; ++i) {
        const auto& tensor = record.tensors[i];
        if (!tensor.ggml_type.has_value() || tensor.shape.size() < 2U || identities[i] == 0U)
            return make_error(ErrorCode::invalid_format, "Expert pack tensor has no storage type, matrix shape or identity",
                              tensor.name);
        Layout layout{};
        if (!layout_for(*tensor.ggml_type, &layout)) {
            try {
                ++stats_.declined_by_type[*tensor.ggml_type];
            } catch (const std::bad_alloc&) {
            }
            return false;
        }
        const std::uint64_t cols = tensor.shape[0], rows = tensor.shape[1];
        if (rows == 0U || cols == 0U || rows > 0xffffffffULL || cols > 0xffffffffULL ||
            cols % layout.block_elements != 0U || cols % 32U != 0U)
            return false;  // a shape the kernels do not take
        const ByteCount expected = rows * (cols / layout.block_elements) * layout.block_bytes;
        if (tensor.bytes != expected || tensor.packed_offset > record.bytes ||
            tensor.bytes > record.bytes - tensor.packed_offset)
            return make_error(ErrorCode::invalid_format, "Expert pack tensor span does not match its shape", tensor.name);
        tensors[i] = vlb_record_tensor{identities[i], *tensor.ggml_type, 0U, rows, cols, tensor.packed_offset,
                                       tensor.bytes};
        tensor_bytes[i] = tensor.bytes;
    }
    // already resident, or on its way
    std::size_t present = 0U;
    for (const std::uint64_t identity : identities) present += resident_.contains(identity) ? 1U : 0U;
    if (present == n) {
        for (const std::uint64_t identity : identities) resident_.find(identity)->second.last_used = ++clock_;
        return true;
    }
    for (const auto& pending : pending_)
        for (const std::uint64_t identity : identities)
            if (std::find(pending.group->identities.begin(), pending.group->identities.end(), identity) !=
                pending.group->identities.end())
                return true;
    // some of them resident on their own (the per-row seam uploaded them): the record replaces them
    for (const std::uint64_t identity : identities) {
        auto found = resident_.find(identity);
        if (found != resident_.end())
            if (auto evicted = evict(found); !evicted) return evicted.error();
    }
    if (record.bytes > options_.maximum_resident_bytes || n > options_.maximum_matrices) return false;
    if (auto room = make_room(record.bytes, n); !room) return room.error();
    if (stats_.resident_bytes + pending_bytes_ + record.bytes > options_.maximum_resident_bytes ||
        resident_.size() + pending_matrices_ + n > options_.maximum_matrices)
        return false;

    auto object = model::ResidencyObject::create(where, record.bytes);
    if (!object) return object.error();
    std::shared_ptr<RecordGroup> group;
    try {
        group = std::make_shared<RecordGroup>(RecordGroup{object.take_value(),
                                                          std::vector<std::uint64_t>(identities.begin(), identities.end()),
                                                          pack.layer, record.expert});
    } catch (const std::bad_alloc&) {
        return make_error(ErrorCode::resource_exhausted, "Unable to record an expert pack upload", where);
    }
    // nvme -> reading: RAM destination and read staging reserved
    if (auto reading = group->object.begin_read(*governor_, record.bytes); !reading) {
        if (refused(reading.error())) return false;
        return reading.error();
    }
    void* host = nullptr;
    const int pinned = api_.host_alloc(handle_, record.bytes, &host);
    if (pinned != VLB_OK) {
        (void)group->object.fail("page-locked staging refused");
        if (pinned == VLB_ERR_RESOURCE_EXHAUSTED) return false;
        return api_error(pinned, "host_alloc");
    }
    const auto give_up = [&](std::string_view reason) {
        api_.host_free(handle_, host);
        (void)group->object.fail(std::string(reason));
    };
    {
        auto transfer = group->object.acquire_transfer();
        if (!transfer) {
            give_up("no read transfer");
            return transfer.error();
        }
        const auto started = std::chrono::steady_clock::now();
        auto read = read_span(pack.payload_path, record.offset, record.bytes, host);
        stats_.record_read_ms += std::chrono::duration<double, std::milli>(
                                     std::chrono::steady_clock::now() - started).count();
        transfer.value().release();
        if (!read) {
            give_up(read.error().message);
            return read.error();
        }
    }
    if (options_.verify_record_sha256) {
        util::Sha256 digest;
        digest.update(std::span<const std::uint8_t>(static_cast<const std::uint8_t*>(host), record.bytes));
        if (digest.finalize_hex() != record.sha256) {
            give_up("record SHA-256 mismatch");
            return make_error(ErrorCode::integrity_error, "Expert pack record does not match its SHA-256", where);
        }
    }
    // reading -> ram_ready -> copying_to_vram: the record's VRAM reserved by the object
    if (auto ready = group->object.publish_ram_ready(); !ready) {
        give_up("publish_ram_ready failed");
        return ready.error();
    }
    if (auto copying = group->object.begin_vram_copy(*governor_); !copying) {
        give_up("VRAM reservation refused");
        if (refused(copying.error())) return false;
        return copying.error();
    }
    auto transfer = group->object.acquire_transfer();
    if (!transfer) {
        give_up("no copy transfer");
        return transfer.error();
    }
    vlb_upload* upload = nullptr;
    const int started = api_.upload_record_async(handle_, host, record.bytes, tensors.data(),
                                                 static_cast<std::uint32_t>(n), record.bytes, &upload);
    if (started != VLB_OK) {
        auto error = api_error(started, "upload_record_async");
        transfer.value().release();
        give_up(error.message);
        if (started == VLB_ERR_RESOURCE_EXHAUSTED || started == VLB_ERR_UNSUPPORTED) return false;
        return error;
    }
    try {
        pending_.push_back(PendingRecord{group, transfer.take_value(), upload, host, std::move(tensor_bytes),
                                         record.bytes});
        records_[{pack.layer, record.expert}] = group;
    } catch (const std::bad_alloc&) {
        return make_error(ErrorCode::resource_exhausted, "Unable to record an expert pack upload", where);
    }
    pending_bytes_ += record.bytes;
    pending_matrices_ += n;
    return true;
}

Result<void> B200MatvecAccelerator::finish_record(std::size_t index) {
    PendingRecord pending = std::move(pending_[index]);
    pending_.erase(pending_.begin() + static_cast<std::ptrdiff_t>(index));
    const std::size_t n = pending.group->identities.size();
    pending_bytes_ -= pending.bytes;
    pending_matrices_ -= n;
    std::vector<vlb_matrix*> matrices(n, nullptr);
    const auto started = std::chrono::steady_clock::now();
    const int finished = api_.upload_finish(handle_, pending.upload, matrices.data(), static_cast<std::uint32_t>(n));
    stats_.record_wait_ms += std::chrono::duration<double, std::milli>(
                                 std::chrono::steady_clock::now() - started).count();
    pending.transfer.release();
    api_.host_free(handle_, pending.host);
    const auto forget = [&] {
        auto record = records_.find({pending.group->layer, pending.group->expert});
        if (record != records_.end() && record->second == pending.group) records_.erase(record);
    };
    if (finished != VLB_OK) {
        auto error = api_error(finished, "upload_finish");
        (void)pending.group->object.fail(error.message);
        forget();
        return error;
    }
    const auto release_all = [&] {
        for (vlb_matrix* matrix : matrices) api_.release_matrix(handle_, matrix);
    };
    // copying_to_vram -> vram_ready; the RAM copy is not kept (its page-locked buffer is gone)
    if (auto ready = pending.group->object.publish_vram_ready(false); !ready) {
        release_all();
        forget();
        return ready.error();
    }
    try {
        for (std::size_t i = 0; i < n; ++i)
            resident_.emplace(pending.group->identities[i],
                              Resident{matrices[i], pending.tensor_bytes[i], ++clock_, false, pending.group});
    } catch (const std::bad_alloc&) {
        for (const std::uint64_t identity : pending.group->identities) resident_.erase(identity);
        release_all();
        (void)pending.group->object.evict_vram();
        forget();
        return make_error(ErrorCode::resource_exhausted, "Unable to record resident B200 matrices");
    }
    stats_.uploaded_bytes += pending.bytes;
    stats_.resident_bytes += pending.bytes;
    stats_.resident_matrices = resident_.size();
    stats_.record_bytes += pending.bytes;
    ++stats_.records_loaded;
    return {};
}

Result<std::size_t> B200MatvecAccelerator::finish_expert_pack_records() {
    std::size_t finished = 0U;
    while (!pending_.empty()) {
        if (auto done = finish_record(0U); !done) return done.error();
        ++finished;
    }
    return finished;
}

void B200MatvecAccelerator::abandon_record(PendingRecord& pending, std::string_view reason) noexcept {
    if (pending.upload != nullptr && handle_ != nullptr) {
        std::vector<vlb_matrix*> matrices(pending.group->identities.size(), nullptr);
        if (api_.upload_finish(handle_, pending.upload, matrices.data(),
                               static_cast<std::uint32_t>(matrices.size())) == VLB_OK)
            for (vlb_matrix* matrix : matrices) api_.release_matrix(handle_, matrix);
        pending.upload = nullptr;
    }
    pending.transfer.release();
    if (pending.host != nullptr && handle_ != nullptr) api_.host_free(handle_, pending.host);
    pending.host = nullptr;
    try {
        (void)pending.group->object.fail(std::string(reason));
    } catch (...) {
    }
}

Result<model::ResidencySnapshot> B200MatvecAccelerator::expert_record_residency(std::uint32_t layer,
                                                                               std::uint32_t expert) const {
    auto found = records_.find({layer, expert});
    if (found == records_.end())
        return make_error(ErrorCode::not_found, "No expert pack record of this expert is on the device",
                          "layer " + std::to_string(layer) + " expert " + std::to_string(expert));
    return found->second->object.snapshot();
}

}  // namespace vastloom::b200
