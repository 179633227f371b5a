// B200MatvecAccelerator: vastloom's DeepseekV4MatvecAccelerator over the vlb200 C ABI.
//
// Drop-in for vastloom::cuda::CudaMatvecAccelerator (include/vastloom/cuda/
// cuda_matvec_accelerator.hpp:17-121, src/cuda/cuda_matvec_accelerator.cpp): the same options,
// statistics, refusal rules and eviction policy, with the device work done by libvlb200 (sm_100a
// kernels) instead of the embedded sm_52 PTX. Compiled against the reference's own headers; the
// graph code that offers rows (linear_packed_matrix, deepseek_v4_graph.cpp:769-874) is unchanged.
//
//   * residency keyed on DeepseekV4PackedMatrix::cache_identity, never a host address
//     (deepseek_v4_reference.hpp:125-132);
//   * refusals (return false, output untouched): recurring matrices when experts_only; storage
//     types without a device kernel (counted per type); identity 0; shapes the kernels do not
//     take; no space under the resident-byte ceiling; device allocation refused
//     (cuda_matvec_accelerator.cpp:102-200);
//   * eviction: non-recurring matrices first, then least recently used (cpp:176-193);
//   * every device byte is reserved from the ResourceGovernor (kind vram) before the library
//     allocates it, through the ABI's governor hooks (CudaDriver::allocate, cuda_driver.cpp:
//     2929-3005); a release the device refuses keeps its accounting charged.
//
// Expert-pack records to device, through the residency tier (deepseek_v4_expert_pack.hpp:24-41;
// ResidencyObject, residency.hpp:114-145, residency.cpp:140-212):
//   * begin_expert_pack_record reads one record's contiguous span from the pack payload in one
//     read into page-locked memory (a ResidencyObject in `reading`, its RAM and staging reserved),
//     publishes it RAM-ready, moves it to `copying_to_vram` (begin_vram_copy reserves the record's
//     VRAM bytes) and enqueues the one host-to-device copy plus the device re-layout on the
//     library's upload stream; it returns without waiting, so the next read overlaps this copy;
//   * the upload finishes on demand (the first matvec that offers one of its identities) or in
//     finish_expert_pack_records: the object is published VRAM-ready without its RAM copy, and
//     the record's matrices become resident under their cache identities;
//   * the library charges the governor hooks only for device bytes above the object's VRAM
//     reservation, so nothing is reserved twice;
//   * eviction takes a record's matrices out together and then calls evict_vram.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <span>
#include <string>
#include <vector>

#include "vastloom/core/bytes.hpp"
#include "vastloom/core/status.hpp"
#include "vastloom/inference/deepseek_v4_expert_pack.hpp"
#include "vastloom/inference/deepseek_v4_reference.hpp"
#include "vastloom/model/residency.hpp"
#include "vastloom/safety/resource_governor.hpp"
#include "vlb200.h"

namespace vastloom::b200 {

// The slice of the C ABI this adapter uses. default_vlb_api() binds libvlb200; tests bind fakes.
struct VlbApi {
    int (*open)(int, const vlb_governor*, uint64_t, vlb_handle**);
    void (*close)(vlb_handle*);
    int (*last_error)(const vlb_handle*, char*, size_t);
    int (*set_codebook)(vlb_handle*, uint32_t, const void*, size_t);
    int (*upload_matrix)(vlb_handle*, uint64_t, uint32_t, size_t, size_t, const void*, size_t,
                         vlb_matrix**);
    int (*release_matrix)(vlb_handle*, vlb_matrix*);
    int (*matvec)(vlb_handle*, const vlb_matrix*, const float*, float*);
    int (*upload_record_async)(vlb_handle*, const void*, size_t, const vlb_record_tensor*, uint32_t,
                               uint64_t, vlb_upload**);
    int (*upload_finish)(vlb_handle*, vlb_upload*, vlb_matrix**, uint32_t);
    int (*host_alloc)(vlb_handle*, size_t, void**);
    int (*host_free)(vlb_handle*, void*);
};

[[nodiscard]] const VlbApi& default_vlb_api() noexcept;

struct B200MatvecAcceleratorOptions {
    int device_ordinal{0};
    ByteCount minimum_free_vram_after{1U * GiB};
    ByteCount maximum_resident_bytes{6U * GiB};
    std::size_t maximum_matrices{512U};
    bool experts_only{false};
    // Check each expert-pack record read against its manifest SHA-256 (the pack verifier checks
    // the whole payload once, verify_deepseek_v4_expert_pack; this re-checks every read).
    bool verify_record_sha256{false};
};

struct B200MatvecAcceleratorStats {
    std::size_t offered{0U};
    std::size_t accelerated{0U};
    std::size_t declined{0U};
    std::size_t evicted{0U};
    std::size_t declined_recurring{0U};
    std::map<std::uint32_t, std::size_t> declined_by_type;
    std::size_t resident_matrices{0U};
    ByteCount resident_bytes{0U};
    ByteCount uploaded_bytes{0U};
    double kernel_ms{0.0};
    double upload_ms{0.0};
    std::size_t records_loaded{0U};
    ByteCount record_bytes{0U};
    double record_read_ms{0.0};
    double record_wait_ms{0.0};
};

class B200MatvecAccelerator final : public inference::DeepseekV4MatvecAccelerator {
public:
    [[nodiscard]] static Result<std::unique_ptr<B200MatvecAccelerator>> create(
        safety::ResourceGovernor& governor,
        const B200MatvecAcceleratorOptions& options = {},
        const VlbApi& api = default_vlb_api());

    ~B200MatvecAccelerator() override;

    [[nodiscard]] Result<bool> matvec(const inference::DeepseekV4PackedMatrix& matrix,
                                      std::span<const float> input,
                                      std::span<float> output) override;

    [[nodiscard]] const B200MatvecAcceleratorStats& stats() const noexcept { return stats_; }

    // Whether these exact weights are device-resident now (a snapshot; reporting only).
    [[nodiscard]] bool holds(std::uint64_t cache_identity) const noexcept {
        return cache_identity != 0U && resident_.contains(cache_identity);
    }

    // Reserved VRAM bytes this accelerator holds in the governor (matrices + codebooks + seam).
    [[nodiscard]] ByteCount reserved_bytes() const noexcept;

    // The cache identity of a routed expert's matrix (deepseek_v4_expert_provider.cpp:75-90:
    // FNV-1a 64 over the little-endian bytes of layer, expert and catalog tensor index, low bit
    // set), so pack uploads and the provider's matrices meet in one residency map.
    [[nodiscard]] static std::uint64_t expert_matrix_identity(std::uint32_t layer, std::uint32_t expert,
                                                              std::uint64_t catalog_tensor_index) noexcept;

    // Starts moving one verified expert-pack record to the device (see the file comment).
    // identities: one per record tensor, in record order. true = enqueued (or every identity is
    // resident already); false = declined (a storage type without a kernel, counted per type;
    // no room under the resident-byte ceiling; governor or device memory refused); Error = a
    // malformed record, a failed read or a device failure.
    [[nodiscard]] Result<bool> begin_expert_pack_record(const inference::DeepseekV4ExpertPack& pack,
                                                        const inference::DeepseekV4ExpertPackRecord& record,
                                                        std::span<const std::uint64_t> identities);
    // Finishes every record upload in flight; returns how many finished.
    [[nodiscard]] Result<std::size_t> finish_expert_pack_records();
    [[nodiscard]] std::size_t records_in_flight() const noexcept { return pending_.size(); }
    // The residency state of a record this accelerator moved (layer, expert), if it still has it.
    [[nodiscard]] Result<model::ResidencySnapshot> expert_record_residency(std::uint32_t layer,
                                                                           std::uint32_t expert) const;

private:
    // The matrices of one expert-pack record and the residency object that accounts for them.
    struct RecordGroup {
        model::ResidencyObject object;
        std::vector<std::uint64_t> identities;
        std::uint32_t layer{0U};
        std::uint32_t expert{0U};
    };
    struct Resident {
        vlb_matrix* matrix{nullptr};
        ByteCount bytes{0U};
        std::uint64_t last_used{0U};
        bool recurring{false};
        std::shared_ptr<RecordGroup> group;
    };
    struct PendingRecord {
        std::shared_ptr<RecordGroup> group;
        model::ResidencyTransfer transfer;
        vlb_upload* upload{nullptr};
        void* host{nullptr};
        std::vector<ByteCount> tensor_bytes;
        ByteCount bytes{0U};
    };

    B200MatvecAccelerator(safety::ResourceGovernor& governor, B200MatvecAcceleratorOptions options,
                          const VlbApi& api);
    [[nodiscard]] Result<Resident*> ensure_resident(const inference::DeepseekV4PackedMatrix& matrix);
    [[nodiscard]] Error api_error(int status, std::string_view operation) const;
    // Evicts (non-recurring first, then least recently used; a record's matrices together) until
    // `bytes` more fit under the ceiling and the matrix count allows `count` more.
    [[nodiscard]] Result<void> make_room(ByteCount bytes, std::size_t count);
    [[nodiscard]] Result<void> evict(std::map<std::uint64_t, Resident>::iterator victim);
    [[nodiscard]] Result<void> finish_record(std::size_t index);
    void abandon_record(PendingRecord& pending, std::string_view reason) noexcept;

    static int reserve_hook(void* ctx, uint64_t bytes, const char* tag);
    static void release_hook(void* ctx, uint64_t bytes, const char* tag);

    safety::ResourceGovernor* governor_{nullptr};
    B200MatvecAcceleratorOptions options_;
    VlbApi api_{};
    vlb_governor hooks_{};
    vlb_handle* handle_{nullptr};
    // Governor reservations held for live device allocations, matched on release by size and tag.
    std::multimap<std::pair<ByteCount, std::string>, safety::Reservation> reservations_;
    std::map<std::uint64_t, Resident> resident_;
    std::vector<PendingRecord> pending_;
    ByteCount pending_bytes_{0U};
    std::size_t pending_matrices_{0U};
    std::map<std::pair<std::uint32_t, std::uint32_t>, std::shared_ptr<RecordGroup>> records_;
    std::uint64_t clock_{0U};
    B200MatvecAcceleratorStats stats_;
};

}  // namespace vastloom::b200
