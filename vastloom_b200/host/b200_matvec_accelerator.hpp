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
#include "vastloom/inference/deepseek_v4_reference.hpp"
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
};

[[nodiscard]] const VlbApi& default_vlb_api() noexcept;

struct B200MatvecAcceleratorOptions {
    int device_ordinal{0};
    ByteCount minimum_free_vram_after{1U * GiB};
    ByteCount maximum_resident_bytes{6U * GiB};
    std::size_t maximum_matrices{512U};
    bool experts_only{false};
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

private:
    struct Resident {
        vlb_matrix* matrix{nullptr};
        ByteCount bytes{0U};
        std::uint64_t last_used{0U};
        bool recurring{false};
    };

    B200MatvecAccelerator(safety::ResourceGovernor& governor, B200MatvecAcceleratorOptions options,
                          const VlbApi& api);
    [[nodiscard]] Result<Resident*> ensure_resident(const inference::DeepseekV4PackedMatrix& matrix);
    [[nodiscard]] Error api_error(int status, std::string_view operation) const;

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
    std::uint64_t clock_{0U};
    B200MatvecAcceleratorStats stats_;
};

}  // namespace vastloom::b200
