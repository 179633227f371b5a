// Host-side tests of B200MatvecAccelerator over a fake vlb200 API held in host memory, in the
// style of the reference's FakeCudaBackend (tests/test_cuda_driver.cpp:60-460): refusal rules,
// eviction order, Governor-first reservation, hard errors. No GPU.
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <vector>

#include "b200_matvec_accelerator.hpp"
#include "vastloom/inference/ggml_quantization.hpp"

namespace {

int failures = 0;
#define CHECK(cond)                                                          \
    do {                                                                     \
        if (!(cond)) {                                                       \
            ++failures;                                                      \
            std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #cond); \
        }                                                                    \
    } while (0)

using vastloom::ByteCount;
using vastloom::inference::DeepseekV4PackedMatrix;

struct FakeMatrix {
    uint32_t type;
    size_t rows, cols;
    std::vector<std::byte> payload;
};

struct FakeState {
    vlb_governor gov{};
    vastloom::safety::ResourceGovernor* governor = nullptr;
    int upload_status = VLB_OK;
    int matvec_status = VLB_OK;
    int uploads = 0, releases = 0, codebooks = 0;
    bool reservation_visible = true;
    std::map<vlb_matrix*, std::unique_ptr<FakeMatrix>> live;
} fake;

vastloom::ByteCount reserved_vram() {
    return fake.governor->snapshot().reserved[static_cast<size_t>(vastloom::safety::ResourceKind::vram)];
}

int f_open(int, const vlb_governor* g, uint64_t, vlb_handle** out) {
    fake.gov = *g;
    *out = reinterpret_cast<vlb_handle*>(0x1);
    return VLB_OK;
}
void f_close(vlb_handle*) {
    for (auto& kv : fake.live) fake.gov.release(fake.gov.ctx, kv.second->payload.size(), "vlb-resident-matrix");
    fake.live.clear();
}
int f_last_error(const vlb_handle*, char* buf, size_t cap) {
    std::snprintf(buf, cap, "fake failure");
    return VLB_OK;
}
int f_set_codebook(vlb_handle*, uint32_t, const void*, size_t) {
    ++fake.codebooks;
    return VLB_OK;
}
int f_upload(vlb_handle*, uint64_t, uint32_t type, size_t rows, size_t cols, const void* p,
             size_t n, vlb_matrix** out) {
    if (fake.upload_status != VLB_OK) return fake.upload_status;
    const ByteCount before = reserved_vram();
    if (fake.gov.reserve(fake.gov.ctx, n, "vlb-resident-matrix") != 0) return VLB_ERR_RESOURCE_EXHAUSTED;
    // Governor first: the reservation is visible before the "device" allocation exists.
    fake.reservation_visible = fake.reservation_visible && reserved_vram() == before + n;
    auto m = std::make_unique<FakeMatrix>();
    m->type = type;
    m->rows = rows;
    m->cols = cols;
    m->payload.assign(static_cast<const std::byte*>(p), static_cast<const std::byte*>(p) + n);
    auto* key = reinterpret_cast<vlb_matrix*>(m.get());
    fake.live[key] = std::move(m);
    *out = key;
    ++fake.uploads;
    return VLB_OK;
}
int f_release(vlb_handle*, vlb_matrix* m) {
    auto it = fake.live.find(m);
    if (it == fake.live.end()) return VLB_ERR_NOT_FOUND;
    fake.gov.release(fake.gov.ctx, it->second->payload.size(), "vlb-resident-matrix");
    fake.live.erase(it);
    ++fake.releases;
    return VLB_OK;
}
int f_matvec(vlb_handle*, const vlb_matrix* m, const float* x, float* y) {
    if (fake.matvec_status != VLB_OK) return fake.matvec_status;
    auto& fm = *fake.live.at(const_cast<vlb_matrix*>(m));
    std::vector<float> scratch(fm.rows);
    auto r = vastloom::inference::matvec_ggml_f32_transactional(fm.type, fm.payload, fm.rows, fm.cols,
                                                                {x, fm.cols}, scratch, {y, fm.rows});
    return r ? VLB_OK : VLB_ERR_INVALID_FORMAT;
}

const vastloom::b200::VlbApi kFake{&f_open, &f_close, &f_last_error, &f_set_codebook, &f_upload,
                                   &f_release, &f_matvec};

vastloom::safety::ResourceLimits limits(ByteCount vram) {
    vastloom::safety::ResourceLimits l;
    l.ram_hard_limit = 64U * vastloom::MiB;
    l.vram_hard_limit = vram;
    l.staging_hard_limit = 1U * vastloom::MiB;
    l.scratch_hard_limit = 1U * vastloom::MiB;
    l.minimum_system_ram_available = 0;
    l.minimum_storage_available = 0;
    return l;
}

std::vector<std::byte> q8_payload(size_t rows, size_t cols, unsigned seed) {
    std::vector<std::byte> p(rows * (cols / 32) * 34);
    for (size_t b = 0; b < rows * (cols / 32); ++b) {
        p[b * 34] = std::byte{0x00};
        p[b * 34 + 1] = std::byte{0x3c};  // d = 1.0
        for (size_t i = 0; i < 32; ++i) p[b * 34 + 2 + i] = std::byte(static_cast<uint8_t>((b * 7 + i * 13 + seed) & 0x7f));
    }
    return p;
}

void test_refusals() {
    vastloom::safety::ResourceGovernor governor(limits(16U * vastloom::MiB));
    fake = FakeState{};
    fake.governor = &governor;
    std::vector<float> input(32, 0.25F), output(1, 17.0F);
    vastloom::b200::B200MatvecAcceleratorOptions experts_only;
    experts_only.experts_only = true;
    experts_only.maximum_resident_bytes = 8U * vastloom::MiB;
    auto acc = vastloom::b200::B200MatvecAccelerator::create(governor, experts_only, kFake);
    CHECK(acc);
    CHECK(fake.codebooks == 4);
    DeepseekV4PackedMatrix recurring(8U, 1U, 32U, 32U, q8_payload(1, 32, 1));
    recurring.cache_identity = 11U;
    recurring.recurring = true;
    auto r = acc.value()->matvec(recurring, input, output);
    CHECK(r && !r.value());
    CHECK(output[0] == 17.0F);  // declined: output untouched
    CHECK(acc.value()->stats().declined_recurring == 1U && acc.value()->stats().declined == 1U);

    vastloom::b200::B200MatvecAcceleratorOptions plain;
    plain.maximum_resident_bytes = 8U * vastloom::MiB;
    auto acc2 = vastloom::b200::B200MatvecAccelerator::create(governor, plain, kFake);
    DeepseekV4PackedMatrix anonymous(8U, 1U, 32U, 32U, q8_payload(1, 32, 2));
    r = acc2.value()->matvec(anonymous, input, output);
    CHECK(r && !r.value());  // identity 0: never cached
    DeepseekV4PackedMatrix unsupported(999U, 1U, 32U, 32U, {});
    unsupported.cache_identity = 12U;
    r = acc2.value()->matvec(unsupported, input, output);
    CHECK(r && !r.value());
    CHECK(acc2.value()->stats().declined_by_type.at(999U) == 1U);
    DeepseekV4PackedMatrix q2k(10U, 1U, 256U, 256U, std::vector<std::byte>(84));  // Q2_K
    q2k.cache_identity = 14U;
    std::vector<float> in256(256, 0.f);
    r = acc2.value()->matvec(q2k, in256, output);
    CHECK(r && !r.value());  // a ggml type the sm_100a kernels do not take is counted too
    CHECK(acc2.value()->stats().declined_by_type.at(10U) == 1U);

    vastloom::b200::B200MatvecAcceleratorOptions tiny;
    tiny.maximum_resident_bytes = 1U;
    auto acc3 = vastloom::b200::B200MatvecAccelerator::create(governor, tiny, kFake);
    DeepseekV4PackedMatrix m(8U, 1U, 32U, 32U, q8_payload(1, 32, 3));
    m.cache_identity = 13U;
    r = acc3.value()->matvec(m, input, output);
    CHECK(r && !r.value());
    CHECK(acc3.value()->stats().resident_matrices == 0U);
}

void test_success_eviction_and_governor() {
    vastloom::safety::ResourceGovernor governor(limits(16U * vastloom::MiB));
    fake = FakeState{};
    fake.governor = &governor;
    vastloom::b200::B200MatvecAcceleratorOptions opts;
    opts.maximum_matrices = 2;
    auto acc = vastloom::b200::B200MatvecAccelerator::create(governor, opts, kFake).take_value();
    std::vector<float> x(64);
    for (size_t i = 0; i < x.size(); ++i) x[i] = static_cast<float>(i % 7) - 3.0F;
    std::vector<float> y(4), want(4), scratch(4);
    DeepseekV4PackedMatrix a(8U, 4U, 64U, 64U, q8_payload(4, 64, 1));
    a.cache_identity = 101U;
    a.recurring = true;
    auto r = acc->matvec(a, x, y);
    CHECK(r && r.value());
    CHECK(vastloom::inference::matvec_ggml_f32_transactional(8U, a.encoded, 4, 64, x, scratch, want));
    CHECK(y == want);
    CHECK(acc->holds(101U));
    CHECK(fake.reservation_visible);
    CHECK(reserved_vram() == a.encoded.size());
    DeepseekV4PackedMatrix b(8U, 4U, 64U, 64U, q8_payload(4, 64, 2));
    b.cache_identity = 102U;
    DeepseekV4PackedMatrix c(8U, 4U, 64U, 64U, q8_payload(4, 64, 3));
    c.cache_identity = 103U;
    CHECK(acc->matvec(b, x, y).value());
    CHECK(acc->matvec(a, x, y).value());  // a is now the most recent, and recurring
    CHECK(acc->matvec(c, x, y).value());  // full: evicts the non-recurring b, keeps a
    CHECK(acc->holds(101U) && !acc->holds(102U) && acc->holds(103U));
    CHECK(acc->stats().evicted == 1U && fake.releases == 1);
    CHECK(reserved_vram() == a.encoded.size() + c.encoded.size());
    CHECK(acc->stats().accelerated == 4U && acc->stats().uploaded_bytes == 3 * a.encoded.size());
    // a device error is a hard error, propagated with its code
    fake.matvec_status = VLB_ERR_IO_ERROR;
    r = acc->matvec(a, x, y);
    CHECK(!r && r.error().code == vastloom::ErrorCode::io_error);
    fake.matvec_status = VLB_OK;
    // out of device memory is a refusal, not a failure
    fake.upload_status = VLB_ERR_RESOURCE_EXHAUSTED;
    DeepseekV4PackedMatrix d(8U, 4U, 64U, 64U, q8_payload(4, 64, 4));
    d.cache_identity = 104U;
    r = acc->matvec(d, x, y);
    CHECK(r && !r.value());
    fake.upload_status = VLB_OK;
    acc.reset();
    CHECK(reserved_vram() == 0U);  // closing releases every reservation
}

void test_governor_refusal_is_a_decline() {
    vastloom::safety::ResourceGovernor governor(limits(64U));  // 64 bytes of VRAM budget
    fake = FakeState{};
    fake.governor = &governor;
    auto acc = vastloom::b200::B200MatvecAccelerator::create(governor, {}, kFake).take_value();
    std::vector<float> x(64, 1.0F), y(4, 5.0F);
    DeepseekV4PackedMatrix a(8U, 4U, 64U, 64U, q8_payload(4, 64, 9));
    a.cache_identity = 7U;
    auto r = acc->matvec(a, x, y);
    CHECK(r && !r.value());
    CHECK(y[0] == 5.0F);
    CHECK(reserved_vram() == 0U && fake.live.empty());
}

}  // namespace

int main() {
    test_refusals();
    test_success_eviction_and_governor();
    test_governor_refusal_is_a_decline();
    if (failures) {
        std::fprintf(stderr, "%d failures\n", failures);
        return 1;
    }
    std::printf("accelerator host tests passed\n");
    return 0;
}
