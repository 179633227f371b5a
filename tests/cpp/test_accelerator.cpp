// Host-side tests of B200MatvecAccelerator over a fake vlb200 API held in host memory, in the
// style of the reference's FakeCudaBackend (tests/test_cuda_driver.cpp:60-460): refusal rules,
// eviction order, Governor-first reservation, hard errors. No GPU.
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <map>
#include <memory>
#include <vector>

#include "b200_matvec_accelerator.hpp"
#include "vastloom/inference/ggml_quantization.hpp"
#include "vastloom/util/sha256.hpp"

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
    size_t hooked = 0;  // bytes charged through the governor hooks
};

// A record upload in flight: its matrices exist but are not handed out yet.
struct FakeRecordUpload {
    std::vector<std::unique_ptr<FakeMatrix>> mats;
};

struct FakeState {
    vlb_governor gov{};
    vastloom::safety::ResourceGovernor* governor = nullptr;
    int upload_status = VLB_OK;
    int matvec_status = VLB_OK;
    int uploads = 0, releases = 0, codebooks = 0, record_uploads = 0;
    int record_status = VLB_OK;
    int finish_status = VLB_OK;
    bool reservation_visible = true;
    std::map<vlb_matrix*, std::unique_ptr<FakeMatrix>> live;
    std::map<vlb_upload*, std::unique_ptr<FakeRecordUpload>> in_flight;
    std::map<void*, std::unique_ptr<std::byte[]>> pinned;
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
    for (auto& kv : fake.live)
        if (kv.second->hooked) fake.gov.release(fake.gov.ctx, kv.second->hooked, "vlb-resident-matrix");
    fake.live.clear();
    for (auto& kv : fake.in_flight)
        for (auto& m : kv.second->mats)
            if (m->hooked) fake.gov.release(fake.gov.ctx, m->hooked, "vlb-resident-matrix");
    fake.in_flight.clear();
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
    m->hooked = n;
    auto* key = reinterpret_cast<vlb_matrix*>(m.get());
    fake.live[key] = std::move(m);
    *out = key;
    ++fake.uploads;
    return VLB_OK;
}
int f_release(vlb_handle*, vlb_matrix* m) {
    auto it = fake.live.find(m);
    if (it == fake.live.end()) return VLB_ERR_NOT_FOUND;
    if (it->second->hooked) fake.gov.release(fake.gov.ctx, it->second->hooked, "vlb-resident-matrix");
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

// The record path as the library keeps it: images (here: the payload bytes) charged through the
// hooks only above the caller's reservation, in tensor order.
int f_upload_record(vlb_handle*, const void* record, size_t bytes, const vlb_record_tensor* t, uint32_t n,
                    uint64_t reserved, vlb_upload** out) {
    if (fake.record_status != VLB_OK) return fake.record_status;
    auto up = std::make_unique<FakeRecordUpload>();
    uint64_t prepaid = reserved;
    for (uint32_t i = 0; i < n; ++i) {
        if (t[i].offset + t[i].bytes > bytes) return VLB_ERR_INVALID_FORMAT;
        auto m = std::make_unique<FakeMatrix>();
        m->type = t[i].ggml_type;
        m->rows = t[i].rows;
        m->cols = t[i].storage_cols;
        const auto* src = static_cast<const std::byte*>(record) + t[i].offset;
        m->payload.assign(src, src + t[i].bytes);
        const uint64_t covered = std::min<uint64_t>(prepaid, t[i].bytes);
        prepaid -= covered;
        m->hooked = t[i].bytes - covered;
        if (m->hooked && fake.gov.reserve(fake.gov.ctx, m->hooked, "vlb-resident-matrix") != 0) {
            for (auto& done : up->mats)
                if (done->hooked) fake.gov.release(fake.gov.ctx, done->hooked, "vlb-resident-matrix");
            return VLB_ERR_RESOURCE_EXHAUSTED;
        }
        up->mats.push_back(std::move(m));
    }
    auto* key = reinterpret_cast<vlb_upload*>(up.get());
    fake.in_flight[key] = std::move(up);
    *out = key;
    ++fake.record_uploads;
    return VLB_OK;
}
int f_upload_finish(vlb_handle*, vlb_upload* u, vlb_matrix** out, uint32_t n) {
    auto it = fake.in_flight.find(u);
    if (it == fake.in_flight.end()) return VLB_ERR_INVALID_ARGUMENT;
    auto up = std::move(it->second);
    fake.in_flight.erase(it);
    if (fake.finish_status != VLB_OK || n != up->mats.size()) {
        for (auto& m : up->mats)
            if (m->hooked) fake.gov.release(fake.gov.ctx, m->hooked, "vlb-resident-matrix");
        return fake.finish_status != VLB_OK ? fake.finish_status : VLB_ERR_INVALID_ARGUMENT;
    }
    for (uint32_t i = 0; i < n; ++i) {
        auto* key = reinterpret_cast<vlb_matrix*>(up->mats[i].get());
        fake.live[key] = std::move(up->mats[i]);
        out[i] = key;
    }
    return VLB_OK;
}
int f_host_alloc(vlb_handle*, size_t bytes, void** out) {
    auto buf = std::make_unique<std::byte[]>(bytes);
    *out = buf.get();
    fake.pinned[*out] = std::move(buf);
    return VLB_OK;
}
int f_host_free(vlb_handle*, void* p) {
    return fake.pinned.erase(p) ? VLB_OK : VLB_ERR_NOT_FOUND;
}

const vastloom::b200::VlbApi kFake{&f_open, &f_close, &f_last_error, &f_set_codebook, &f_upload,
                                   &f_release, &f_matvec, &f_upload_record, &f_upload_finish,
                                   &f_host_alloc, &f_host_free};

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

ByteCount reserved(vastloom::safety::ResourceKind kind) {
    return fake.governor->snapshot().reserved[static_cast<size_t>(kind)];
}

// Two expert-pack records (three Q8_0 4 x 64 tensors each) in a payload file, 4 KiB aligned as a
// pack lays them out (kDeepseekV4ExpertPackAlignment).
struct PackFixture {
    std::filesystem::path path;
    vastloom::inference::DeepseekV4ExpertPack pack;
    std::vector<std::vector<std::byte>> tensors;  // [record * 3 + j]
};

PackFixture make_pack(const std::string& name) {
    PackFixture f;
    f.path = std::filesystem::temp_directory_path() / name;
    std::vector<std::byte> payload(4096 + 3 * 272);
    f.pack.payload_path = f.path;
    f.pack.layer = 3U;
    for (uint32_t e = 0; e < 2; ++e) {
        vastloom::inference::DeepseekV4ExpertPackRecord record;
        record.expert = 5U + e;
        record.offset = 4096U * e;
        record.bytes = 3U * 272U;
        for (uint32_t j = 0; j < 3; ++j) {
            auto bytes = q8_payload(4, 64, 10U * e + j);
            std::copy(bytes.begin(), bytes.end(), payload.begin() + record.offset + 272U * j);
            vastloom::inference::DeepseekV4ExpertPackTensor t;
            t.name = "blk.3.ffn_" + std::to_string(j) + "_exps.weight";
            t.packed_offset = 272U * j;
            t.bytes = 272U;
            t.ggml_type = 8U;
            t.shape = {64U, 4U, 256U};
            record.tensors.push_back(t);
            f.tensors.push_back(bytes);
        }
        vastloom::util::Sha256 digest;
        digest.update(std::span<const std::byte>(payload.data() + record.offset, record.bytes));
        record.sha256 = digest.finalize_hex();
        f.pack.records.push_back(record);
    }
    std::ofstream(f.path, std::ios::binary).write(reinterpret_cast<const char*>(payload.data()),
                                                  static_cast<std::streamsize>(payload.size()));
    return f;
}

std::vector<uint64_t> identities(uint32_t expert) {
    std::vector<uint64_t> ids;
    for (uint64_t j = 0; j < 3; ++j)
        ids.push_back(vastloom::b200::B200MatvecAccelerator::expert_matrix_identity(3U, expert, 40U + j));
    return ids;
}

void test_expert_pack_records() {
    using vastloom::model::ResidencyState;
    using vastloom::safety::ResourceKind;
    // the provider's identity (deepseek_v4_expert_provider.cpp:75-90), computed here independently
    uint64_t want = 14695981039346656037ULL;
    for (uint64_t part : {3ULL, 5ULL, 41ULL})
        for (unsigned sh = 0; sh < 64; sh += 8) {
            want ^= (part >> sh) & 0xffU;
            want *= 1099511628211ULL;
        }
    CHECK(identities(5)[1] == (want | 1ULL));

    auto f = make_pack("vlb_pack_records.bin");
    vastloom::safety::ResourceGovernor governor(limits(16U * vastloom::MiB));
    fake = FakeState{};
    fake.governor = &governor;
    vastloom::b200::B200MatvecAcceleratorOptions opts;
    opts.maximum_matrices = 4U;
    opts.verify_record_sha256 = true;
    auto acc = vastloom::b200::B200MatvecAccelerator::create(governor, opts, kFake).take_value();
    const auto ids5 = identities(5), ids6 = identities(6);

    // record 5 in flight: RAM and VRAM held by its residency object, nothing charged twice
    auto begun = acc->begin_expert_pack_record(f.pack, f.pack.records[0], ids5);
    CHECK(begun && begun.value());
    CHECK(acc->records_in_flight() == 1U && fake.record_uploads == 1 && fake.uploads == 0);
    auto snap = acc->expert_record_residency(3U, 5U);
    CHECK(snap && snap.value().state == ResidencyState::copying_to_vram);
    CHECK(snap.value().active_transfers == 1U && snap.value().vram_reserved_bytes == 816U);
    CHECK(reserved(ResourceKind::vram) == 816U && reserved(ResourceKind::ram) == 816U);
    CHECK(reserved(ResourceKind::staging) == 0U);  // released at publish_ram_ready
    CHECK(!acc->holds(ids5[0]));

    // the seam offering one of its matrices finishes the upload (no second upload)
    std::vector<float> x(64), y(4), expect(4), scratch(4);
    for (size_t i = 0; i < x.size(); ++i) x[i] = static_cast<float>(i % 5) - 2.0F;
    DeepseekV4PackedMatrix w3(8U, 4U, 64U, 64U, f.tensors[1]);
    w3.cache_identity = ids5[1];
    auto r = acc->matvec(w3, x, y);
    CHECK(r && r.value());
    CHECK(vastloom::inference::matvec_ggml_f32_transactional(8U, f.tensors[1], 4, 64, x, scratch, expect));
    CHECK(y == expect);
    CHECK(fake.uploads == 0 && acc->records_in_flight() == 0U);
    CHECK(acc->holds(ids5[0]) && acc->holds(ids5[1]) && acc->holds(ids5[2]));
    snap = acc->expert_record_residency(3U, 5U);
    CHECK(snap && snap.value().state == ResidencyState::vram_ready && snap.value().ram_reserved_bytes == 0U);
    CHECK(reserved(ResourceKind::vram) == 816U && reserved(ResourceKind::ram) == 0U);
    CHECK(fake.pinned.empty());
    CHECK(acc->stats().records_loaded == 1U && acc->stats().record_bytes == 816U);
    // a record already resident is not read again
    CHECK(acc->begin_expert_pack_record(f.pack, f.pack.records[0], ids5).value());
    CHECK(fake.record_uploads == 1);

    // record 6 needs three more matrices (ceiling 4): record 5 leaves as a whole, then evict_vram
    CHECK(acc->begin_expert_pack_record(f.pack, f.pack.records[1], ids6).value());
    CHECK(!acc->holds(ids5[0]) && !acc->holds(ids5[1]) && !acc->holds(ids5[2]));
    CHECK(acc->stats().evicted == 3U);
    CHECK(!acc->expert_record_residency(3U, 5U));
    auto finished = acc->finish_expert_pack_records();
    CHECK(finished && finished.value() == 1U);
    CHECK(acc->holds(ids6[2]) && reserved(ResourceKind::vram) == 816U);

    // a storage type without a kernel is a counted decline; a bad digest an integrity error
    auto odd = f.pack.records[0];
    odd.tensors[2].ggml_type = 10U;  // Q2_K
    auto declined = acc->begin_expert_pack_record(f.pack, odd, ids5);
    CHECK(declined && !declined.value());
    CHECK(acc->stats().declined_by_type.at(10U) == 1U);
    auto tampered = f.pack.records[0];
    tampered.sha256[0] = tampered.sha256[0] == '0' ? '1' : '0';
    auto bad = acc->begin_expert_pack_record(f.pack, tampered, ids5);
    CHECK(!bad && bad.error().code == vastloom::ErrorCode::integrity_error);
    CHECK(fake.pinned.empty() && reserved(ResourceKind::ram) == 0U);
    auto wrong_ids = acc->begin_expert_pack_record(f.pack, f.pack.records[0], std::span(ids5).first(2));
    CHECK(!wrong_ids && wrong_ids.error().code == vastloom::ErrorCode::invalid_argument);

    // a block the device rejects fails the record and releases everything it held
    fake.finish_status = VLB_ERR_INVALID_FORMAT;
    CHECK(acc->begin_expert_pack_record(f.pack, f.pack.records[0], ids5).value());
    finished = acc->finish_expert_pack_records();
    CHECK(!finished && finished.error().code == vastloom::ErrorCode::invalid_format);
    CHECK(!acc->holds(ids5[0]) && !acc->expert_record_residency(3U, 5U));
    CHECK(!acc->holds(ids6[0]));  // evicted to make room for the record that then failed
    CHECK(reserved(ResourceKind::vram) == 0U && reserved(ResourceKind::ram) == 0U && fake.pinned.empty());
    fake.finish_status = VLB_OK;

    // the governor refusing the VRAM destination is a decline
    vastloom::safety::ResourceGovernor small(limits(1000U));
    fake = FakeState{};
    fake.governor = &small;
    auto acc2 = vastloom::b200::B200MatvecAccelerator::create(small, {}, kFake).take_value();
    CHECK(acc2->begin_expert_pack_record(f.pack, f.pack.records[0], ids5).value());
    auto refused = acc2->begin_expert_pack_record(f.pack, f.pack.records[1], ids6);
    CHECK(refused && !refused.value());
    CHECK(reserved(ResourceKind::ram) == 816U && fake.pinned.size() == 1U);
    // destroyed with a record in flight: every reservation and buffer goes back
    acc2.reset();
    CHECK(reserved(ResourceKind::vram) == 0U && reserved(ResourceKind::ram) == 0U && fake.pinned.empty());
    acc.reset();
    std::filesystem::remove(f.path);
}

}  // namespace

int main() {
    test_refusals();
    test_success_eviction_and_governor();
    test_governor_refusal_is_a_decline();
    test_expert_pack_records();
    if (failures) {
        std::fprintf(stderr, "%d failures\n", failures);
        return 1;
    }
    std::printf("accelerator host tests passed\n");
    return 0;
}
