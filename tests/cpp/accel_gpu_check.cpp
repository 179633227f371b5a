// GPU check of B200MatvecAccelerator with the real vlb200 library: the reference's
// DeepseekV4PackedMatrix descriptors go through accelerator->matvec exactly as
// linear_packed_matrix offers them (deepseek_v4_graph.cpp:832-844), and the results are compared
// with the reference's own CPU kernel (matvec_ggml_f32_transactional) on the same bytes.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <filesystem>
#include <fstream>
#include <random>
#include <vector>

#include "b200_matvec_accelerator.hpp"
#include "vastloom/inference/ggml_quantization.hpp"

int main() {
    vastloom::safety::ResourceLimits limits;
    limits.ram_hard_limit = 1ULL << 30;
    limits.vram_hard_limit = 8ULL << 30;
    limits.staging_hard_limit = 64ULL << 20;  // one whole expert record is one read
    limits.scratch_hard_limit = 1ULL << 20;
    limits.minimum_system_ram_available = 0;
    limits.minimum_storage_available = 0;
    vastloom::safety::ResourceGovernor governor(limits);
    vastloom::b200::B200MatvecAcceleratorOptions options;
    options.minimum_free_vram_after = 0;
    int failures = 0;
    {
        auto created = vastloom::b200::B200MatvecAccelerator::create(governor, options);
        if (!created) {
            std::fprintf(stderr, "create failed: %s (%s)\n", created.error().message.c_str(),
                         created.error().context.c_str());
            return 2;
        }
        auto acc = created.take_value();
        std::mt19937_64 rng(42);
        struct Case { uint32_t type; size_t rows, cols, be, bb; };
        const Case cases[] = {{8, 256, 4096, 32, 34}, {16, 2048, 4096, 256, 66},
                              {18, 4096, 2048, 256, 98}, {19, 2048, 4096, 256, 50}};
        uint64_t identity = 1001;
        for (const auto& c : cases) {
            std::vector<std::byte> payload(c.rows * (c.cols / c.be) * c.bb);
            for (auto& b : payload) b = std::byte(static_cast<uint8_t>(rng()));
            for (size_t b = 0; b < payload.size(); b += c.bb) {  // finite fp16 scale ~ 0.01
                payload[b] = std::byte{0x1f};
                payload[b + 1] = std::byte{0x21};
            }
            vastloom::inference::DeepseekV4PackedMatrix m(c.type, c.rows, c.cols, c.cols, payload);
            m.cache_identity = identity += 2;
            std::vector<float> x(c.cols), y(c.rows, 0.f), want(c.rows), scratch(c.rows);
            std::normal_distribution<float> nd;
            for (auto& v : x) v = nd(rng);
            for (int pass = 0; pass < 2; ++pass) {
                auto r = acc->matvec(m, x, y);
                if (!r || !r.value()) {
                    std::fprintf(stderr, "type %u: matvec not served\n", c.type);
                    ++failures;
                    continue;
                }
            }
            auto ok = vastloom::inference::matvec_ggml_f32_transactional(c.type, payload, c.rows, c.cols, x,
                                                                         scratch, want);
            if (!ok) { ++failures; continue; }
            double num = 0, den = 0;
            for (size_t i = 0; i < c.rows; ++i) {
                num = std::max(num, std::fabs((double)y[i] - (double)want[i]));
                den = std::max(den, std::fabs((double)want[i]));
            }
            const double rel = num / den;
            std::printf("type %u %zux%zu rel_err %.3e resident %d\n", c.type, c.rows, c.cols, rel,
                        acc->holds(m.cache_identity) ? 1 : 0);
            if (!(rel <= 1e-5) || !acc->holds(m.cache_identity)) ++failures;
        }
        if (acc->stats().accelerated != 8 || acc->stats().resident_matrices != 4) ++failures;
        if (acc->reserved_bytes() == 0) ++failures;

        // Expert-pack records through the residency tier: a config-1 expert (IQ2_XXS W1 / W3
        // 2048 x 4096, W2 4096 x 2048) per record, read from a payload file, moved in one copy,
        // then offered through the seam like any expert matrix.
        const auto path = std::filesystem::temp_directory_path() / "vlb_accel_gpu_pack.bin";
        vastloom::inference::DeepseekV4ExpertPack pack;
        pack.payload_path = path;
        pack.layer = 7U;
        const size_t tensor_bytes = 2048ULL * 16ULL * 66ULL;
        std::vector<std::byte> file_bytes;
        const uint32_t n_records = 4;
        for (uint32_t e = 0; e < n_records; ++e) {
            vastloom::inference::DeepseekV4ExpertPackRecord record;
            record.expert = e;
            record.offset = file_bytes.size();
            record.bytes = 3 * tensor_bytes;
            for (uint32_t j = 0; j < 3; ++j) {
                vastloom::inference::DeepseekV4ExpertPackTensor t;
                t.name = "w" + std::to_string(j);
                t.packed_offset = j * tensor_bytes;
                t.bytes = tensor_bytes;
                t.ggml_type = 16U;
                t.shape = j < 2 ? std::vector<uint64_t>{4096U, 2048U} : std::vector<uint64_t>{2048U, 4096U};
                record.tensors.push_back(t);
            }
            const size_t at = file_bytes.size();
            file_bytes.resize(at + (record.bytes + 4095) / 4096 * 4096);
            for (size_t i = 0; i < record.bytes; ++i) file_bytes[at + i] = std::byte(static_cast<uint8_t>(rng()));
            for (size_t b = 0; b < record.bytes; b += 66) {
                file_bytes[at + b] = std::byte{0x1f};
                file_bytes[at + b + 1] = std::byte{0x21};
            }
            pack.records.push_back(record);
        }
        std::ofstream(path, std::ios::binary).write(reinterpret_cast<const char*>(file_bytes.data()),
                                                    static_cast<std::streamsize>(file_bytes.size()));
        const auto t0 = std::chrono::steady_clock::now();
        for (const auto& record : pack.records) {
            std::vector<uint64_t> ids;
            for (uint64_t j = 0; j < 3; ++j)
                ids.push_back(vastloom::b200::B200MatvecAccelerator::expert_matrix_identity(7U, record.expert, j));
            auto begun = acc->begin_expert_pack_record(pack, record, ids);
            if (!begun || !begun.value()) {
                std::fprintf(stderr, "record %u not started: %s\n", record.expert,
                             begun ? "declined" : begun.error().message.c_str());
                ++failures;
            }
        }
        auto finished = acc->finish_expert_pack_records();
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        if (!finished || finished.value() != n_records) ++failures;
        std::printf("records: %u x %.2f MB in %.2f ms (read %.2f ms, waited %.2f ms): %.2f GB/s\n", n_records,
                    3.0 * tensor_bytes / 1e6, ms, acc->stats().record_read_ms, acc->stats().record_wait_ms,
                    n_records * 3.0 * tensor_bytes / ms / 1e6);
        for (const auto& record : pack.records) {
            auto snap = acc->expert_record_residency(7U, record.expert);
            if (!snap || snap.value().state != vastloom::model::ResidencyState::vram_ready) ++failures;
            for (uint32_t j = 0; j < 3; ++j) {
                const size_t rows = j < 2 ? 2048 : 4096, cols = j < 2 ? 4096 : 2048;
                const auto* src = file_bytes.data() + record.offset + j * tensor_bytes;
                std::vector<std::byte> payload(src, src + tensor_bytes);
                vastloom::inference::DeepseekV4PackedMatrix m(16U, rows, cols, cols, payload);
                m.cache_identity = vastloom::b200::B200MatvecAccelerator::expert_matrix_identity(7U, record.expert, j);
                if (!acc->holds(m.cache_identity)) ++failures;
                std::vector<float> x(cols), y(rows), want(rows), scratch(rows);
                std::normal_distribution<float> nd;
                for (auto& v : x) v = nd(rng);
                const size_t before = acc->stats().uploaded_bytes;
                auto r = acc->matvec(m, x, y);
                if (!r || !r.value() || acc->stats().uploaded_bytes != before) ++failures;  // served, not re-uploaded
                if (!vastloom::inference::matvec_ggml_f32_transactional(16U, payload, rows, cols, x, scratch, want)) {
                    ++failures;
                    continue;
                }
                double num = 0, den = 0;
                for (size_t i = 0; i < rows; ++i) {
                    num = std::max(num, std::fabs((double)y[i] - (double)want[i]));
                    den = std::max(den, std::fabs((double)want[i]));
                }
                if (!(num / den <= 1e-5)) {
                    std::fprintf(stderr, "record %u tensor %u rel_err %.3e\n", record.expert, j, num / den);
                    ++failures;
                }
            }
        }
        std::printf("records resident: %zu matrices, %llu bytes\n", acc->stats().resident_matrices,
                    (unsigned long long)acc->stats().resident_bytes);
        std::filesystem::remove(path);
    }
    const auto vram = governor.snapshot().reserved[1];
    std::printf("vram reserved after close: %llu\n", (unsigned long long)vram);
    if (vram != 0) ++failures;
    std::printf(failures ? "FAILED\n" : "accelerator gpu check passed\n");
    return failures ? 1 : 0;
}
