// GPU check of B200MatvecAccelerator with the real vlb200 library: the reference's
// DeepseekV4PackedMatrix descriptors go through accelerator->matvec exactly as
// linear_packed_matrix offers them (deepseek_v4_graph.cpp:832-844), and the results are compared
// with the reference's own CPU kernel (matvec_ggml_f32_transactional) on the same bytes.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

#include "b200_matvec_accelerator.hpp"
#include "vastloom/inference/ggml_quantization.hpp"

int main() {
    vastloom::safety::ResourceLimits limits;
    limits.ram_hard_limit = 1ULL << 30;
    limits.vram_hard_limit = 8ULL << 30;
    limits.staging_hard_limit = 1ULL << 20;
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
    }
    const auto vram = governor.snapshot().reserved[1];
    std::printf("vram reserved after close: %llu\n", (unsigned long long)vram);
    if (vram != 0) ++failures;
    std::printf(failures ? "FAILED\n" : "accelerator gpu check passed\n");
    return failures ? 1 : 0;
}
