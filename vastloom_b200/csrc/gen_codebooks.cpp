// Build-time tool: writes the IQ codebooks a caller hands to vlb_set_codebook into one data file.
//
// The library itself carries no codebook; in the reference runtime the caller passes
// iq1_s_grid_table() / iq2_xxs_grid_table() / iq3_xxs_grid_table() / iq2_s_grid_table()
// (ggml_quantization.hpp:73-81).
// For this package's own callers (tests, bench) the same tables are read at build time from the
// reference tree's data files (src/inference/iq*_grid.inc, ggml commit 30bf8685, MIT) and stored
// in vastloom_b200/data/iq_grids.bin, which is a build artefact, not a source file. The output
// records each table's FNV-1a fingerprint; the ABI checks it against the pinned values again.
//
// Usage: gen_codebooks <out.bin>   (compiled with -I <reference>/src/inference)
#include <cstdint>
#include <cstdio>
#include <cstring>

static const uint64_t kIq1S[2048] = {
#include "iq1s_grid.inc"
};
static const uint64_t kIq2Xxs[256] = {
#include "iq2xxs_grid.inc"
};
static const uint32_t kIq3Xxs[256] = {
#include "iq3xxs_grid.inc"
};
static const uint64_t kIq2S[1024] = {
#include "iq2s_grid.inc"
};

static uint64_t fnv1a(const void* p, size_t n) {
    const unsigned char* b = static_cast<const unsigned char*>(p);
    uint64_t h = 14695981039346656037ull;
    for (size_t i = 0; i < n; ++i) {
        h ^= b[i];
        h *= 1099511628211ull;
    }
    return h;
}

static int put(FILE* f, uint32_t type, const void* data, uint32_t bytes) {
    const uint64_t fp = fnv1a(data, bytes);
    return fwrite(&type, 4, 1, f) == 1 && fwrite(&bytes, 4, 1, f) == 1 &&
                   fwrite(&fp, 8, 1, f) == 1 && fwrite(data, 1, bytes, f) == bytes
               ? 0
               : 1;
}

int main(int argc, char** argv) {
    if (argc != 2) {
        std::fprintf(stderr, "usage: gen_codebooks <out.bin>\n");
        return 2;
    }
    FILE* f = std::fopen(argv[1], "wb");
    if (!f) return 1;
    const char magic[8] = {'V', 'L', 'B', 'G', 'R', 'I', 'D', '1'};
    const uint32_t count = 4;
    int bad = fwrite(magic, 1, 8, f) != 8 || fwrite(&count, 4, 1, f) != 1;
    bad |= put(f, 19u, kIq1S, sizeof(kIq1S));
    bad |= put(f, 16u, kIq2Xxs, sizeof(kIq2Xxs));
    bad |= put(f, 18u, kIq3Xxs, sizeof(kIq3Xxs));
    bad |= put(f, 22u, kIq2S, sizeof(kIq2S));
    bad |= std::fclose(f) != 0;
    return bad;
}
