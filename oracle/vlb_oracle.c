/*
 * TEST INFRASTRUCTURE ONLY - CPU restatement of the vastloom reference arithmetic for the MoE
 * routed-expert path (see vlb_oracle.h). Built with -O2 -ffp-contract=off so that every float
 * operation rounds exactly where the reference's does (the reference is built for x86-64 without
 * FMA, so it never contracts a multiply into an add).
 *
 * Citations are vastloom source paths (file:line).
 */
#include "vlb_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ggml_quantization.hpp:12-31 */
int vlo_block_layout(uint32_t type, size_t* block_elems, size_t* block_bytes) {
    switch (type) {
        case VLO_TYPE_F32: *block_elems = 1; *block_bytes = 4; return 0;
        case VLO_TYPE_Q8_0: *block_elems = 32; *block_bytes = 34; return 0;
        case VLO_TYPE_IQ2_XXS: *block_elems = 256; *block_bytes = 66; return 0;
        case VLO_TYPE_IQ3_XXS: *block_elems = 256; *block_bytes = 98; return 0;
        case VLO_TYPE_IQ1_S: *block_elems = 256; *block_bytes = 50; return 0;
        case VLO_TYPE_Q4_K: *block_elems = 256; *block_bytes = 144; return 0;
        case VLO_TYPE_Q5_K: *block_elems = 256; *block_bytes = 176; return 0;
        case VLO_TYPE_Q6_K: *block_elems = 256; *block_bytes = 210; return 0;
        case VLO_TYPE_IQ2_S: *block_elems = 256; *block_bytes = 82; return 0;
        case VLO_TYPE_MXFP4: *block_elems = 32; *block_bytes = 17; return 0;
        default: return -1;
    }
}

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* fp16_to_float, ggml_quantization.cpp:101-124: IEEE half with subnormals normalised by hand. */
float vlo_fp16_to_float(uint16_t value) {
    uint32_t sign = (uint32_t)(value & 0x8000u) << 16;
    uint32_t exponent = (value >> 10) & 0x1fu;
    uint32_t mantissa = value & 0x03ffu;
    uint32_t bits = sign;
    if (exponent == 0u) {
        if (mantissa != 0u) {
            exponent = 113u;
            while ((mantissa & 0x0400u) == 0u) { mantissa <<= 1; --exponent; }
            mantissa &= 0x03ffu;
            bits |= exponent << 23;
            bits |= mantissa << 13;
        }
    } else if (exponent == 0x1fu) {
        bits |= 0x7f800000u | (mantissa << 13);
    } else {
        bits |= (exponent + 112u) << 23;
        bits |= mantissa << 13;
    }
    return u2f(bits);
}

/* float_to_fp16, ggml_quantization.cpp:126-145: round-to-nearest-even through the
 * scale-to-infinity / scale-to-zero construction. */
uint16_t vlo_float_to_fp16(float value) {
    const float scale_to_infinity = 0x1.0p+112f;
    const float scale_to_zero = 0x1.0p-110f;
    float base = (fabsf(value) * scale_to_infinity) * scale_to_zero;
    const uint32_t word = f2u(value);
    const uint32_t shifted = word + word;
    const uint32_t sign = word & 0x80000000u;
    uint32_t bias = shifted & 0xff000000u;
    if (bias < 0x71000000u) bias = 0x71000000u;
    base = u2f((bias >> 1) + 0x07800000u) + base;
    const uint32_t bits = f2u(base);
    const uint32_t exponent = (bits >> 13) & 0x00007c00u;
    const uint32_t mantissa = bits & 0x00000fffu;
    const uint32_t non_sign = exponent + mantissa;
    return (uint16_t)((sign >> 16) | (shifted > 0xff000000u ? 0x7e00u : non_sign));
}

uint64_t vlo_fnv1a_bytes(const void* v, size_t n) {
    const uint8_t* p = (const uint8_t*)v;
    uint64_t h = 14695981039346656037ull;
    for (size_t i = 0; i < n; ++i) { h ^= p[i]; h *= 1099511628211ull; }
    return h;
}

/* The float fingerprint of tests/test_main.cpp:1332-1339: FNV-1a over each value's bits, low
 * byte first. On a little-endian host that is the byte FNV of the array. */
uint64_t vlo_fnv1a_f32(const float* v, size_t n) {
    uint64_t h = 14695981039346656037ull;
    for (size_t i = 0; i < n; ++i) {
        uint32_t bits = f2u(v[i]);
        for (unsigned s = 0; s < 32; s += 8) { h ^= (bits >> s) & 0xffu; h *= 1099511628211ull; }
    }
    return h;
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static uint32_t rd32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static int parity7(uint32_t v) { return __builtin_popcount(v) & 1; }

/* decode_q8_0_block, ggml_quantization.cpp:419-435: w = d * float(int8 q) */
static int decode_q8_0(const uint8_t* b, float* out) {
    const float d = vlo_fp16_to_float(rd16(b));
    if (!isfinite(d)) return -1;
    for (int i = 0; i < 32; ++i) out[i] = d * (float)(int8_t)b[2 + i];
    return 0;
}

/* decode_iq2_xxs_block, ggml_quantization.cpp:250-283 */
static int decode_iq2_xxs(const uint8_t* b, const uint64_t* grid, float* out) {
    const float d = vlo_fp16_to_float(rd16(b));
    if (!isfinite(d)) return -1;
    const uint8_t* q = b + 2;
    for (int g = 0; g < 8; ++g) {
        const uint8_t* packed = q + g * 8;
        const uint32_t aux = rd32(packed + 4);
        const float ls = d * (0.5f + (float)(aux >> 28)) * 0.25f;
        for (int j = 0; j < 4; ++j) {
            const uint64_t gv = grid[packed[j]];
            const uint32_t si = (aux >> (7 * j)) & 127u;
            const uint32_t signs = si | ((uint32_t)parity7(si) << 7);
            for (int l = 0; l < 8; ++l) {
                const uint8_t m = (uint8_t)((gv >> (8 * l)) & 0xffu);
                const float s = (signs & (1u << l)) ? -1.0f : 1.0f;
                out[g * 32 + j * 8 + l] = ls * (float)m * s;
            }
        }
    }
    return 0;
}

/* decode_iq3_xxs_block, ggml_quantization.cpp:336-379 */
static int decode_iq3_xxs(const uint8_t* b, const uint32_t* grid, float* out) {
    const float d = vlo_fp16_to_float(rd16(b));
    if (!isfinite(d)) return -1;
    const uint8_t* q = b + 2;
    const uint8_t* ss = q + 64;
    for (int g = 0; g < 8; ++g) {
        const uint32_t aux = rd32(ss + g * 4);
        const float ls = d * (0.5f + (float)(aux >> 28)) * 0.5f;
        for (int j = 0; j < 4; ++j) {
            const uint32_t si = (aux >> (7 * j)) & 127u;
            const uint32_t signs = si | ((uint32_t)parity7(si) << 7);
            const uint32_t g1 = grid[q[g * 8 + j * 2]];
            const uint32_t g2 = grid[q[g * 8 + j * 2 + 1]];
            for (int l = 0; l < 4; ++l) {
                const float s1 = (signs & (1u << l)) ? -1.0f : 1.0f;
                const float s2 = (signs & (1u << (l + 4))) ? -1.0f : 1.0f;
                const uint8_t m1 = (uint8_t)((g1 >> (8 * l)) & 0xffu);
                const uint8_t m2 = (uint8_t)((g2 >> (8 * l)) & 0xffu);
                out[g * 32 + j * 8 + l] = ls * (float)m1 * s1;
                out[g * 32 + j * 8 + l + 4] = ls * (float)m2 * s2;
            }
        }
    }
    return 0;
}

/* decode_iq1_s_block, ggml_quantization.cpp:217-248 */
static int decode_iq1_s(const uint8_t* b, const uint64_t* grid, float* out) {
    const float d = vlo_fp16_to_float(rd16(b));
    if (!isfinite(d)) return -1;
    const uint8_t* qs = b + 2;
    const uint8_t* qh = b + 34;
    for (int g = 0; g < 8; ++g) {
        const uint16_t h = rd16(qh + g * 2);
        const float ls = d * (float)(2u * ((h >> 12) & 7u) + 1u);
        const float delta = (h & 0x8000u) ? -0.125f : 0.125f;
        for (int j = 0; j < 4; ++j) {
            const uint32_t idx = (uint32_t)qs[g * 4 + j] | ((uint32_t)((h >> (3 * j)) & 7u) << 8);
            const uint64_t gv = grid[idx];
            for (int l = 0; l < 8; ++l) {
                const int8_t v = (int8_t)((gv >> (8 * l)) & 0xffu);
                out[g * 32 + j * 8 + l] = ls * ((float)v + delta);
            }
        }
    }
    return 0;
}

/* qk_scale_min, ggml_quantization.cpp:437-455: the 6-bit scale and minimum of sub-block j of a
 * Q4_K / Q5_K block from its 12 packed bytes (j < 4: low six bits of bytes j and j + 4; else four
 * bits of byte j + 4 and the top two bits of bytes j - 4 and j). */
static void qk_scale_min(uint32_t j, const uint8_t* s, uint32_t* sc, uint32_t* mn) {
    if (j < 4) {
        *sc = s[j] & 63u;
        *mn = s[j + 4] & 63u;
    } else {
        *sc = (s[j + 4] & 15u) | ((uint32_t)(s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
    }
}

/* decode_q4_k_block, ggml_quantization.cpp:457-493: d, dmin, 12 scale bytes, 128 nibble bytes; the
 * 32 bytes of pair p hold sub-block 2p in their low nibbles and 2p + 1 in their high nibbles;
 * w = d * sc - dmin * m rounded as (d * sc) * q - (dmin * m). */
static int decode_q4_k(const uint8_t* b, float* out) {
    const float d = vlo_fp16_to_float(rd16(b)), dmin = vlo_fp16_to_float(rd16(b + 2));
    if (!isfinite(d) || !isfinite(dmin)) return -1;
    const uint8_t* q = b + 16;
    for (uint32_t p = 0; p < 4; ++p) {
        uint32_t s1, m1, s2, m2;
        qk_scale_min(2 * p, b + 4, &s1, &m1);
        qk_scale_min(2 * p + 1, b + 4, &s2, &m2);
        const float d1 = d * (float)s1, n1 = dmin * (float)m1, d2 = d * (float)s2, n2 = dmin * (float)m2;
        for (uint32_t l = 0; l < 32; ++l) {
            out[64 * p + l] = d1 * (float)(q[32 * p + l] & 15u) - n1;
            out[64 * p + 32 + l] = d2 * (float)(q[32 * p + l] >> 4) - n2;
        }
    }
    return 0;
}

/* decode_q5_k_block, ggml_quantization.cpp:495-539: as Q4_K with a fifth bit per weight from the 32
 * qh bytes: sub-block 2p takes bit 2p of qh[l], sub-block 2p + 1 bit 2p + 1. */
static int decode_q5_k(const uint8_t* b, float* out) {
    const float d = vlo_fp16_to_float(rd16(b)), dmin = vlo_fp16_to_float(rd16(b + 2));
    if (!isfinite(d) || !isfinite(dmin)) return -1;
    const uint8_t* qh = b + 16;
    const uint8_t* q = b + 48;
    for (uint32_t p = 0; p < 4; ++p) {
        uint32_t s1, m1, s2, m2;
        qk_scale_min(2 * p, b + 4, &s1, &m1);
        qk_scale_min(2 * p + 1, b + 4, &s2, &m2);
        const float d1 = d * (float)s1, n1 = dmin * (float)m1, d2 = d * (float)s2, n2 = dmin * (float)m2;
        for (uint32_t l = 0; l < 32; ++l) {
            const uint32_t v1 = (q[32 * p + l] & 15u) + ((qh[l] >> (2 * p)) & 1u ? 16u : 0u);
            const uint32_t v2 = (q[32 * p + l] >> 4) + ((qh[l] >> (2 * p + 1)) & 1u ? 16u : 0u);
            out[64 * p + l] = d1 * (float)v1 - n1;
            out[64 * p + 32 + l] = d2 * (float)v2 - n2;
        }
    }
    return 0;
}

/* decode_q6_k_block, ggml_quantization.cpp:541-590: 128 low-nibble bytes, 64 high-bit bytes, 16
 * int8 scales, then the fp16 d (last). Per half h of 128 weights and l < 32, the four weights
 * h*128 + 32 i + l take nibble (i / 2) of low byte 64 h + 32 (i % 2) + l and bits 2 i of high byte
 * 32 h + l, minus 32; w = (d * scale[8 h + l / 16 + 2 i]) * q. */
static int decode_q6_k(const uint8_t* b, float* out) {
    const float d = vlo_fp16_to_float(rd16(b + 208));
    if (!isfinite(d)) return -1;
    for (uint32_t h = 0; h < 2; ++h) {
        const uint8_t* lo = b + 64 * h;
        const uint8_t* hi = b + 128 + 32 * h;
        const int8_t* sc = (const int8_t*)(b + 192 + 8 * h);
        for (uint32_t l = 0; l < 32; ++l) {
            for (uint32_t i = 0; i < 4; ++i) {
                const uint32_t byte = lo[32 * (i & 1) + l];
                const int q = (int)((i < 2 ? byte & 15u : byte >> 4) | (((hi[l] >> (2 * i)) & 3u) << 4)) - 32;
                out[128 * h + 32 * i + l] = d * (float)sc[l / 16 + 2 * i] * (float)q;
            }
        }
    }
    return 0;
}

/* decode_iq2_s_block, ggml_quantization.cpp:285-334: d, 32 grid-index bytes, 32 sign bytes, 8 qh
 * bytes (two high index bits per sub-block), 8 scale bytes (low nibble for sub-blocks 0-1 of the
 * group, high nibble for 2-3); w = ((d * (0.5 + s)) * 0.25) * m, negated where the sign bit is set. */
static int decode_iq2_s(const uint8_t* b, const uint64_t* grid, float* out) {
    const float d = vlo_fp16_to_float(rd16(b));
    if (!isfinite(d)) return -1;
    const uint8_t* qs = b + 2;
    const uint8_t* signs = b + 34;
    const uint8_t* qh = b + 66;
    const uint8_t* scales = b + 74;
    for (uint32_t g = 0; g < 8; ++g) {
        const float lo = d * (0.5f + (float)(scales[g] & 15u)) * 0.25f;
        const float hi = d * (0.5f + (float)(scales[g] >> 4)) * 0.25f;
        for (uint32_t s = 0; s < 4; ++s) {
            const float ls = s < 2 ? lo : hi;
            const uint32_t idx = qs[4 * g + s] | (((uint32_t)qh[g] << (8 - 2 * s)) & 0x300u);
            const uint64_t gv = grid[idx];
            const uint32_t sg = signs[4 * g + s];
            for (uint32_t l = 0; l < 8; ++l) {
                const float m = ls * (float)((gv >> (8 * l)) & 0xffu);
                out[32 * g + 8 * s + l] = (sg >> l) & 1u ? -m : m;
            }
        }
    }
    return 0;
}

/* e8m0_to_float_half, ggml_quantization.cpp:112-120, and decode_mxfp4_block :381-398: half the
 * power of two of the E8M0 byte (bytes 0 and 1: the two smallest half-scaled powers) times the
 * doubled E2M1 value of each nibble; byte i holds weight i (low nibble) and i + 16 (high). */
static const int8_t kMxfp4[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
static int decode_mxfp4(const uint8_t* b, float* out) {
    const uint32_t e = b[0];
    const float scale = u2f(e < 2 ? 0x00200000u << e : (e - 1u) << 23);
    for (uint32_t i = 0; i < 16; ++i) {
        const float lo = (float)kMxfp4[b[1 + i] & 15u] * scale, hi = (float)kMxfp4[b[1 + i] >> 4] * scale;
        if (!isfinite(lo) || !isfinite(hi)) return -1;
        out[i] = lo;
        out[i + 16] = hi;
    }
    return 0;
}

static int decode_block(uint32_t type, const uint8_t* b, const void* grid, float* out) {
    switch (type) {
        case VLO_TYPE_Q8_0: return decode_q8_0(b, out);
        case VLO_TYPE_IQ2_XXS: return decode_iq2_xxs(b, (const uint64_t*)grid, out);
        case VLO_TYPE_IQ3_XXS: return decode_iq3_xxs(b, (const uint32_t*)grid, out);
        case VLO_TYPE_IQ1_S: return decode_iq1_s(b, (const uint64_t*)grid, out);
        case VLO_TYPE_Q4_K: return decode_q4_k(b, out);
        case VLO_TYPE_Q5_K: return decode_q5_k(b, out);
        case VLO_TYPE_Q6_K: return decode_q6_k(b, out);
        case VLO_TYPE_IQ2_S: return decode_iq2_s(b, (const uint64_t*)grid, out);
        case VLO_TYPE_MXFP4: return decode_mxfp4(b, out);
        case VLO_TYPE_F32: memcpy(out, b, 4); return isfinite(out[0]) ? 0 : -1;
        default: return -2;
    }
}

/* dequantize_blocked, ggml_quantization.cpp:600-628 */
int vlo_dequantize(uint32_t type, const uint8_t* enc, size_t n_blocks, const void* grid,
                   float* out) {
    size_t be, bb;
    if (vlo_block_layout(type, &be, &bb) != 0) return -2;
    for (size_t i = 0; i < n_blocks; ++i) {
        int st = decode_block(type, enc + i * bb, grid, out + i * be);
        if (st) return st;
    }
    return 0;
}

/* matvec_blocked, ggml_quantization.cpp:768-809 (and the serial twins matvec_iq1_s_f32 :1331,
 * matvec_iq3_xxs_f32 :1409): one double accumulator per row, columns in order, cast once. */
int vlo_matvec(uint32_t type, const uint8_t* enc, size_t rows, size_t cols, const float* x,
               float* y, const void* grid) {
    size_t be, bb;
    if (vlo_block_layout(type, &be, &bb) != 0 || cols % be) return -2;
    float dec[256];
    const size_t bpr = cols / be;
    for (size_t r = 0; r < rows; ++r) {
        double sum = 0.0;
        for (size_t b = 0; b < bpr; ++b) {
            int st = decode_block(type, enc + (r * bpr + b) * bb, grid, dec);
            if (st) return st;
            for (size_t c = 0; c < be; ++c) sum += (double)dec[c] * (double)x[b * be + c];
        }
        y[r] = (float)sum;
        if (!isfinite(y[r])) return -3;
    }
    return 0;
}

/* quantize_q8_0_reference, ggml_quantization.cpp:944-1004 */
int vlo_quantize_q8_0(const float* m, size_t rows, size_t lc, size_t sc, uint8_t* out) {
    if (lc == 0 || lc > sc || sc % 32) return -1;
    const size_t bpr = sc / 32;
    for (size_t r = 0; r < rows; ++r) {
        for (size_t b = 0; b < bpr; ++b) {
            float v[32];
            float maximum = 0.0f;
            for (size_t i = 0; i < 32; ++i) {
                const size_t c = b * 32 + i;
                const float val = c < lc ? m[r * lc + c] : 0.0f;
                if (!isfinite(val)) return -1;
                v[i] = val;
                maximum = fmaxf(maximum, fabsf(val));
            }
            const float scale = maximum / 127.0f;
            const float inverse = scale != 0.0f ? 1.0f / scale : 0.0f;
            uint8_t* o = out + (r * bpr + b) * 34;
            const uint16_t es = vlo_float_to_fp16(scale);
            if (!isfinite(vlo_fp16_to_float(es))) return -1;
            o[0] = (uint8_t)(es & 0xffu);
            o[1] = (uint8_t)(es >> 8);
            for (size_t i = 0; i < 32; ++i) {
                float rounded = roundf(v[i] * inverse);
                if (rounded < -127.0f) rounded = -127.0f;
                if (rounded > 127.0f) rounded = 127.0f;
                o[2 + i] = (uint8_t)(int8_t)rounded;
            }
        }
    }
    return 0;
}

/* sqrt_softplus, deepseek_v4_reference.cpp:65-69 */
float vlo_sqrt_softplus(float value) {
    const double p = (double)value;
    const double softplus = (p > 0.0 ? p : 0.0) + log1p(exp(-fabs(p)));
    return (float)sqrt(softplus);
}

/* sigmoid, deepseek_v4_reference.cpp:71-78 */
float vlo_sigmoid(float value) {
    const double p = (double)value;
    if (p >= 0.0) return (float)(1.0 / (1.0 + exp(-p)));
    const double e = exp(p);
    return (float)(e / (1.0 + e));
}

/* gate_logits, deepseek_v4_reference.cpp:123-160 (also linear, deepseek_v4_graph.cpp:735-767) */
void vlo_router_logits(const float* x, const float* w, size_t T, size_t H, size_t E,
                       float* logits) {
    for (size_t t = 0; t < T; ++t)
        for (size_t e = 0; e < E; ++e) {
            double sum = 0.0;
            for (size_t c = 0; c < H; ++c) sum += (double)x[t * H + c] * (double)w[e * H + c];
            logits[t * E + e] = (float)sum;
        }
}

/* Ordering used by every reference router: larger key first, ties to the lower expert id
 * (deepseek_v4_reference.cpp:240-244, olmoe_runtime.cpp:1128-1137). */
static void top_k_by_key(const float* key, size_t E, size_t k, uint32_t* out) {
    /* selection sort of the first k: identical result to std::partial_sort with a strict
     * total order (no NaN can reach here: inputs are finite). */
    unsigned char* used = (unsigned char*)calloc(E, 1);
    for (size_t s = 0; s < k; ++s) {
        size_t best = E;
        for (size_t e = 0; e < E; ++e) {
            if (used[e]) continue;
            if (best == E || key[e] > key[best]) best = e;
        }
        used[best] = 1;
        out[s] = (uint32_t)best;
    }
    free(used);
}

/* route_from_indices, deepseek_v4_reference.cpp:80-121: weights are the UNBIASED scores of the
 * chosen experts, normalised in double and multiplied by route_scale. */
static int route_from_indices(const float* scores, const uint32_t* idx, size_t t, size_t E,
                              size_t k, float route_scale, float* weights) {
    double sum = 0.0;
    for (size_t s = 0; s < k; ++s) {
        if (idx[t * k + s] >= E) return -1;
        const float v = scores[t * E + idx[t * k + s]];
        weights[t * k + s] = v;
        sum += (double)v;
    }
    if (!isfinite(sum) || sum <= 0.0) return -1;
    for (size_t s = 0; s < k; ++s)
        weights[t * k + s] = (float)((double)weights[t * k + s] / sum * (double)route_scale);
    return 0;
}

static void score_logits(const float* logits, size_t n, int score, float* out) {
    for (size_t i = 0; i < n; ++i)
        out[i] = score == VLO_SCORE_SIGMOID ? vlo_sigmoid(logits[i]) : vlo_sqrt_softplus(logits[i]);
}

/* deepseek_v4_route_learned_logits, deepseek_v4_reference.cpp:223-255 */
int vlo_route_learned(const float* logits, const float* bias, size_t T, size_t E, size_t k,
                      float route_scale, int score, uint32_t* idx, float* weights) {
    if (k == 0 || k > E || !(route_scale > 0.0f)) return -1;
    float* scores = (float*)malloc(T * E * sizeof(float));
    float* key = (float*)malloc(E * sizeof(float));
    score_logits(logits, T * E, score, scores);
    int st = 0;
    for (size_t t = 0; t < T && !st; ++t) {
        for (size_t e = 0; e < E; ++e) key[e] = scores[t * E + e] + bias[e];
        top_k_by_key(key, E, k, idx + t * k);
        st = route_from_indices(scores, idx, t, E, k, route_scale, weights);
    }
    free(scores);
    free(key);
    return st;
}

/* deepseek_v4_route_hash_logits, deepseek_v4_reference.cpp:275-307 */
int vlo_route_hash(const float* logits, const uint32_t* token_ids, const uint32_t* table,
                   size_t T, size_t V, size_t E, size_t k, float route_scale, int score,
                   uint32_t* idx, float* weights) {
    if (k == 0 || k > E || !(route_scale > 0.0f)) return -1;
    float* scores = (float*)malloc(T * E * sizeof(float));
    score_logits(logits, T * E, score, scores);
    int st = 0;
    for (size_t t = 0; t < T && !st; ++t) {
        if (token_ids[t] >= V) { st = -1; break; }
        for (size_t s = 0; s < k; ++s) idx[t * k + s] = table[(size_t)token_ids[t] * k + s];
        st = route_from_indices(scores, idx, t, E, k, route_scale, weights);
    }
    free(scores);
    return st;
}

/* OLMoE router, olmoe_runtime.cpp:1120-1137: float exp of (logit - max), double denominator,
 * float division, top-k by probability, no renormalisation. */
int vlo_route_softmax(const float* logits, size_t T, size_t E, size_t k, uint32_t* idx,
                      float* weights) {
    if (k == 0 || k > E) return -1;
    float* p = (float*)malloc(E * sizeof(float));
    for (size_t t = 0; t < T; ++t) {
        const float* l = logits + t * E;
        float mx = l[0];
        for (size_t e = 1; e < E; ++e) if (l[e] > mx) mx = l[e];
        double den = 0.0;
        for (size_t e = 0; e < E; ++e) { p[e] = expf(l[e] - mx); den += (double)p[e]; }
        for (size_t e = 0; e < E; ++e) p[e] /= (float)den;
        top_k_by_key(p, E, k, idx + t * k);
        for (size_t s = 0; s < k; ++s) weights[t * k + s] = p[idx[t * k + s]];
    }
    free(p);
    return 0;
}

/* Qwen router, qwen38_moe_route (qwen3_8_flash_next_reference.cpp:1186-1239) on given logits:
 * probs = exp(double(l) - max) in double, summed in expert order, prob = probs * (1 / sum); all
 * experts ranked by prob (larger first, ties to the lower id); weights = f32(prob), and with
 * norm_topk_prob each weight becomes f32(double(weight) * (1 / top_sum)) where top_sum adds the
 * selected probs in rank order. */
int vlo_route_softmax_f64(const float* logits, size_t T, size_t E, size_t k, int norm,
                          uint32_t* idx, float* weights) {
    if (k == 0 || k > E) return -1;
    double* p = (double*)malloc(E * sizeof(double));
    unsigned char* used = (unsigned char*)malloc(E);
    for (size_t t = 0; t < T; ++t) {
        const float* l = logits + t * E;
        double mx = (double)l[0];
        for (size_t e = 0; e < E; ++e) if ((double)l[e] > mx) mx = (double)l[e];
        double sum = 0.0;
        for (size_t e = 0; e < E; ++e) { p[e] = exp((double)l[e] - mx); sum += p[e]; }
        const double inv = sum > 0.0 ? 1.0 / sum : 0.0;
        for (size_t e = 0; e < E; ++e) p[e] = p[e] * inv;
        memset(used, 0, E);
        double top = 0.0;
        for (size_t s = 0; s < k; ++s) {
            size_t best = E;
            for (size_t e = 0; e < E; ++e) {
                if (used[e]) continue;
                if (best == E || p[e] > p[best]) best = e;
            }
            used[best] = 1;
            idx[t * k + s] = (uint32_t)best;
            weights[t * k + s] = (float)p[best];
            top += p[best];
        }
        if (norm && top > 0.0) {
            const double sc = 1.0 / top;
            for (size_t s = 0; s < k; ++s)
                weights[t * k + s] = (float)((double)weights[t * k + s] * sc);
        }
    }
    free(p);
    free(used);
    return 0;
}

/* The dispatch permutation. The reference visits experts in ascending id, then tokens, then
 * slots (deepseek_v4_graph.cpp:2134-2223); this is that visit order written out as a stable
 * counting sort. */
void vlo_dispatch(const uint32_t* idx, size_t T, size_t k, size_t E, uint32_t* offsets,
                  uint32_t* pair_token, uint32_t* pair_slot) {
    memset(offsets, 0, (E + 1) * sizeof(uint32_t));
    for (size_t i = 0; i < T * k; ++i) offsets[idx[i] + 1]++;
    for (size_t e = 0; e < E; ++e) offsets[e + 1] += offsets[e];
    uint32_t* cursor = (uint32_t*)malloc(E * sizeof(uint32_t));
    memcpy(cursor, offsets, E * sizeof(uint32_t));
    for (size_t t = 0; t < T; ++t)
        for (size_t s = 0; s < k; ++s) {
            const uint32_t e = idx[t * k + s];
            pair_token[cursor[e]] = (uint32_t)t;
            pair_slot[cursor[e]] = (uint32_t)s;
            cursor[e]++;
        }
    free(cursor);
}

/* deepseek_v4_rms_norm, deepseek_v4_reference.cpp:170-206 */
int vlo_rms_norm(const float* x, const float* w, size_t rows, size_t width, float eps,
                 float* out) {
    for (size_t r = 0; r < rows; ++r) {
        double sq = 0.0;
        for (size_t c = 0; c < width; ++c) { const double v = x[r * width + c]; sq += v * v; }
        const double inv = 1.0 / sqrt(sq / (double)width + (double)eps);
        for (size_t c = 0; c < width; ++c)
            out[r * width + c] = (float)((double)x[r * width + c] * inv * (double)w[c]);
    }
    return 0;
}

/* deepseek_v4_hc_split_sinkhorn, deepseek_v4_reference.cpp:387-477. mixes [T x (2+m)m]: per token
 * the m pre logits, the m post logits, then the m x m combination logits (row-major,
 * [source][destination]). */
int vlo_hc_split_sinkhorn(const float* mixes, const float* scale, const float* base, size_t T, size_t m,
                          size_t iters, float eps, float* pre, float* post, float* comb) {
    if (T == 0 || m == 0 || m > 16 || iters == 0) return -1;
    const size_t mw = (2 + m) * m;
    for (size_t t = 0; t < T; ++t) {
        const float* mx = mixes + t * mw;
        for (size_t i = 0; i < m; ++i) {
            pre[t * m + i] = vlo_sigmoid(mx[i] * scale[0] + base[i]) + eps;
            post[t * m + i] = 2.0f * vlo_sigmoid(mx[m + i] * scale[1] + base[m + i]);
        }
        float* c = comb + t * m * m;
        for (size_t r = 0; r < m; ++r) {  /* softmax over each row, plus eps */
            float mxv = -INFINITY;
            for (size_t j = 0; j < m; ++j) {
                const size_t at = 2 * m + r * m + j;
                c[r * m + j] = mx[at] * scale[2] + base[at];
                if (c[r * m + j] > mxv) mxv = c[r * m + j];
            }
            double sum = 0.0;
            for (size_t j = 0; j < m; ++j) {
                c[r * m + j] = (float)exp((double)(c[r * m + j] - mxv));
                sum += (double)c[r * m + j];
            }
            for (size_t j = 0; j < m; ++j) c[r * m + j] = (float)((double)c[r * m + j] / sum) + eps;
        }
        for (size_t it = 0; it < iters; ++it) {
            if (it > 0)
                for (size_t r = 0; r < m; ++r) {  /* rows */
                    double sum = 0.0;
                    for (size_t j = 0; j < m; ++j) sum += (double)c[r * m + j];
                    for (size_t j = 0; j < m; ++j) c[r * m + j] = (float)((double)c[r * m + j] / (sum + (double)eps));
                }
            for (size_t j = 0; j < m; ++j) {  /* columns */
                double sum = 0.0;
                for (size_t r = 0; r < m; ++r) sum += (double)c[r * m + j];
                for (size_t r = 0; r < m; ++r) c[r * m + j] = (float)((double)c[r * m + j] / (sum + (double)eps));
            }
        }
    }
    return 0;
}

/* deepseek_v4_hc_pre, deepseek_v4_reference.cpp:479-547 (the f32 mixing-weight form; the graph's
 * hc_pre, deepseek_v4_graph.cpp:2276-2295). x [T x m x W], fn [(2+m)m x mW]; reduced [T x W]. */
int vlo_hc_pre(const float* x, const float* fn, const float* scale, const float* base, size_t T, size_t m,
               size_t W, size_t iters, float norm_eps, float hc_eps, float* reduced, float* pre, float* post,
               float* comb) {
    if (T == 0 || m == 0 || m > 16 || W == 0) return -1;
    const size_t fw = m * W, mw = (2 + m) * m;
    float* mixes = (float*)malloc(T * mw * sizeof(float));
    if (!mixes) return -1;
    for (size_t t = 0; t < T; ++t) {
        const float* row = x + t * fw;
        double sq = 0.0;
        for (size_t c = 0; c < fw; ++c) { const double v = (double)row[c]; sq += v * v; }
        const double inv = 1.0 / sqrt(sq / (double)fw + (double)norm_eps);
        for (size_t r = 0; r < mw; ++r) {
            double sum = 0.0;
            for (size_t c = 0; c < fw; ++c) sum += (double)row[c] * (double)fn[r * fw + c];
            mixes[t * mw + r] = (float)(sum * inv);
        }
    }
    const int st = vlo_hc_split_sinkhorn(mixes, scale, base, T, m, iters, hc_eps, pre, post, comb);
    free(mixes);
    if (st) return st;
    for (size_t t = 0; t < T; ++t)
        for (size_t c = 0; c < W; ++c) {
            double sum = 0.0;
            for (size_t j = 0; j < m; ++j) sum += (double)pre[t * m + j] * (double)x[(t * m + j) * W + c];
            reduced[t * W + c] = (float)sum;
            if (!isfinite(reduced[t * W + c])) return -1;
        }
    return 0;
}

/* deepseek_v4_hc_post, deepseek_v4_reference.cpp:549-610: out[t, d] = post[d] * sub[t] +
 * sum over sources s of comb[s][d] * residual[t, s], in f64. */
int vlo_hc_post(const float* sub, const float* residual, const float* post, const float* comb, size_t T,
                size_t m, size_t W, float* out) {
    for (size_t t = 0; t < T; ++t)
        for (size_t d = 0; d < m; ++d)
            for (size_t c = 0; c < W; ++c) {
                double v = (double)post[t * m + d] * (double)sub[t * W + c];
                for (size_t s2 = 0; s2 < m; ++s2)
                    v += (double)comb[(t * m + s2) * m + d] * (double)residual[(t * m + s2) * W + c];
                out[(t * m + d) * W + c] = (float)v;
                if (!isfinite(out[(t * m + d) * W + c])) return -1;
            }
    return 0;
}

static const void* grid_for(const vlo_moe_layer* L, uint32_t type) {
    switch (type) {
        case VLO_TYPE_IQ1_S: return L->grid_iq1_s;
        case VLO_TYPE_IQ2_XXS: return L->grid_iq2_xxs;
        case VLO_TYPE_IQ3_XXS: return L->grid_iq3_xxs;
        case VLO_TYPE_IQ2_S: return L->grid_iq2_s;
        default: return NULL;
    }
}

static int mv(const vlo_moe_layer* L, const vlo_matrix* m, const float* x, float* y) {
    return vlo_matvec(m->type, m->data, m->rows, m->cols, x, y, grid_for(L, m->type));
}

/* The DeepSeek V4 SwiGLU of one gate/up pair, in double: with a positive limit L the gate is
 * clamped to min(g, L) and the up value to [-L, L]; silu(g) * u, times the route weight when one
 * is given. Shared by execute_expert (deepseek_v4_graph.cpp:1865-1890) and
 * deepseek_v4_expert_swiglu (deepseek_v4_reference.cpp:350-365), which differ only in where g and
 * u come from (f32 matvec outputs there, f64 sums here). */
static double v4_swiglu(double g, double u, float limit, const float* route_w) {
    if (limit > 0.0f) {
        if (g > (double)limit) g = (double)limit;
        if (u < -(double)limit) u = -(double)limit;
        if (u > (double)limit) u = (double)limit;
    }
    double v = g / (1.0 + exp(-g)) * u;
    if (route_w) v *= (double)*route_w;
    return v;
}

/* deepseek_v4_expert_swiglu, deepseek_v4_reference.cpp:309-385: float weights, gate and up kept in
 * double (column-order sums), clamp and SwiGLU in double, activation rounded to f32, down product
 * in double. routing_weights may be NULL. */
int vlo_expert_swiglu(const float* x, const float* gate_w, const float* down_w, const float* up_w,
                      const float* routing_weights, size_t T, size_t width, size_t inter,
                      float limit, float* out) {
    if (T == 0 || width == 0 || inter == 0 || !(limit >= 0.0f) || !isfinite(limit)) return -1;
    float* act = (float*)malloc(T * inter * sizeof(float));
    for (size_t t = 0; t < T; ++t)
        for (size_t r = 0; r < inter; ++r) {
            double g = 0.0, u = 0.0;
            for (size_t c = 0; c < width; ++c) {
                const double v = (double)x[t * width + c];
                g += v * (double)gate_w[r * width + c];
                u += v * (double)up_w[r * width + c];
            }
            act[t * inter + r] = (float)v4_swiglu(g, u, limit, routing_weights ? routing_weights + t : NULL);
        }
    for (size_t t = 0; t < T; ++t)
        for (size_t r = 0; r < width; ++r) {
            double sum = 0.0;
            for (size_t c = 0; c < inter; ++c)
                sum += (double)act[t * inter + c] * (double)down_w[r * inter + c];
            out[t * width + r] = (float)sum;
        }
    free(act);
    return 0;
}

/* execute_expert, deepseek_v4_graph.cpp:1826-1895, for one token: gate and up products, SwiGLU
 * in double with the optional clamp, route weight applied BEFORE the down product. */
static int v4_expert(const vlo_moe_layer* L, const vlo_matrix* w1, const vlo_matrix* w3,
                     const vlo_matrix* w2, const float* x, const float* route_w, float limit,
                     float* gate, float* up, float* act, float* out) {
    int st = mv(L, w1, x, gate);
    if (!st) st = mv(L, w3, x, up);
    if (st) return st;
    for (size_t c = 0; c < L->intermediate; ++c)
        act[c] = (float)v4_swiglu((double)gate[c], (double)up[c], limit, route_w);
    return mv(L, w2, act, out);
}

/* The activation row execute_expert hands to the down product (deepseek_v4_graph.cpp:1855-1890:
 * gate and up products, the optional clamp, SwiGLU in double, route weight when given), act f32[I]
 * for one token. Exposed so that tests can compare it with the down-projection input the
 * reference graph offers to its matvec accelerator. */
int vlo_v4_expert_activation(uint32_t type, const uint8_t* w1, const uint8_t* w3, size_t I, size_t H,
                             const float* x, const float* route_w, float limit, const void* grid,
                             float* act) {
    float* gate = (float*)malloc(I * sizeof(float));
    float* up = (float*)malloc(I * sizeof(float));
    int st = vlo_matvec(type, w1, I, H, x, gate, grid);
    if (!st) st = vlo_matvec(type, w3, I, H, x, up, grid);
    for (size_t c = 0; c < I && !st; ++c)
        act[c] = (float)v4_swiglu((double)gate[c], (double)up[c], limit, route_w);
    free(gate);
    free(up);
    return st;
}

/* OLMoE expert, olmoe_runtime.cpp:1276-1281: SwiGLU in float with expf. */
static int olmoe_expert(const vlo_moe_layer* L, const vlo_matrix* w1, const vlo_matrix* w3,
                        const vlo_matrix* w2, const float* x, float* gate, float* up,
                        float* act, float* out) {
    int st = mv(L, w1, x, gate);
    if (!st) st = mv(L, w3, x, up);
    if (st) return st;
    for (size_t c = 0; c < L->intermediate; ++c)
        act[c] = (gate[c] / (1.0f + expf(-gate[c]))) * up[c];
    return mv(L, w2, act, out);
}

/* moe_forward, deepseek_v4_graph.cpp:1902-2274 (DeepSeek V4: route, shared expert over all
 * tokens, routed experts in ascending id / token / slot order with float +=, shared added last),
 * and the OLMoE layer loop, olmoe_runtime.cpp:1119-1290 (rank-order combine, weight after down,
 * no shared expert). */
int vlo_moe_forward(const vlo_moe_layer* L, const float* x, const uint32_t* token_ids,
                    size_t T, const float* logits_in, float* out, uint32_t* idx,
                    float* weights) {
    const size_t H = L->hidden, I = L->intermediate, E = L->experts, k = L->top_k;
    float* logits = (float*)malloc(T * E * sizeof(float));
    float* gate = (float*)malloc(I * sizeof(float));
    float* up = (float*)malloc(I * sizeof(float));
    float* act = (float*)malloc(I * sizeof(float));
    float* eo = (float*)malloc(H * sizeof(float));
    int st = 0;
    if (logits_in) memcpy(logits, logits_in, T * E * sizeof(float));
    else vlo_router_logits(x, L->router, T, H, E, logits);
    if (L->score == VLO_SCORE_SOFTMAX) st = vlo_route_softmax(logits, T, E, k, idx, weights);
    else if (L->score == VLO_SCORE_SOFTMAX_F64 || L->score == VLO_SCORE_SOFTMAX_F64_NORM)
        st = vlo_route_softmax_f64(logits, T, E, k, L->score == VLO_SCORE_SOFTMAX_F64_NORM, idx, weights);
    else if (L->hash_routing)
        st = vlo_route_hash(logits, token_ids, L->tid2eid, T, L->vocab, E, k, L->route_scale,
                            L->score, idx, weights);
    else
        st = vlo_route_learned(logits, L->bias, T, E, k, L->route_scale, L->score, idx, weights);
    memset(out, 0, T * H * sizeof(float));
    if (!st && L->weight_after_down) {
        for (size_t t = 0; t < T && !st; ++t)
            for (size_t s = 0; s < k && !st; ++s) {
                const uint32_t e = idx[t * k + s];
                st = olmoe_expert(L, &L->w1[e], &L->w3[e], &L->w2[e], x + t * H, gate, up, act,
                                  eo);
                const float w = weights[t * k + s];
                for (size_t c = 0; c < H && !st; ++c) out[t * H + c] += w * eo[c];
            }
    } else if (!st) {
        float* shared = NULL;
        if (L->shared_w1) {
            shared = (float*)malloc(T * H * sizeof(float));
            for (size_t t = 0; t < T && !st; ++t)
                st = v4_expert(L, L->shared_w1, L->shared_w3, L->shared_w2, x + t * H, NULL,
                               L->shared_swiglu_limit, gate, up, act, shared + t * H);
        }
        for (size_t e = 0; e < E && !st; ++e)
            for (size_t t = 0; t < T && !st; ++t)
                for (size_t s = 0; s < k && !st; ++s) {
                    if (idx[t * k + s] != e) continue;
                    st = v4_expert(L, &L->w1[e], &L->w3[e], &L->w2[e], x + t * H,
                                   &weights[t * k + s], L->routed_swiglu_limit, gate, up, act, eo);
                    for (size_t c = 0; c < H && !st; ++c) out[t * H + c] += eo[c];
                }
        if (shared && !st)
            for (size_t i = 0; i < T * H; ++i) out[i] += shared[i];
        free(shared);
    }
    free(logits); free(gate); free(up); free(act); free(eo);
    return st;
}
