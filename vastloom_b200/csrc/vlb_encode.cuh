// The resident image of one ggml matrix, written block by block by both upload paths: the
// host one (vlb_upload_matrix re-lays the payload out in host memory and copies the image) and the
// device one (vlb_upload_record_async copies a whole expert record's ggml bytes and re-lays every
// block out with one thread per block). Both call encode_block, so their images are identical.
//
//   split formats (Q8_0, IQ2_XXS, IQ3_XXS, IQ1_S):
//     [fp16 d per slot, 256-byte padded][IQ2/IQ3: u32 group scales per slot, 256-byte padded]
//     [body per slot]
//   whole-block formats (vlb_formats.cuh): [slot per block]
// Slots are tiled by blk_index and rows are padded to a multiple of 128 with zero blocks.
#pragma once

#include "vlb_formats.cuh"

namespace vlb {

struct MatrixImage {
    size_t nslots;    // rows padded to the tile x blocks per row
    size_t d_bytes;   // 0 for the whole-block formats
    size_t sc_bytes;  // IQ2_XXS / IQ3_XXS only
    size_t total;     // allocation size
    size_t resident;  // bytes the kernels read (what vlb_matrix_bytes reports for split formats)
};

__host__ __device__ inline MatrixImage matrix_image(uint32_t type, const TypeLayout& L, size_t rows, size_t cols) {
    MatrixImage m{};
    const size_t bpr = cols / L.block_elems;
    m.nslots = (rows + kTileRows - 1) / kTileRows * kTileRows * bpr;
    if (raw_type(type)) {
        m.total = m.nslots * L.body_bytes;
        m.resident = m.total;
        return m;
    }
    const bool scaled = type == kTypeIq2Xxs || type == kTypeIq3Xxs;
    m.d_bytes = (m.nslots * 2 + 255) / 256 * 256;
    m.sc_bytes = scaled ? (m.nslots * 4 + 255) / 256 * 256 : 0;
    m.total = m.d_bytes + m.sc_bytes + m.nslots * L.body_bytes;
    m.resident = m.nslots * 2 + (scaled ? m.nslots * 4 : 0) + m.nslots * L.body_bytes;
    return m;
}

__host__ __device__ inline uint16_t ld_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
__host__ __device__ inline uint32_t ld_u32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
__host__ __device__ inline void st_u32(uint8_t* p, uint32_t v) {
    p[0] = (uint8_t)v;
    p[1] = (uint8_t)(v >> 8);
    p[2] = (uint8_t)(v >> 16);
    p[3] = (uint8_t)(v >> 24);
}
__host__ __device__ inline bool half_bits_finite(uint16_t bits) { return ((bits >> 10) & 0x1fu) != 0x1fu; }

// Whether the reference's decoder accepts a block (validate_block_scales, ggml_quantization.cpp:
// 205-215: every fp16 scale finite; decode_mxfp4_block :381-398: every value finite, i.e. the
// largest doubled E2M1 magnitude m times the half scale 2^(e - 128) below 2^128).
__host__ __device__ inline bool block_finite(uint32_t type, const uint8_t* blk) {
    switch (type) {
        case kTypeQ4K:
        case kTypeQ5K:
            return half_bits_finite(ld_u16(blk)) && half_bits_finite(ld_u16(blk + 2));
        case kTypeQ6K:
            return half_bits_finite(ld_u16(blk + 208));
        case kTypeMxfp4: {
            uint32_t mx = 0;
            for (int i = 0; i < 16; ++i) {
                const uint32_t lo = blk[1 + i] & 7u, hi = (blk[1 + i] >> 4) & 7u;
                mx = mx > lo ? mx : lo;
                mx = mx > hi ? mx : hi;
            }
            // codes 0..7 double to 0 1 2 3 4 6 8 12 (increasing), and m x 2^(e - 128) is exact
            // until it reaches 2^128: m < 2 at e = 255, m < 4 at e = 254, m < 8 at e = 253
            // (6 x 2^125 < 2^128 = 8 x 2^125), any m below that
            const uint32_t e = blk[0];
            if (e == 255u) return mx <= 1u;
            if (e == 254u) return mx <= 3u;
            if (e == 253u) return mx <= 5u;
            return true;
        }
        default:
            return half_bits_finite(ld_u16(blk));
    }
}

// Writes block `blk` (ggml bytes) into slot `at` of the image at `img`.
__host__ __device__ inline void encode_block(uint32_t type, const TypeLayout& L, const MatrixImage& m,
                                             const uint8_t* blk, size_t at, uint8_t* img) {
    if (raw_type(type)) {
        uint8_t* dst = img + at * L.body_bytes;
        if (type == kTypeIq2S) {
            dst[0] = blk[0];
            dst[1] = blk[1];
            for (uint32_t i = 2; i < L.block_bytes; ++i) dst[i + 2] = blk[i];
        } else if (type == kTypeMxfp4) {
            for (uint32_t i = 0; i < 16; ++i) dst[i] = blk[1 + i];
            dst[16] = blk[0];
        } else {
            for (uint32_t i = 0; i < L.block_bytes; ++i) dst[i] = blk[i];
        }
        return;
    }
    img[2 * at] = blk[0];
    img[2 * at + 1] = blk[1];
    uint8_t* body = img + m.d_bytes + m.sc_bytes + at * L.body_bytes;
    for (uint32_t i = 0; i + 2 < L.block_bytes; ++i) body[i] = blk[2 + i];
    if (type == kTypeIq2Xxs || type == kTypeIq3Xxs) {
        // group words (IQ2_XXS: after each group's 4 index bytes; IQ3_XXS: after the 64 index
        // bytes) -> pair-layout sign words, the 4-bit group scales gathered per block
        uint32_t scales = 0;
        for (uint32_t g = 0; g < 8; ++g) {
            uint8_t* word = type == kTypeIq2Xxs ? body + g * 8 + 4 : body + 64 + g * 4;
            const uint32_t aux = ld_u32(word);
            scales |= (aux >> 28) << (4 * g);
            st_u32(word, iq2_pair_signs(aux));
        }
        st_u32(img + m.d_bytes + 4 * at, scales);
    }
}

}  // namespace vlb
