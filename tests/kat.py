"""Known-answer inputs of the vastloom reference's own unit tests, rebuilt from the integer
formulas those tests use, with the answers they pin.

Every block set uses the six fp16 scales {0x3c00, 0xb800, 0x3555, 0x4000, 0x0400, 0x0001}
(1.0, -0.5, ~0.333, 2.0, the smallest normal, the smallest subnormal) and the non-dyadic input
x[c] = ((c % 29) - 14) * 0.03125 + (c % 3) * 0.0078125.
"""

from __future__ import annotations

import numpy as np

SCALES = (0x3C00, 0xB800, 0x3555, 0x4000, 0x0400, 0x0001)


def kat_input(n: int) -> np.ndarray:
    c = np.arange(n)
    return (((c % 29) - 14).astype(np.float32) * np.float32(0.03125)
            + (c % 3).astype(np.float32) * np.float32(0.0078125)).astype(np.float32)


def _put16(b: bytearray, off: int, v: int) -> None:
    b[off] = v & 0xFF
    b[off + 1] = (v >> 8) & 0xFF


def iq1_s_blocks() -> np.ndarray:
    """tests/test_main.cpp:1295-1318 (test_iq1_s_reference_kernel)."""
    b = bytearray(len(SCALES) * 50)
    for blk, s in enumerate(SCALES):
        base = blk * 50
        _put16(b, base, s)
        for i in range(32):
            b[base + 2 + i] = (blk * 37 + i * 53 + 11) & 0xFF
        for g in range(8):
            high = ((((g * 5 + blk) & 7) << 12) | (0x8000 if ((g + blk) & 1) else 0)
                    | ((blk * 733 + g * 97 + 0x123) & 0x0FFF))
            _put16(b, base + 34 + g * 2, high)
    return np.frombuffer(bytes(b), np.uint8).copy()


def iq2_xxs_blocks() -> np.ndarray:
    """tests/test_main.cpp:1367-1381 (test_iq2_xxs_reference_kernel)."""
    b = bytearray(len(SCALES) * 66)
    for blk, s in enumerate(SCALES):
        base = blk * 66
        _put16(b, base, s)
        for i in range(32):
            _put16(b, base + 2 + i * 2, (blk * 733 + i * 977 + 0x1234) & 0xFFFF)
    return np.frombuffer(bytes(b), np.uint8).copy()


def iq3_xxs_blocks() -> np.ndarray:
    """tests/test_main.cpp:1832-1858 (test_iq3_xxs_reference_kernel)."""
    b = bytearray(len(SCALES) * 98)
    for blk, s in enumerate(SCALES):
        base = blk * 98
        _put16(b, base, s)
        for i in range(64):
            b[base + 2 + i] = (blk * 37 + i * 53 + 11) & 0xFF
        for g in range(8):
            aux = ((blk * 3 + g * 5) & 15) << 28
            for j in range(4):
                aux |= ((blk * 19 + g * 13 + j * 23 + 7) & 127) << (7 * j)
            for byte in range(4):
                b[base + 66 + g * 4 + byte] = (aux >> (8 * byte)) & 0xFF
    return np.frombuffer(bytes(b), np.uint8).copy()


def q8_0_blocks() -> np.ndarray:
    """tests/test_main.cpp:944-957 (test_trunk_storage_reference_kernels, Q8_0 part)."""
    b = bytearray(len(SCALES) * 34)
    for blk, s in enumerate(SCALES):
        base = blk * 34
        _put16(b, base, s)
        for i in range(32):
            b[base + 2 + i] = (blk * 37 + i * 53 + 11) & 0xFF
    return np.frombuffer(bytes(b), np.uint8).copy()


def q8_0_encoder_source() -> np.ndarray:
    """tests/test_main.cpp:906-913: 3 x 17 floats for quantize_q8_0_reference(.., 3, 17, 32)."""
    r = np.arange(3)[:, None]
    c = np.arange(17)[None, :]
    centered = ((r * 19 + c * 7) % 31) - 15
    return (centered.astype(np.float32) * np.float32(0.017578125)
            + (c % 5).astype(np.float32) * np.float32(0.00390625)).astype(np.float32)


MIN_SCALES = (0x3800, 0xBC00, 0x3000, 0x3C00, 0x0001, 0x0400)  # tests/test_main.cpp:946-947


def q4_k_blocks() -> np.ndarray:
    """tests/test_main.cpp:976-989 (Q4_K part of test_trunk_storage_reference_kernels)."""
    b = bytearray(len(SCALES) * 144)
    for blk, s in enumerate(SCALES):
        base = blk * 144
        _put16(b, base, s)
        _put16(b, base + 2, MIN_SCALES[blk])
        for i in range(12):
            b[base + 4 + i] = (blk * 29 + i * 47 + 7) & 0xFF
        for i in range(128):
            b[base + 16 + i] = (blk * 37 + i * 53 + 11) & 0xFF
    return np.frombuffer(bytes(b), np.uint8).copy()


def q5_k_blocks() -> np.ndarray:
    """tests/test_main.cpp:1019-1037 (Q5_K part)."""
    b = bytearray(len(SCALES) * 176)
    for blk, s in enumerate(SCALES):
        base = blk * 176
        _put16(b, base, s)
        _put16(b, base + 2, MIN_SCALES[blk])
        for i in range(12):
            b[base + 4 + i] = (blk * 29 + i * 47 + 7) & 0xFF
        for i in range(32):
            b[base + 16 + i] = (blk * 41 + i * 31 + 13) & 0xFF
        for i in range(128):
            b[base + 48 + i] = (blk * 37 + i * 53 + 11) & 0xFF
    return np.frombuffer(bytes(b), np.uint8).copy()


def q6_k_blocks() -> np.ndarray:
    """tests/test_main.cpp:1057-1072 (Q6_K part)."""
    b = bytearray(len(SCALES) * 210)
    for blk, s in enumerate(SCALES):
        base = blk * 210
        for i in range(128):
            b[base + i] = (blk * 37 + i * 53 + 11) & 0xFF
        for i in range(64):
            b[base + 128 + i] = (blk * 41 + i * 31 + 13) & 0xFF
        for i in range(16):
            b[base + 192 + i] = (blk * 59 + i * 43 + 17) & 0xFF
        _put16(b, base + 208, s)
    return np.frombuffer(bytes(b), np.uint8).copy()


def iq2_s_blocks() -> np.ndarray:
    """tests/test_main.cpp:1725-1753 (test_iq2_s_reference_kernel)."""
    b = bytearray(len(SCALES) * 82)
    for blk, s in enumerate(SCALES):
        base = blk * 82
        _put16(b, base, s)
        for i in range(32):
            b[base + 2 + i] = (blk * 733 + i * 977 + 0x1234) & 0xFF
        for i in range(32):
            b[base + 34 + i] = (blk * 251 + i * 131 + 0x5AA5) & 0xFF
        for i in range(8):
            b[base + 66 + i] = (blk * 97 + i * 43 + 0x3C) & 0xFF
        for i in range(8):
            b[base + 74 + i] = (blk * 61 + i * 29 + 0x17) & 0xFF
    return np.frombuffer(bytes(b), np.uint8).copy()


PARITY_MINIMUMS = (0x3800, 0x3555, 0xBC00, 0x0001, 0x4200, 0x0400)  # tests/test_main.cpp:1666-1667


def q4_k_parity_blocks() -> np.ndarray:
    """tests/test_main.cpp:1668-1683 (test_q4k_mxfp4_reference_parity, Q4_K part)."""
    b = bytearray(len(SCALES) * 144)
    for blk, s in enumerate(SCALES):
        base = blk * 144
        _put16(b, base, s)
        _put16(b, base + 2, PARITY_MINIMUMS[blk])
        for i in range(12):
            b[base + 4 + i] = (blk * 37 + i * 53 + 0x2B) & 0xFF
        for i in range(128):
            b[base + 16 + i] = (blk * 733 + i * 977 + 0x1234) & 0xFF
    return np.frombuffer(bytes(b), np.uint8).copy()


def mxfp4_blocks() -> np.ndarray:
    """tests/test_main.cpp:1701-1709 (test_q4k_mxfp4_reference_parity, MXFP4 part)."""
    b = bytearray(len(SCALES) * 17)
    for blk in range(len(SCALES)):
        base = blk * 17
        b[base] = 120 + blk * 3
        for i in range(16):
            b[base + 1 + i] = (blk * 91 + i * 167 + 0x5A) & 0xFF
    return np.frombuffer(bytes(b), np.uint8).copy()


# Pinned answers. (hash of all decoded f32 bits, selected decoded values, 3-row matvec outputs
# with an absolute tolerance where the reference uses one.)
ANSWERS = {
    "iq1_s": dict(  # tests/test_main.cpp:1329-1352
        hash=0x9B66DE452B7F3C8D,
        values={0: 0.125, 7: 0.125, 8: -0.875, 31: -0.875, 32: 9.625, 255: -7.875, 256: 1.6875, 511: -0.5625},
        matvec=[(-4.8994140625, 0.0), (22.142812728881836, 1e-6), (-0.0021024104207754135, 1e-9)]),
    "iq2_xxs": dict(  # tests/test_main.cpp:1385-1412
        hash=0x9BCA8E03F48DAFE9,
        values={0: 9.375, 7: 3.0, 8: -16.125, 31: -3.0, 32: 5.0, 63: -5.0, 127: -9.0, 255: 17.0,
                256: 2.5, 511: 8.5},
        matvec=[(-32.86767578125, 0.0), (-284.89828491210938, 0.0), (-0.011499286629259586, 1e-9)]),
    "iq3_xxs": dict(  # tests/test_main.cpp:1862-1886
        hash=0xF36989DCC58B1664,
        values={0: -11.0, 7: -3.0, 8: 5.0, 31: -5.0, 32: 170.5, 255: 7.0, 256: -54.25, 511: -19.5},
        matvec=[(-347.998046875, 0.0), (2887.319580078125, 1e-4), (0.064146831631660461, 1e-8)]),
    "q8_0": dict(  # tests/test_main.cpp:958-971
        hash=0x25EDD1A40129EE99,
        values={0: 11.0, 7: 126.0, 8: -77.0, 31: 118.0, 32: -24.0, 63: 50.5, 127: -54.0},
        matvec=[(-168.55859375, 0.0), (-2.8284435272216797, 0.0), (0.0058367089368402958, 0.0)]),
    "q4_k": dict(  # tests/test_main.cpp:992-1005
        hash=0x84E8E84336EA0AD7,
        values={0: 75.5, 7: 96.5, 8: 19.5, 31: 40.5, 32: -25.0, 63: 353.0, 127: 12.0, 255: 212.0, 256: 32.0,
                511: -125.5},
        matvec=[(281.6796875, 0.0), (-792.12872314453125, 0.0), (0.0096547976136207581, 0.0)]),
    "q5_k": dict(  # tests/test_main.cpp:1040-1054
        hash=0x3EC4A59589931118,
        values={0: 187.5, 7: 96.5, 8: 131.5, 31: 40.5, 32: -25.0, 63: 1217.0, 127: 332.0, 255: 916.0,
                256: 32.0, 511: -453.5},
        matvec=[(668.2421875, 0.0), (1631.9100341796875, 0.0), (-0.046117834746837616, 0.0)]),
    "q6_k": dict(  # tests/test_main.cpp:1074-1088
        hash=0xCD39C3F1219AFBC9,
        values={0: -85.0, 7: 238.0, 8: -221.0, 31: 360.0, 32: 2781.0, 63: -2420.0, 127: 1054.0, 255: -530.0,
                511: 540.5},
        matvec=[(-4684.79296875, 0.0), (7494.287109375, 0.0), (0.5950310230255127, 0.0)]),
    "iq2_s": dict(  # tests/test_main.cpp:1766-1783
        hash=0x785968D455DE0695,
        values={0: -15.0, 7: -15.0, 8: 15.0, 31: 3.0, 32: -9.0, 63: 21.875, 127: 40.625, 255: -29.0,
                256: -4.5, 511: -8.0625},
        matvec=[(209.540527, 0.0), (274.050537, 0.0), (0.0192997903, 1e-9)]),
    "q4_k_parity": dict(  # tests/test_main.cpp:1694-1699
        hash=0x4A61F0F8094737CC,
        values={0: 140.5, 1: 183.5, 31: 97.5, 32: 70.0, 127: 85.0, 255: 680.5},
        matvec=None),
    "mxfp4": dict(  # tests/test_main.cpp:1720-1722
        hash=0xCE2B9AA19EF0E448,
        values={0: -0.0078125, 1: 0.00390625, 2: 0.0, 3: -0.046875, 4: 0.03125},
        matvec=None),
}
Q8_0_ENCODER_FINGERPRINT = 0x083A653165A92C21  # tests/test_main.cpp:920

# (blocks, ggml type, matvec columns) per KAT
KAT_SETS = {
    "iq1_s": (iq1_s_blocks, 19, 512),
    "iq2_xxs": (iq2_xxs_blocks, 16, 512),
    "iq3_xxs": (iq3_xxs_blocks, 18, 512),
    "q8_0": (q8_0_blocks, 8, 64),
    "q4_k": (q4_k_blocks, 12, 512),
    "q5_k": (q5_k_blocks, 13, 512),
    "q6_k": (q6_k_blocks, 14, 512),
    "iq2_s": (iq2_s_blocks, 22, 512),
    "q4_k_parity": (q4_k_parity_blocks, 12, 512),
    "mxfp4": (mxfp4_blocks, 39, 64),
}


def fnv1a_f32(values: np.ndarray) -> int:
    h = 14695981039346656037
    for byte in np.ascontiguousarray(values, dtype=np.float32).view(np.uint8).tobytes():
        h ^= byte
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def fnv1a_bytes(data: bytes) -> int:
    h = 14695981039346656037
    for byte in data:
        h ^= byte
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h
