"""Seeded synthetic inputs for the routed-expert path, following the benchmark configurations.

No checkpoint or dataset is available, so every weight and activation is drawn from a seeded
numpy PCG64 generator with the distributions the configurations specify. Block bytes use the
reference's ggml layouts exactly (ggml_quantization.cpp:217-435): a little-endian fp16 scale
followed by the block body. Scales are rounded to fp16 with numpy's round-to-nearest-even, the
same rounding as the reference encoder's float_to_fp16 (ggml_quantization.cpp:126-145) for
normal values.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from . import (BLOCK_LAYOUT, SCORE_SIGMOID, SCORE_SOFTMAX, SCORE_SQRT_SOFTPLUS, TYPE_IQ1_S, TYPE_IQ2_S,
               TYPE_IQ2_XXS, TYPE_IQ3_XXS, TYPE_MXFP4, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K, TYPE_Q8_0)


def _fp16_bits(v: np.ndarray) -> np.ndarray:
    return np.asarray(v, dtype=np.float32).astype(np.float16).view(np.uint16)


def blocks(rng: np.random.Generator, ggml_type: int, n_blocks: int, d_scale: float) -> np.ndarray:
    """n_blocks ggml blocks of one type as a flat uint8 array.

    Q8_0    : d = |N(0,1)| * d_scale, 32 int8 uniform in [-127, 127]          (34 B)
    IQ2_XXS : d = |N(0,1)| * d_scale, 32 uniformly random u16 qs words         (66 B)
    IQ3_XXS : d = |N(0,1)| * d_scale, 96 random packed bytes                   (98 B)
    IQ1_S   : d = |N(0,1)| * d_scale, 32 random qs bytes, 8 random u16 qh      (50 B)
    Q4_K/Q5_K: d and dmin = |N(0,1)| * d_scale, the rest random bytes       (144 / 176 B)
    Q6_K    : 208 random bytes, then d = |N(0,1)| * d_scale                  (210 B)
    IQ2_S   : d = |N(0,1)| * d_scale, 80 random bytes                        (82 B)
    MXFP4   : an E8M0 scale byte in [118, 126] (2^-10 .. 2^-2), 16 random nibble bytes (17 B)
    """
    _, bb = BLOCK_LAYOUT[ggml_type]
    out = np.empty((n_blocks, bb), dtype=np.uint8)
    if ggml_type == TYPE_MXFP4:
        out[:, 0] = rng.integers(118, 127, size=n_blocks, dtype=np.uint8)
        out[:, 1:] = rng.integers(0, 256, size=(n_blocks, bb - 1), dtype=np.uint8)
        return out.reshape(-1)
    d = _fp16_bits(np.abs(rng.standard_normal(n_blocks)) * d_scale)
    at = 208 if ggml_type == TYPE_Q6_K else 0
    if ggml_type == TYPE_Q6_K:
        out[:, :208] = rng.integers(0, 256, size=(n_blocks, 208), dtype=np.uint8)
    elif ggml_type == TYPE_Q8_0:
        out[:, 2:] = rng.integers(-127, 128, size=(n_blocks, 32), dtype=np.int16).astype(np.int8).view(np.uint8)
    else:
        out[:, 2:] = rng.integers(0, 256, size=(n_blocks, bb - 2), dtype=np.uint8)
    out[:, at] = d & 0xFF
    out[:, at + 1] = d >> 8
    if ggml_type in (TYPE_Q4_K, TYPE_Q5_K):
        dmin = _fp16_bits(np.abs(rng.standard_normal(n_blocks)) * d_scale)
        out[:, 2] = dmin & 0xFF
        out[:, 3] = dmin >> 8
    return out.reshape(-1)


def matrix(rng: np.random.Generator, ggml_type: int, rows: int, cols: int, d_scale: float) -> np.ndarray:
    be, _ = BLOCK_LAYOUT[ggml_type]
    return blocks(rng, ggml_type, rows * (cols // be), d_scale)


D_SCALE = {TYPE_Q8_0: 0.002, TYPE_IQ2_XXS: 0.01, TYPE_IQ3_XXS: 0.01, TYPE_IQ1_S: 0.01, TYPE_Q4_K: 0.001,
           TYPE_Q5_K: 0.0005, TYPE_Q6_K: 0.0005, TYPE_IQ2_S: 0.01, TYPE_MXFP4: 1.0}


@dataclass
class LayerSpec:
    """One MoE layer configuration (all sizes in elements)."""

    name: str
    hidden: int
    intermediate: int
    experts: int
    top_k: int
    score: int
    gate_type: int           # routed gate/up type
    down_type: int           # routed down type
    shared_type: Optional[int] = None
    hash_routing: bool = False
    vocab: int = 0
    weight_after_down: bool = False
    route_scale: float = 1.0
    zero_router: bool = False      # config 2: equal combine weights inside the reference's math
    mixed_types: bool = False      # config 3: experts alternate IQ2_XXS / Q8_0 by seeded coin
    logits_given: bool = False     # config 3/4: routing logits are an input
    zipf_s: float = 0.0            # config 4: Zipf-skewed popularity of the given logits
    routed_swiglu_limit: float = 0.0   # SwiGLU clamp of the routed / shared experts (0: off)
    shared_swiglu_limit: float = 0.0


def config(n: int, scale: str = "full") -> LayerSpec:
    """The benchmark configurations (BASELINE.json configs[n]); scale='small' keeps every
    structural property but shrinks H/I/E so the CPU oracle finishes in seconds."""
    small = scale == "small"
    if n == 0:
        return LayerSpec("cfg0-olmoe-q8_0", 512 if small else 2048, 256 if small else 1024,
                         16 if small else 64, 4 if small else 8, SCORE_SOFTMAX, TYPE_Q8_0, TYPE_Q8_0,
                         weight_after_down=True)
    if n == 1:
        return LayerSpec("cfg1-v4flash-decode", 512 if small else 4096, 256 if small else 2048,
                         16 if small else 256, 4 if small else 8, SCORE_SQRT_SOFTPLUS, TYPE_IQ2_XXS,
                         TYPE_IQ2_XXS, shared_type=TYPE_Q8_0)
    if n == 2:
        return LayerSpec("cfg2-hash-chain", 512 if small else 4096, 256 if small else 2048,
                         16 if small else 256, 6, SCORE_SQRT_SOFTPLUS, TYPE_IQ1_S, TYPE_IQ3_XXS,
                         shared_type=TYPE_Q8_0, hash_routing=True, vocab=1000 if small else 129280,
                         zero_router=True)
    if n == 3:
        return LayerSpec("cfg3-prefill-mixed", 512 if small else 4096, 256 if small else 2048,
                         16 if small else 256, 4 if small else 8, SCORE_SQRT_SOFTPLUS, TYPE_IQ2_XXS,
                         TYPE_IQ2_XXS, shared_type=TYPE_Q8_0, mixed_types=True, logits_given=True)
    if n == 4:
        return LayerSpec("cfg4-ep-zipf", 512 if small else 4096, 256 if small else 2048,
                         16 if small else 256, 4 if small else 8, SCORE_SQRT_SOFTPLUS, TYPE_IQ2_XXS,
                         TYPE_IQ2_XXS, shared_type=TYPE_Q8_0, logits_given=True, zipf_s=1.1)
    raise ValueError(n)


@dataclass
class LayerWeights:
    spec: LayerSpec
    router: np.ndarray                     # f32 [E, H]
    bias: Optional[np.ndarray]             # f32 [E]
    tid2eid: Optional[np.ndarray]          # u32 [V, k]
    w1: list = field(default_factory=list)  # (type, bytes) per expert
    w3: list = field(default_factory=list)
    w2: list = field(default_factory=list)
    shared: Optional[tuple] = None         # ((type, bytes) x 3)


def layer_weights(spec: LayerSpec, seed: int) -> LayerWeights:
    rng = np.random.Generator(np.random.PCG64(seed))
    H, I, E, k = spec.hidden, spec.intermediate, spec.experts, spec.top_k
    if spec.zero_router:
        router = np.zeros((E, H), np.float32)
    else:
        router = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    bias = None
    if not spec.hash_routing and spec.score in (SCORE_SQRT_SOFTPLUS, SCORE_SIGMOID):
        bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    tid2eid = None
    if spec.hash_routing:
        # distinct experts per row: the first k of a random permutation (argsort of uniforms),
        # drawn in row chunks (the same stream as one draw) to bound the memory at full vocabulary
        tid2eid = np.empty((spec.vocab, k), np.uint32)
        for r0 in range(0, spec.vocab, 8192):
            r1 = min(spec.vocab, r0 + 8192)
            tid2eid[r0:r1] = np.argsort(rng.random((r1 - r0, E)), axis=1)[:, :k]
    W = LayerWeights(spec, router, bias, tid2eid)
    for e in range(E):
        gt, dt = spec.gate_type, spec.down_type
        if spec.mixed_types and rng.random() < 0.5:
            gt = dt = TYPE_Q8_0
        W.w1.append((gt, matrix(rng, gt, I, H, D_SCALE[gt])))
        W.w3.append((gt, matrix(rng, gt, I, H, D_SCALE[gt])))
        W.w2.append((dt, matrix(rng, dt, H, I, D_SCALE[dt])))
    if spec.shared_type is not None:
        st = spec.shared_type
        W.shared = tuple((st, matrix(rng, st, r, c, D_SCALE[st])) for r, c in ((I, H), (I, H), (H, I)))
    return W


def activations(spec: LayerSpec, T: int, seed: int):
    """x f32 [T, H] ~ N(0,1); token ids u32 [T] uniform over the vocabulary (hash routing);
    logits f32 [T, E] for configurations whose routing logits are an input."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal((T, spec.hidden)).astype(np.float32)
    tok = None
    if spec.hash_routing:
        tok = rng.integers(0, spec.vocab, size=T, dtype=np.uint32)
    logits = None
    if spec.logits_given:
        if spec.zipf_s > 0:
            # logits = ln p_e + Gumbel(0,1), p_e proportional to rank^-s over a seeded permutation
            ranks = rng.permutation(spec.experts) + 1
            p = ranks.astype(np.float64) ** (-spec.zipf_s)
            p /= p.sum()
            g = -np.log(-np.log(rng.random((T, spec.experts))))
            logits = (np.log(p)[None, :] + g).astype(np.float32)
        else:
            logits = rng.standard_normal((T, spec.experts)).astype(np.float32)
    return x, tok, logits


def expert_record(W: LayerWeights, e: int, identities) -> tuple:
    """Expert e's record as an expert pack holds it (its W1, W3, W2 ggml bytes back to back) and
    its (identity, type, rows, storage_cols, offset, bytes) tensor list."""
    H, I = W.spec.hidden, W.spec.intermediate
    parts, tensors, off = [], [], 0
    for ident, (name, rows, cols) in zip(identities, (("w1", I, H), ("w3", I, H), ("w2", H, I))):
        t, b = getattr(W, name)[e]
        parts.append(np.asarray(b, np.uint8).reshape(-1))
        tensors.append((ident, t, rows, cols, off, parts[-1].nbytes))
        off += parts[-1].nbytes
    return np.concatenate(parts), tensors


def upload_layer(dev, W: LayerWeights, max_tokens: int, layer_index: int = 0, records: bool = False):
    """Uploads every matrix (identities in the reference's expert style: nonzero, stable per
    (layer, expert, role)) and creates the device layer. records=True moves each routed expert
    as one record (vlb_upload_record_async), up to 64 in flight."""
    from . import MoeLayer

    spec = W.spec
    H, I = spec.hidden, spec.intermediate

    def ident(e, role):
        return ((layer_index * 1_000_003 + e) * 4 + role) * 2 + 1

    mats = {"w1": [], "w3": [], "w2": []}
    if records:
        pending = []

        def drain(keep):
            while len(pending) > keep:
                for name, m in zip(("w1", "w3", "w2"), pending.pop(0).finish()):
                    mats[name].append(m)

        for e in range(spec.experts):
            rec, tensors = expert_record(W, e, [ident(e, role) for role in range(3)])
            pending.append(dev.upload_record(rec, tensors))
            drain(63)
        drain(0)
    for e in range(0 if records else spec.experts):
        for role, (name, rows, cols) in enumerate((("w1", I, H), ("w3", I, H), ("w2", H, I))):
            t, b = getattr(W, name)[e]
            mats[name].append(dev.upload_matrix(t, rows, cols, b, identity=ident(e, role)))
    shared = None
    if W.shared is not None:
        shared = tuple(dev.upload_matrix(t, r, c, b, identity=ident(spec.experts, i))
                       for i, ((t, b), (r, c)) in enumerate(zip(W.shared, ((I, H), (I, H), (H, I)))))
    layer = MoeLayer(dev, hidden=H, intermediate=I, experts=spec.experts, top_k=spec.top_k,
                     router=W.router, w1=mats["w1"], w3=mats["w3"], w2=mats["w2"], score=spec.score,
                     bias=W.bias, route_scale=spec.route_scale, hash_table=W.tid2eid,
                     weight_after_down=spec.weight_after_down, shared=shared, max_tokens=max_tokens,
                     routed_swiglu_limit=spec.routed_swiglu_limit, shared_swiglu_limit=spec.shared_swiglu_limit)
    layer.matrices = mats
    layer.shared_matrices = shared
    return layer
