"""Parity of the CUDA path (through the vlb200 C ABI) with the CPU oracle on the same seeded
inputs. Bit-exact: dequantized weights, routing indices, hash choices, permutation maps.
Floating point: layer and matvec outputs within 1e-5 norm-wise relative error (fp32
accumulation against the reference's f64 accumulation); route weights within 1 ulp where the
only difference is the device's double exp/log1p against glibc's (2 ulp for the softmax router,
whose probabilities use glibc expf on the CPU)."""

import json
from pathlib import Path

import numpy as np
import pytest

import kat
import vastloom_b200 as vb
from conftest import rel_err
from vastloom_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-5
GOLDEN = json.loads((Path(__file__).parent / "golden" / "deepseek_v4_operators.json").read_text())


def ulp_diff(a, b):
    a = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    return int(np.max(np.abs(a - b))) if a.size else 0


# ---- dequant / matvec ------------------------------------------------------------------------

KAT_NAMES = ["iq1_s", "iq2_xxs", "iq3_xxs", "q8_0", "q4_k", "q5_k", "q6_k", "iq2_s", "q4_k_parity", "mxfp4"]
ALL_TYPES = [8, 16, 18, 19, 12, 13, 14, 22, 39]  # the four MoE formats, then Q4_K Q5_K Q6_K IQ2_S MXFP4


@pytest.mark.parametrize("name", KAT_NAMES)
def test_gpu_dequant_and_matvec_kats(device, oracle, name):
    make, t, cols = kat.KAT_SETS[name]
    enc = make()
    m = device.upload_matrix(t, 3, cols, enc, identity=0x101)
    try:
        dec = device.dequantize(m).reshape(-1)
        assert kat.fnv1a_f32(dec) == kat.ANSWERS[name]["hash"]
        be = vb.BLOCK_LAYOUT[t][0]
        assert dec.tobytes() == oracle.dequantize(t, enc, len(kat.SCALES), be).tobytes()
        y = device.matvec(m, kat.kat_input(cols))
        if kat.ANSWERS[name]["matvec"] is not None:
            want = np.array([v for v, _ in kat.ANSWERS[name]["matvec"]])
            assert rel_err(y, want) <= TOL
        assert rel_err(y, oracle.matvec(t, enc, 3, cols, kat.kat_input(cols))) <= TOL
    finally:
        device.release_matrix(m)


@pytest.mark.parametrize("t", ALL_TYPES)
@pytest.mark.parametrize("shape", [(64, 512), (40, 1024), (7, 256)])
def test_gpu_dequant_bit_exact_random(device, oracle, t, shape):
    rows, cols = shape
    be, _ = vb.BLOCK_LAYOUT[t]
    rng = np.random.default_rng(rows * 131 + t)
    enc = synth.matrix(rng, t, rows, cols, synth.D_SCALE[t])
    m = device.upload_matrix(t, rows, cols, enc, identity=7)
    try:
        dev = device.dequantize(m).reshape(-1)
        ref = oracle.dequantize(t, enc, rows * cols // be, be)
        assert dev.view(np.uint32).tolist() == ref.view(np.uint32).tolist()
    finally:
        device.release_matrix(m)


@pytest.mark.parametrize("t", ALL_TYPES)
@pytest.mark.parametrize("ntok", [1, 2, 3, 5, 9])
def test_gpu_matvec_multi_token(device, oracle, t, ntok):
    rows, cols = 136, 1024
    rng = np.random.default_rng(ntok * 17 + t)
    enc = synth.matrix(rng, t, rows, cols, synth.D_SCALE[t])
    x = rng.standard_normal((ntok, cols)).astype(np.float32)
    m = device.upload_matrix(t, rows, cols, enc, identity=9)
    try:
        y = device.matvec_tokens(m, x)
        for i in range(ntok):
            assert rel_err(y[i], oracle.matvec(t, enc, rows, cols, x[i])) <= TOL
        # the single-token seam agrees with the batched path bit for bit
        assert device.matvec(m, x[0]).tobytes() == y[0].tobytes()
    finally:
        device.release_matrix(m)


# ---- routing ---------------------------------------------------------------------------------

def test_gpu_route_fixtures(device, oracle):
    for key in ("learned_route", "hash_route"):
        f = GOLDEN[key]
        x = np.array(f["input"], np.float32).reshape(f["tokens"], f["width"])
        w = np.array(f["gate_weight"], np.float32).reshape(f["experts"], f["width"])
        logits = device.router_logits(x, w)
        assert logits.tobytes() == oracle.router_logits(x, w).tobytes()
        if key == "learned_route":
            idx, wts = device.route(logits, f["top_k"], f["route_scale"],
                                    bias=np.array(f["selection_bias"], np.float32))
        else:
            idx, wts = device.route(logits, f["top_k"], f["route_scale"],
                                    token_ids=np.array(f["token_ids"]),
                                    tid2eid=np.array(f["token_to_experts"]))
        assert idx.reshape(-1).tolist() == f["expected_indices"]
        assert np.max(np.abs(wts.reshape(-1) - np.array(f["expected_weights"]))) <= GOLDEN["absolute_tolerance"]


@pytest.mark.parametrize("score", [vb.SCORE_SQRT_SOFTPLUS, vb.SCORE_SIGMOID, vb.SCORE_SOFTMAX])
@pytest.mark.parametrize("T,E,k", [(64, 256, 8), (17, 64, 8), (4096, 256, 8), (3, 512, 16)])
def test_gpu_route_random(device, oracle, score, T, E, k):
    rng = np.random.default_rng(T + E + score)
    logits = rng.standard_normal((T, E)).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    if score == vb.SCORE_SOFTMAX:
        idx, w = device.route(logits, k, score=score)
        ri, rw = oracle.route_softmax(logits, k)
        assert np.array_equal(idx, ri)
        assert ulp_diff(w, rw) <= 2
    else:
        idx, w = device.route(logits, k, 1.5, score=score, bias=bias)
        ri, rw = oracle.route_learned(logits, bias, k, 1.5, score)
        assert np.array_equal(idx, ri)
        assert ulp_diff(w, rw) <= 1


def test_gpu_route_ties_go_to_the_lower_id(device, oracle):
    logits = np.zeros((4, 64), np.float32)  # every score equal
    bias = np.zeros(64, np.float32)
    idx, _ = device.route(logits, 8, bias=bias)
    assert idx.tolist() == [list(range(8))] * 4


def test_gpu_hash_route_rejects_out_of_range_token(device):
    logits = np.zeros((2, 16), np.float32)
    table = np.tile(np.arange(4, dtype=np.uint32), (10, 1))
    with pytest.raises(vb.VlbError) as e:
        device.route(logits, 4, token_ids=np.array([1, 10]), tid2eid=table)
    assert e.value.code == "invalid_argument"


# ---- the MoE layer ---------------------------------------------------------------------------

@pytest.mark.parametrize("cfg", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("T", [1, 5, 16, 37])
def test_gpu_layer_small_configs(device, oracle, cfg, T):
    """Every configuration's structure at small scale through the decode path; T = 37 gives the
    Q8_0 shared expert three wide units (16 + 16 + 5 tokens)."""
    spec = synth.config(cfg, "small")
    W = synth.layer_weights(spec, seed=300 + cfg)
    x, tok, logits = synth.activations(spec, T, seed=400 + cfg + T)
    layer = synth.upload_layer(device, W, max_tokens=64)
    try:
        out = layer.forward(x, tok, logits)
        ref, ridx, rw = oracle.moe_forward(W, x, tok, logits)
        idx, w, off, pt, ps = layer.last_route(T)
        assert np.array_equal(idx, ridx)
        assert ulp_diff(w, rw) <= 2
        roff, rpt, rps = oracle.dispatch(ridx, spec.experts)
        assert np.array_equal(off, roff) and np.array_equal(pt, rpt) and np.array_equal(ps, rps)
        assert rel_err(out, ref) <= TOL
    finally:
        layer.destroy()
        for lst in layer.matrices.values():
            for m in lst:
                device.release_matrix(m)
        for m in layer.shared_matrices or ():
            device.release_matrix(m)


# Layers whose experts use the formats served on the CUDA cores only: Q4_K gate/up with Q6_K down
# beside a Q8_0 shared expert (DeepSeek V4 semantics), IQ2_S and MXFP4 experts (OLMoE semantics),
# Q5_K with IQ2_S down; against the oracle layer loop.
WHOLE_BLOCK = {
    "q4k-q6k-v4": synth.LayerSpec("wb-q4k-q6k", 512, 256, 12, 3, synth.SCORE_SQRT_SOFTPLUS, vb.TYPE_Q4_K,
                                  vb.TYPE_Q6_K, shared_type=synth.TYPE_Q8_0),
    "iq2s-mxfp4-olmoe": synth.LayerSpec("wb-iq2s-mxfp4", 512, 256, 12, 3, synth.SCORE_SOFTMAX, vb.TYPE_IQ2_S,
                                        vb.TYPE_MXFP4, weight_after_down=True),
    "q5k-iq2s-v4": synth.LayerSpec("wb-q5k-iq2s", 768, 512, 8, 2, synth.SCORE_SQRT_SOFTPLUS, vb.TYPE_Q5_K,
                                   vb.TYPE_IQ2_S, shared_type=synth.TYPE_Q8_0),
}


@pytest.mark.parametrize("name", list(WHOLE_BLOCK))
@pytest.mark.parametrize("T", [1, 9])
def test_gpu_layer_whole_block_formats(device, oracle, name, T):
    spec = WHOLE_BLOCK[name]
    W = synth.layer_weights(spec, seed=700 + T)
    x, tok, logits = synth.activations(spec, T, seed=710 + T)
    layer = synth.upload_layer(device, W, max_tokens=16)
    try:
        out = layer.forward(x, tok, logits)
        ref, ridx, _ = oracle.moe_forward(W, x, tok, logits)
        idx, _, _, _, _ = layer.last_route(T)
        assert np.array_equal(idx, ridx)
        assert rel_err(out, ref) <= TOL
    finally:
        layer.destroy()
        for lst in layer.matrices.values():
            for m in lst:
                device.release_matrix(m)
        for m in layer.shared_matrices or ():
            device.release_matrix(m)


RAGGED = {
    # Q8_0, OLMoE semantics: 6 row tiles of W1/W3 and of W2 (gate/up row groups of 2 tiles fill
    # exactly, down row groups of 4 tiles leave 2 empty)
    "q8-olmoe": synth.LayerSpec("ragged-q8", 768, 768, 12, 3, synth.SCORE_SOFTMAX, synth.TYPE_Q8_0,
                                synth.TYPE_Q8_0, weight_after_down=True),
    # IQ2_XXS, 3 row tiles of W1/W3: the second gate/up row group has one empty slice
    "iq2-odd-tiles": synth.LayerSpec("ragged-iq2-odd", 512, 768, 12, 3, synth.SCORE_SQRT_SOFTPLUS,
                                     synth.TYPE_IQ2_XXS, synth.TYPE_IQ2_XXS),
    # IQ2_XXS with a Q8_0 shared expert, DeepSeek-V4 semantics: 6 W2 tiles, 2 of the second down row
    # group empty
    "iq2-v4": synth.LayerSpec("ragged-iq2", 768, 512, 12, 3, synth.SCORE_SQRT_SOFTPLUS, synth.TYPE_IQ2_XXS,
                              synth.TYPE_IQ2_XXS, shared_type=synth.TYPE_Q8_0),
    # IQ1_S gate/up and IQ3_XXS down (configuration 2's types) with a Q8_0 shared expert: 6 W2
    # tiles, 2 of the second down row group empty
    "iq1-iq3-v4": synth.LayerSpec("ragged-iq1-iq3", 768, 512, 12, 3, synth.SCORE_SQRT_SOFTPLUS, synth.TYPE_IQ1_S,
                                  synth.TYPE_IQ3_XXS, shared_type=synth.TYPE_Q8_0),
}


@pytest.mark.parametrize("name", sorted(RAGGED))
@pytest.mark.parametrize("T", [1, 9])
def test_gpu_layer_ragged_tiles(device, oracle, name, T):
    """Shapes whose row counts are not whole row groups of the decode kernel (row groups with
    empty 128-row slices), for every storage type and both layer semantics."""
    spec = RAGGED[name]
    W = synth.layer_weights(spec, seed=500 + T)
    x, tok, logits = synth.activations(spec, T, seed=510 + T)
    layer = synth.upload_layer(device, W, max_tokens=16)
    try:
        out = layer.forward(x, tok, logits)
        ref, ridx, _ = oracle.moe_forward(W, x, tok, logits)
        idx, _, _, _, _ = layer.last_route(T)
        assert np.array_equal(idx, ridx)
        assert np.all(np.isfinite(out))
        assert rel_err(out, ref) <= TOL
    finally:
        layer.destroy()
        for lst in layer.matrices.values():
            for m in lst:
                device.release_matrix(m)
        for m in layer.shared_matrices or ():
            device.release_matrix(m)


@pytest.fixture(scope="module")
def full_cfg1(device):
    spec = synth.config(1)
    W = synth.layer_weights(spec, seed=1)
    layer = synth.upload_layer(device, W, max_tokens=64)
    yield spec, W, layer
    layer.destroy()
    for lst in layer.matrices.values():
        for m in lst:
            device.release_matrix(m)
    for m in layer.shared_matrices or ():
        device.release_matrix(m)


def test_gpu_layer_full_cfg1_single_token(full_cfg1, oracle):
    spec, W, layer = full_cfg1
    x, _, _ = synth.activations(spec, 1, seed=5)
    out = layer.forward(x)
    ref, ridx, rw = oracle.moe_forward(W, x)
    idx, w, *_ = layer.last_route(1)
    assert np.array_equal(idx, ridx)
    assert ulp_diff(w, rw) <= 1
    assert rel_err(out, ref) <= TOL


def test_gpu_layer_full_cfg1_batch_properties(full_cfg1, oracle):
    """T=64 at full size: the route and permutation are bit-exact against the oracle (router in
    f64 on the CPU); tokens taken from the batch match the oracle run on them alone; and every
    token's output agrees with running it alone to 1e-6 (the kernels' column-split shape depends
    on the batch size, so the f32 summation order - not the arithmetic - differs)."""
    spec, W, layer = full_cfg1
    x, _, _ = synth.activations(spec, 64, seed=6)
    out = layer.forward(x)
    idx, w, off, pt, ps = layer.last_route(64)
    logits = oracle.router_logits(x, W.router)
    ridx, rw = oracle.route_learned(logits, W.bias, spec.top_k, spec.route_scale)
    assert np.array_equal(idx, ridx)
    assert ulp_diff(w, rw) <= 1
    roff, rpt, rps = oracle.dispatch(ridx, spec.experts)
    assert np.array_equal(off, roff) and np.array_equal(pt, rpt) and np.array_equal(ps, rps)
    for t in (0, 37):
        ref, _, _ = oracle.moe_forward(W, x[t:t + 1])
        assert rel_err(out[t:t + 1], ref) <= TOL
    for t in (0, 13, 63):
        single = layer.forward(x[t:t + 1])
        assert rel_err(single, out[t:t + 1]) <= 1e-6
    assert np.all(np.isfinite(out))


def test_gpu_layer_rejects_too_many_tokens(full_cfg1):
    spec, W, layer = full_cfg1
    x = np.zeros((65, spec.hidden), np.float32)
    with pytest.raises(vb.VlbError) as e:
        layer.forward(x)
    assert e.value.code == "invalid_argument"


def test_gpu_upload_rejects_non_finite_scale_and_bad_codebook(device, grids):
    enc = kat.iq2_xxs_blocks()
    enc[4 * 66 + 1] = 0x7C
    enc[4 * 66] = 0x00
    with pytest.raises(vb.VlbError) as e:
        device.upload_matrix(16, 3, 512, enc)
    assert e.value.code == "invalid_format"
    bad = bytearray(grids[16])
    bad[5] ^= 1
    with pytest.raises(vb.VlbError) as e:
        device.set_codebook(16, bytes(bad))
    assert e.value.code == "integrity_error"


def test_gpu_governor_reserves_before_every_allocation():
    class Gov:
        def __init__(self, limit):
            self.limit, self.used, self.log = limit, 0, []

        def reserve(self, n, tag):
            if self.used + n > self.limit:
                self.log.append(("refuse", n, tag))
                return False
            self.used += n
            self.log.append(("reserve", n, tag))
            return True

        def release(self, n, tag):
            self.used -= n
            self.log.append(("release", n, tag))

    gov = Gov(limit=64 * 1024)
    with vb.Device(0, governor=gov, install_codebooks=False) as dev:
        assert gov.used == 0
        buf = dev.buffer(4096, "probe")
        assert gov.used == 4096 and dev.allocated_bytes() == 4096
        with pytest.raises(vb.VlbError) as e:
            dev.buffer(1 << 20, "too-big")
        assert e.value.code == "resource_exhausted"
        assert gov.log[-1][0] == "refuse"
        buf.free()
        assert gov.used == 0 and dev.allocated_bytes() == 0
