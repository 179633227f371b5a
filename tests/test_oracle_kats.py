"""Pins the CPU oracle (oracle/vlb_oracle.c) to the reference's own known answers and to the
reference library compiled from its sources (oracle/_ref). No GPU."""

import json
from pathlib import Path

import numpy as np
import pytest

import kat
from conftest import rel_err

GOLDEN = json.loads((Path(__file__).parent / "golden" / "deepseek_v4_operators.json").read_text())
PINNED_GRIDS = {19: 0x6703ED863501AE2E, 16: 0xBB4EE025B5AC6E8E, 18: 0xDFA5DC83D6A155D5, 22: 0x123EDD38A3B62B90}


def test_codebook_fingerprints(grids):
    # ggml_quantization.cpp:60,73,99 static_asserts
    for t, fp in PINNED_GRIDS.items():
        assert kat.fnv1a_bytes(grids[t]) == fp


def test_codebooks_equal_reference_tables(grids, reference):
    for t in PINNED_GRIDS:
        assert grids[t] == reference.grid(t)


KAT_NAMES = ["iq1_s", "iq2_xxs", "iq3_xxs", "q8_0", "q4_k", "q5_k", "q6_k", "iq2_s", "q4_k_parity", "mxfp4"]


@pytest.mark.parametrize("name", KAT_NAMES)
def test_oracle_decode_and_matvec_kats(oracle, name):
    make, t, cols = kat.KAT_SETS[name]
    enc = make()
    be = 32 if t in (8, 39) else 256
    dec = oracle.dequantize(t, enc, len(kat.SCALES), be)
    ans = kat.ANSWERS[name]
    assert kat.fnv1a_f32(dec) == ans["hash"]
    for i, v in ans["values"].items():
        assert dec[i] == np.float32(v), (i, dec[i], v)
    if ans["matvec"] is None:
        return
    y = oracle.matvec(t, enc, 3, cols, kat.kat_input(cols))
    for got, (want, tol) in zip(y, ans["matvec"]):
        if tol == 0.0:
            assert got == np.float32(want)
        else:
            assert abs(float(got) - want) <= tol


def test_oracle_q8_0_encoder_kat(oracle):
    enc = oracle.quantize_q8_0(kat.q8_0_encoder_source(), 3, 17, 32)
    assert kat.fnv1a_bytes(enc.tobytes()) == kat.Q8_0_ENCODER_FINGERPRINT
    dec = oracle.dequantize(8, enc, 3, 32).reshape(3, 32)
    assert np.all(dec[:, 17:] == 0.0)  # zero padding beyond the logical columns


def test_oracle_rejects_non_finite_scale(oracle):
    enc = kat.iq2_xxs_blocks()
    enc[4 * 66] = 0x00
    enc[4 * 66 + 1] = 0x7C  # +inf fp16 scale, tests/test_main.cpp:1427-1431
    with pytest.raises(ValueError):
        oracle.dequantize(16, enc, 6, 256)


def test_oracle_learned_route_fixture(oracle):
    f = GOLDEN["learned_route"]
    x = np.array(f["input"], np.float32).reshape(f["tokens"], f["width"])
    w = np.array(f["gate_weight"], np.float32).reshape(f["experts"], f["width"])
    logits = oracle.router_logits(x, w)
    idx, wts = oracle.route_learned(logits, np.array(f["selection_bias"], np.float32), f["top_k"],
                                    f["route_scale"])
    assert idx.reshape(-1).tolist() == f["expected_indices"]
    assert np.max(np.abs(wts.reshape(-1) - np.array(f["expected_weights"]))) <= GOLDEN["absolute_tolerance"]


def test_oracle_hash_route_fixture(oracle):
    f = GOLDEN["hash_route"]
    x = np.array(f["input"], np.float32).reshape(f["tokens"], f["width"])
    w = np.array(f["gate_weight"], np.float32).reshape(f["experts"], f["width"])
    logits = oracle.router_logits(x, w)
    idx, wts = oracle.route_hash(logits, np.array(f["token_ids"], np.uint32),
                                 np.array(f["token_to_experts"], np.uint32), f["top_k"], f["route_scale"])
    assert idx.reshape(-1).tolist() == f["expected_indices"]
    assert np.max(np.abs(wts.reshape(-1) - np.array(f["expected_weights"]))) <= GOLDEN["absolute_tolerance"]


def test_oracle_rms_norm_fixture(oracle):
    f = GOLDEN["rms_norm"]
    x = np.array(f["input"], np.float32).reshape(f["rows"], f["width"])
    out = oracle.rms_norm(x, np.array(f["weight"], np.float32), f["epsilon"])
    assert np.max(np.abs(out.reshape(-1) - np.array(f["expected"]))) <= GOLDEN["absolute_tolerance"]


def test_oracle_dispatch_is_the_reference_visit_order(oracle):
    rng = np.random.default_rng(3)
    idx = rng.integers(0, 16, size=(40, 4)).astype(np.uint32)
    off, pt, ps = oracle.dispatch(idx, 16)
    visit = [(t, s) for e in range(16) for t in range(40) for s in range(4) if idx[t, s] == e]
    assert list(zip(pt.tolist(), ps.tolist())) == visit
    assert off[-1] == 160 and np.all(np.diff(off.astype(np.int64)) >= 0)


# ---- restatement vs the reference compiled from its sources -------------------------------

@pytest.mark.parametrize("t", [8, 16, 18, 19, 12, 13, 14, 22, 39])
def test_oracle_matches_reference_decode_and_matvec(oracle, reference, t):
    from vastloom_b200 import synth, BLOCK_LAYOUT

    rng = np.random.default_rng(t)
    be, bb = BLOCK_LAYOUT[t]
    rows, cols = 24, 512
    enc = synth.matrix(rng, t, rows, cols, synth.D_SCALE[t])
    a = oracle.dequantize(t, enc, rows * cols // be, be)
    b = reference.dequantize(t, enc, rows * cols)
    assert a.view(np.uint32).tolist() == b.view(np.uint32).tolist()
    x = rng.standard_normal(cols).astype(np.float32)
    assert oracle.matvec(t, enc, rows, cols, x).tobytes() == reference.matvec(t, enc, rows, cols, x).tobytes()
    # the reference's row split (RowWorkPool) is bit-identical to serial
    rows2 = 256
    enc2 = synth.matrix(rng, t, rows2, cols, synth.D_SCALE[t])
    assert reference.matvec(t, enc2, rows2, cols, x, threads=4).tobytes() == \
        oracle.matvec(t, enc2, rows2, cols, x).tobytes()


def test_oracle_matches_reference_q8_0_encoder(oracle, reference):
    rng = np.random.default_rng(11)
    m = rng.standard_normal((5, 70)).astype(np.float32)
    assert oracle.quantize_q8_0(m, 5, 70, 96).tobytes() == reference.quantize_q8_0(m, 5, 70, 96).tobytes()


def test_oracle_matches_reference_routing(oracle, reference):
    rng = np.random.default_rng(5)
    logits = rng.standard_normal((64, 256)).astype(np.float32)
    bias = (rng.standard_normal(256) * 0.01).astype(np.float32)
    i1, w1 = oracle.route_learned(logits, bias, 8, 1.5)
    i2, w2 = reference.route_learned(logits, bias, 8, 1.5)
    assert np.array_equal(i1, i2) and w1.tobytes() == w2.tobytes()
    table = np.argsort(rng.random((100, 256)), axis=1)[:, :6].astype(np.uint32)
    tok = rng.integers(0, 100, 64).astype(np.uint32)
    i1, w1 = oracle.route_hash(logits, tok, table, 6, 1.0)
    i2, w2 = reference.route_hash(logits, tok, table, 6, 1.0)
    assert np.array_equal(i1, i2) and w1.tobytes() == w2.tobytes()


def test_oracle_matches_reference_rms_norm(oracle, reference):
    rng = np.random.default_rng(9)
    x = rng.standard_normal((3, 512)).astype(np.float32)
    w = np.ones(512, np.float32)
    assert oracle.rms_norm(x, w, 1e-6).tobytes() == reference.rms_norm(x, w, 1e-6).tobytes()


@pytest.mark.parametrize("cfg", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("T", [1, 5, 13])
def test_oracle_layer_matches_reference_layer(oracle, reference, cfg, T):
    """The restated MoE layer loop against the reference-kernel layer loop: bit-identical, for a
    single token and ragged batches."""
    from vastloom_b200 import synth

    spec = synth.config(cfg, "small")
    W = synth.layer_weights(spec, seed=100 + cfg)
    x, tok, logits = synth.activations(spec, T, seed=200 + cfg + 10 * T)
    a = oracle.moe_forward(W, x, tok, logits)
    b = reference.moe_forward(W, x, tok, logits)
    assert np.array_equal(a[1], b[1])
    assert a[2].tobytes() == b[2].tobytes()
    assert a[0].tobytes() == b[0].tobytes()


def test_hash_config_equal_weights_in_reference_math(oracle):
    """Config 2: a zero gate matrix and route_scale 1 give sqrt_softplus(0) for every slot, so
    every combine weight is exactly float(1/6) in the reference's own arithmetic."""
    from vastloom_b200 import synth

    spec = synth.config(2, "small")
    W = synth.layer_weights(spec, seed=7)
    x, tok, _ = synth.activations(spec, 5, seed=8)
    _, idx, w = oracle.moe_forward(W, x, tok)
    assert np.all(w == np.float32(1.0 / 6.0))
    assert np.array_equal(idx, W.tid2eid[tok])


def test_routed_expert_zero_weights_give_zero(oracle):
    """tests/test_main.cpp:2006-2017: zero weights -> zero output."""
    rng = np.random.default_rng(1)
    enc = np.zeros(256 * 50, np.uint8)  # IQ1_S 256 x 256, all-zero (d = 0)
    y = oracle.matvec(19, enc, 256, 256, np.full(256, 0.25, np.float32))
    assert np.all(y == 0.0)
    assert rel_err(y, y) == 0.0


# ---- SwiGLU clamp and the Qwen router -----------------------------------------------------

def test_oracle_expert_swiglu_fixture(oracle, reference):
    """The clamped SwiGLU the layer loops share, pinned to the reference's `expert` fixture
    (swiglu_limit 0.35, consumed by tests/test_main.cpp:4503-4516) and to the reference's
    deepseek_v4_expert_swiglu itself, bit for bit."""
    f = GOLDEN["expert"]
    T, H, I = f["tokens"], f["width"], f["intermediate"]
    x = np.array(f["input"], np.float32).reshape(T, H)
    g = np.array(f["gate_weight"], np.float32).reshape(I, H)
    u = np.array(f["up_weight"], np.float32).reshape(I, H)
    d = np.array(f["down_weight"], np.float32).reshape(H, I)
    rw = np.array(f["routing_weights"], np.float32)
    out = oracle.expert_swiglu(x, g, d, u, rw, f["swiglu_limit"])
    assert np.max(np.abs(out.reshape(-1) - np.array(f["expected"]))) <= GOLDEN["absolute_tolerance"]
    assert out.tobytes() == reference.expert_swiglu(x, g, d, u, rw, f["swiglu_limit"]).tobytes()
    # the clamp changes this fixture's result (the limit is active)
    assert out.tobytes() != oracle.expert_swiglu(x, g, d, u, rw, 0.0).tobytes()


@pytest.mark.parametrize("limit", [0.05, 0.35, 10.0])
def test_oracle_expert_swiglu_matches_reference_random(oracle, reference, limit):
    rng = np.random.default_rng(int(limit * 100))
    T, H, I = 3, 64, 48
    x = rng.standard_normal((T, H)).astype(np.float32)
    g, u = (rng.standard_normal((I, H)).astype(np.float32) for _ in range(2))
    d = rng.standard_normal((H, I)).astype(np.float32)
    rw = rng.random(T).astype(np.float32)
    for w in (rw, None):
        assert oracle.expert_swiglu(x, g, d, u, w, limit).tobytes() == \
            reference.expert_swiglu(x, g, d, u, w, limit).tobytes()


@pytest.mark.parametrize("cfg", [1, 2])
@pytest.mark.parametrize("limits", [(0.01, 0.02), (10.0, 10.0)])
def test_oracle_layer_with_clamp_matches_reference(oracle, reference, cfg, limits):
    """The layer loops with the SwiGLU clamp on (routed and shared limits): 10.0 is the real
    model's limit (tests/test_main.cpp:2836), 0.01 / 0.02 clamp most gate and up values of these
    synthetic layers."""
    from dataclasses import replace

    from vastloom_b200 import synth

    spec = replace(synth.config(cfg, "small"), routed_swiglu_limit=limits[0], shared_swiglu_limit=limits[1])
    W = synth.layer_weights(spec, seed=600 + cfg)
    x, tok, logits = synth.activations(spec, 5, seed=610 + cfg)
    a = oracle.moe_forward(W, x, tok, logits)
    b = reference.moe_forward(W, x, tok, logits)
    assert np.array_equal(a[1], b[1]) and a[0].tobytes() == b[0].tobytes()
    off = oracle.moe_forward(replace(W, spec=replace(spec, routed_swiglu_limit=0.0, shared_swiglu_limit=0.0)),
                             x, tok, logits)[0]
    if limits[0] < 1.0:
        assert a[0].tobytes() != off.tobytes()  # the small limits do clamp


def test_oracle_qwen_route_reference_test_vector(oracle):
    """tests/test_main.cpp:3966-3990: hidden (1, 0), three experts, top-2 with renormalisation."""
    x = np.array([[1.0, 0.0]], np.float32)
    r = np.array([[1, 0], [0, 1], [1, 1]], np.float32)
    logits = oracle.router_logits(x, r)
    assert logits.tolist() == [[1.0, 0.0, 1.0]]
    idx, w = oracle.route_softmax_f64(logits, 2, norm=True)
    assert idx.tolist() == [[0, 2]]
    assert np.all(np.abs(w - 0.5) < 1e-5)


@pytest.mark.parametrize("norm", [True, False])
@pytest.mark.parametrize("E,k", [(512, 10), (64, 8)])
def test_oracle_qwen_route_matches_reference(oracle, reference, norm, E, k):
    rng = np.random.default_rng(E + k + norm)
    T, H = 6, 256
    hidden = rng.standard_normal((T, H)).astype(np.float32)
    router = (rng.standard_normal((E, H)) * 0.05).astype(np.float32)
    logits = oracle.router_logits(hidden, router)
    idx, w = oracle.route_softmax_f64(logits, k, norm=norm)
    rl, ri, rw = reference.qwen_route(hidden, router, k, norm=norm)
    assert logits.tobytes() == rl.tobytes()
    assert np.array_equal(idx, ri) and w.tobytes() == rw.tobytes()
