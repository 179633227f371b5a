"""Cross-checks the restated MoE layer loop against the reference's own graph.

The reference's layer loop (`execute_expert` / `moe_forward`, deepseek_v4_graph.cpp:1826-2274) is
file-static; its only public entry is `deepseek_v4_reference_prefill` (deepseek_v4_graph.cpp:4651).
These tests run that prefill, from the reference compiled from its sources (oracle/_ref), on the
reference's reduced graph fixture (tests/fixtures/deepseek_v4_graph.json in the reference tree:
2 layers + 1 MTP layer, 4 experts, top-2, token-id hash routing in layer 0, SwiGLU limit 0.35):

* with the fixture's float weights, the build reproduces the fixture's expected routes and logits
  (the fixture was produced by the official model code, so this pins the compiled reference);
* with every expert matrix packed as Q8_0, a matvec accelerator that declines every row records
  what the graph's own MoE offered it: the MoE input (the shared expert's gate rows), and each
  expert's down-projection input in the order the loop runs. The oracle, given the same input and
  weights, must produce the same routes bit for bit, the same down-projection inputs bit for bit
  (gate/up products, the clamp, SwiGLU in double, route weight before the down product) and the
  same loop order (shared expert, then expert id ascending, token, slot);
* the same with seeded random blocks of the checkpoints' storage types (IQ1_S / IQ3_XXS as in
  configuration 2, IQ2_XXS, Q4_K / Q6_K, IQ2_S / Q5_K, MXFP4 / Q8_0) in place of the Q8_0 weights:
  the graph decodes them with its own kernels and the oracle with its restated decoders.

CPU only; skipped when the reference tree or oracle/_ref is absent."""

import json

import numpy as np
import pytest

import vastloom_b200 as vb
from vastloom_b200 import synth
from vastloom_b200.build import reference_root

FIXTURE = reference_root() / "tests" / "fixtures" / "deepseek_v4_graph.json"
Q8_0 = 8
PAD = 32  # Q8_0 block width: matrices are stored with their columns zero-padded to 32

pytestmark = pytest.mark.skipif(not FIXTURE.exists(), reason="reference graph fixture is not present")


def _load():
    d = json.loads(FIXTURE.read_text())
    tensors = {}
    for name, vals in d["tensors"].items():
        kind = d["tensor_dtypes"][name]
        tensors[name] = np.asarray(vals, np.float32 if kind == "F32" else np.uint32)
    return d, d["config"], tensors


def _blocks(cfg):
    return [f"layers.{i}" for i in range(cfg["layers"])] + [f"mtp.{i}" for i in range(cfg.get("mtp_layers", 0))]


def test_reference_build_reproduces_graph_fixture(reference):
    d, cfg, tensors = _load()
    logits, routes, _ = reference.graph_prefill(cfg, tensors, {}, d["token_ids"])
    exp = d["expected"]
    tol = float(d["absolute_tolerance"])
    for i, r in enumerate(exp["routes"] + exp["mtp_routes"]):
        idx, w = routes[i]
        assert idx.ravel().tolist() == r["indices"], f"routed layer {i}"
        np.testing.assert_allclose(w.ravel(), np.asarray(r["weights"], np.float32), rtol=0, atol=tol)
    np.testing.assert_allclose(logits, np.asarray(exp["logits"], np.float32), rtol=0, atol=tol)


def _ident(block, expert, w):
    # block slot, expert (0xE: shared expert), projection (1 gate, 2 down, 3 up)
    return (block + 1) << 16 | (expert + 1) << 4 | w


def _cross_check(reference, oracle, make):
    """Runs the reference graph with every expert matrix packed by make(name, w, float matrix)
    -> (ggml type, storage columns, encoded rows [rows x row bytes]) and checks its own MoE
    against the oracle: routes, every expert's down-projection input and the loop order."""
    d, cfg, tensors = _load()
    H, I, E, k = cfg["width"], cfg["intermediate_width"], cfg["experts"], cfg["experts_per_token"]
    limit, scale = float(cfg["swiglu_limit"]), float(cfg["route_scale"])
    floats = dict(tensors)
    packed, enc_of = {}, {}
    for b, block in enumerate(_blocks(cfg)):
        experts = [(e, f"{block}.ffn.experts.{e}") for e in range(E)] + [(0xE, f"{block}.ffn.shared_experts")]
        for e, pre in experts:
            for w, (rows, cols) in ((1, (I, H)), (3, (I, H)), (2, (H, I))):
                name = f"{pre}.w{w}.weight"
                t, sc, enc = make(name, w, floats.pop(name).reshape(rows, cols))
                enc_of[(b, e, w)] = (t, sc, enc)
                packed[name] = (t, rows, cols, sc, enc.ravel(), _ident(b, e, w))
    width = max(sc for _, sc, _ in enc_of.values())
    _, routes, (ids, rows) = reference.graph_prefill(cfg, floats, packed, d["token_ids"], rec_cols=width,
                                                     rec_cap=8192)
    token_ids = np.asarray(d["token_ids"], np.uint32)
    for b, block in enumerate(_blocks(cfg)):
        x = np.ascontiguousarray(rows[ids == _ident(b, 0xE, 1)])  # [T x width], zero past H
        T = x.shape[0]
        assert T > 0 and not x[:, H:].any()
        # routes: router projection (f64 column-order sums), then hash or learned routing
        logits = oracle.router_logits(x[:, :H], tensors[f"{block}.ffn.gate.weight"].reshape(E, H))
        if block.startswith("layers.") and b < cfg["hash_layers"]:
            table = tensors[f"{block}.ffn.gate.tid2eid"].reshape(-1, k)
            idx, wts = oracle.route_hash(logits, token_ids[:T], table, k, scale)
        else:
            idx, wts = oracle.route_learned(logits, tensors[f"{block}.ffn.gate.bias"], k, scale)
        idx, wts = idx.reshape(T, k).astype(np.uint32), np.asarray(wts, np.float32).reshape(T, k)
        gidx, gw = routes[b]
        assert idx.tobytes() == gidx[:T].tobytes(), f"{block} route indices"
        assert wts.tobytes() == gw[:T].tobytes(), f"{block} route weights"

        def act(e, t, rw):
            gt, sc, w1 = enc_of[(b, e, 1)]
            _, _, w3 = enc_of[(b, e, 3)]
            a = np.zeros(width, np.float32)
            a[:I] = oracle.v4_expert_activation(gt, w1, w3, I, sc, x[t, :sc], rw, limit)
            return a

        # shared expert: its down-projection inputs, token by token
        got = rows[ids == _ident(b, 0xE, 2)]
        want = np.stack([act(0xE, t, None) for t in range(T)])
        assert got.tobytes() == want.tobytes(), f"{block} shared expert"
        # routed experts: the loop order (expert id ascending, token, slot) and every down input
        order, want_rows = [], []
        for e in range(E):
            for t in range(T):
                for s_ in range(k):
                    if idx[t, s_] == e:
                        order.append(_ident(b, e, 2))
                        want_rows.append(act(e, t, float(wts[t, s_])))
        mask = np.isin(ids, [_ident(b, e, 2) for e in range(E)])
        assert ids[mask].tolist() == order, f"{block} routed loop order"
        assert rows[mask].tobytes() == np.stack(want_rows).tobytes(), f"{block} routed down inputs"
        # every routed gate offer carries the MoE input row of its token
        for e in range(E):
            toks = [t for t in range(T) for s_ in range(k) if idx[t, s_] == e]
            assert rows[ids == _ident(b, e, 1)].tobytes() == x[toks].tobytes(), f"{block} expert {e} input"


def test_oracle_layer_loop_matches_reference_graph(reference, oracle):
    """The fixture's own expert weights, quantized to Q8_0 by the reference's encoder (columns
    zero-padded to one 32-wide block)."""

    def make(name, w, m):
        rows, cols = m.shape
        p = np.zeros((rows, PAD), np.float32)
        p[:, :cols] = m
        return Q8_0, PAD, reference.quantize_q8_0(p, rows, PAD, PAD).reshape(rows, -1)

    _cross_check(reference, oracle, make)


@pytest.mark.parametrize("gate_type,down_type", [
    (vb.TYPE_IQ1_S, vb.TYPE_IQ3_XXS),   # configuration 2's routed experts
    (vb.TYPE_IQ2_XXS, vb.TYPE_IQ2_XXS),  # configuration 1
    (vb.TYPE_Q4_K, vb.TYPE_Q6_K),
    (vb.TYPE_IQ2_S, vb.TYPE_Q5_K),
    (vb.TYPE_MXFP4, vb.TYPE_Q8_0),
])
def test_oracle_layer_loop_matches_reference_graph_quantized(reference, oracle, gate_type, down_type):
    """The same cross-check with seeded random blocks of the real checkpoints' storage types as
    the expert weights (gate and up of one type, down of another, the shared expert likewise):
    the graph decodes them with its own kernels, the oracle with its restated decoders. One
    256-column storage row per matrix row; columns past the logical width meet zero inputs."""
    rng = np.random.default_rng(gate_type * 100 + down_type)
    sc = 256

    def make(name, w, m):
        t = down_type if w == 2 else gate_type
        be, bb = vb.BLOCK_LAYOUT[t]
        rows = m.shape[0]
        enc = synth.matrix(rng, t, rows, sc, synth.D_SCALE[t] * 20)
        return t, sc, enc.reshape(rows, (sc // be) * bb)

    _cross_check(reference, oracle, make)
