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
  same loop order (shared expert, then expert id ascending, token, slot).

CPU only; skipped when the reference tree or oracle/_ref is absent."""

import json

import numpy as np
import pytest

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
    # block slot, expert (0xF: shared expert), projection (1 gate, 2 down, 3 up)
    return (block + 1) << 16 | (expert + 1) << 4 | w


def _pack(reference, m, rows_pad=PAD):
    """Q8_0 bytes of the zero-padded [rows_pad x 32] matrix (rows beyond m's are zero blocks)."""
    p = np.zeros((rows_pad, PAD), np.float32)
    p[: m.shape[0], : m.shape[1]] = m
    return reference.quantize_q8_0(p, rows_pad, PAD, PAD).reshape(rows_pad, -1)


def test_oracle_layer_loop_matches_reference_graph(reference, oracle):
    d, cfg, tensors = _load()
    H, I, E, k = cfg["width"], cfg["intermediate_width"], cfg["experts"], cfg["experts_per_token"]
    limit, scale = float(cfg["swiglu_limit"]), float(cfg["route_scale"])
    assert H <= PAD and I <= PAD
    floats = dict(tensors)
    packed, padded = {}, {}
    for b, block in enumerate(_blocks(cfg)):
        experts = [(e, f"{block}.ffn.experts.{e}") for e in range(E)] + [(0xE, f"{block}.ffn.shared_experts")]
        for e, pre in experts:
            for w, (rows, cols) in ((1, (I, H)), (3, (I, H)), (2, (H, I))):
                name = f"{pre}.w{w}.weight"
                m = floats.pop(name).reshape(rows, cols)
                enc = _pack(reference, m)
                padded[(b, e, w)] = enc  # 32 x 32 for the oracle's zero-padded products
                packed[name] = (Q8_0, rows, cols, PAD, enc[:rows].ravel(), _ident(b, e, w))
    _, routes, (ids, rows) = reference.graph_prefill(cfg, floats, packed, d["token_ids"], rec_cols=PAD,
                                                     rec_cap=8192)
    token_ids = np.asarray(d["token_ids"], np.uint32)
    for b, block in enumerate(_blocks(cfg)):
        shared_in = rows[ids == _ident(b, 0xE, 1)]
        T = shared_in.shape[0]
        assert T > 0
        x = np.ascontiguousarray(shared_in)  # [T x 32], columns beyond H are zero
        # routes: router projection (f64 column-order sums), then hash or learned routing
        gate_w = np.zeros((E, PAD), np.float32)
        gate_w[:, :H] = tensors[f"{block}.ffn.gate.weight"].reshape(E, H)
        logits = oracle.router_logits(x, gate_w)
        if block.startswith("layers.") and b < cfg["hash_layers"]:
            table = tensors[f"{block}.ffn.gate.tid2eid"].reshape(-1, k)
            idx, wts = oracle.route_hash(logits, token_ids[:T], table, k, scale)
        else:
            idx, wts = oracle.route_learned(logits, tensors[f"{block}.ffn.gate.bias"], k, scale)
        gidx, gw = routes[b]
        assert np.array_equal(idx.reshape(T, k), gidx[:T]), block
        assert idx.reshape(T, k).astype(np.uint32).tobytes() == gidx[:T].tobytes(), block
        assert np.asarray(wts, np.float32).reshape(T, k).tobytes() == gw[:T].tobytes(), block

        def act(e, xt, rw):
            a = np.zeros(PAD, np.float32)
            a[:] = oracle.v4_expert_activation(Q8_0, padded[(b, e, 1)], padded[(b, e, 3)], PAD, PAD, xt, rw, limit)
            return a

        # shared expert: its down-projection inputs, token by token
        got = rows[ids == _ident(b, 0xE, 2)]
        want = np.stack([act(0xE, x[t], None) for t in range(T)])
        assert got[:, I:].max(initial=0) == 0 and want[:, I:].max(initial=0) == 0
        assert got.tobytes() == want.tobytes(), f"{block} shared expert"
        # routed experts: the loop order (expert id ascending, token, slot) and every down input
        idx2, w2 = idx.reshape(T, k), np.asarray(wts, np.float32).reshape(T, k)
        order, want_rows = [], []
        for e in range(E):
            for t in range(T):
                for s in range(k):
                    if idx2[t, s] == e:
                        order.append(_ident(b, e, 2))
                        want_rows.append(act(e, x[t], float(w2[t, s])))
        mask = np.isin(ids, [_ident(b, e, 2) for e in range(E)])
        assert ids[mask].tolist() == order, f"{block} routed loop order"
        assert rows[mask].tobytes() == np.stack(want_rows).tobytes(), f"{block} routed down inputs"
        # every routed gate offer carries the MoE input row of its token
        for e in range(E):
            toks = [t for t in range(T) for s in range(k) if idx2[t, s] == e]
            assert rows[ids == _ident(b, e, 1)].tobytes() == x[toks].tobytes(), f"{block} expert {e} input"
