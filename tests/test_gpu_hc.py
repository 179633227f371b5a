"""Hyper-Connection entry and exit fused around the MoE layer (vlb_layer_set_hyper_connection): the
ffn half of a DeepSeek V4 block, out = hc_post(MoE(RMSNorm(hc_pre(x))), x)
(deepseek_v4_graph.cpp:2391-2408). Checked against the oracle composed the same way
(hc_pre -> rms_norm -> moe_forward -> hc_post, each pinned to the reference):

  * the split (pre, post, combination): within 1 ulp (only CUDA's double exp can differ from the
    host's; in practice the bits match);
  * routes and permutation: bit-exact (they depend on the normalised reduced row, whose bits
    follow from the split);
  * the m output copies: within 1e-5 norm-wise (the MoE's f32 accumulation), 2e-2 on the
    tensor-core prefill path."""

import numpy as np
import pytest

import vastloom_b200 as vb
from conftest import rel_err
from oracle.oracle import per_token
from vastloom_b200 import synth

pytestmark = pytest.mark.gpu


def ulp_diff(a, b):
    a = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    return int(np.max(np.abs(a - b))) if a.size else 0


def hc_params(seed, m, H):
    rng = np.random.default_rng(seed)
    mw = (2 + m) * m
    fn = (rng.standard_normal((mw, m * H)) * 0.02).astype(np.float32)
    scale = (rng.random(3) + 0.5).astype(np.float32)
    base = (rng.standard_normal(mw) * 0.1).astype(np.float32)
    norm_w = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    return fn, scale, base, norm_w


def run_case(device, oracle, cfg, T, m, iters, prefill=False, seed=0):
    spec = synth.config(cfg, "small")
    W = synth.layer_weights(spec, seed=900 + cfg)
    _, tok, logits = synth.activations(spec, T, seed=901 + cfg)
    H = spec.hidden
    x = np.random.default_rng(seed + T).standard_normal((T, m, H)).astype(np.float32)
    fn, scale, base, norm_w = hc_params(seed + m, m, H)
    eps, hc_eps = 1e-6, 1e-6
    # the oracle composition
    red, pre, post, comb = oracle.hc_pre(x, fn, scale, base, iters, eps, hc_eps)
    xn = oracle.rms_norm(red, norm_w, eps)
    moe, ridx, _ = per_token(oracle.moe_forward, W, xn, tok, logits)
    want = oracle.hc_post(moe, x, post, comb)
    layer = synth.upload_layer(device, W, max_tokens=max(T, 8))
    try:
        layer.set_hyper_connection(m, fn, scale, base, norm_w, sinkhorn_iterations=iters, norm_eps=eps, hc_eps=hc_eps)
        if prefill:
            layer.set_prefill_tokens(1)
        out = layer.forward(x, tok, logits)
        dpre, dpost, dcomb = layer.last_hyper_split(T)
        idx, *_ = layer.last_route(T)
    finally:
        layer.destroy()
        for lst in layer.matrices.values():
            for mm in lst:
                device.release_matrix(mm)
        for mm in layer.shared_matrices or ():
            device.release_matrix(mm)
    assert ulp_diff(dpre, pre) <= 1 and ulp_diff(dpost, post) <= 1 and ulp_diff(dcomb, comb) <= 1
    assert out.shape == (T, m, H) and np.all(np.isfinite(out))
    if not prefill:
        assert np.array_equal(idx, ridx)
    assert rel_err(out, want) <= (2e-2 if prefill else 1e-5), rel_err(out, want)
    return out


@pytest.mark.parametrize("cfg,T,m,iters", [(1, 5, 4, 20), (1, 37, 4, 20), (0, 9, 2, 4), (2, 3, 4, 20), (1, 1, 16, 7)])
def test_gpu_hc_layer_matches_oracle(device, oracle, cfg, T, m, iters):
    run_case(device, oracle, cfg, T, m, iters)


def test_gpu_hc_layer_prefill_path(device, oracle):
    run_case(device, oracle, 3, 64, 4, 20, prefill=True)


def test_gpu_hc_set_and_remove(device, oracle):
    """Removing the Hyper-Connection restores the plain layer (same outputs as a fresh one); bad
    descriptors are refused before anything changes."""
    spec = synth.config(1, "small")
    W = synth.layer_weights(spec, seed=5)
    x, tok, logits = synth.activations(spec, 4, seed=6)
    layer = synth.upload_layer(device, W, max_tokens=8)
    try:
        plain = layer.forward(x, tok, logits)
        fn, scale, base, norm_w = hc_params(1, 4, spec.hidden)
        bad = fn.copy()
        bad[3, 7] = np.inf
        with pytest.raises(vb.VlbError) as e:
            layer.set_hyper_connection(4, bad, scale, base, norm_w)
        assert e.value.code == "invalid_argument"
        layer.set_hyper_connection(4, fn, scale, base, norm_w)
        with pytest.raises(vb.VlbError):
            layer.set_input_norm(norm_w)
        hx = np.repeat(x[:, None, :], 4, axis=1)
        assert layer.forward(hx, tok, logits).shape == (4, 4, spec.hidden)
        layer.set_hyper_connection(0, None, None, None, None)
        assert layer.forward(x, tok, logits).tobytes() == plain.tobytes()
    finally:
        layer.destroy()
        for lst in layer.matrices.values():
            for mm in lst:
                device.release_matrix(mm)
        for mm in layer.shared_matrices or ():
            device.release_matrix(mm)
