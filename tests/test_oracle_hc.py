"""The Hyper-Connection restatement (deepseek_v4_hc_split_sinkhorn / hc_pre / hc_post,
deepseek_v4_reference.cpp:387-610) pinned two ways: against the reference's own operator fixture
(tests/fixtures/deepseek_v4_operators.json "hyper_connection", consumed by the reference at
tests/test_main.cpp:4519-4541 within its absolute tolerance 3e-5) and bit-for-bit against the
reference compiled from its sources on random inputs."""

import json
from pathlib import Path

import numpy as np
import pytest

GOLDEN = json.loads((Path(__file__).parent / "golden" / "deepseek_v4_operators.json").read_text())


def _fixture():
    hc = GOLDEN["hyper_connection"]
    T, m, W = hc["tokens"], hc["multiplier"], hc["width"]
    x = np.array(hc["input"], np.float32).reshape(T, m, W)
    fn = np.array(hc["mixing_weight"], np.float32)
    return hc, T, m, W, x, fn


def _impls(oracle, request):
    out = [("oracle", oracle)]
    from oracle.oracle import Reference

    if Reference.available():
        out.append(("reference", request.getfixturevalue("reference")))
    return out


def test_hc_matches_reference_fixture(oracle, request):
    hc, T, m, W, x, fn = _fixture()
    tol = GOLDEN["absolute_tolerance"]
    for _name, impl in _impls(oracle, request):
        red, pre, post, comb = impl.hc_pre(x, fn, hc["scale"], hc["base"], hc["sinkhorn_iterations"],
                                           hc["norm_epsilon"], hc["hc_epsilon"])
        assert np.max(np.abs(red.reshape(-1) - hc["expected_reduced"])) <= tol
        assert np.max(np.abs(pre.reshape(-1) - hc["expected_pre"])) <= tol
        assert np.max(np.abs(post.reshape(-1) - hc["expected_post"])) <= tol
        assert np.max(np.abs(comb.reshape(-1) - hc["expected_combination"])) <= tol
        sub = np.array(hc["sublayer"], np.float32).reshape(T, W)
        out = impl.hc_post(sub, x, post, comb)
        assert np.max(np.abs(out.reshape(-1) - hc["expected_output"])) <= tol


def hc_case(seed, T, m, W):
    rng = np.random.default_rng(seed)
    mw = (2 + m) * m
    x = rng.standard_normal((T, m, W)).astype(np.float32)
    fn = (rng.standard_normal((mw, m * W)) * 0.05).astype(np.float32)
    scale = (rng.random(3) + 0.5).astype(np.float32)
    base = (rng.standard_normal(mw) * 0.1).astype(np.float32)
    sub = rng.standard_normal((T, W)).astype(np.float32)
    return x, fn, scale, base, sub


@pytest.mark.parametrize("T,m,W,iters", [(5, 4, 64, 20), (3, 2, 48, 4), (2, 16, 8, 7), (1, 1, 32, 1)])
def test_hc_bit_identical_to_reference(oracle, reference, T, m, W, iters):
    x, fn, scale, base, sub = hc_case(T * 100 + m, T, m, W)
    a = oracle.hc_pre(x, fn, scale, base, iters, 1e-6, 1e-6)
    b = reference.hc_pre(x, fn, scale, base, iters, 1e-6, 1e-6)
    for u, v in zip(a, b):
        assert u.tobytes() == v.tobytes()
    assert oracle.hc_post(sub, x, a[2], a[3]).tobytes() == reference.hc_post(sub, x, b[2], b[3]).tobytes()
    mixes = np.random.default_rng(T).standard_normal((T, (2 + m) * m)).astype(np.float32)
    for u, v in zip(oracle.hc_split_sinkhorn(mixes, scale, base, m, iters, 1e-6),
                    reference.hc_split_sinkhorn(mixes, scale, base, m, iters, 1e-6)):
        assert u.tobytes() == v.tobytes()


def test_hc_rejects_invalid_dimensions(oracle):
    x, fn, scale, base, _ = hc_case(1, 2, 2, 8)
    with pytest.raises(ValueError):
        oracle.hc_pre(x, fn, scale, base, 0, 1e-6, 1e-6)
    with pytest.raises(ValueError):
        oracle.hc_split_sinkhorn(np.zeros((1, 8), np.float32), scale, base[:8], 2, 0, 1e-6)
