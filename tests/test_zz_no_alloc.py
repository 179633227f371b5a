"""vlb_route_device_noalloc: the router for callers that cannot allocate device memory (code in a
CUDA host callback, a runtime whose memory governor refuses new reservations, decode loops that
cannot take the synchronisation of cudaMalloc/cudaFree). Its scratch is a fixed array inside the
library instead of a per-call allocation.

Called through the C ABI and compared with the allocating entry point, vlb_route_device, on two
calls in a row with different inputs (the shared scratch keeps the previous call's contents, so
the second call checks that nothing leaks between calls). This file is collected last on purpose.
"""

import ctypes as C

import numpy as np
import pytest

import vastloom_b200 as vb

pytestmark = pytest.mark.gpu


def _noalloc_route(dev, logits_b, bias_b, tok_b, tab_b, vocab, T, E, k, score, scale):
    idx_b = dev.buffer(T * k * 4, "test-idx")
    w_b = dev.buffer(T * k * 4, "test-w")
    try:
        st = dev.lib.vlb_route_device_noalloc(
            dev.ordinal, score, 1 if tab_b else 0, logits_b.ptr, bias_b.ptr if bias_b else None,
            tok_b.ptr if tok_b else None, tab_b.ptr if tab_b else None, vocab, T, E, k, scale,
            idx_b.ptr, w_b.ptr, C.c_void_p(dev.stream))
        if st != 0:
            buf = C.create_string_buffer(512)
            dev.lib.vlb_thread_error(buf, 512)
            raise vb.VlbError(st, buf.value.decode())
        return (idx_b.download(np.uint32, T * k).reshape(T, k),
                w_b.download(np.float32, T * k).reshape(T, k))
    finally:
        idx_b.free()
        w_b.free()


@pytest.mark.parametrize("score", [vb.SCORE_SQRT_SOFTPLUS, vb.SCORE_SOFTMAX])
def test_noalloc_route_matches_allocating_route_twice(device, score):
    rng = np.random.default_rng(1234 + score)
    for T, E, k in ((64, 256, 8), (7, 64, 4)):  # two calls in a row, different sizes and inputs
        logits = rng.standard_normal((T, E)).astype(np.float32)
        bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
        use_bias = score != vb.SCORE_SOFTMAX
        want_idx, want_w = device.route(logits, k, 1.5, score=score, bias=bias if use_bias else None)
        lb = device.to_device(logits, "test-logits")
        bb = device.to_device(bias, "test-bias") if use_bias else None
        try:
            idx, w = _noalloc_route(device, lb, bb, None, None, 0, T, E, k, score, 1.5)
        finally:
            lb.free()
            if bb:
                bb.free()
        assert np.array_equal(idx, want_idx)
        assert w.tobytes() == want_w.tobytes()


def test_noalloc_hash_route_and_size_limit(device):
    rng = np.random.default_rng(99)
    T, E, k, V = 5, 256, 6, 1000
    logits = np.zeros((T, E), np.float32)
    table = np.argsort(rng.random((V, E)), axis=1)[:, :k].astype(np.uint32)
    tok = rng.integers(0, V, T).astype(np.uint32)
    want_idx, want_w = device.route(logits, k, 1.0, token_ids=tok, tid2eid=table)
    lb, tb, kb = device.to_device(logits), device.to_device(tok), device.to_device(table)
    try:
        for _ in range(2):
            idx, w = _noalloc_route(device, lb, None, tb, kb, V, T, E, k, vb.SCORE_SQRT_SOFTPLUS, 1.0)
            assert np.array_equal(idx, want_idx) and w.tobytes() == want_w.tobytes()
        # beyond the fixed scratch: a clear error, nothing launched
        big = 262_080 // E + 1
        with pytest.raises(vb.VlbError) as e:
            _noalloc_route(device, lb, None, None, None, 0, big, E, k, vb.SCORE_SQRT_SOFTPLUS, 1.0)
        assert e.value.code == "resource_exhausted" and "at most 262080" in str(e.value)
    finally:
        for b in (lb, tb, kb):
            b.free()
