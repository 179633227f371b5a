"""vlb_route_device_noalloc: the router for callers that cannot allocate device memory (a runtime
whose memory governor refuses new reservations, callers that may not call cudaMalloc, decode loops
that cannot take the synchronisation of cudaMalloc/cudaFree). Its scratch is a fixed array inside
the library instead of an allocation; it is called from ordinary host code (it synchronises its
stream).

Called through the C ABI and compared with the allocating entry point, vlb_route_device, and with
the CPU oracle, on two calls in a row with different inputs (the shared scratch keeps the previous
call's contents, so the second call checks that nothing leaks between calls). This file is
collected last on purpose.
"""

import ctypes as C

import numpy as np
import pytest

import vastloom_b200 as vb

pytestmark = pytest.mark.gpu


def _call_noalloc(dev, logits_b, bias_b, tok_b, tab_b, vocab, T, E, k, score, scale, idx_b, w_b):
    """One vlb_route_device_noalloc call on dev's ordinal and stream; returns (status, message)."""
    st = dev.lib.vlb_route_device_noalloc(
        dev.ordinal, score, 1 if tab_b else 0, logits_b.ptr, bias_b.ptr if bias_b else None,
        tok_b.ptr if tok_b else None, tab_b.ptr if tab_b else None, vocab, T, E, k, scale,
        idx_b.ptr, w_b.ptr, C.c_void_p(dev.stream))
    if st == 0:
        return st, ""
    buf = C.create_string_buffer(512)
    dev.lib.vlb_thread_error(buf, 512)
    return st, buf.value.decode()


def _noalloc_route(dev, logits_b, bias_b, tok_b, tab_b, vocab, T, E, k, score, scale):
    idx_b = dev.buffer(T * k * 4, "test-idx")
    w_b = dev.buffer(T * k * 4, "test-w")
    try:
        st, msg = _call_noalloc(dev, logits_b, bias_b, tok_b, tab_b, vocab, T, E, k, score, scale, idx_b, w_b)
        if st != 0:
            raise vb.VlbError(st, msg)
        return (idx_b.download(np.uint32, T * k).reshape(T, k),
                w_b.download(np.float32, T * k).reshape(T, k))
    finally:
        idx_b.free()
        w_b.free()


def _ulp(a, b):
    a = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    return int(np.max(np.abs(a - b)))


@pytest.mark.parametrize("score", [vb.SCORE_SQRT_SOFTPLUS, vb.SCORE_SIGMOID, vb.SCORE_SOFTMAX,
                                   vb.SCORE_SOFTMAX_F64_NORM])
def test_noalloc_route_matches_allocating_route_twice(device, oracle, score):
    rng = np.random.default_rng(1234 + score)
    for T, E, k in ((64, 256, 8), (7, 64, 4)):  # two calls in a row, different sizes and inputs
        logits = rng.standard_normal((T, E)).astype(np.float32)
        bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
        use_bias = score in (vb.SCORE_SQRT_SOFTPLUS, vb.SCORE_SIGMOID)
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
        if score == vb.SCORE_SOFTMAX:
            ri, rw = oracle.route_softmax(logits, k)
        elif score == vb.SCORE_SOFTMAX_F64_NORM:
            ri, rw = oracle.route_softmax_f64(logits, k, norm=True)
        else:
            ri, rw = oracle.route_learned(logits, bias, k, 1.5, score)
        assert np.array_equal(idx, ri) and _ulp(w, rw) <= (2 if score == vb.SCORE_SOFTMAX else 1)


def test_noalloc_route_on_another_device_restores_the_current_one():
    """With two GPUs: device 0 current, a call for ordinal 1 runs there (its own copy of the fixed
    array, looked up on its first call) and leaves device 0 current. The handle's own calls
    (allocations, copies) make the handle's device current, so every buffer is allocated first
    and device 0 is made current right before the no-allocation call."""
    if vb.device_count() < 2:
        pytest.skip("needs two GPUs")
    import ctypes

    rt = ctypes.CDLL("libcudart.so.12")  # the runtime instance libvlb200.so is linked against
    cur = ctypes.c_int(-1)
    T, E, k = 9, 64, 4
    with vb.Device(1) as dev1:
        rng = np.random.default_rng(5)
        logits = rng.standard_normal((T, E)).astype(np.float32)
        bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
        want_idx, want_w = dev1.route(logits, k, 1.0, bias=bias)
        lb, bb = dev1.to_device(logits), dev1.to_device(bias)
        idx_b, w_b = dev1.buffer(T * k * 4, "test-idx"), dev1.buffer(T * k * 4, "test-w")
        try:
            assert rt.cudaSetDevice(0) == 0
            st, msg = _call_noalloc(dev1, lb, bb, None, None, 0, T, E, k, vb.SCORE_SQRT_SOFTPLUS, 1.0, idx_b, w_b)
            assert rt.cudaGetDevice(ctypes.byref(cur)) == 0 and cur.value == 0
            assert st == 0, msg
            idx = idx_b.download(np.uint32, T * k).reshape(T, k)
            w = w_b.download(np.float32, T * k).reshape(T, k)
        finally:
            for b in (lb, bb, idx_b, w_b):
                b.free()
        assert np.array_equal(idx, want_idx) and w.tobytes() == want_w.tobytes()


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
