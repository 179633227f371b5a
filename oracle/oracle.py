"""TEST INFRASTRUCTURE ONLY - ctypes bindings of the two CPU checkers.

``Oracle``     the plain-C restatement (oracle/vlb_oracle.c -> oracle/liboracle.so)
``Reference``  the vastloom reference library itself, compiled from its own sources by
               oracle/Makefile into oracle/_ref/libvlref.so, with the extern "C" shim
               oracle/ref_shim.cpp

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline leg load this module; the
product package (vastloom_b200) never does.
"""

from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libvlref.so"


def build(reference: Optional[str] = None, jobs: int = 8) -> None:
    """Builds liboracle.so, and _ref/libvlref.so when the reference tree is present."""
    args = ["make", "-C", str(HERE), f"-j{jobs}", "oracle"]
    subprocess.run(args, check=True, capture_output=True)
    from vastloom_b200.build import reference_root

    ref = Path(reference) if reference else reference_root()
    if (ref / "src" / "inference" / "ggml_quantization.cpp").exists():
        subprocess.run(["make", "-C", str(HERE), f"-j{jobs}", "ref", f"REF={ref}"], check=True,
                       capture_output=True)


def _p(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return C.c_void_p(a.ctypes.data)


class _Mat(C.Structure):
    _fields_ = [("type", C.c_uint32), ("rows", C.c_size_t), ("cols", C.c_size_t), ("data", C.c_void_p)]


_LAYER_FIELDS = [
    ("hidden", C.c_size_t), ("intermediate", C.c_size_t), ("experts", C.c_size_t),
    ("top_k", C.c_size_t), ("score", C.c_int), ("hash_routing", C.c_int),
    ("weight_after_down", C.c_int), ("route_scale", C.c_float),
    ("routed_swiglu_limit", C.c_float), ("shared_swiglu_limit", C.c_float),
    ("router", C.c_void_p), ("bias", C.c_void_p), ("tid2eid", C.c_void_p), ("vocab", C.c_size_t),
    ("w1", C.POINTER(_Mat)), ("w3", C.POINTER(_Mat)), ("w2", C.POINTER(_Mat)),
    ("shared_w1", C.POINTER(_Mat)), ("shared_w3", C.POINTER(_Mat)), ("shared_w2", C.POINTER(_Mat)),
]


class _OracleLayer(C.Structure):
    _fields_ = _LAYER_FIELDS + [("grid_iq1_s", C.c_void_p), ("grid_iq2_xxs", C.c_void_p),
                                ("grid_iq3_xxs", C.c_void_p), ("grid_iq2_s", C.c_void_p)]


class _RefLayer(C.Structure):
    _fields_ = list(_LAYER_FIELDS)


class _LayerBuilder:
    """Holds the ctypes mirror of one synthetic layer (vastloom_b200.synth.LayerWeights)."""

    def __init__(self, W, struct_type, grids: Optional[dict] = None):
        s = W.spec
        self.keep = []
        L = struct_type()
        L.hidden, L.intermediate, L.experts, L.top_k = s.hidden, s.intermediate, s.experts, s.top_k
        L.score = s.score
        L.hash_routing = 1 if s.hash_routing else 0
        L.weight_after_down = 1 if s.weight_after_down else 0
        L.route_scale = s.route_scale
        L.routed_swiglu_limit = s.routed_swiglu_limit
        L.shared_swiglu_limit = s.shared_swiglu_limit
        self.keep += [W.router, W.bias, W.tid2eid]
        L.router = W.router.ctypes.data
        L.bias = None if W.bias is None else W.bias.ctypes.data
        L.tid2eid = None if W.tid2eid is None else W.tid2eid.ctypes.data
        L.vocab = 0 if W.tid2eid is None else W.tid2eid.shape[0]
        H, I = s.hidden, s.intermediate

        def mats(lst, rows, cols):
            arr = (_Mat * len(lst))()
            for i, (t, b) in enumerate(lst):
                arr[i] = _Mat(t, rows, cols, b.ctypes.data)
                self.keep.append(b)
            self.keep.append(arr)
            return arr

        L.w1 = mats(W.w1, I, H)
        L.w3 = mats(W.w3, I, H)
        L.w2 = mats(W.w2, H, I)
        if W.shared is not None:
            sm = [mats([W.shared[0]], I, H), mats([W.shared[1]], I, H), mats([W.shared[2]], H, I)]
            L.shared_w1, L.shared_w3, L.shared_w2 = sm
        if grids is not None:
            gb = {t: np.frombuffer(v, dtype=np.uint8).copy() for t, v in grids.items()}
            self.keep.append(gb)
            L.grid_iq1_s = gb[19].ctypes.data
            L.grid_iq2_xxs = gb[16].ctypes.data
            L.grid_iq3_xxs = gb[18].ctypes.data
            if 22 in gb:
                L.grid_iq2_s = gb[22].ctypes.data
        self.layer = L


def _hc_argtypes(L, pre):
    P, SZ, F = C.c_void_p, C.c_size_t, C.c_float
    getattr(L, pre + "_hc_split_sinkhorn").argtypes = [P, P, P, SZ, SZ, SZ, F, P, P, P]
    getattr(L, pre + "_hc_pre").argtypes = [P, P, P, P, SZ, SZ, SZ, SZ, F, F, P, P, P, P]
    getattr(L, pre + "_hc_post").argtypes = [P, P, P, P, SZ, SZ, SZ, P]


def _f32(a):
    return np.ascontiguousarray(a, np.float32)


def _hc_split(lib, pre, mixes, scale, base, m, iters, eps):
    """deepseek_v4_hc_split_sinkhorn: mixes [T, (2+m)m] -> pre [T, m], post [T, m], comb [T, m, m]."""
    mixes = _f32(mixes)
    T = mixes.shape[0]
    p, q, c = np.empty((T, m), np.float32), np.empty((T, m), np.float32), np.empty((T, m, m), np.float32)
    if getattr(lib, pre + "_hc_split_sinkhorn")(_p(mixes), _p(_f32(scale)), _p(_f32(base)), T, m, iters, eps,
                                                _p(p), _p(q), _p(c)):
        raise ValueError("hc_split_sinkhorn failed")
    return p, q, c


def _hc_pre(lib, pre, x, fn, scale, base, iters, norm_eps, hc_eps):
    """deepseek_v4_hc_pre: x [T, m, W] -> reduced [T, W] and the split."""
    x = _f32(x)
    T, m, W = x.shape
    red = np.empty((T, W), np.float32)
    p, q, c = np.empty((T, m), np.float32), np.empty((T, m), np.float32), np.empty((T, m, m), np.float32)
    if getattr(lib, pre + "_hc_pre")(_p(x), _p(_f32(fn)), _p(_f32(scale)), _p(_f32(base)), T, m, W, iters,
                                     norm_eps, hc_eps, _p(red), _p(p), _p(q), _p(c)):
        raise ValueError("hc_pre failed")
    return red, p, q, c


def _hc_post(lib, pre, sub, residual, post, comb):
    """deepseek_v4_hc_post: sub [T, W], residual [T, m, W] -> [T, m, W]."""
    residual = _f32(residual)
    T, m, W = residual.shape
    out = np.empty_like(residual)
    if getattr(lib, pre + "_hc_post")(_p(_f32(sub)), _p(residual), _p(_f32(post)), _p(_f32(comb)), T, m, W, _p(out)):
        raise ValueError("hc_post failed")
    return out


class Oracle:
    """The plain-C restatement (parity checker)."""

    def __init__(self, grids: dict[int, bytes]):
        if not ORACLE_LIB.exists():
            build()
        self.lib = C.CDLL(str(ORACLE_LIB))
        self.grids = {t: np.frombuffer(v, dtype=np.uint8).copy() for t, v in grids.items()}
        self._grids_raw = grids
        L = self.lib
        P, SZ, U32, F, I = C.c_void_p, C.c_size_t, C.c_uint32, C.c_float, C.c_int
        L.vlo_fp16_to_float.restype = F
        L.vlo_fp16_to_float.argtypes = [C.c_uint16]
        L.vlo_float_to_fp16.restype = C.c_uint16
        L.vlo_float_to_fp16.argtypes = [F]
        L.vlo_fnv1a_f32.restype = C.c_uint64
        L.vlo_fnv1a_f32.argtypes = [P, SZ]
        L.vlo_fnv1a_bytes.restype = C.c_uint64
        L.vlo_fnv1a_bytes.argtypes = [P, SZ]
        L.vlo_dequantize.argtypes = [U32, P, SZ, P, P]
        L.vlo_matvec.argtypes = [U32, P, SZ, SZ, P, P, P]
        L.vlo_quantize_q8_0.argtypes = [P, SZ, SZ, SZ, P]
        L.vlo_sqrt_softplus.restype = F
        L.vlo_sqrt_softplus.argtypes = [F]
        L.vlo_sigmoid.restype = F
        L.vlo_sigmoid.argtypes = [F]
        L.vlo_router_logits.argtypes = [P, P, SZ, SZ, SZ, P]
        L.vlo_route_learned.argtypes = [P, P, SZ, SZ, SZ, F, I, P, P]
        L.vlo_route_hash.argtypes = [P, P, P, SZ, SZ, SZ, SZ, F, I, P, P]
        L.vlo_route_softmax.argtypes = [P, SZ, SZ, SZ, P, P]
        L.vlo_route_softmax_f64.argtypes = [P, SZ, SZ, SZ, I, P, P]
        L.vlo_expert_swiglu.argtypes = [P, P, P, P, P, SZ, SZ, SZ, F, P]
        L.vlo_dispatch.argtypes = [P, SZ, SZ, SZ, P, P, P]
        L.vlo_dispatch.restype = None
        L.vlo_rms_norm.argtypes = [P, P, SZ, SZ, F, P]
        _hc_argtypes(L, "vlo")
        L.vlo_moe_forward.argtypes = [C.POINTER(_OracleLayer), P, P, SZ, P, P, P, P]
        L.vlo_v4_expert_activation.argtypes = [U32, P, P, SZ, SZ, P, P, F, P, P]

    def grid(self, t):
        g = self.grids.get(t)
        return None if g is None else _p(g)

    def dequantize(self, t: int, enc: np.ndarray, n_blocks: int, block_elems: int) -> np.ndarray:
        out = np.empty(n_blocks * block_elems, np.float32)
        st = self.lib.vlo_dequantize(t, _p(enc), n_blocks, self.grid(t), _p(out))
        if st:
            raise ValueError(f"oracle dequantize failed ({st})")
        return out

    def matvec(self, t: int, enc: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(rows, np.float32)
        st = self.lib.vlo_matvec(t, _p(enc), rows, cols, _p(x), _p(y), self.grid(t))
        if st:
            raise ValueError(f"oracle matvec failed ({st})")
        return y

    def quantize_q8_0(self, m: np.ndarray, rows: int, lc: int, sc: int) -> np.ndarray:
        m = np.ascontiguousarray(m, np.float32)
        out = np.empty(rows * (sc // 32) * 34, np.uint8)
        if self.lib.vlo_quantize_q8_0(_p(m), rows, lc, sc, _p(out)):
            raise ValueError("oracle Q8_0 encode failed")
        return out

    def router_logits(self, x, w):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        T, H = x.shape
        E = w.shape[0]
        out = np.empty((T, E), np.float32)
        self.lib.vlo_router_logits(_p(x), _p(w), T, H, E, _p(out))
        return out

    def route_learned(self, logits, bias, k, route_scale, score=0):
        logits = np.ascontiguousarray(logits, np.float32)
        T, E = logits.shape
        idx = np.empty((T, k), np.uint32)
        w = np.empty((T, k), np.float32)
        bias = np.ascontiguousarray(bias, np.float32)
        if self.lib.vlo_route_learned(_p(logits), _p(bias), T, E, k, route_scale, score, _p(idx), _p(w)):
            raise ValueError("oracle route failed")
        return idx, w

    def route_hash(self, logits, token_ids, table, k, route_scale, score=0):
        logits = np.ascontiguousarray(logits, np.float32)
        T, E = logits.shape
        token_ids = np.ascontiguousarray(token_ids, np.uint32)
        table = np.ascontiguousarray(table, np.uint32)
        idx = np.empty((T, k), np.uint32)
        w = np.empty((T, k), np.float32)
        if self.lib.vlo_route_hash(_p(logits), _p(token_ids), _p(table), T, table.size // k, E, k,
                                   route_scale, score, _p(idx), _p(w)):
            raise ValueError("oracle hash route failed")
        return idx, w

    def route_softmax(self, logits, k):
        logits = np.ascontiguousarray(logits, np.float32)
        T, E = logits.shape
        idx = np.empty((T, k), np.uint32)
        w = np.empty((T, k), np.float32)
        self.lib.vlo_route_softmax(_p(logits), T, E, k, _p(idx), _p(w))
        return idx, w

    def route_softmax_f64(self, logits, k, norm=True):
        """qwen38_moe_route on given logits (f64 softmax, top-k, optional norm_topk_prob)."""
        logits = np.ascontiguousarray(logits, np.float32)
        T, E = logits.shape
        idx = np.empty((T, k), np.uint32)
        w = np.empty((T, k), np.float32)
        if self.lib.vlo_route_softmax_f64(_p(logits), T, E, k, 1 if norm else 0, _p(idx), _p(w)):
            raise ValueError("oracle f64 softmax route failed")
        return idx, w

    def expert_swiglu(self, x, gate_w, down_w, up_w, routing_weights, limit):
        """deepseek_v4_expert_swiglu on float weights (gate/up [I, H], down [H, I])."""
        x = np.ascontiguousarray(x, np.float32)
        T, H = x.shape
        I = gate_w.shape[0]
        out = np.empty((T, H), np.float32)
        rw = None if routing_weights is None else np.ascontiguousarray(routing_weights, np.float32)
        if self.lib.vlo_expert_swiglu(_p(x), _p(np.ascontiguousarray(gate_w, np.float32)),
                                      _p(np.ascontiguousarray(down_w, np.float32)),
                                      _p(np.ascontiguousarray(up_w, np.float32)), _p(rw), T, H, I, limit, _p(out)):
            raise ValueError("oracle expert_swiglu failed")
        return out

    def dispatch(self, idx, E):
        idx = np.ascontiguousarray(idx, np.uint32)
        T, k = idx.shape
        off = np.empty(E + 1, np.uint32)
        pt = np.empty(T * k, np.uint32)
        ps = np.empty(T * k, np.uint32)
        self.lib.vlo_dispatch(_p(idx), T, k, E, _p(off), _p(pt), _p(ps))
        return off, pt, ps

    def v4_expert_activation(self, t, w1, w3, I, H, x, route_w, limit):
        """Down-projection input of one DeepSeek V4 expert for one token (f32 [I])."""
        x = np.ascontiguousarray(x, np.float32)
        act = np.empty(I, np.float32)
        rw = None if route_w is None else np.array([route_w], np.float32)
        if self.lib.vlo_v4_expert_activation(t, _p(w1), _p(w3), I, H, _p(x), _p(rw), limit, self.grid(t), _p(act)):
            raise ValueError("oracle expert activation failed")
        return act

    def hc_split_sinkhorn(self, mixes, scale, base, m, iters, eps):
        return _hc_split(self.lib, "vlo", mixes, scale, base, m, iters, eps)

    def hc_pre(self, x, fn, scale, base, iters, norm_eps, hc_eps):
        return _hc_pre(self.lib, "vlo", x, fn, scale, base, iters, norm_eps, hc_eps)

    def hc_post(self, sub, residual, post, comb):
        return _hc_post(self.lib, "vlo", sub, residual, post, comb)

    def rms_norm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        rows, width = x.shape
        out = np.empty_like(x)
        self.lib.vlo_rms_norm(_p(x), _p(np.ascontiguousarray(w, np.float32)), rows, width, eps, _p(out))
        return out

    def moe_forward(self, W, x, token_ids=None, logits=None):
        b = _LayerBuilder(W, _OracleLayer, self._grids_raw)
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        k = W.spec.top_k
        out = np.empty((T, W.spec.hidden), np.float32)
        idx = np.empty((T, k), np.uint32)
        w = np.empty((T, k), np.float32)
        tok = None if token_ids is None else np.ascontiguousarray(token_ids, np.uint32)
        lg = None if logits is None else np.ascontiguousarray(logits, np.float32)
        st = self.lib.vlo_moe_forward(C.byref(b.layer), _p(x), _p(tok), T, _p(lg), _p(out), _p(idx), _p(w))
        if st:
            raise ValueError(f"oracle moe_forward failed ({st})")
        return out, idx, w


def per_token(forward, W, x, token_ids=None, logits=None, threads: int = 0):
    """Runs a layer forward one token at a time on a thread pool and stacks the results.

    Every reference router and layer loop treats the tokens of a batch independently (per-token
    routing; each token's output is the sum of its own expert outputs in a fixed order), so the
    per-token results equal the batched call's. ctypes releases the GIL during the foreign call,
    so the threads run in parallel; this keeps full-size parity checks to seconds."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    T = x.shape[0]
    n = threads or min(T, os.cpu_count() or 1)

    def one(t):
        tok = None if token_ids is None else token_ids[t:t + 1]
        lg = None if logits is None else logits[t:t + 1]
        return forward(W, x[t:t + 1], tok, lg)

    with ThreadPoolExecutor(max_workers=max(1, n)) as ex:
        parts = list(ex.map(one, range(T)))
    return (np.concatenate([p[0] for p in parts]), np.concatenate([p[1] for p in parts]),
            np.concatenate([p[2] for p in parts]))


class Reference:
    """The vastloom reference compiled from its sources (oracle/_ref)."""

    @staticmethod
    def available() -> bool:
        return REF_LIB.exists()

    def __init__(self):
        if not REF_LIB.exists():
            raise FileNotFoundError(f"{REF_LIB} is not built (oracle/Makefile ref)")
        self.lib = C.CDLL(str(REF_LIB))
        L = self.lib
        P, SZ, U32, F, I = C.c_void_p, C.c_size_t, C.c_uint32, C.c_float, C.c_int
        L.vlr_grid.restype = SZ
        L.vlr_grid.argtypes = [U32, P, SZ]
        L.vlr_dequantize.argtypes = [U32, P, SZ, P, SZ]
        L.vlr_matvec.argtypes = [U32, P, SZ, SZ, P, P, C.c_uint]
        L.vlr_quantize_q8_0.argtypes = [P, SZ, SZ, SZ, P]
        L.vlr_route_learned.argtypes = [P, P, SZ, SZ, SZ, F, P, P]
        L.vlr_route_hash.argtypes = [P, P, P, SZ, SZ, SZ, SZ, F, P, P]
        L.vlr_rms_norm.argtypes = [P, P, SZ, SZ, F, P]
        _hc_argtypes(L, "vlr")
        L.vlr_moe_forward.argtypes = [C.POINTER(_RefLayer), P, P, SZ, P, P, P, P, C.c_uint]
        L.vlr_qwen_route.argtypes = [P, P, SZ, SZ, SZ, SZ, I, P, P, P]
        L.vlr_expert_swiglu.argtypes = [P, P, P, P, P, SZ, SZ, SZ, F, P]
        L.vlr_graph_prefill.argtypes = [P, SZ, P, SZ, P, SZ, P, SZ, P, P, SZ, P, P, SZ, SZ,
                                        C.POINTER(SZ), C.c_char_p, SZ]

    def grid(self, t: int) -> bytes:
        n = self.lib.vlr_grid(t, None, 0)
        buf = (C.c_char * n)()
        self.lib.vlr_grid(t, C.cast(buf, C.c_void_p), n)
        return bytes(buf)

    def dequantize(self, t, enc, n_out):
        out = np.empty(n_out, np.float32)
        if self.lib.vlr_dequantize(t, _p(enc), enc.nbytes, _p(out), n_out):
            raise ValueError("reference dequantize failed")
        return out

    def matvec(self, t, enc, rows, cols, x, threads=1):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(rows, np.float32)
        if self.lib.vlr_matvec(t, _p(enc), rows, cols, _p(x), _p(y), threads):
            raise ValueError("reference matvec failed")
        return y

    def quantize_q8_0(self, m, rows, lc, sc):
        m = np.ascontiguousarray(m, np.float32)
        out = np.empty(rows * (sc // 32) * 34, np.uint8)
        if self.lib.vlr_quantize_q8_0(_p(m), rows, lc, sc, _p(out)):
            raise ValueError("reference Q8_0 encode failed")
        return out

    def route_learned(self, logits, bias, k, route_scale):
        logits = np.ascontiguousarray(logits, np.float32)
        T, E = logits.shape
        idx = np.empty((T, k), np.uint32)
        w = np.empty((T, k), np.float32)
        if self.lib.vlr_route_learned(_p(logits), _p(np.ascontiguousarray(bias, np.float32)), T, E, k,
                                      route_scale, _p(idx), _p(w)):
            raise ValueError("reference route failed")
        return idx, w

    def route_hash(self, logits, token_ids, table, k, route_scale):
        logits = np.ascontiguousarray(logits, np.float32)
        T, E = logits.shape
        table = np.ascontiguousarray(table, np.uint32)
        idx = np.empty((T, k), np.uint32)
        w = np.empty((T, k), np.float32)
        if self.lib.vlr_route_hash(_p(logits), _p(np.ascontiguousarray(token_ids, np.uint32)), _p(table),
                                   T, table.size // k, E, k, route_scale, _p(idx), _p(w)):
            raise ValueError("reference hash route failed")
        return idx, w

    def qwen_route(self, hidden, router, k, norm=True):
        """qwen38_moe_route per token: returns (logits, indices, weights)."""
        hidden = np.ascontiguousarray(hidden, np.float32)
        router = np.ascontiguousarray(router, np.float32)
        T, H = hidden.shape
        E = router.shape[0]
        lg = np.empty((T, E), np.float32)
        idx = np.empty((T, k), np.uint32)
        w = np.empty((T, k), np.float32)
        if self.lib.vlr_qwen_route(_p(hidden), _p(router), T, H, E, k, 1 if norm else 0, _p(lg), _p(idx), _p(w)):
            raise ValueError("reference qwen route failed")
        return lg, idx, w

    def expert_swiglu(self, x, gate_w, down_w, up_w, routing_weights, limit):
        x = np.ascontiguousarray(x, np.float32)
        T, H = x.shape
        I = gate_w.shape[0]
        out = np.empty((T, H), np.float32)
        rw = None if routing_weights is None else np.ascontiguousarray(routing_weights, np.float32)
        if self.lib.vlr_expert_swiglu(_p(x), _p(np.ascontiguousarray(gate_w, np.float32)),
                                      _p(np.ascontiguousarray(down_w, np.float32)),
                                      _p(np.ascontiguousarray(up_w, np.float32)), _p(rw), T, H, I, limit, _p(out)):
            raise ValueError("reference expert_swiglu failed")
        return out

    def hc_split_sinkhorn(self, mixes, scale, base, m, iters, eps):
        return _hc_split(self.lib, "vlr", mixes, scale, base, m, iters, eps)

    def hc_pre(self, x, fn, scale, base, iters, norm_eps, hc_eps):
        return _hc_pre(self.lib, "vlr", x, fn, scale, base, iters, norm_eps, hc_eps)

    def hc_post(self, sub, residual, post, comb):
        return _hc_post(self.lib, "vlr", sub, residual, post, comb)

    def rms_norm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        if self.lib.vlr_rms_norm(_p(x), _p(np.ascontiguousarray(w, np.float32)), x.shape[0], x.shape[1], eps, _p(out)):
            raise ValueError("reference rms_norm failed")
        return out

    def moe_forward(self, W, x, token_ids=None, logits=None, threads=1):
        b = _LayerBuilder(W, _RefLayer)
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        k = W.spec.top_k
        out = np.empty((T, W.spec.hidden), np.float32)
        idx = np.empty((T, k), np.uint32)
        w = np.empty((T, k), np.float32)
        tok = None if token_ids is None else np.ascontiguousarray(token_ids, np.uint32)
        lg = None if logits is None else np.ascontiguousarray(logits, np.float32)
        st = self.lib.vlr_moe_forward(C.byref(b.layer), _p(x), _p(tok), T, _p(lg), _p(out), _p(idx), _p(w), threads)
        if st:
            raise ValueError(f"reference moe_forward failed ({st})")
        return out, idx, w

    def graph_prefill(self, config: dict, tensors: dict, packed: dict, token_ids, rec_cols: int = 64,
                      rec_cap: int = 4096):
        """deepseek_v4_reference_prefill over a reduced graph (deepseek_v4_graph.cpp:4651).

        config: the fixture's configuration (list-valued fields as lists); tensors: name ->
        (numpy f32 or u32 array); packed: name -> (ggml type, rows, logical columns, storage
        columns, encoded uint8 bytes, cache identity). Returns (logits, [(indices, weights)] per
        routed layer, main layers first, then the offered rows as (identities, inputs [n x rec_cols]))."""
        entries, keep = [], []
        for key, v in config.items():
            for item in (v if isinstance(v, list) else [v]):
                kb = key.encode()
                keep.append(kb)
                entries.append((kb, float(item)))
        cfg = (_GraphConfigEntry * len(entries))(*[_GraphConfigEntry(k, v) for k, v in entries])
        items = []
        for name, arr in tensors.items():
            a = np.ascontiguousarray(arr)
            kind = 0 if a.dtype == np.float32 else 1
            if kind == 1:
                a = np.ascontiguousarray(a, np.uint32)
            nb = name.encode()
            keep += [a, nb]
            items.append(_GraphTensor(nb, kind, a.ctypes.data, a.size, 0, 0, 0, 0, 0))
        for name, (t, rows, lc, sc, enc, ident) in packed.items():
            e = np.ascontiguousarray(enc, np.uint8)
            nb = name.encode()
            keep += [e, nb]
            items.append(_GraphTensor(nb, 2, e.ctypes.data, e.size, t, rows, lc, sc, ident))
        arr = (_GraphTensor * len(items))(*items)
        tok = np.ascontiguousarray(token_ids, np.uint32)
        T = tok.size
        V = int(config["vocabulary_size"])
        k = int(config["experts_per_token"])
        n_layers = int(config["layers"]) + int(config.get("mtp_layers", 0))
        logits = np.empty(V, np.float32)
        ridx = np.empty((n_layers, T, k), np.uint32)
        rw = np.empty((n_layers, T, k), np.float32)
        ids = np.zeros(rec_cap, np.uint64)
        rows = np.zeros((rec_cap, rec_cols), np.float32)
        n = C.c_size_t(0)
        err = C.create_string_buffer(512)
        st = self.lib.vlr_graph_prefill(cfg, len(entries), arr, len(items), _p(tok), T, _p(logits), V,
                                        _p(ridx), _p(rw), n_layers, _p(ids), _p(rows), rec_cols, rec_cap,
                                        C.byref(n), err, len(err))
        if st:
            raise ValueError(f"reference prefill failed: {err.value.decode()}")
        if n.value > rec_cap:
            raise ValueError(f"{n.value} offered rows exceed the recording capacity {rec_cap}")
        return logits, [(ridx[i], rw[i]) for i in range(n_layers)], (ids[: n.value], rows[: n.value])


class _GraphConfigEntry(C.Structure):
    _fields_ = [("key", C.c_char_p), ("value", C.c_double)]


class _GraphTensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("kind", C.c_int), ("data", C.c_void_p), ("n", C.c_size_t),
                ("ggml_type", C.c_uint32), ("rows", C.c_size_t), ("logical_columns", C.c_size_t),
                ("storage_columns", C.c_size_t), ("identity", C.c_uint64)]
