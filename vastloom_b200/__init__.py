"""vastloom_b200 - B200 (sm_100a) MoE routed-expert path behind the vlb200 C ABI.

This package is the Python host mirror of vastloom's operator surface for the routed-expert hot
path. Every call goes through the C ABI of ``libvlb200.so`` (``include/vlb200.h``); there is no
CPU fallback: importing works without a GPU, but opening a device fails loudly when the CUDA
library or a B200 is missing.

Reference interfaces mirrored here (vastloom source paths):
  * ``Device.matvec``            DeepseekV4MatvecAccelerator::matvec
                                 (include/vastloom/inference/deepseek_v4_reference.hpp:440-451)
  * ``Device.dequantize``        dequantize_q8_0/_iq2_xxs/_iq3_xxs/_iq1_s
                                 (include/vastloom/inference/ggml_quantization.hpp:98-297)
  * ``Device.route``             deepseek_v4_route_learned_logits / _hash_logits
                                 (include/vastloom/inference/deepseek_v4_reference.hpp:634-650)
  * ``MoeLayer.forward``         moe_forward (src/inference/deepseek_v4_graph.cpp:1902-2274) and
                                 the OLMoE layer loop (src/inference/olmoe_runtime.cpp:1119-1290)
Errors raise ``VlbError`` whose ``code`` names the reference ErrorCode
(include/vastloom/core/status.hpp:10-21).
"""

from __future__ import annotations

import ctypes as C
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Optional, Sequence

import numpy as np

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libvlb200.so"
GRIDS_PATH = _PKG / "data" / "iq_grids.bin"

TYPE_F32 = 0
TYPE_Q8_0 = 8
TYPE_IQ2_XXS = 16
TYPE_IQ3_XXS = 18
TYPE_IQ1_S = 19
TYPE_Q4_K = 12
TYPE_Q5_K = 13
TYPE_Q6_K = 14
TYPE_IQ2_S = 22
TYPE_MXFP4 = 39

SCORE_SQRT_SOFTPLUS = 0
SCORE_SIGMOID = 1
SCORE_SOFTMAX = 2
SCORE_SOFTMAX_F64 = 3       # Qwen router (qwen38_moe_route), norm_topk_prob = false
SCORE_SOFTMAX_F64_NORM = 4  # Qwen router with norm_topk_prob = true

# (weights per block, ggml block bytes) - ggml_quantization.hpp:12-31
BLOCK_LAYOUT = {
    TYPE_Q8_0: (32, 34),
    TYPE_IQ2_XXS: (256, 66),
    TYPE_IQ3_XXS: (256, 98),
    TYPE_IQ1_S: (256, 50),
    TYPE_Q4_K: (256, 144),
    TYPE_Q5_K: (256, 176),
    TYPE_Q6_K: (256, 210),
    TYPE_IQ2_S: (256, 82),
    TYPE_MXFP4: (32, 17),
}

ERROR_CODES = {
    0: "ok",
    1: "invalid_argument",
    2: "invalid_format",
    3: "not_found",
    4: "permission_denied",
    5: "io_error",
    6: "integrity_error",
    7: "unsafe_path",
    8: "unsupported",
    9: "resource_exhausted",
    10: "internal_error",
    100: "declined",
}


class VlbError(RuntimeError):
    def __init__(self, status: int, message: str):
        self.status = status
        self.code = ERROR_CODES.get(status, f"status_{status}")
        super().__init__(f"{self.code}: {message}")


def matrix_bytes(ggml_type: int, rows: int, cols: int) -> int:
    be, bb = BLOCK_LAYOUT[ggml_type]
    if cols % be:
        raise ValueError("columns must be a multiple of the block size")
    return rows * (cols // be) * bb


class _DeviceInfo(C.Structure):
    _fields_ = [
        ("ordinal", C.c_int),
        ("sm_count", C.c_int),
        ("cc_major", C.c_int),
        ("cc_minor", C.c_int),
        ("total_bytes", C.c_uint64),
        ("free_bytes", C.c_uint64),
        ("name", C.c_char * 96),
    ]


RESERVE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_uint64, C.c_char_p)
RELEASE_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_uint64, C.c_char_p)


class _Governor(C.Structure):
    _fields_ = [("ctx", C.c_void_p), ("reserve", RESERVE_FN), ("release", RELEASE_FN)]


class _RecordTensor(C.Structure):
    _fields_ = [("cache_identity", C.c_uint64), ("ggml_type", C.c_uint32), ("reserved0", C.c_uint32),
                ("rows", C.c_uint64), ("storage_cols", C.c_uint64), ("offset", C.c_uint64),
                ("bytes", C.c_uint64)]


class _HcDesc(C.Structure):
    _fields_ = [("multiplier", C.c_uint32), ("sinkhorn_iterations", C.c_uint32), ("norm_epsilon", C.c_float),
                ("hc_epsilon", C.c_float), ("mixing_weight", C.c_void_p), ("scale", C.c_void_p),
                ("base", C.c_void_p), ("norm_weight", C.c_void_p)]


class _LayerDesc(C.Structure):
    _fields_ = [
        ("hidden", C.c_uint32),
        ("intermediate", C.c_uint32),
        ("experts", C.c_uint32),
        ("top_k", C.c_uint32),
        ("score", C.c_int),
        ("hash_routing", C.c_int),
        ("weight_after_down", C.c_int),
        ("route_scale", C.c_float),
        ("routed_swiglu_limit", C.c_float),
        ("shared_swiglu_limit", C.c_float),
        ("max_tokens", C.c_uint32),
        ("vocab", C.c_uint32),
        ("router", C.c_void_p),
        ("bias", C.c_void_p),
        ("tid2eid", C.c_void_p),
        ("w1", C.c_void_p),
        ("w3", C.c_void_p),
        ("w2", C.c_void_p),
        ("shared_w1", C.c_void_p),
        ("shared_w3", C.c_void_p),
        ("shared_w2", C.c_void_p),
    ]


_lib: Optional[C.CDLL] = None

# exported symbols of include/vlb200.h (checked by the CPU test suite)
EXPORTS = (
    "vlb_abi_version vlb_thread_error vlb_device_count vlb_probe vlb_open vlb_close "
    "vlb_last_error vlb_stream vlb_synchronize vlb_set_codebook vlb_alloc vlb_free "
    "vlb_memcpy_h2d vlb_memcpy_d2h vlb_allocated_bytes vlb_upload_matrix vlb_release_matrix "
    "vlb_matrix_bytes vlb_matvec vlb_matvec_device vlb_dequantize_device vlb_layer_create "
    "vlb_layer_destroy vlb_layer_forward_device vlb_layer_forward vlb_layer_last_route "
    "vlb_layer_last_weight_bytes vlb_layer_set_profiling vlb_layer_phase_times vlb_layer_set_prefill_tokens "
    "vlb_layer_prefill_tokens vlb_layer_set_input_norm vlb_layer_forward_routes_device vlb_layer_status vlb_ep_workspace_bytes "
    "vlb_ep_plan_device vlb_ep_plan_half_device vlb_ep_pack_half_device vlb_ep_combine_half_device vlb_layer_forward_rows_half_device vlb_ep_combine_device vlb_route_device vlb_route_device_noalloc vlb_router_logits_device vlb_rms_norm_device "
    "vlb_ep_nccl_version vlb_ep_unique_id vlb_ep_comm_init vlb_ep_comm_destroy vlb_ep_comm_abort "
    "vlb_ep_all_to_all_device vlb_ep_layer_create vlb_ep_layer_destroy vlb_ep_forward_device vlb_ep_last_phases "
    "vlb_upload_record_async vlb_upload_query vlb_upload_finish vlb_host_alloc vlb_host_free "
    "vlb_layer_set_hyper_connection vlb_layer_last_hyper_split"
).split()


def load_library() -> C.CDLL:
    """Loads libvlb200.so. Raises when it has not been built: there is no fallback path."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m vastloom_b200.build` "
            "(the MoE path has no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH))
    P, U32, U64, SZ, I, F = C.c_void_p, C.c_uint32, C.c_uint64, C.c_size_t, C.c_int, C.c_float
    sig = {
        "vlb_abi_version": (I, []),
        "vlb_thread_error": (I, [C.c_char_p, SZ]),
        "vlb_device_count": (I, [C.POINTER(C.c_int)]),
        "vlb_probe": (I, [I, C.POINTER(_DeviceInfo)]),
        "vlb_open": (I, [I, P, U64, C.POINTER(P)]),
        "vlb_close": (None, [P]),
        "vlb_last_error": (I, [P, C.c_char_p, SZ]),
        "vlb_stream": (P, [P]),
        "vlb_synchronize": (I, [P]),
        "vlb_set_codebook": (I, [P, U32, P, SZ]),
        "vlb_alloc": (I, [P, SZ, C.c_char_p, C.POINTER(P)]),
        "vlb_free": (I, [P, P]),
        "vlb_memcpy_h2d": (I, [P, P, P, SZ]),
        "vlb_memcpy_d2h": (I, [P, P, P, SZ]),
        "vlb_allocated_bytes": (U64, [P]),
        "vlb_upload_matrix": (I, [P, U64, U32, SZ, SZ, P, SZ, C.POINTER(P)]),
        "vlb_release_matrix": (I, [P, P]),
        "vlb_matrix_bytes": (U64, [P]),
        "vlb_matvec": (I, [P, P, P, P]),
        "vlb_matvec_device": (I, [P, P, P, SZ, SZ, P, SZ, P]),
        "vlb_dequantize_device": (I, [P, P, P, P]),
        "vlb_layer_create": (I, [P, C.POINTER(_LayerDesc), C.POINTER(P)]),
        "vlb_layer_destroy": (I, [P, P]),
        "vlb_layer_forward_device": (I, [P, P, P, P, P, U32, P, P]),
        "vlb_layer_forward": (I, [P, P, P, P, P, U32, P]),
        "vlb_layer_last_route": (I, [P, P, U32, P, P, P, P, P]),
        "vlb_layer_last_weight_bytes": (U64, [P, P]),
        "vlb_layer_set_profiling": (I, [P, P, I]),
        "vlb_layer_phase_times": (I, [P, P, C.POINTER(C.c_float), I]),
        "vlb_layer_set_prefill_tokens": (I, [P, P, U32]),
        "vlb_layer_set_input_norm": (I, [P, P, P, F]),
        "vlb_layer_forward_routes_device": (I, [P, P, P, P, P, U32, P, P]),
        "vlb_layer_status": (I, [P, P, P]),
        "vlb_ep_workspace_bytes": (SZ, [U32, U32, U32]),
        "vlb_ep_plan_device": (I, [P, P, P, U32, U32, U32, U32, P, U32, P, P, P, P, P, P, P, P]),
        "vlb_ep_combine_device": (I, [P, P, P, U32, U32, P, U32, P, P]),
        "vlb_ep_plan_half_device": (I, [P, P, P, U32, U32, U32, U32, P, P, U32, P, P, P, P, P, P, P, P, P]),
        "vlb_ep_pack_half_device": (I, [P, P, U32, U32, P, P, P]),
        "vlb_ep_combine_half_device": (I, [P, P, P, P, U32, U32, P, U32, P, P]),
        "vlb_layer_forward_rows_half_device": (I, [P, P, P, P, U32, P, P]),
        "vlb_layer_prefill_tokens": (U32, [P, P]),
        "vlb_route_device": (I, [P, I, I, P, P, P, P, U32, U32, U32, U32, F, P, P, P]),
        "vlb_route_device_noalloc": (I, [I, I, I, P, P, P, P, U32, U32, U32, U32, F, P, P, P]),
        "vlb_router_logits_device": (I, [P, P, P, U32, U32, U32, P, P]),
        "vlb_rms_norm_device": (I, [P, P, P, U32, U32, F, P, P]),
        "vlb_ep_nccl_version": (I, [C.POINTER(I)]),
        "vlb_ep_unique_id": (I, [P]),
        "vlb_ep_comm_init": (I, [P, P, I, I, U32, C.POINTER(P)]),
        "vlb_ep_comm_destroy": (I, [P]),
        "vlb_ep_comm_abort": (I, [P]),
        "vlb_ep_all_to_all_device": (I, [P, P, P, P, P, P]),
        "vlb_ep_layer_create": (I, [P, P, P, C.POINTER(P)]),
        "vlb_ep_layer_destroy": (I, [P, P]),
        "vlb_ep_forward_device": (I, [P, P, P, P, U32, P, P]),
        "vlb_ep_last_phases": (I, [P, C.POINTER(C.c_float), C.POINTER(U64)]),
        "vlb_upload_record_async": (I, [P, P, SZ, C.POINTER(_RecordTensor), U32, U64, C.POINTER(P)]),
        "vlb_upload_query": (I, [P, P, C.POINTER(C.c_int)]),
        "vlb_upload_finish": (I, [P, P, C.POINTER(P), U32]),
        "vlb_host_alloc": (I, [P, SZ, C.POINTER(P)]),
        "vlb_host_free": (I, [P, P]),
        "vlb_layer_set_hyper_connection": (I, [P, P, C.POINTER(_HcDesc)]),
        "vlb_layer_last_hyper_split": (I, [P, P, U32, P, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _ptr(a: np.ndarray) -> C.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return C.c_void_p(a.ctypes.data)


def read_codebooks(path: Path = GRIDS_PATH) -> dict[int, bytes]:
    """Reads the codebook data file written at build time (see csrc/gen_codebooks.cpp)."""
    raw = Path(path).read_bytes()
    if raw[:8] != b"VLBGRID1":
        raise VlbError(2, f"{path} is not a codebook file")
    (count,) = struct.unpack_from("<I", raw, 8)
    off = 12
    out = {}
    for _ in range(count):
        t, n, _fp = struct.unpack_from("<IIQ", raw, off)
        off += 16
        out[t] = raw[off: off + n]
        off += n
    return out


def device_count() -> int:
    lib = load_library()
    n = C.c_int(0)
    st = lib.vlb_device_count(C.byref(n))
    return n.value if st == 0 else 0


@dataclass
class Matrix:
    ptr: C.c_void_p
    ggml_type: int
    rows: int
    cols: int
    identity: int
    payload_bytes: int


class DeviceBuffer:
    """A governed device allocation owned by a Device."""

    def __init__(self, dev: "Device", nbytes: int, tag: str = "py-buffer"):
        self.dev = dev
        self.nbytes = nbytes
        p = C.c_void_p()
        dev._check(dev.lib.vlb_alloc(dev.h, nbytes, tag.encode(), C.byref(p)))
        self.ptr = p

    @property
    def address(self) -> int:
        return self.ptr.value or 0

    def upload(self, a: np.ndarray) -> "DeviceBuffer":
        a = np.ascontiguousarray(a)
        assert a.nbytes <= self.nbytes
        self.dev._check(self.dev.lib.vlb_memcpy_h2d(self.dev.h, self.ptr, _ptr(a), a.nbytes))
        return self

    def download(self, dtype, count: int) -> np.ndarray:
        out = np.empty(count, dtype=dtype)
        self.dev._check(self.dev.lib.vlb_memcpy_d2h(self.dev.h, _ptr(out), self.ptr, out.nbytes))
        return out

    def free(self) -> None:
        if self.ptr:
            self.dev._check(self.dev.lib.vlb_free(self.dev.h, self.ptr))
            self.ptr = C.c_void_p()


class RecordUpload:
    """An expert record on its way to the device (vlb_upload_record_async)."""

    def __init__(self, dev: "Device", ptr: C.c_void_p, record: np.ndarray, tensors: list):
        self.dev, self.ptr, self.record, self.tensors = dev, ptr, record, tensors

    def done(self) -> bool:
        d = C.c_int(0)
        self.dev._check(self.dev.lib.vlb_upload_query(self.dev.h, self.ptr, C.byref(d)))
        return bool(d.value)

    def finish(self) -> list:
        n = len(self.tensors)
        out = (C.c_void_p * n)()
        ptr, self.ptr = self.ptr, None
        self.dev._check(self.dev.lib.vlb_upload_finish(self.dev.h, ptr, out, n))
        self.record = None
        return [Matrix(C.c_void_p(out[i]), t, rows, cols, ident, nb)
                for i, (ident, t, rows, cols, _off, nb) in enumerate(self.tensors)]


class PinnedBuffer:
    """Page-locked host memory from the library (vlb_host_alloc), viewed as a uint8 array."""

    def __init__(self, dev: "Device", nbytes: int):
        self.dev = dev
        p = C.c_void_p()
        dev._check(dev.lib.vlb_host_alloc(dev.h, nbytes, C.byref(p)))
        self.ptr = p
        self.array = np.ctypeslib.as_array((C.c_uint8 * nbytes).from_address(p.value))

    def free(self) -> None:
        if self.ptr:
            self.array = None
            self.dev._check(self.dev.lib.vlb_host_free(self.dev.h, self.ptr))
            self.ptr = None


class Device:
    """One vlb200 handle on one GPU (cf. CudaMatvecAccelerator::create,
    src/cuda/cuda_matvec_accelerator.cpp:68-90)."""

    def __init__(self, ordinal: int = 0, governor=None, min_free_after: int = 0,
                 install_codebooks: bool = True):
        self.lib = load_library()
        self._gov_keep = None
        gov_ptr = None
        if governor is not None:
            # governor: object with reserve(bytes, tag) -> bool and release(bytes, tag)
            def _res(_ctx, n, tag):
                return 0 if governor.reserve(int(n), tag.decode() if tag else "") else 1

            def _rel(_ctx, n, tag):
                governor.release(int(n), tag.decode() if tag else "")

            g = _Governor(None, RESERVE_FN(_res), RELEASE_FN(_rel))
            self._gov_keep = g
            gov_ptr = C.byref(g)
        h = C.c_void_p()
        st = self.lib.vlb_open(ordinal, gov_ptr, min_free_after, C.byref(h))
        if st != 0:
            buf = C.create_string_buffer(512)
            self.lib.vlb_thread_error(buf, 512)
            raise VlbError(st, buf.value.decode())
        self.h = h
        self.ordinal = ordinal
        if install_codebooks:
            for t, table in read_codebooks().items():
                self.set_codebook(t, table)

    # -- plumbing --
    def _check(self, st: int) -> None:
        if st != 0:
            buf = C.create_string_buffer(1024)
            self.lib.vlb_last_error(self.h, buf, 1024)
            raise VlbError(st, buf.value.decode())

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.vlb_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def stream(self) -> int:
        return self.lib.vlb_stream(self.h) or 0

    def synchronize(self) -> None:
        self._check(self.lib.vlb_synchronize(self.h))

    def allocated_bytes(self) -> int:
        return int(self.lib.vlb_allocated_bytes(self.h))

    def buffer(self, nbytes: int, tag: str = "py-buffer") -> DeviceBuffer:
        return DeviceBuffer(self, nbytes, tag)

    def to_device(self, a: np.ndarray, tag: str = "py-buffer") -> DeviceBuffer:
        a = np.ascontiguousarray(a)
        return DeviceBuffer(self, max(a.nbytes, 4), tag).upload(a)

    # -- operators --
    def set_codebook(self, ggml_type: int, table: bytes) -> None:
        b = (C.c_char * len(table)).from_buffer_copy(table)
        self._check(self.lib.vlb_set_codebook(self.h, ggml_type, C.cast(b, C.c_void_p), len(table)))

    def upload_matrix(self, ggml_type: int, rows: int, cols: int, payload, identity: int = 1) -> Matrix:
        payload = np.ascontiguousarray(np.frombuffer(payload, dtype=np.uint8) if isinstance(payload, (bytes, bytearray)) else payload)
        m = C.c_void_p()
        self._check(self.lib.vlb_upload_matrix(self.h, identity, ggml_type, rows, cols, _ptr(payload),
                                               payload.nbytes, C.byref(m)))
        return Matrix(m, ggml_type, rows, cols, identity, int(payload.nbytes))

    def upload_record(self, record, tensors, reserved_bytes: int = 0) -> "RecordUpload":
        """Starts the device upload of one expert record (vlb_upload_record_async). `record`: the
        record's bytes (kept alive by the returned object until finish); `tensors`: one
        (identity, ggml_type, rows, storage_cols, offset, nbytes) tuple per tensor."""
        record = np.ascontiguousarray(np.frombuffer(record, dtype=np.uint8) if isinstance(record, (bytes, bytearray)) else record)
        arr = (_RecordTensor * len(tensors))()
        for i, (ident, t, rows, cols, off, nb) in enumerate(tensors):
            arr[i] = _RecordTensor(ident, t, 0, rows, cols, off, nb)
        u = C.c_void_p()
        self._check(self.lib.vlb_upload_record_async(self.h, _ptr(record), record.nbytes, arr, len(tensors),
                                                     reserved_bytes, C.byref(u)))
        return RecordUpload(self, u, record, list(tensors))

    def host_buffer(self, nbytes: int) -> "PinnedBuffer":
        return PinnedBuffer(self, nbytes)

    def release_matrix(self, m: Matrix) -> None:
        if m.ptr:
            self._check(self.lib.vlb_release_matrix(self.h, m.ptr))
            m.ptr = C.c_void_p()

    def matvec(self, m: Matrix, x: np.ndarray) -> np.ndarray:
        """The per-row seam (host input of storage_cols floats, host output of rows floats)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.shape != (m.cols,):
            raise ValueError("input must have storage_columns elements")
        y = np.empty(m.rows, dtype=np.float32)
        self._check(self.lib.vlb_matvec(self.h, m.ptr, _ptr(x), _ptr(y)))
        return y

    def matvec_tokens(self, m: Matrix, x: np.ndarray) -> np.ndarray:
        """Multi-token product through the device entry point: x [n, cols] -> y [n, rows]."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        n = x.shape[0]
        xb = self.to_device(x, "py-x")
        yb = self.buffer(n * m.rows * 4, "py-y")
        try:
            self._check(self.lib.vlb_matvec_device(self.h, m.ptr, xb.ptr, n, m.cols, yb.ptr, m.rows, None))
            return yb.download(np.float32, n * m.rows).reshape(n, m.rows)
        finally:
            xb.free()
            yb.free()

    def dequantize(self, m: Matrix) -> np.ndarray:
        ob = self.buffer(m.rows * m.cols * 4, "py-dequant")
        try:
            self._check(self.lib.vlb_dequantize_device(self.h, m.ptr, ob.ptr, None))
            return ob.download(np.float32, m.rows * m.cols).reshape(m.rows, m.cols)
        finally:
            ob.free()

    def route(self, logits: np.ndarray, top_k: int, route_scale: float = 1.0,
              score: int = SCORE_SQRT_SOFTPLUS, bias: Optional[np.ndarray] = None,
              token_ids: Optional[np.ndarray] = None, tid2eid: Optional[np.ndarray] = None):
        """deepseek_v4_route_learned_logits / deepseek_v4_route_hash_logits (and the OLMoE
        softmax router with score=SCORE_SOFTMAX) on the device. Returns (indices, weights)."""
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        T, E = logits.shape
        bufs = [self.to_device(logits, "py-logits")]
        bias_b = tok_b = tab_b = None
        if bias is not None:
            bias_b = self.to_device(np.ascontiguousarray(bias, dtype=np.float32), "py-bias")
            bufs.append(bias_b)
        hashing = tid2eid is not None
        vocab = 0
        if hashing:
            tab = np.ascontiguousarray(tid2eid, dtype=np.uint32)
            vocab = tab.size // top_k
            tok_b = self.to_device(np.ascontiguousarray(token_ids, dtype=np.uint32), "py-tokens")
            tab_b = self.to_device(tab, "py-tid2eid")
            bufs += [tok_b, tab_b]
        idx_b = self.buffer(T * top_k * 4, "py-idx")
        w_b = self.buffer(T * top_k * 4, "py-w")
        bufs += [idx_b, w_b]
        try:
            self._check(self.lib.vlb_route_device(
                self.h, score, 1 if hashing else 0, bufs[0].ptr, bias_b.ptr if bias_b else None,
                tok_b.ptr if tok_b else None, tab_b.ptr if tab_b else None, vocab, T, E, top_k,
                route_scale, idx_b.ptr, w_b.ptr, None))
            idx = idx_b.download(np.uint32, T * top_k).reshape(T, top_k)
            w = w_b.download(np.float32, T * top_k).reshape(T, top_k)
            return idx, w
        finally:
            for b in bufs:
                b.free()

    def router_logits(self, x: np.ndarray, w: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        T, H = x.shape
        E = w.shape[0]
        xb, wb, lb = self.to_device(x), self.to_device(w), self.buffer(T * E * 4)
        try:
            self._check(self.lib.vlb_router_logits_device(self.h, xb.ptr, wb.ptr, T, H, E, lb.ptr, None))
            return lb.download(np.float32, T * E).reshape(T, E)
        finally:
            for b in (xb, wb, lb):
                b.free()

    def rms_norm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, width = x.shape
        xb, wb, ob = self.to_device(x), self.to_device(np.ascontiguousarray(w, dtype=np.float32)), self.buffer(x.nbytes)
        try:
            self._check(self.lib.vlb_rms_norm_device(self.h, xb.ptr, wb.ptr, rows, width, eps, ob.ptr, None))
            self.synchronize()
            return ob.download(np.float32, rows * width).reshape(rows, width)
        finally:
            for b in (xb, wb, ob):
                b.free()


class MoeLayer:
    """One resident MoE layer (router, routed experts, optional shared expert)."""

    def __init__(self, dev: Device, *, hidden: int, intermediate: int, experts: int, top_k: int,
                 router: np.ndarray, w1: Sequence[Matrix], w3: Sequence[Matrix],
                 w2: Sequence[Matrix], score: int = SCORE_SQRT_SOFTPLUS,
                 bias: Optional[np.ndarray] = None, route_scale: float = 1.0,
                 hash_table: Optional[np.ndarray] = None, weight_after_down: bool = False,
                 routed_swiglu_limit: float = 0.0, shared_swiglu_limit: float = 0.0,
                 shared: Optional[tuple[Matrix, Matrix, Matrix]] = None, max_tokens: int = 64):
        self.dev = dev
        self.H, self.I, self.E, self.k = hidden, intermediate, experts, top_k
        self.max_tokens = max_tokens
        self._router = np.ascontiguousarray(router, dtype=np.float32)
        self._bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self._table = None if hash_table is None else np.ascontiguousarray(hash_table, dtype=np.uint32)
        arr = C.c_void_p * experts
        self._w1 = arr(*[m.ptr.value for m in w1])
        self._w3 = arr(*[m.ptr.value for m in w3])
        self._w2 = arr(*[m.ptr.value for m in w2])
        d = _LayerDesc()
        d.hidden, d.intermediate, d.experts, d.top_k = hidden, intermediate, experts, top_k
        d.score = score
        d.hash_routing = 1 if hash_table is not None else 0
        d.weight_after_down = 1 if weight_after_down else 0
        d.route_scale = route_scale
        d.routed_swiglu_limit = routed_swiglu_limit
        d.shared_swiglu_limit = shared_swiglu_limit
        d.max_tokens = max_tokens
        d.vocab = 0 if self._table is None else self._table.size // top_k
        d.router = self._router.ctypes.data
        d.bias = None if self._bias is None else self._bias.ctypes.data
        d.tid2eid = None if self._table is None else self._table.ctypes.data
        d.w1 = C.cast(self._w1, C.c_void_p)
        d.w3 = C.cast(self._w3, C.c_void_p)
        d.w2 = C.cast(self._w2, C.c_void_p)
        if shared is not None:
            d.shared_w1, d.shared_w3, d.shared_w2 = (m.ptr.value for m in shared)
        p = C.c_void_p()
        dev._check(dev.lib.vlb_layer_create(dev.h, C.byref(d), C.byref(p)))
        self.ptr = p

    def forward(self, x: np.ndarray, token_ids: Optional[np.ndarray] = None,
                logits: Optional[np.ndarray] = None, out: Optional[np.ndarray] = None) -> np.ndarray:
        """Host-memory forward (H2D inputs, layer, D2H output) - the end-to-end call. `out`
        (f32 [T, H], C-contiguous) may be supplied, e.g. page-locked, to receive the output."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0]
        shape = (T, self.hc_m, self.H) if self.hc_m else (T, self.H)
        if x.shape != shape:
            raise ValueError(f"x must have shape {shape}")
        if out is None:
            out = np.empty(shape, dtype=np.float32)
        elif out.dtype != np.float32 or out.shape != shape or not out.flags["C_CONTIGUOUS"]:
            raise ValueError(f"out must be a C-contiguous float32 array of shape {shape}")
        tok = None if token_ids is None else np.ascontiguousarray(token_ids, dtype=np.uint32)
        lg = None if logits is None else np.ascontiguousarray(logits, dtype=np.float32)
        self.dev._check(self.dev.lib.vlb_layer_forward(
            self.dev.h, self.ptr, _ptr(x), None if tok is None else _ptr(tok),
            None if lg is None else _ptr(lg), T, _ptr(out)))
        return out

    def forward_device(self, x_ptr: int, T: int, out_ptr: int, token_ids_ptr: int = 0,
                       logits_ptr: int = 0, stream: int = 0) -> None:
        """Device-resident forward on raw device pointers, enqueued on `stream`."""
        self.dev._check(self.dev.lib.vlb_layer_forward_device(
            self.dev.h, self.ptr, C.c_void_p(x_ptr), C.c_void_p(token_ids_ptr or None),
            C.c_void_p(logits_ptr or None), T, C.c_void_p(out_ptr), C.c_void_p(stream or None)))

    def last_route(self, T: int):
        n = T * self.k
        idx = np.empty(n, np.uint32)
        w = np.empty(n, np.float32)
        off = np.empty(self.E + 1, np.uint32)
        pt = np.empty(n, np.uint32)
        ps = np.empty(n, np.uint32)
        self.dev._check(self.dev.lib.vlb_layer_last_route(self.dev.h, self.ptr, T, _ptr(idx), _ptr(w),
                                                          _ptr(off), _ptr(pt), _ptr(ps)))
        return idx.reshape(T, self.k), w.reshape(T, self.k), off, pt, ps

    PHASES = ("route", "dispatch", "gate_up", "down", "combine")

    def set_profiling(self, enable: bool) -> None:
        self.dev._check(self.dev.lib.vlb_layer_set_profiling(self.dev.h, self.ptr, 1 if enable else 0))

    def phase_times(self) -> dict:
        ms = (C.c_float * 5)()
        self.dev._check(self.dev.lib.vlb_layer_phase_times(self.dev.h, self.ptr, ms, 5))
        return dict(zip(self.PHASES, [float(v) for v in ms]))

    def last_weight_bytes(self) -> int:
        return int(self.dev.lib.vlb_layer_last_weight_bytes(self.dev.h, self.ptr))

    def forward_routes_device(self, x_ptr: int, idx_ptr: int, w_ptr: int, T: int, out_ptr: int,
                              stream: int = 0) -> None:
        """Forward with given routes (device u32 ids [T x k], f32 weights): router and top-k skipped."""
        self.dev._check(self.dev.lib.vlb_layer_forward_routes_device(
            self.dev.h, self.ptr, C.c_void_p(x_ptr), C.c_void_p(idx_ptr), C.c_void_p(w_ptr), T,
            C.c_void_p(out_ptr), C.c_void_p(stream or None)))

    def forward_rows_half_device(self, rows_ptr: int, meta_ptr: int, T: int, out_ptr: int, stream: int = 0) -> None:
        """Forward of fp16 rows with one route each (meta u32 [T x 3]: expert, weight bits, max|x| bits)."""
        self.dev._check(self.dev.lib.vlb_layer_forward_rows_half_device(
            self.dev.h, self.ptr, C.c_void_p(rows_ptr), C.c_void_p(meta_ptr), T, C.c_void_p(out_ptr),
            C.c_void_p(stream or None)))

    def status(self, stream: int = 0) -> None:
        """Raises the error the last device forward flagged (synchronises `stream`)."""
        self.dev._check(self.dev.lib.vlb_layer_status(self.dev.h, self.ptr, C.c_void_p(stream or None)))

    def set_input_norm(self, weight: Optional[np.ndarray], eps: float = 1e-6) -> None:
        """Makes every forward a residual block out = x + MoE(RMSNorm(x)) (weight f32 [hidden]);
        None removes the entry norm and the residual."""
        if weight is None:
            self.dev._check(self.dev.lib.vlb_layer_set_input_norm(self.dev.h, self.ptr, None, 0.0))
            self._norm_w = None
            return
        w = np.ascontiguousarray(weight, dtype=np.float32)
        if w.shape != (self.H,):
            raise ValueError("the norm weight must have `hidden` elements")
        self.dev._check(self.dev.lib.vlb_layer_set_input_norm(self.dev.h, self.ptr, _ptr(w), eps))
        self._norm_w = w

    hc_m = 0

    def set_hyper_connection(self, multiplier: int, mixing_weight, scale, base, norm_weight,
                             sinkhorn_iterations: int = 20, norm_eps: float = 1e-6, hc_eps: float = 1e-6) -> None:
        """Hyper-Connection entry and exit around the MoE (vlb_layer_set_hyper_connection): x and
        out become [T, multiplier, hidden]. multiplier 0 removes it (and the norm)."""
        if multiplier == 0:
            self.dev._check(self.dev.lib.vlb_layer_set_hyper_connection(self.dev.h, self.ptr, None))
            self.hc_m = 0
            return
        m, H = multiplier, self.H
        fn = np.ascontiguousarray(mixing_weight, np.float32)
        sc, ba = np.ascontiguousarray(scale, np.float32), np.ascontiguousarray(base, np.float32)
        nw = np.ascontiguousarray(norm_weight, np.float32)
        if fn.size != (2 + m) * m * m * H or sc.size != 3 or ba.size != (2 + m) * m or nw.size != H:
            raise ValueError("Hyper-Connection tensors have the wrong sizes")
        d = _HcDesc(m, sinkhorn_iterations, norm_eps, hc_eps, _ptr(fn), _ptr(sc), _ptr(ba), _ptr(nw))
        self.dev._check(self.dev.lib.vlb_layer_set_hyper_connection(self.dev.h, self.ptr, C.byref(d)))
        self.hc_m = m

    def last_hyper_split(self, T: int):
        """(pre [T, m], post [T, m], combination [T, m, m]) of the last forward."""
        m = self.hc_m
        pre, post, comb = np.empty((T, m), np.float32), np.empty((T, m), np.float32), np.empty((T, m, m), np.float32)
        self.dev._check(self.dev.lib.vlb_layer_last_hyper_split(self.dev.h, self.ptr, T, _ptr(pre), _ptr(post),
                                                                _ptr(comb)))
        return pre, post, comb

    PREFILL_NEVER = 0xFFFFFFFF

    def set_prefill_tokens(self, min_tokens: int) -> None:
        """Forwards of at least `min_tokens` tokens run the expert products on the tensor-core
        prefill kernels (2e-2 contract); 0 = the default threshold, PREFILL_NEVER = never."""
        self.dev._check(self.dev.lib.vlb_layer_set_prefill_tokens(self.dev.h, self.ptr, min_tokens))

    def prefill_tokens(self) -> int:
        return int(self.dev.lib.vlb_layer_prefill_tokens(self.dev.h, self.ptr))

    def destroy(self) -> None:
        if self.ptr:
            self.dev._check(self.dev.lib.vlb_layer_destroy(self.dev.h, self.ptr))
            self.ptr = C.c_void_p()


class LayerChain:
    """Layers applied one after another on the device, x_{l+1} = layer_l(x_l), with one host copy
    in and one out. With an input norm set on every layer (MoeLayer.set_input_norm) this is the
    residual chain x <- x + MoE(RMSNorm(x)) of the hash-routed configuration; every layer reads the
    same token ids (each with its own token-to-expert table)."""

    def __init__(self, dev: Device, layers: Sequence[MoeLayer], max_tokens: int):
        if not layers or any(l.H != layers[0].H for l in layers):
            raise ValueError("a chain needs layers of one hidden size")
        self.dev, self.layers, self.max_tokens = dev, list(layers), max_tokens
        H = layers[0].H
        self._bufs = [dev.buffer(max_tokens * H * 4, "chain-x0"), dev.buffer(max_tokens * H * 4, "chain-x1")]
        self._tok = dev.buffer(max_tokens * 4, "chain-tokens")

    def forward(self, x: np.ndarray, token_ids: Optional[np.ndarray] = None) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        T, H = x.shape
        if T == 0 or T > self.max_tokens or H != self.layers[0].H:
            raise ValueError("chain input has the wrong shape")
        self._bufs[0].upload(x)
        tok_ptr = 0
        if token_ids is not None:
            self._tok.upload(np.ascontiguousarray(token_ids, dtype=np.uint32))
            tok_ptr = self._tok.address
        cur = 0
        for layer in self.layers:
            layer.forward_device(self._bufs[cur].address, T, self._bufs[1 - cur].address, token_ids_ptr=tok_ptr)
            cur = 1 - cur
        out = self._bufs[cur].download(np.float32, T * H).reshape(T, H)
        for layer in self.layers:
            layer.status()
        return out

    def close(self) -> None:
        for b in self._bufs + [self._tok]:
            b.free()
