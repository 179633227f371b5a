"""Expert parallelism for the MoE layer (benchmark configuration 4): the routed experts are
sharded over the ranks of a process group (contiguous ranges of ids, or a placement balanced by
expert load), every rank routes its own tokens, sends each (token, slot) pair's activation row to
the rank that owns the expert (all-to-all), computes the pairs it received on its expert shard,
and sends the results back for the combine.

The layer math is the reference's (moe_forward, deepseek_v4_graph.cpp:1902-2274): route weights
are applied before the down product, each token's pairs are summed and the shared expert's row is
added. The shared expert is replicated: every rank computes it for its own tokens, as one more
expert of its local group (weight 1).

    rank r:  route (own logits) -> plan (stable order by expert = by owner rank, x rows gathered)
             -> all-to-all counts, rows, expert ids, weights
             -> group forward over [received rows ; own tokens for the shared expert]
             -> all-to-all results back -> combine

The orchestration is written once against two small interfaces: `ops` (the compute steps; the
device implementation, DeviceEpOps, calls the vlb200 C ABI) and `comm` (the exchange;
TorchComm wraps torch.distributed, NCCL on GPUs, gloo on CPU tensors).

Failure detection is the process group's: give it a short timeout. A rank that fails, leaves or
never reaches an exchange makes the exchange raise on its peers (after the timeout, or at once
when its connections close); the layer turns that into EpExchangeError naming the exchange and
refuses further forwards, since the peers' state is unknown. Rebuild the group and the layer to
continue.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

import numpy as np


class EpExchangeError(RuntimeError):
    """An exchange of the expert-parallel layer failed: a peer rank failed, left the group or did
    not join within the process group's timeout. `phase` is "counts", "dispatch" or "return"."""

    def __init__(self, phase: str, cause: BaseException):
        super().__init__(f"expert-parallel {phase} exchange failed: {cause}")
        self.phase = phase


def balanced_slots(loads, world: int) -> np.ndarray:
    """Expert placement balanced by load: slot[e] for every expert (rank slot // epr, local expert
    slot % epr), experts_per_rank = E / world experts on every rank. Longest-processing-time
    greedy: experts by load, heaviest first (ties to the lower id), each to the least-loaded rank
    that still has room (ties to the lower rank); within a rank in assignment order. Every rank
    computes the same placement from the same loads."""
    loads = np.asarray(loads, dtype=np.float64)
    E = loads.size
    if E % world:
        raise ValueError("experts must divide evenly over the ranks")
    epr = E // world
    order = sorted(range(E), key=lambda e: (-loads[e], e))
    rank_load = [0.0] * world
    fill = [0] * world
    slot = np.empty(E, np.uint32)
    for e in order:
        r = min((r for r in range(world) if fill[r] < epr), key=lambda r: (rank_load[r], r))
        slot[e] = r * epr + fill[r]
        fill[r] += 1
        rank_load[r] += loads[e]
    return slot


def owner_counts(offsets_host: np.ndarray, world: int, experts_per_rank: int) -> list:
    """Pairs destined to each rank from the per-expert starts of a plan (expert-sorted order)."""
    return [int(offsets_host[(r + 1) * experts_per_rank]) - int(offsets_host[r * experts_per_rank])
            for r in range(world)]


class TorchComm:
    """All-to-all exchange through torch.distributed (NCCL for CUDA tensors, gloo for CPU)."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def exchange_counts(self, send_counts: list, like) -> list:
        import torch

        s = torch.tensor(send_counts, dtype=torch.int64, device=like.device)
        r = torch.empty_like(s)
        self.dist.all_to_all_single(r, s, group=self.group)
        return [int(v) for v in r.cpu().tolist()]

    def all_to_all(self, out, inp, out_splits: list, in_splits: list) -> None:
        self.dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def max_over_ranks(self, v: float, like) -> float:
        import torch

        t = torch.tensor([v], dtype=torch.float64, device=like.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX, group=self.group)
        return float(t.item())

    def min_over_ranks(self, v: float, like) -> float:
        import torch

        t = torch.tensor([v], dtype=torch.float64, device=like.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MIN, group=self.group)
        return float(t.item())


@dataclass
class EpBuffers:
    send_rows: object   # [T*k, H] activation rows in send (plan) order; the ops choose the format
    send_meta: object   # [T*k, 3] per row: local expert id, route weight, row scale information
    elem_row: object    # [T*k] element (t * k + slot) -> send row
    group_rows: object  # [capacity, H] received rows, then this rank's own rows for the shared expert
    group_meta: object  # [capacity, 3]
    group_y: object     # [capacity, H] f32 expert outputs of the group rows
    back_y: object      # [T*k, H] results returned to this rank, in send order (the ops' format)
    out: object         # [T, H] f32
    group_ys: object = None  # [capacity] per-row scales of packed return rows (ops with pack_return)
    back_ys: object = None   # [T*k] their returned copies


class ExpertParallelLayer:
    """One rank's share of an expert-parallel MoE layer. `ops` provides route / plan / group
    forward / combine on this rank's device (or host, for the CPU tests); `comm` the exchange.
    Rows travel in the format `ops` allocates for them (fp16 with per-row scale information on
    GPUs: half the bytes of f32, and exactly the operands the tensor-core expert kernels use)."""

    def __init__(self, ops, comm, experts: int, top_k: int, hidden: int, max_tokens: int):
        if experts % comm.world:
            raise ValueError("experts must divide evenly over the ranks")
        self.ops = ops
        self.comm = comm
        self.E = experts
        self.k = top_k
        self.H = hidden
        self.epr = experts // comm.world
        self.max_tokens = max_tokens
        n = max_tokens * top_k
        # ops with pack_return send the expert outputs back in their own (smaller) row format
        self.packed = hasattr(ops, "pack_return")
        self.buf = EpBuffers(
            send_rows=ops.empty((n, hidden), "rows"), send_meta=ops.empty((n, 3), "meta"),
            elem_row=ops.empty((n,), "i32"), group_rows=None, group_meta=None, group_y=None,
            back_y=ops.empty((n, hidden), "rows" if self.packed else "f32"), out=ops.empty((max_tokens, hidden), "f32"),
            back_ys=ops.empty((n,), "f32") if self.packed else None)
        self.capacity = 0  # group rows the receive side is sized for (grown on demand)
        self._marks = None
        self._rows = (0, 0)
        self.failed: Optional[str] = None  # the exchange that failed, once one has

    def _exchange(self, phase: str, fn):
        """Runs one exchange step; a failure of the process group becomes EpExchangeError and
        marks the layer failed."""
        try:
            with self.ops.comm_scope():
                return fn()
        except Exception as e:  # torch.distributed raises RuntimeError (or a subclass) here
            self.failed = phase
            raise EpExchangeError(phase, e) from e

    def _reserve(self, rows: int) -> None:
        """Receive-side buffers for `rows` group rows (received pairs + own shared rows). The worst
        case (every rank's pairs on this rank) is world x the balanced load, so capacity follows
        the observed load with headroom instead."""
        if rows <= self.capacity:
            return
        cap = int(rows * 1.25) + 16
        b, ops = self.buf, self.ops
        b.group_rows = ops.empty((cap, self.H), "rows")
        b.group_meta = ops.empty((cap, 3), "meta")
        b.group_y = ops.empty((cap, self.H), "f32")
        if self.packed:
            b.group_yh = ops.empty((cap, self.H), "rows")
            b.group_ys = ops.empty((cap,), "f32")
        ops.reserve_group(cap)
        self.capacity = cap

    def forward(self, x, logits, T: int):
        """x [T, H] f32 and logits [T, E] f32 of this rank's tokens (in the ops' memory); returns
        out [T, H]. The phase boundaries are marked on the device (no host synchronisation beyond
        the two count read-backs the exchange sizes need); `last` reads them afterwards."""
        if T > self.max_tokens:
            raise ValueError("more tokens than the layer was sized for")
        if self.failed:
            raise EpExchangeError(self.failed, RuntimeError("an earlier exchange of this layer failed"))
        ops, comm, b, k = self.ops, self.comm, self.buf, self.k
        n = T * k
        m0 = ops.mark()
        idx, w = ops.route(logits, T)
        offsets = ops.plan(idx, w, x, T, self.epr, b)
        send_counts = owner_counts(offsets, comm.world, self.epr)
        recv_counts = self._exchange("counts", lambda: comm.exchange_counts(send_counts, b.out))
        R = sum(recv_counts)
        self._reserve(R + T)
        m1 = ops.mark()
        def dispatch():
            comm.all_to_all(b.group_rows[:R], b.send_rows[:n], recv_counts, send_counts)
            comm.all_to_all(b.group_meta[:R], b.send_meta[:n], recv_counts, send_counts)

        self._exchange("dispatch", dispatch)
        ops.append_shared_rows(b, R, x, T, self.epr)
        m2 = ops.mark()
        ops.group_forward(b, R + T)
        m3 = ops.mark()
        if self.packed:
            ops.pack_return(b, R)

            def ret():
                comm.all_to_all(b.back_y[:n], b.group_yh[:R], send_counts, recv_counts)
                comm.all_to_all(b.back_ys[:n], b.group_ys[:R], send_counts, recv_counts)

            self._exchange("return", ret)
        else:
            self._exchange("return", lambda: comm.all_to_all(b.back_y[:n], b.group_y[:R], send_counts, recv_counts))
        m4 = ops.mark()
        out = ops.combine(b, T, k, R)
        m5 = ops.mark()
        ops.check()
        self._marks = (m0, m1, m2, m3, m4, m5)
        self._rows = (R, n)
        return out

    @property
    def last(self) -> dict:
        """Phase times (seconds) and row counts of the last forward on this rank."""
        if not getattr(self, "_marks", None):
            return {}
        t = self.ops.elapsed(self._marks)
        names = ("plan_s", "dispatch_s", "experts_s", "return_s", "combine_s")
        d = {name: t[i] for i, name in enumerate(names)}
        d["received_rows"], d["sent_rows"] = self._rows
        return d


class DeviceEpOps:
    """The compute steps on this rank's GPU through the vlb200 C ABI (buffers are torch CUDA
    tensors on the handle's stream). The local group layer holds the rank's routed experts plus
    the shared expert as local expert `experts_per_rank`."""

    def __init__(self, dev, group_mats, spec, bias, score: int, route_scale: float, experts: int, top_k: int,
                 hidden: int, max_tokens: int, slots: Optional[np.ndarray] = None):
        import torch

        self.torch = torch
        self.dev = dev
        self.lib = dev.lib
        self.group_mats = group_mats
        self.spec = spec
        self.group = None
        self.score = score
        self.route_scale = route_scale
        self.E = experts
        self.k = top_k
        self.H = hidden
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.stream = torch.cuda.ExternalStream(dev.stream, device=self.device)
        self.bias = None if bias is None else torch.from_numpy(np.ascontiguousarray(bias, np.float32)).to(self.device)
        self.slots = None if slots is None else torch.from_numpy(
            np.ascontiguousarray(slots, np.uint32).view(np.int32)).to(self.device)
        n = max_tokens * top_k
        self.idx = torch.empty((n,), dtype=torch.int32, device=self.device)
        self.w = torch.empty((n,), dtype=torch.float32, device=self.device)
        self.offsets = torch.empty((experts + 2,), dtype=torch.int32, device=self.device)
        self.offsets_host = np.zeros(experts + 1, np.uint32)
        self.ws = torch.empty((int(self.lib.vlb_ep_workspace_bytes(max_tokens, top_k, experts)),),
                              dtype=torch.uint8, device=self.device)
        # this rank's own tokens as half rows for its shared expert (written by the plan)
        self.own_rows = torch.empty((max_tokens, hidden), dtype=torch.float16, device=self.device)
        self.own_meta = torch.empty((max_tokens, 3), dtype=torch.int32, device=self.device)

    def reserve_group(self, rows: int) -> None:
        """(Re)creates the local group layer with a workspace for `rows` given-route rows."""
        from . import MoeLayer

        if self.group is not None:
            self.group.destroy()
        m = self.group_mats
        spec = self.spec
        e_local = len(m["w1"])
        self.group = MoeLayer(self.dev, hidden=spec.hidden, intermediate=spec.intermediate, experts=e_local,
                              top_k=1, router=np.zeros((e_local, spec.hidden), np.float32), w1=m["w1"],
                              w3=m["w3"], w2=m["w2"], score=spec.score, bias=None, route_scale=1.0,
                              weight_after_down=spec.weight_after_down, shared=None, max_tokens=rows)

    def close(self) -> None:
        if self.group is not None:
            self.group.destroy()
            self.group = None
        for lst in self.group_mats.values():
            for mtx in lst:
                self.dev.release_matrix(mtx)

    def empty(self, shape, kind):
        # rows travel as fp16(x * 2^e); meta rows are u32 (expert, weight bits, max|x| bits)
        dt = {"f32": self.torch.float32, "i32": self.torch.int32, "rows": self.torch.float16,
              "meta": self.torch.int32}[kind]
        return self.torch.empty(shape, dtype=dt, device=self.device)

    @staticmethod
    def _p(t):
        return C.c_void_p(t.data_ptr())

    def mark(self):
        """A phase boundary: an event on the library stream (no host synchronisation)."""
        ev = self.torch.cuda.Event(enable_timing=True)
        ev.record(self.stream)
        return ev

    def elapsed(self, marks) -> list:
        marks[-1].synchronize()
        return [marks[i].elapsed_time(marks[i + 1]) / 1000.0 for i in range(len(marks) - 1)]

    def comm_scope(self):
        """The collectives run on the library stream, ordered with the kernels without host syncs."""
        return self.torch.cuda.stream(self.stream)

    def check(self) -> None:
        """Raises the error the step's group forward flagged (one synchronisation per step)."""
        self.group.status(stream=self.dev.stream)

    def route(self, logits, T):
        self.dev._check(self.lib.vlb_route_device(
            self.dev.h, self.score, 0, self._p(logits), None if self.bias is None else self._p(self.bias), None, None,
            0, T, self.E, self.k, self.route_scale, self._p(self.idx), self._p(self.w), C.c_void_p(self.dev.stream)))
        return self.idx, self.w

    def plan(self, idx, w, x, T, epr, b):
        self.dev._check(self.lib.vlb_ep_plan_half_device(
            self.dev.h, self._p(idx), self._p(w), T, self.k, self.E, epr,
            None if self.slots is None else self._p(self.slots), self._p(x), self.H, self._p(self.ws),
            self._p(self.offsets), self.offsets_host.ctypes.data_as(C.c_void_p), self._p(b.send_rows),
            self._p(b.send_meta), self._p(b.elem_row), self._p(self.own_rows), self._p(self.own_meta),
            C.c_void_p(self.dev.stream)))
        return self.offsets_host

    def append_shared_rows(self, b, R, x, T, epr):
        with self.torch.cuda.stream(self.stream):
            b.group_rows[R:R + T].copy_(self.own_rows[:T])
            b.group_meta[R:R + T].copy_(self.own_meta[:T])

    def group_forward(self, b, rows):
        self.group.forward_rows_half_device(b.group_rows.data_ptr(), b.group_meta.data_ptr(), rows,
                                            b.group_y.data_ptr(), stream=self.dev.stream)

    def pack_return(self, b, R):
        """The received pairs' outputs as fp16 rows with a power-of-two scale per row: half the
        bytes of the f32 rows on the return exchange (11 significant bits, like the operands)."""
        self.dev._check(self.lib.vlb_ep_pack_half_device(
            self.dev.h, self._p(b.group_y), R, self.H, self._p(b.group_yh), self._p(b.group_ys),
            C.c_void_p(self.dev.stream)))

    def combine(self, b, T, k, R):
        self.dev._check(self.lib.vlb_ep_combine_half_device(
            self.dev.h, self._p(b.back_y), self._p(b.back_ys), self._p(b.elem_row), T, k,
            self._p(b.group_y[R:R + T]), self.H, self._p(b.out), C.c_void_p(self.dev.stream)))
        return b.out[:T]


def upload_group(dev, W, rank: int, world: int, layer_index: int = 0, slots: Optional[np.ndarray] = None) -> dict:
    """This rank's expert group matrices: the routed experts placed on it (slots [rank * E/world,
    (rank + 1) * E/world) in slot order; without slots the contiguous range of ids) plus the shared
    expert as local expert E/world (w1 / w3 / w2 lists)."""
    spec = W.spec
    E, H, I = spec.experts, spec.hidden, spec.intermediate
    epr = E // world
    if slots is None:
        local = list(range(rank * epr, (rank + 1) * epr))
    else:
        by_slot = np.argsort(np.asarray(slots, np.int64))
        local = [int(e) for e in by_slot[rank * epr:(rank + 1) * epr]]

    def ident(e, role):
        return ((layer_index * 1_000_003 + e) * 4 + role) * 2 + 1

    mats = {"w1": [], "w3": [], "w2": []}
    for e in local:
        for role, (name, rows, cols) in enumerate((("w1", I, H), ("w3", I, H), ("w2", H, I))):
            t, blob = getattr(W, name)[e]
            mats[name].append(dev.upload_matrix(t, rows, cols, blob, identity=ident(e, role)))
    if W.shared is None:
        raise ValueError("the expert-parallel layer expects a shared expert")
    for role, ((t, blob), (rows, cols), name) in enumerate(zip(W.shared, ((I, H), (I, H), (H, I)), ("w1", "w3", "w2"))):
        mats[name].append(dev.upload_matrix(t, rows, cols, blob, identity=ident(E, role)))
    return mats


def make_device_layer(dev, W, comm, max_tokens: int, slots: Optional[np.ndarray] = None):
    """The expert-parallel layer of this rank on device `dev` (weights W of the whole layer; only
    this rank's shard and the shared expert are uploaded). `slots` places the experts (see
    balanced_slots; None: contiguous ranges of ids)."""
    spec = W.spec
    mats = upload_group(dev, W, comm.rank, comm.world, slots=slots)
    ops = DeviceEpOps(dev, mats, spec, W.bias, spec.score, spec.route_scale, spec.experts, spec.top_k,
                      spec.hidden, max_tokens, slots=slots)
    return ExpertParallelLayer(ops, comm, spec.experts, spec.top_k, spec.hidden, max_tokens), ops


class _EpLayerDesc(C.Structure):
    _fields_ = [
        ("hidden", C.c_uint32), ("intermediate", C.c_uint32), ("experts", C.c_uint32), ("top_k", C.c_uint32),
        ("score", C.c_int), ("weight_after_down", C.c_int), ("route_scale", C.c_float),
        ("routed_swiglu_limit", C.c_float), ("shared_swiglu_limit", C.c_float), ("max_tokens", C.c_uint32),
        ("bias", C.c_void_p), ("expert_slot", C.c_void_p), ("w1", C.c_void_p), ("w3", C.c_void_p),
        ("w2", C.c_void_p),
    ]


def _native_check(lib, st: int, phase: Optional[str] = None) -> None:
    if st != 0:
        from . import VlbError

        buf = C.create_string_buffer(1024)
        lib.vlb_thread_error(buf, 1024)
        msg = buf.value.decode()
        if phase is not None:
            raise EpExchangeError(phase, VlbError(st, msg))
        raise VlbError(st, msg)


def native_unique_id() -> bytes:
    """ncclGetUniqueId through the library (rank 0 makes it; every rank passes the same bytes to
    NativeEpComm)."""
    import torch  # noqa: F401  (torch's NCCL first: see NativeEpComm)

    from . import load_library

    lib = load_library()
    buf = (C.c_uint8 * 128)()
    _native_check(lib, lib.vlb_ep_unique_id(buf))
    return bytes(buf)


class NativeEpComm:
    """The library's own NCCL communicator for one rank (vlb_ep_comm_init): non-blocking, every
    wait bounded by `timeout_ms`, aborted by the library when an exchange fails.

    The library binds the NCCL copy already loaded in the process when there is one. torch is
    imported before the first NCCL call, so that copy is torch's own: a process that loaded
    another libnccl.so.2 first could no longer import torch (one soname per process)."""

    def __init__(self, dev, unique_id: bytes, rank: int, world: int, timeout_ms: int = 120_000):
        import torch  # noqa: F401

        if len(unique_id) != 128:
            raise ValueError("an NCCL unique id is 128 bytes")
        self.dev, self.lib, self.rank, self.world = dev, dev.lib, rank, world
        uid = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        p = C.c_void_p()
        _native_check(self.lib, self.lib.vlb_ep_comm_init(dev.h, uid, rank, world, timeout_ms, C.byref(p)))
        self.ptr = p

    def abort(self) -> None:
        _native_check(self.lib, self.lib.vlb_ep_comm_abort(self.ptr))

    def all_to_all(self, send_ptr: int, send_bytes, recv_ptr: int, recv_bytes, stream: int = 0) -> None:
        sb = (C.c_uint64 * self.world)(*[int(v) for v in send_bytes])
        rb = (C.c_uint64 * self.world)(*[int(v) for v in recv_bytes])
        _native_check(self.lib, self.lib.vlb_ep_all_to_all_device(self.ptr, C.c_void_p(send_ptr), sb,
                                                                  C.c_void_p(recv_ptr), rb, C.c_void_p(stream)))

    def close(self) -> None:
        if self.ptr:
            st = self.lib.vlb_ep_comm_destroy(self.ptr)
            self.ptr = C.c_void_p()
            _native_check(self.lib, st)


class NativeEpLayer:
    """One rank's expert-parallel layer run by the library's C++ driver (vlb_ep_layer_create /
    vlb_ep_forward_device): route, plan, the NCCL exchanges, the group forward and the combine in
    one call per step. A failed exchange raises EpExchangeError with the phase the library names
    and leaves the layer refusing further forwards."""

    PHASES = ("plan_s", "dispatch_s", "experts_s", "return_s", "combine_s")

    def __init__(self, dev, comm: NativeEpComm, W, max_tokens: int, slots: Optional[np.ndarray] = None,
                 layer_index: int = 0):
        spec = W.spec
        self.dev, self.lib, self.comm, self.spec = dev, dev.lib, comm, spec
        self.mats = upload_group(dev, W, comm.rank, comm.world, layer_index=layer_index, slots=slots)
        self._keep = []

        def arr(lst):
            a = (C.c_void_p * len(lst))(*[m.ptr.value for m in lst])
            self._keep.append(a)
            return C.cast(a, C.c_void_p)

        bias = None if W.bias is None else np.ascontiguousarray(W.bias, np.float32)
        sl = None if slots is None else np.ascontiguousarray(slots, np.uint32)
        self._keep += [bias, sl]
        d = _EpLayerDesc(spec.hidden, spec.intermediate, spec.experts, spec.top_k, spec.score,
                         spec.weight_after_down, spec.route_scale, spec.routed_swiglu_limit,
                         spec.shared_swiglu_limit, max_tokens,
                         None if bias is None else bias.ctypes.data, None if sl is None else sl.ctypes.data,
                         arr(self.mats["w1"]), arr(self.mats["w3"]), arr(self.mats["w2"]))
        p = C.c_void_p()
        try:
            _native_check(self.lib, self.lib.vlb_ep_layer_create(dev.h, comm.ptr, C.byref(d), C.byref(p)))
        except Exception:
            self._release_mats()
            raise
        self.ptr = p
        self.max_tokens = max_tokens
        self.failed: Optional[str] = None

    def forward_device(self, x_ptr: int, logits_ptr: int, T: int, out_ptr: int, stream: int = 0) -> None:
        """x [T, H] f32, logits [T, E] f32 and out [T, H] f32 device addresses."""
        st = self.lib.vlb_ep_forward_device(self.dev.h, self.ptr, C.c_void_p(x_ptr), C.c_void_p(logits_ptr), T,
                                            C.c_void_p(out_ptr), C.c_void_p(stream))
        if st != 0:
            buf = C.create_string_buffer(1024)
            self.lib.vlb_thread_error(buf, 1024)
            msg = buf.value.decode()
            # the driver prefixes an exchange failure with its phase ("counts: ...") and refuses a
            # failed layer with "an earlier exchange (<phase>) ..."
            phase = next((p for p in ("counts", "dispatch", "return", "communicator")
                          if msg.startswith(p + ":") or msg.startswith(f"an earlier exchange ({p})")), None)
            if phase is not None:
                from . import VlbError

                self.failed = phase
                raise EpExchangeError(phase, VlbError(st, msg))
            _native_check(self.lib, st)

    def forward(self, x, logits, T: int):
        """torch CUDA tensors x [T, H], logits [T, E] (f32); returns out [T, H] on the library
        stream's device."""
        import torch

        out = torch.empty((T, self.spec.hidden), dtype=torch.float32, device=x.device)
        lib_stream = torch.cuda.ExternalStream(self.dev.stream, device=x.device)
        lib_stream.wait_stream(torch.cuda.current_stream(x.device))  # inputs written on torch's stream
        # the step ends with a synchronisation of the library stream (its status read), so `out`
        # is complete when this returns
        self.forward_device(x.data_ptr(), logits.data_ptr(), T, out.data_ptr(), self.dev.stream)
        return out

    @property
    def last(self) -> dict:
        ms = (C.c_float * 5)()
        rows = (C.c_uint64 * 2)()
        if self.lib.vlb_ep_last_phases(self.ptr, ms, rows) != 0:
            return {}
        d = {name: ms[i] / 1000.0 for i, name in enumerate(self.PHASES)}
        d["received_rows"], d["sent_rows"] = int(rows[0]), int(rows[1])
        return d

    def _release_mats(self) -> None:
        for lst in self.mats.values():
            for m in lst:
                self.dev.release_matrix(m)

    def close(self) -> None:
        if getattr(self, "ptr", None):
            st = self.lib.vlb_ep_layer_destroy(self.dev.h, self.ptr)
            self.ptr = C.c_void_p()
            self._release_mats()
            _native_check(self.lib, st)
