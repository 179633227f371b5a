"""Expert-parallel orchestration (vastloom_b200/ep.py) on CPU: two gloo ranks exchange real
tensors through torch.distributed all-to-all; the compute steps are a NumPy implementation
(oracle decode + f64 products) so that the routing, plan, exchange, shared-expert rows and combine
can be checked without a GPU. Each rank's output must equal the single-process layer computed
with the same NumPy steps on the same tokens."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vastloom_b200 import synth
from vastloom_b200.ep import ExpertParallelLayer, TorchComm, owner_counts


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


class NumpyExperts:
    """f64 expert products from the oracle's dequantized weights (V4 semantics: route weight
    before the down product, weight 1 for the shared expert)."""

    def __init__(self, oracle, W):
        spec = W.spec
        self.H, self.I = spec.hidden, spec.intermediate
        def deq(tb, r, c):
            be = 32 if tb[0] == synth.TYPE_Q8_0 else 256
            enc = np.frombuffer(bytes(tb[1]), np.uint8) if not isinstance(tb[1], np.ndarray) else tb[1]
            return oracle.dequantize(tb[0], enc, r * c // be, be).reshape(r, c).astype(np.float64)

        self.w = [tuple(deq(getattr(W, n)[e], *rc) for n, rc in (("w1", (self.I, self.H)), ("w3", (self.I, self.H)),
                                                                  ("w2", (self.H, self.I))))
                  for e in range(spec.experts)]
        self.shared = tuple(deq(tb, *rc) for tb, rc in zip(W.shared, ((self.I, self.H), (self.I, self.H), (self.H, self.I))))

    def apply(self, mats, x, w):
        g = mats[0] @ x
        u = mats[1] @ x
        act = g / (1.0 + np.exp(-g)) * u * w
        return mats[2] @ act


class NumpyEpOps:
    def __init__(self, oracle, W, rank, world):
        self.oracle = oracle
        self.spec = W.spec
        self.bias = W.bias
        self.ex = NumpyExperts(oracle, W)
        self.rank = rank
        self.epr = self.spec.experts // world

    def empty(self, shape, kind):
        return torch.zeros(shape, dtype={"f32": torch.float64, "i32": torch.int32, "rows": torch.float64,
                                         "meta": torch.float64}[kind])

    def mark(self):
        import time

        return time.perf_counter()

    def elapsed(self, marks):
        return [marks[i + 1] - marks[i] for i in range(len(marks) - 1)]

    def comm_scope(self):
        import contextlib

        return contextlib.nullcontext()

    def check(self):
        pass

    def reserve_group(self, rows):
        pass

    def route(self, logits, T):
        idx, w = self.oracle.route_learned(logits.numpy(), self.bias, self.spec.top_k, self.spec.route_scale,
                                           self.spec.score)
        return idx, w

    def plan(self, idx, w, x, T, epr, b):
        k = self.spec.top_k
        flat = idx.reshape(-1).astype(np.int64)
        order = np.argsort(flat, kind="stable")  # expert ascending, then element (token, slot)
        n = flat.size
        b.send_rows[:n] = torch.from_numpy(x.numpy()[order // k].astype(np.float64))
        b.send_meta[:n, 0] = torch.from_numpy((flat[order] % epr).astype(np.float64))
        b.send_meta[:n, 1] = torch.from_numpy(w.reshape(-1)[order].astype(np.float64))
        rows = np.empty(n, np.int32)
        rows[order] = np.arange(n, dtype=np.int32)
        b.elem_row[:n] = torch.from_numpy(rows)
        counts = np.bincount(flat, minlength=self.spec.experts)
        return np.concatenate([[0], np.cumsum(counts)]).astype(np.uint32)

    def append_shared_rows(self, b, R, x, T, epr):
        b.group_rows[R:R + T] = torch.from_numpy(x.numpy().astype(np.float64))
        b.group_meta[R:R + T, 0] = epr
        b.group_meta[R:R + T, 1] = 1.0

    def group_forward(self, b, rows):
        lo = self.rank * self.epr
        for r in range(rows):
            e = int(b.group_meta[r, 0])
            mats = self.ex.shared if e == self.epr else self.ex.w[lo + e]
            b.group_y[r] = torch.from_numpy(self.ex.apply(mats, b.group_rows[r].numpy(), float(b.group_meta[r, 1])))

    def combine(self, b, T, k, R):
        y = b.back_y.numpy()
        rows = b.elem_row.numpy()
        out = np.zeros((T, self.spec.hidden))
        for t in range(T):
            for j in range(k):
                out[t] += y[rows[t * k + j]]
            out[t] += b.group_y[R + t].numpy()
        return torch.from_numpy(out)


def _rank_main(rank, world, port, spec_args, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.oracle import Oracle

        oracle = Oracle(spec_args["grids"])
        spec = synth.config(4, "small")
        W = synth.layer_weights(spec, seed=spec_args["seed"])
        T = spec_args["T"]
        x, _, logits = synth.activations(spec, T, seed=spec_args["seed"] + 1 + rank)
        comm = TorchComm()
        ops = NumpyEpOps(oracle, W, rank, world)
        layer = ExpertParallelLayer(ops, comm, spec.experts, spec.top_k, spec.hidden, max_tokens=T)
        out = layer.forward(torch.from_numpy(x), torch.from_numpy(logits), T).numpy()
        # single-process reference on this rank's tokens
        idx, w = oracle.route_learned(logits, W.bias, spec.top_k, spec.route_scale, spec.score)
        ex = NumpyExperts(oracle, W)
        ref = np.zeros((T, spec.hidden))
        for t in range(T):
            for j in np.argsort(idx[t], kind="stable"):  # expert ascending, as the reference sums
                ref[t] += ex.apply(ex.w[int(idx[t, j])], x[t].astype(np.float64), float(w[t, j]))
            ref[t] += ex.apply(ex.shared, x[t].astype(np.float64), 1.0)
        err = float(np.max(np.abs(out - ref)) / max(np.max(np.abs(ref)), 1e-300))
        result_q.put((rank, err, layer.last["received_rows"], layer.last["sent_rows"]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,T", [(2, 9), (2, 1), (4, 5)])
def test_ep_orchestration_matches_single_process(grids, world, T):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    args = {"seed": 70 + T, "T": T, "grids": grids}
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, args, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    results = sorted(q.get(timeout=10) for _ in range(world))
    spec = synth.config(4, "small")
    assert sum(r[3] for r in results) == world * T * spec.top_k  # every pair sent once
    assert sum(r[2] for r in results) == world * T * spec.top_k  # and received once
    for rank, err, received, sent in results:
        assert err < 1e-12, (rank, err)


def test_owner_counts_split_expert_sorted_offsets():
    offsets = np.array([0, 2, 2, 5, 9, 9, 12, 12, 13], np.uint32)  # 8 experts, 2 per rank
    assert owner_counts(offsets, 4, 2) == [2, 7, 3, 1]


class _InjectedFailure(RuntimeError):
    pass


class FailingEpOps(NumpyEpOps):
    """NumpyEpOps whose rank raises at one step (a host-side stand-in for a rank that fails)."""

    def __init__(self, *args, fail_at=None):
        super().__init__(*args)
        self.fail_at = fail_at

    def plan(self, *args):
        if self.fail_at == "plan":
            raise _InjectedFailure("injected failure before the first exchange")
        return super().plan(*args)

    def group_forward(self, *args):
        if self.fail_at == "group_forward":
            raise _InjectedFailure("injected failure between the dispatch and the return exchange")
        return super().group_forward(*args)


def _failure_rank_main(rank, world, port, mode, grids, result_q):
    """Rank world - 1 fails (raises at `mode`, or never reaches the layer when mode is "absent");
    the other ranks must end their forward with EpExchangeError instead of waiting for it."""
    import datetime
    import time

    from vastloom_b200.ep import EpExchangeError

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=4))
    failing = rank == world - 1
    if failing and mode == "absent":
        time.sleep(12)  # alive but never joins an exchange; longer than the group's timeout
        os._exit(0)
    from oracle.oracle import Oracle

    oracle = Oracle(grids)
    spec = synth.config(4, "small")
    W = synth.layer_weights(spec, seed=91)
    T = 3
    x, _, logits = synth.activations(spec, T, seed=92 + rank)
    ops = FailingEpOps(oracle, W, rank, world, fail_at=mode if failing else None)
    layer = ExpertParallelLayer(ops, TorchComm(), spec.experts, spec.top_k, spec.hidden, max_tokens=T)
    if failing:
        layer.forward(torch.from_numpy(x), torch.from_numpy(logits), T)  # raises: the process ends with it
        os._exit(5)  # not reached
    t0 = time.perf_counter()
    try:
        layer.forward(torch.from_numpy(x), torch.from_numpy(logits), T)
        outcome = ("no error", None)
    except EpExchangeError as e:
        outcome = ("EpExchangeError", e.phase)
    elapsed = time.perf_counter() - t0
    try:  # the layer refuses further forwards at once
        t1 = time.perf_counter()
        layer.forward(torch.from_numpy(x), torch.from_numpy(logits), T)
        again = ("no error", None, 0.0)
    except EpExchangeError as e:
        again = ("EpExchangeError", e.phase, time.perf_counter() - t1)
    result_q.put((rank, outcome, elapsed, again))
    result_q.close()
    result_q.join_thread()
    os._exit(0)  # no destroy_process_group: a peer is gone


@pytest.mark.parametrize("mode,phase", [("plan", "counts"), ("group_forward", "return"), ("absent", "counts")])
def test_ep_failed_rank_ends_the_step_with_an_error(grids, mode, phase):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failure_rank_main, args=(r, world, port, mode, grids, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes[0] == 0, codes
    assert codes[1] == (0 if mode == "absent" else 1), codes
    rank, outcome, elapsed, again = q.get(timeout=10)
    assert rank == 0
    assert outcome == ("EpExchangeError", phase), outcome
    assert elapsed < 60.0, elapsed
    assert again[:2] == ("EpExchangeError", phase) and again[2] < 1.0, again


@pytest.mark.parametrize("zipf", [0.6, 1.1])
def test_balanced_slots_is_a_balanced_permutation(zipf):
    """LPT placement: a permutation of the expert ids, E / world experts per rank, Zipf loads
    spread within a few percent of the mean when no expert outweighs a rank's share, and the
    heaviest rank no heavier than the heaviest expert plus the lightest others when one does;
    always better than contiguous ranges."""
    from vastloom_b200.ep import balanced_slots

    E, world = 256, 8
    epr = E // world
    ranks = np.random.default_rng(3).permutation(E) + 1
    loads = ranks.astype(np.float64) ** -zipf * 1e6
    slots = balanced_slots(loads, world)
    assert sorted(slots.tolist()) == list(range(E))
    assert np.bincount(slots // epr, minlength=world).tolist() == [epr] * world
    per_rank = np.zeros(world)
    for e in range(E):
        per_rank[slots[e] // epr] += loads[e]
    mean = per_rank.mean()
    bound = max(1.05 * mean, loads.max() + np.sort(loads)[:epr - 1].sum())
    assert per_rank.max() <= bound * (1 + 1e-12)
    contiguous = loads.reshape(world, -1).sum(axis=1)
    assert contiguous.max() > per_rank.max()
    assert np.array_equal(slots, balanced_slots(loads, world))  # deterministic
