"""Benchmark of the B200 MoE routed-expert path (one JSON line on rank 0).

Workload (default): the DeepSeek-V4-Flash-shaped decode layer of the benchmark configurations
(config 1): H=4096, 256 routed IQ2_XXS experts + 1 Q8_0 shared expert, top-8 learned routing
(sqrt-softplus + bias, renormalised), I=2048, a decode batch of 64 tokens. A step is one layer
forward over the batch: router projection, top-k, dispatch, gate/up + SwiGLU, down, combine.
The same line carries a "prefill" object: configuration 3 (the same shapes, 4096 tokens,
N(0,1) routing logits, mixed IQ2_XXS / Q8_0 experts) through the tensor-core prefill path, with
its tensor roofline; and an "expert_parallel" object: configuration 4 (8192 tokens per GPU with
Zipf-skewed routing, the 256 experts sharded over the N GPUs, NCCL all-to-all exchange), whose
per-N values are the expert-parallel scaling. All inputs are seeded synthetic data with the
configurations' distributions (no checkpoint).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--tokens T] [--no-prefill]

--impl reference times the reference's own CPU implementation (the vastloom library compiled
from its sources into oracle/_ref, driven by the restated layer loop) on the host cores.
Multi-GPU (torchrun): every rank runs an independent replica of the layer on its own batch
(replicas only - no collective on the data path), value = all ranks' tokens / max rank time.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer tokens/s decode & prefill at 1/2/4/8 B200; % HBM / tensor roofline"
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0
L2_FLUSH_BYTES = 256 << 20


FALLBACK_BF16_TFLOPS = 1590.0
FALLBACK_BF16_SUSTAINED_TFLOPS = 1400.0


def load_peaks():
    if PEAKS_FILE.exists():
        p = json.loads(PEAKS_FILE.read_text())
        return float(p["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def load_tensor_peaks():
    """(burst, sustained) dense bf16 TFLOP/s; fp16 operands run at the same tensor rate."""
    if PEAKS_FILE.exists():
        p = json.loads(PEAKS_FILE.read_text())
        return float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured"
    return FALLBACK_BF16_TFLOPS, FALLBACK_BF16_SUSTAINED_TFLOPS, "fallback"


class ClockSampler:
    """SM clocks and throttle reasons sampled through NVML (read-only queries) every few
    milliseconds while the timed region runs. Without NVML (pynvml missing or failing) nothing is
    sampled and stop() returns {"samples": 0, "source": "unavailable: ..."}."""

    REASONS = {  # nvmlClocksEventReason bits
        "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, index: int, period_s: float = 0.005):
        self.index = index
        self.period = period_s
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = False
        self._thread = None
        self.unavailable = None

    def start(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 - any NVML failure means no clock record
            self.unavailable = f"unavailable: NVML ({type(e).__name__})"
            return

        def run():
            while not self._stop:
                try:
                    self.samples.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    self.reasons |= pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                except Exception:
                    pass
                time.sleep(self.period)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()

    def stop(self):
        if self._thread is None:
            return {"samples": 0, "source": self.unavailable or "unavailable: sampler not started"}
        self._stop = True
        self._thread.join(timeout=2)
        if not self.samples:
            return {"samples": 0, "source": "nvml (no sample inside the timed region)"}
        names = sorted(n for n, bit in self.REASONS.items() if self.reasons & bit)
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples), "source": "nvml"}


def phase_bytes(spec, W, layer, T, offsets):
    """Algorithmic bytes per phase of one forward (weights of the experts actually selected,
    activations read and written once)."""
    E, H, I, k = spec.experts, spec.hidden, spec.intermediate, spec.top_k
    active = [e for e in range(E) if offsets[e + 1] > offsets[e]]
    sz = lambda m: m.payload_bytes
    gu = sum(sz(layer.matrices["w1"][e]) + sz(layer.matrices["w3"][e]) for e in active)
    dn = sum(sz(layer.matrices["w2"][e]) for e in active)
    P = T * k
    if layer.shared_matrices:
        s1, s3, s2 = layer.shared_matrices
        gu += sz(s1) + sz(s3)
        dn += sz(s2)
        P += T
    return {
        "route": E * H * 4 + T * H * 4 + T * E * 8,
        "gate_up": gu + T * H * 4 + P * I * 4,
        "down": dn + P * I * 4 + P * H * 4,
        "combine": P * H * 4 + T * H * 4,
        "weights": gu + dn + E * H * 4,
        "active_experts": len(active),
    }


def traffic_from_profiles(kernel: str):
    f = ROOT / "profiles" / "ncu_traffic.json"
    if not f.exists():
        return None
    d = json.loads(f.read_text())
    return d.get(kernel)


def run_ours(args, rank, world, local_rank):
    import torch

    import vastloom_b200 as vb
    from vastloom_b200 import synth

    torch.cuda.set_device(local_rank)
    dev = vb.Device(local_rank)
    if args.only_prefill:
        stream = torch.cuda.ExternalStream(dev.stream, device=torch.device("cuda", local_rank))
        with torch.cuda.stream(stream):
            flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")

        def flush_only():
            with torch.cuda.stream(stream):
                flush.zero_()

        res = {"metric": METRIC, "n_gpus": world, "prefill": run_prefill(args, dev, stream, flush_only, rank, world,
                                                                        local_rank)}
        dev.close()
        return res
    spec = synth.config(1)
    T = args.tokens
    W = synth.layer_weights(spec, seed=1)
    layer = synth.upload_layer(dev, W, max_tokens=max(T, 64))
    x_host, _, _ = synth.activations(spec, T, seed=2 + rank)
    stream = torch.cuda.ExternalStream(dev.stream, device=torch.device("cuda", local_rank))
    with torch.cuda.stream(stream):
        x_dev = torch.from_numpy(x_host).cuda()
        out_dev = torch.empty((T, spec.hidden), dtype=torch.float32, device="cuda")
        flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    def step():
        layer.forward_device(x_dev.data_ptr(), T, out_dev.data_ptr(), stream=dev.stream)

    def flush_l2():
        with torch.cuda.stream(stream):
            flush.zero_()

    if args.only_hc:
        # the Hyper-Connection layer alone at T = --tokens (profiling runs of hc_entry_kernel)
        res = {"metric": METRIC, "n_gpus": world,
               "hyper_connection": run_hc_object(args, dev, stream, flush_l2, W, layer, tokens=(T,), plain=False)}
        layer.destroy()
        dev.close()
        return res
    for _ in range(args.warmup):
        flush_l2()
        step()
    torch.cuda.synchronize()
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        flush_l2()  # outside the events: every timed step starts with a cold L2
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    total_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    if dist:
        t = torch.tensor([total_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = T * world * args.steps / (total_ms / 1000.0)

    # result check against a finite output (parity is the tests' job)
    out = out_dev.cpu().numpy()
    assert np.all(np.isfinite(out))

    # end to end through the host-memory C-ABI call (H2D x, layer, D2H out, synchronise)
    e2e_times = []
    pinned_x = torch.from_numpy(x_host).pin_memory().numpy()
    pinned_out = torch.empty((T, spec.hidden), dtype=torch.float32).pin_memory().numpy()
    for i in range(max(3, args.steps)):
        flush_l2()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        layer.forward(pinned_x, out=pinned_out)
        e2e_times.append(time.perf_counter() - t0)
    e2e_value = T * world / statistics.mean(e2e_times)

    # per-phase device time of the same forward (events inside the library, on its stream)
    layer.set_profiling(True)
    phases = {p: [] for p in layer.PHASES}
    for _ in range(args.steps):
        flush_l2()
        step()
        for p, v in layer.phase_times().items():
            phases[p].append(v)
    layer.set_profiling(False)
    phase_ms = {p: statistics.mean(v) for p, v in phases.items()}
    idx, w, offsets, pt, ps = layer.last_route(T)
    pb = phase_bytes(spec, W, layer, T, offsets)
    hbm, peak_kind = load_peaks()
    dom = max(("gate_up", "down"), key=lambda p: phase_ms[p])
    achieved = pb[dom] / (phase_ms[dom] / 1000.0) / 1e9
    kernel_name = {"gate_up": "decode_experts_kernel<true>", "down": "decode_experts_kernel<false>"}[dom]
    traffic = traffic_from_profiles(kernel_name)
    layer_bytes = pb["route"] + pb["gate_up"] + pb["down"] + pb["combine"]
    result = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded; configuration distributions, no checkpoint)",
        "config": headline_config(spec, T, world),
        "roofline": {
            "bound": "hbm", "kernel": kernel_name, "achieved": round(achieved, 1),
            "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
            "peak_kind": peak_kind, "traffic": traffic,
            "algorithmic_bytes": pb[dom], "kernel_ms": round(phase_ms[dom], 5),
        },
        "layer_roofline": {
            "bytes": layer_bytes, "achieved_gbs": round(layer_bytes / (ms_per_step / 1000.0) / 1e9, 1),
            "frac": round(layer_bytes / (ms_per_step / 1000.0) / 1e9 / hbm, 4),
            "active_experts": pb["active_experts"],
        },
        "phase_ms": {p: round(v, 5) for p, v in phase_ms.items()},
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(x_host.nbytes), "d2h_bytes_per_step": int(out.nbytes),
                "timing": "host wall clock around the synchronous C-ABI call"},
        "clocks": clk,
        "gpu_launches": kernels_per_forward(spec, T) * args.steps,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(W, x_host, budget_s=args.cpu_budget)
        # the same sample on one host thread (the reference's serial matvec path)
        one = cpu_baseline(W, x_host, budget_s=args.cpu_budget / 3, threads=1)
        result["cpu_baseline"]["single_thread"] = {"value": one["value"], "cores": 1, "sample": one["sample"]}
    if not args.no_configs:
        result["configs"] = run_config_objects(args, dev, stream, flush_l2, rank, world, cfg1=(W, layer))
        result["formats"] = run_format_objects(args, dev, stream)
        result["records"] = run_record_objects(args, dev)
        result["hyper_connection"] = run_hc_object(args, dev, stream, flush_l2, W, layer)
    layer.destroy()
    for lst in layer.matrices.values():
        for m in lst:
            dev.release_matrix(m)
    for m in layer.shared_matrices or ():
        dev.release_matrix(m)
    if not args.no_prefill:
        result["prefill"] = run_prefill(args, dev, stream, flush_l2, rank, world, local_rank)
    if not args.no_ep:
        result["expert_parallel"] = run_ep(args, dev, rank, world, local_rank)
    dev.close()
    return result


def run_ep(args, dev, rank, world, local_rank):
    """Configuration 4: 256 experts placed over the N ranks by measured load (N = 1: all local),
    args.ep_tokens tokens per rank with Zipf(1.1)-skewed routing logits; dispatch and return by
    peer stores or NCCL (ep_exchange_label). Device-timed per step (CUDA events on the library
    stream around the whole step), max over ranks; also the per-rank expert-phase time, whose
    spread is the load imbalance, and a check of every token against one GPU holding all
    experts."""
    import torch

    from vastloom_b200 import synth
    from vastloom_b200.ep import TorchComm, balanced_slots, make_device_layer

    spec = synth.config(4)
    T = args.ep_tokens
    W = synth.layer_weights(spec, seed=4)
    x_host, _, logits_host = synth.activations(spec, T, seed=44 + rank)
    created_group = False
    if world == 1 and not torch.distributed.is_initialized():
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29500 + (os.getpid() % 1000)))
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
        created_group = True
    comm = TorchComm()
    # expert placement balanced by the measured load: every rank routes its own batch once, the
    # per-expert counts are summed over the ranks, and every rank computes the same placement
    idx0, _ = dev.route(logits_host, spec.top_k, spec.route_scale, score=spec.score, bias=W.bias)
    counts = torch.from_numpy(np.bincount(idx0.ravel(), minlength=spec.experts).astype(np.float64)).cuda()
    torch.distributed.all_reduce(counts)
    slots = balanced_slots(counts.cpu().numpy(), world)
    epr = spec.experts // world
    load_contig = counts.cpu().numpy().reshape(world, epr).sum(axis=1)
    load_bal = np.zeros(world)
    np.add.at(load_bal, slots // epr, counts.cpu().numpy())
    native = args.ep_driver == "native"
    if native:
        # the library's C++ driver with its own NCCL communicator (id made by rank 0, shared through
        # the process group); torch.distributed carries only the set-up and the timing reductions
        from vastloom_b200.ep import NativeEpComm, NativeEpLayer, native_unique_id

        uid = [native_unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(uid, src=0)
        ncomm = NativeEpComm(dev, uid[0], rank, world, timeout_ms=120_000)
        layer = NativeEpLayer(dev, ncomm, W, max_tokens=T, slots=slots)
        lib_stream = torch.cuda.ExternalStream(dev.stream, device=torch.device("cuda", torch.cuda.current_device()))
    else:
        layer, ops = make_device_layer(dev, W, comm, max_tokens=T, slots=slots)
        lib_stream = ops.stream
    xd = torch.from_numpy(x_host).cuda()
    ld = torch.from_numpy(logits_host).cuda()
    for _ in range(args.warmup):
        layer.forward(xd, ld, T)
    torch.cuda.synchronize()
    torch.distributed.barrier()
    steps = args.ep_steps or args.steps
    times, experts_s = [], []
    for _ in range(steps):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(lib_stream)
        layer.forward(xd, ld, T)
        end.record(lib_stream)
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end))
        experts_s.append(layer.last["experts_s"])
    torch.distributed.barrier()
    ms = statistics.mean(times)
    ms_max = comm.max_over_ranks(ms, xd)
    ex = statistics.mean(experts_s) * 1000.0
    ex_max = comm.max_over_ranks(ex, xd)
    ex_min = comm.min_over_ranks(ex, xd)
    recv = layer.last["received_rows"]
    recv_max = comm.max_over_ranks(float(recv), xd)
    recv_min = comm.min_over_ranks(float(recv), xd)
    out = layer.forward(xd, ld, T).cpu().numpy()
    assert np.all(np.isfinite(out))
    check = ep_parity_check(dev, W, x_host, logits_host, out)
    check_max = comm.max_over_ranks(check["max_rel_err"], xd)
    res = {
        "value": round(T * world / (ms_max / 1000.0), 1), "unit": "tokens/s", "ms_per_step": round(ms_max, 4),
        "steps": steps, "scaling": "weak", "n_gpus": world,
        "config": {"workload": f"cfg4-ep-zipf-T{T}x{world}", "hidden": spec.hidden,
                   "intermediate": spec.intermediate, "experts": spec.experts, "experts_per_gpu": spec.experts // world,
                   "top_k": spec.top_k, "tokens_per_gpu": T, "zipf_s": spec.zipf_s,
                   "exchange": ep_exchange_label(world, native),
                   "driver": ("C++ (vlb_ep_forward_device, the library's own NCCL communicator)" if native
                              else "Python orchestration over torch.distributed"),
                   "placement": "balanced by the measured expert load (longest-processing-time greedy, E/N per GPU)",
                   "expert_path": "tensor-core prefill kernels on the received rows"},
        "expected_rows_per_rank": {"contiguous_max": int(load_contig.max()), "balanced_max": int(load_bal.max()),
                                   "mean": int(load_bal.mean())},
        "timing": "CUDA events on the library stream around each step, max over ranks",
        "load_imbalance": {"experts_ms_max": round(ex_max, 4), "experts_ms_min": round(ex_min, 4),
                           "imbalance_ms": round(ex_max - ex_min, 4), "received_rows_max": int(recv_max),
                           "received_rows_min": int(recv_min), "rows_per_rank_balanced": T * spec.top_k},
        "phases_ms_rank0": {k_: round(v * 1000.0, 4) for k_, v in layer.last.items() if k_.endswith("_s")},
        "check": {"max_rel_err": check_max, "rank0": check, "bound": 4e-3,
                  "against": "the same tokens through one GPU holding all experts, exact decode path"},
    }
    assert check_max <= 4e-3, f"expert-parallel output differs from the single-GPU layer: {check_max}"
    if native and world > 1:
        res["nvlink_all_to_all"] = all_to_all_reference(ncomm, lib_stream, comm, xd, world, T, spec, res)
    if native:
        layer.close()
        ncomm.close()
    else:
        ops.close()
    if created_group:
        torch.distributed.destroy_process_group()
    return res


def ep_exchange_label(world, native):
    """How the expert-parallel step moves its rows (the library's policy; phases_ms shows the cost)."""
    payload = ("fp16 rows + (expert, weight, max|x|) words out, fp16 results with a per-row power-of-two "
               "scale back")
    if world == 1:
        return "one rank: NCCL send/receive to itself; " + payload
    if native and world <= 16 and os.environ.get("VLB_EP_EXCHANGE", "") != "nccl":
        return ("rows and results by peer stores into CUDA-IPC-mapped receive buffers over NVLink when every "
                "rank maps every peer (else NCCL all-to-all); counts and meta words over NCCL; " + payload)
    return "NCCL all-to-all: " + payload


def all_to_all_reference(ncomm, stream, comm, like, world, T, spec, res):
    """The exchange's own roofline: a plain NCCL all-to-all on the same communicator and stream,
    equal splits, at the step's two sizes (dispatch: T*k fp16 rows of H; return: the same rows'
    fp16 results), CUDA events around 5 calls after 2, max over ranks. algbw = bytes a rank sends
    / time; busbw = algbw * (N-1)/N (the bytes that cross NVLink), against the pool's measured
    770 GB/s per direction peer copy. The step's dispatch and return phases are then expressed
    as a fraction of this reference time."""
    import torch

    out = {"timing": "CUDA events on the library stream, 5 calls after 2, max over ranks",
           "peer_copy_gbs_reference": 770.0}
    sizes = {"dispatch": T * spec.top_k * spec.hidden * 2, "return": T * spec.top_k * spec.hidden * 2}
    for name, total in sizes.items():
        per = (total // world) // 256 * 256
        send = torch.empty(per * world, dtype=torch.uint8, device="cuda")
        recv = torch.empty(per * world, dtype=torch.uint8, device="cuda")
        for _ in range(2):
            ncomm.all_to_all(send.data_ptr(), [per] * world, recv.data_ptr(), [per] * world, stream=stream.cuda_stream)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            ncomm.all_to_all(send.data_ptr(), [per] * world, recv.data_ptr(), [per] * world, stream=stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = comm.max_over_ranks(e0.elapsed_time(e1) / 5, like)
        alg = per * world / (ms / 1000.0) / 1e9
        bus = alg * (world - 1) / world
        entry = {"bytes_per_rank": per * world, "ms": round(ms, 4), "algbw_gbs": round(alg, 1),
                 "busbw_gbs": round(bus, 1), "busbw_frac_of_peer_copy": round(bus / 770.0, 4)}
        phase = res["phases_ms_rank0"].get(f"{name}_s")
        if phase:
            entry["step_phase_ms"] = phase
            entry["step_phase_over_reference"] = round(phase / ms, 3)
        out[name] = entry
        del send, recv
    return out


def ep_parity_check(dev, W, x_host, logits_host, out_ep):
    """The expert-parallel output of this rank's tokens against the same tokens through a
    single-GPU layer holding all experts on the exact decode path (f32 accumulation of exact
    products; itself held to 1e-5 against the oracle by the tests). The exchange carries fp16
    rows and the group forward runs the tensor-core path, so ~1e-3 is expected."""
    import vastloom_b200 as vb
    from vastloom_b200 import synth

    T = x_host.shape[0]
    full = synth.upload_layer(dev, W, max_tokens=T)
    try:
        full.set_prefill_tokens(vb.MoeLayer.PREFILL_NEVER)
        ref = full.forward(x_host, None, logits_host)
    finally:
        full.destroy()
        for lst in full.matrices.values():
            for m in lst:
                dev.release_matrix(m)
        for m in full.shared_matrices or ():
            dev.release_matrix(m)
    diff = np.abs(out_ep.astype(np.float64) - ref.astype(np.float64))
    num = np.linalg.norm(out_ep.astype(np.float64) - ref.astype(np.float64), axis=1)
    den = np.maximum(np.linalg.norm(ref.astype(np.float64), axis=1), 1e-30)
    return {"max_rel_err": float(np.max(diff) / max(float(np.max(np.abs(ref))), 1e-30)),
            "max_token_rel_err": float(np.max(num / den)), "tokens": int(T)}


def run_prefill(args, dev, stream, flush_l2, rank, world, local_rank):
    """Configuration 3 at 4096 tokens per GPU through the tensor-core prefill path."""
    import torch

    from vastloom_b200 import synth

    spec = synth.config(3)
    if args.prefill_experts != spec.experts:  # smaller case of the same kernels (profiling)
        import dataclasses
        spec = dataclasses.replace(spec, experts=args.prefill_experts)
    T = args.prefill_tokens
    W = synth.layer_weights(spec, seed=3)
    layer = synth.upload_layer(dev, W, max_tokens=T)
    assert layer.prefill_tokens() <= T
    x_host, _, logits_host = synth.activations(spec, T, seed=33 + rank)
    with torch.cuda.stream(stream):
        x_dev = torch.from_numpy(x_host).cuda()
        lg_dev = torch.from_numpy(logits_host).cuda()
        out_dev = torch.empty((T, spec.hidden), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    def step():
        layer.forward_device(x_dev.data_ptr(), T, out_dev.data_ptr(), logits_ptr=lg_dev.data_ptr(), stream=dev.stream)

    for _ in range(args.warmup):
        flush_l2()
        step()
    torch.cuda.synchronize()
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    steps = args.prefill_steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush_l2()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk = clocks.stop()
    total_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    if dist:
        t = torch.tensor([total_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / steps
    value = T * world * steps / (total_ms / 1000.0)
    out = out_dev.cpu().numpy()
    assert np.all(np.isfinite(out))
    # end to end: host x and logits in, host output back, per call
    pinned_x = torch.from_numpy(x_host).pin_memory().numpy()
    pinned_l = torch.from_numpy(logits_host).pin_memory().numpy()
    pinned_out = torch.empty((T, spec.hidden), dtype=torch.float32).pin_memory().numpy()
    e2e = []
    for _ in range(3):
        flush_l2()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        layer.forward(pinned_x, None, pinned_l, out=pinned_out)
        e2e.append(time.perf_counter() - t0)
    e2e_value = T * world / statistics.mean(e2e)
    layer.set_profiling(True)
    phases = {p: [] for p in layer.PHASES}
    for _ in range(steps):
        flush_l2()
        step()
        for p, v in layer.phase_times().items():
            phases[p].append(v)
    layer.set_profiling(False)
    phase_ms = {p: statistics.mean(v) for p, v in phases.items()}
    pairs = T * spec.top_k + T  # routed pairs + the shared expert's
    flops = {"gate_up": 2.0 * 2 * spec.hidden * spec.intermediate * pairs,
             "down": 2.0 * spec.hidden * spec.intermediate * pairs}
    burst, sustained, kind = load_tensor_peaks()
    dom = max(flops, key=lambda p: phase_ms[p])
    achieved = flops[dom] / (phase_ms[dom] / 1000.0) / 1e12
    layer_tflops = (flops["gate_up"] + flops["down"]) / (ms_per_step / 1000.0) / 1e12
    res = {
        "value": round(value, 1), "unit": "tokens/s", "ms_per_step": round(ms_per_step, 4), "steps": steps,
        "dtype": "fp16 operands, f32 accumulation (tensor cores); routing f32/f64",
        "config": {"workload": f"cfg3-prefill-mixed-T{T}", "hidden": spec.hidden,
                   "intermediate": spec.intermediate, "experts": spec.experts, "top_k": spec.top_k,
                   "shared_experts": 1, "tokens_per_gpu": T, "routed_types": "IQ2_XXS / Q8_0 (seeded coin)",
                   "shared_type": "Q8_0", "routing": "given N(0,1) logits, sqrt_softplus+bias, renorm",
                   "l2": "flushed (256 MiB write) before every timed step"},
        "roofline": {"bound": "tensor", "kernel": f"prefill_gemm_kernel<{'true' if dom == 'gate_up' else 'false'}>",
                     "achieved": round(achieved, 1), "peak": burst, "unit": "TFLOP/s",
                     "frac": round(achieved / burst, 4),
                     "peak_kind": f"{kind} burst bf16 (a kernel of a few ms timed alone; fp16 runs at the same rate)",
                     "frac_of_sustained": round(achieved / sustained, 4), "peak_sustained": sustained,
                     "traffic": traffic_from_profiles(f"prefill_gemm_kernel<{'true' if dom == 'gate_up' else 'false'}>"),
                     "algorithmic_flops": flops[dom], "kernel_ms": round(phase_ms[dom], 5)},
        "layer_tflops": round(layer_tflops, 1),
        "phase_ms": {p: round(v, 5) for p, v in phase_ms.items()},
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(x_host.nbytes + logits_host.nbytes), "d2h_bytes_per_step": int(out.nbytes),
                "timing": "host wall clock around the synchronous C-ABI call"},
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(W, x_host, budget_s=args.cpu_budget / 2, logits=logits_host)
    layer.destroy()
    for lst in layer.matrices.values():
        for m in lst:
            dev.release_matrix(m)
    for m in layer.shared_matrices or ():
        dev.release_matrix(m)
    return res


def cpu_baseline(W, x, budget_s: float, threads: int | None = None, logits=None, token_ids=None):
    """The reference's own CPU path (oracle/_ref) on a bounded sample of the same batch."""
    from oracle.oracle import Reference

    if not Reference.available():
        return {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference",
                "sample": "unavailable: oracle/_ref is not built"}
    ref = Reference()
    cores = os.cpu_count() or 1
    # RowWorkPool has hardware_concurrency()/2 workers plus the caller (ggml_quantization.cpp:761)
    threads = threads or max(1, cores // 2 + 1)
    lg = (lambda a, b: None) if logits is None else (lambda a, b: logits[a:b])
    tk = (lambda a, b: None) if token_ids is None else (lambda a, b: token_ids[a:b])
    t0 = time.perf_counter()
    ref.moe_forward(W, x[:1], tk(0, 1), lg(0, 1), threads=threads)
    t1 = time.perf_counter() - t0
    n = int(max(1, min(x.shape[0], budget_s / max(t1, 1e-6))))
    t0 = time.perf_counter()
    ref.moe_forward(W, x[:n], tk(0, n), lg(0, n), threads=threads)
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 3), "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": f"first {n} of the {x.shape[0]} batch tokens through the reference's layer loop "
                      f"({dt:.1f} s, max_threads={threads} of {cores} host threads)"}


# ---- decode-size objects of the other benchmark configurations ---------------------------------

MMA_TYPES = (8, 16, 18, 19)  # Q8_0, IQ2_XXS, IQ3_XXS, IQ1_S: all on the decode_experts_kernel instances


def kernels_per_forward(spec, T, logits_given=False, norm=False):
    """Kernel launches of one layer forward (the library's launch sequence for this shape)."""
    types = {spec.gate_type, spec.down_type} | ({spec.shared_type} if spec.shared_type is not None else set())
    n = 1  # token prescale, or the RMSNorm entry step of a residual block
    n += 1 if logits_given else 1  # score kernel on given logits, or the router projection
    n += 1  # top-k route
    n += 1 if T * spec.top_k <= 4096 else 3  # dispatch
    if any(t in MMA_TYPES for t in types):
        n += 4  # per phase: the activation image, then the decode kernel
    if any(t not in MMA_TYPES for t in types):
        n += 2
    return n + 1  # combine


def expert_kernel_name(spec, phase):
    t = spec.gate_type if phase == "gate_up" else spec.down_type
    flag = "true" if phase == "gate_up" else "false"
    return f"decode_experts_kernel<{flag}>" if t in MMA_TYPES else f"expert_kernel<{flag}>"


def measure_decode_object(dev, stream, flush_l2, Ws, layers, T, x_host, tok_host, args, rank, world, workload,
                          chain=False, cpu_budget=5.0):
    """One decode-size workload: a single layer (chain=False) or the layers applied in sequence as
    residual blocks (chain=True). Device-timed steps with a cold L2, the host-memory C-ABI call
    end to end, per-phase times, the HBM roofline of the dominant expert kernel, and the
    reference CPU path on a bounded sample."""
    import torch

    import vastloom_b200 as vb

    spec = Ws[0].spec
    H = spec.hidden
    with torch.cuda.stream(stream):
        bufs = [torch.from_numpy(x_host).cuda(), torch.empty((T, H), dtype=torch.float32, device="cuda")]
        if chain:
            bufs.append(torch.empty((T, H), dtype=torch.float32, device="cuda"))
        tok_dev = torch.from_numpy(tok_host.astype(np.uint32).view(np.int32)).cuda() if tok_host is not None else None
    torch.cuda.synchronize()
    tok_ptr = tok_dev.data_ptr() if tok_dev is not None else 0

    def step():
        if not chain:
            layers[0].forward_device(bufs[0].data_ptr(), T, bufs[1].data_ptr(), token_ids_ptr=tok_ptr, stream=dev.stream)
            return
        src = 0
        for i, layer in enumerate(layers):
            dst = 1 if i % 2 == 0 else 2
            layer.forward_device(bufs[src].data_ptr(), T, bufs[dst].data_ptr(), token_ids_ptr=tok_ptr, stream=dev.stream)
            src = dst

    for _ in range(args.warmup):
        flush_l2()
        step()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    steps = args.steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush_l2()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    total_ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends))
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([total_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms = total_ms / steps
    for layer in layers:
        layer.status()
    # end to end through the public host-memory calls
    pinned_x = torch.from_numpy(x_host).pin_memory().numpy()
    e2e = []
    if chain:
        lc = vb.LayerChain(dev, layers, max_tokens=T)
        try:
            for _ in range(max(3, min(steps, 20))):
                flush_l2()
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                out = lc.forward(pinned_x, tok_host)
                e2e.append(time.perf_counter() - t0)
        finally:
            lc.close()
    else:
        out = torch.empty((T, H), dtype=torch.float32).pin_memory().numpy()
        for _ in range(max(3, min(steps, 20))):
            flush_l2()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            layers[0].forward(pinned_x, tok_host, out=out)
            e2e.append(time.perf_counter() - t0)
    assert np.all(np.isfinite(out))
    # phases (summed over the layers of a chain) and algorithmic bytes
    phase_sum = {p: 0.0 for p in vb.MoeLayer.PHASES}
    bytes_sum = {"route": 0, "gate_up": 0, "down": 0, "combine": 0}
    active = []
    for layer in layers:
        layer.set_profiling(True)
    reps = max(3, min(steps, 20))
    for _ in range(reps):
        flush_l2()
        step()
        for layer in layers:
            for p, v in layer.phase_times().items():
                phase_sum[p] += v / reps
    for W, layer in zip(Ws, layers):
        layer.set_profiling(False)
        _, _, offsets, _, _ = layer.last_route(T)
        pb = phase_bytes(W.spec, W, layer, T, offsets)
        for p in bytes_sum:
            bytes_sum[p] += pb[p]
        active.append(pb["active_experts"])
    hbm, peak_kind = load_peaks()
    dom = max(("gate_up", "down"), key=lambda p: phase_sum[p])
    achieved = bytes_sum[dom] / (phase_sum[dom] / 1000.0) / 1e9
    layer_bytes = sum(bytes_sum.values())
    res = {
        "value": round(T * world / (ms / 1000.0), 1), "unit": "tokens/s", "ms_per_step": round(ms, 5),
        "steps": steps, "tokens_per_gpu": T, "workload": workload,
        "roofline": {"bound": "hbm", "kernel": expert_kernel_name(spec, dom), "achieved": round(achieved, 1),
                     "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4), "peak_kind": peak_kind,
                     "traffic": None, "algorithmic_bytes": bytes_sum[dom], "kernel_ms": round(phase_sum[dom], 5)},
        "layer_roofline": {"bytes": layer_bytes, "achieved_gbs": round(layer_bytes / (ms / 1000.0) / 1e9, 1),
                           "frac": round(layer_bytes / (ms / 1000.0) / 1e9 / hbm, 4), "active_experts": active},
        "phase_ms": {p: round(v, 5) for p, v in phase_sum.items()},
        "e2e": {"value": round(T * world / statistics.mean(e2e), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(x_host.nbytes + (0 if tok_host is None else 4 * T)),
                "d2h_bytes_per_step": int(T * H * 4),
                "timing": "host wall clock around the synchronous host-memory call"},
        "gpu_launches": sum(kernels_per_forward(W.spec, T, norm=chain) for W in Ws) * steps,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_chain(Ws, x_host, tok_host, cpu_budget) if chain else \
            cpu_baseline(Ws[0], x_host, budget_s=cpu_budget, token_ids=tok_host)
    return res


def cpu_baseline_chain(Ws, x, tok, budget_s):
    """The reference's CPU path for the residual chain: its RMSNorm and its layer loop per layer,
    f32 residual addition, on the first n tokens of the batch."""
    from oracle.oracle import Reference

    if not Reference.available():
        return {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference",
                "sample": "unavailable: oracle/_ref is not built"}
    ref = Reference()
    cores = os.cpu_count() or 1
    threads = max(1, cores // 2 + 1)
    H = Ws[0].spec.hidden
    ones = np.ones(H, np.float32)

    def run(n):
        h = x[:n].copy()
        for W in Ws:
            o, _, _ = ref.moe_forward(W, ref.rms_norm(h, ones, 1e-6), None if tok is None else tok[:n],
                                      threads=threads)
            h = (h + o).astype(np.float32)
        return h

    t0 = time.perf_counter()
    run(1)
    t1 = time.perf_counter() - t0
    n = int(max(1, min(x.shape[0], budget_s / max(t1, 1e-6))))
    t0 = time.perf_counter()
    run(n)
    dt = time.perf_counter() - t0
    return {"value": round(n / dt, 3), "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": f"first {n} of the {x.shape[0]} prompt tokens through the reference's RMSNorm and layer loop, "
                      f"{len(Ws)} layers ({dt:.1f} s, max_threads={threads} of {cores} host threads)"}


def run_config_objects(args, dev, stream, flush_l2, rank, world, cfg1=None):
    """Decode-size numbers of configurations 0 (T = 1, 16), 1 (T = 1, 8; the headline is T = 64)
    and 2 (the three-layer residual chain, prompts of 1 and 5 tokens)."""
    from vastloom_b200 import synth

    out = {}
    budget = args.cpu_budget / 4

    def release(layer):
        layer.destroy()
        for lst in layer.matrices.values():
            for m in lst:
                dev.release_matrix(m)
        for m in layer.shared_matrices or ():
            dev.release_matrix(m)

    spec0 = synth.config(0)
    W0 = synth.layer_weights(spec0, seed=10)
    L0 = synth.upload_layer(dev, W0, max_tokens=16)
    try:
        for T in (1, 16):
            x, _, _ = synth.activations(spec0, T, seed=20 + T + 100 * rank)
            out[f"cfg0-T{T}"] = measure_decode_object(dev, stream, flush_l2, [W0], [L0], T, x, None, args, rank, world,
                                                     f"cfg0-olmoe-q8_0-T{T}", cpu_budget=budget)
    finally:
        release(L0)
    if cfg1 is not None:
        W1, L1 = cfg1
        for T in (1, 8):
            x, _, _ = synth.activations(W1.spec, T, seed=30 + T + 100 * rank)
            out[f"cfg1-T{T}"] = measure_decode_object(dev, stream, flush_l2, [W1], [L1], T, x, None, args, rank, world,
                                                     f"cfg1-v4flash-decode-T{T}", cpu_budget=budget)
    spec2 = synth.config(2)
    W2 = [synth.layer_weights(spec2, seed=40 + i) for i in range(3)]
    L2 = [synth.upload_layer(dev, W, max_tokens=8, layer_index=i) for i, W in enumerate(W2)]
    try:
        for layer in L2:
            layer.set_input_norm(np.ones(spec2.hidden, np.float32), 1e-6)
        for T in (1, 5):
            x, tok, _ = synth.activations(spec2, T, seed=60 + T + 100 * rank)
            out[f"cfg2-chain-T{T}"] = measure_decode_object(dev, stream, flush_l2, W2, L2, T, x, tok, args, rank, world,
                                                           f"cfg2-hash-chain-3x-T{T}", chain=True, cpu_budget=budget)
    finally:
        for layer in L2:
            release(layer)
    return out


def run_format_objects(args, dev, stream):
    """The operator seam's dequant-matvec (vlb_matvec_device) for every storage type on a 4096 x
    4096 matrix, 1 and 4 tokens: 16 different matrices per type (more bytes than the L2) taken in
    turn, CUDA events around 64 calls; bytes = the matrix's GGUF payload + activations + outputs,
    against the HBM copy peak. The parity of each format is the test suite's."""
    import ctypes as C

    import torch

    import vastloom_b200 as vb
    from vastloom_b200 import synth

    peak, peak_kind = load_peaks()
    rows = cols = 4096
    names = {vb.TYPE_Q8_0: "Q8_0", vb.TYPE_IQ2_XXS: "IQ2_XXS", vb.TYPE_IQ3_XXS: "IQ3_XXS", vb.TYPE_IQ1_S: "IQ1_S",
             vb.TYPE_Q4_K: "Q4_K", vb.TYPE_Q5_K: "Q5_K", vb.TYPE_Q6_K: "Q6_K", vb.TYPE_IQ2_S: "IQ2_S",
             vb.TYPE_MXFP4: "MXFP4"}
    rng = np.random.default_rng(77)
    x = torch.from_numpy(rng.standard_normal((4, cols)).astype(np.float32)).cuda()
    y = torch.empty((4, rows), dtype=torch.float32, device="cuda")
    ext = torch.cuda.ExternalStream(dev.stream, device=x.device)
    out = {}
    for t, name in names.items():
        enc = synth.matrix(rng, t, rows, cols, synth.D_SCALE[t])
        mats = [dev.upload_matrix(t, rows, cols, enc, identity=0x5000 + i) for i in range(16)]
        try:
            res = {"payload_bytes": int(enc.nbytes)}
            for ntok in (1, 4):
                def call(i):
                    dev._check(dev.lib.vlb_matvec_device(dev.h, mats[i % 16].ptr, C.c_void_p(x.data_ptr()), ntok, cols,
                                                         C.c_void_p(y.data_ptr()), rows, C.c_void_p(dev.stream)))
                for i in range(16):
                    call(i)
                dev.synchronize()
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ev0.record(ext)
                for i in range(64):
                    call(i)
                ev1.record(ext)
                ev1.synchronize()
                ms = ev0.elapsed_time(ev1) / 64
                nbytes = enc.nbytes + ntok * cols * 4 + ntok * rows * 4
                gbs = nbytes / (ms * 1e-3) / 1e9
                res[f"T{ntok}"] = {"us_per_call": round(ms * 1000, 2), "achieved_gbs": round(gbs, 1),
                                   "frac": round(gbs / peak, 4), "weights_per_s": round(rows * cols / (ms * 1e-3), 1)}
            res["roofline"] = {"bound": "hbm", "peak": peak, "unit": "GB/s", "peak_kind": peak_kind,
                               "kernel": "gemv_kernel", "frac_T1": res["T1"]["frac"]}
            out[name] = res
        finally:
            for m in mats:
                dev.release_matrix(m)
    return {"workload": "vlb_matvec_device, 4096 x 4096 matrix, 16 matrices in turn (> L2), 64 calls",
            "timing": "CUDA events on the library stream", "by_type": out}


def run_hc_object(args, dev, stream, flush_l2, W, layer, tokens=(1, 64), plain=True):
    """The config-1 layer with and without the Hyper-Connection entry and exit (m = 4 copies of
    the hidden state, 20 Sinkhorn iterations, f32 mixing weight [24 x 16384]) at T = 1 and 64:
    device time per forward (CUDA events, cold L2) and the profiled phases. The entry's mixing
    projection is 24 sequential f64 chains of m x H = 16,384 steps per token (the reference's
    summation order, needed for bit-identical mixes): a latency floor that does not shrink with T."""
    import torch

    H, m = W.spec.hidden, 4
    rng = np.random.default_rng(12)
    mw = (2 + m) * m
    fn = (rng.standard_normal((mw, m * H)) * 0.02).astype(np.float32)
    scale = (rng.random(3) + 0.5).astype(np.float32)
    base = (rng.standard_normal(mw) * 0.1).astype(np.float32)
    norm_w = np.ones(H, np.float32)
    out = {"workload": "cfg1 layer (IQ2_XXS experts + Q8_0 shared), Hyper-Connection m=4, 20 iterations"}

    def timed(T, rows):
        x = torch.from_numpy(rng.standard_normal((T, rows, H)).astype(np.float32)).cuda()
        y = torch.empty_like(x)
        for _ in range(3):
            flush_l2()
            layer.forward_device(x.data_ptr(), T, y.data_ptr(), stream=dev.stream)
        torch.cuda.synchronize()
        n = max(5, min(args.steps, 20))
        tot = 0.0
        for _ in range(n):
            flush_l2()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            layer.forward_device(x.data_ptr(), T, y.data_ptr(), stream=dev.stream)
            e1.record(stream)
            e1.synchronize()
            tot += e0.elapsed_time(e1)
        layer.status()
        layer.set_profiling(True)
        layer.forward_device(x.data_ptr(), T, y.data_ptr(), stream=dev.stream)
        torch.cuda.synchronize()
        phases = {k: round(v, 4) for k, v in layer.phase_times().items()}
        layer.set_profiling(False)
        return tot / n, phases

    try:
        for T in tokens:
            plain_ms, plain_ph = timed(T, 1) if plain else (None, None)
            layer.set_hyper_connection(m, fn, scale, base, norm_w, sinkhorn_iterations=20)
            hc_ms, hc_ph = timed(T, m)
            layer.set_hyper_connection(0, None, None, None, None)
            out[f"T{T}"] = {"ms_plain": plain_ms and round(plain_ms, 4), "ms_hc": round(hc_ms, 4),
                            "added_ms": plain_ms and round(hc_ms - plain_ms, 4), "phases_plain": plain_ph,
                            "phases_hc": hc_ph}
    finally:
        if layer.hc_m:
            layer.set_hyper_connection(0, None, None, None, None)
    return out


def run_record_objects(args, dev):
    """Expert records to device: 32 config-1 expert records (IQ2_XXS W1 / W3 2048 x 4096 and W2
    4096 x 2048, 6.49 MB each, as an expert pack stores them) from page-locked memory through
    vlb_upload_record_async (one host-to-device copy per record, the re-layout on the device),
    host wall clock from the first start to the last finish. Beside it: a plain host-to-device
    copy of the same bytes from page-locked memory (the link's own rate in this run, CUDA events)
    and the host-path upload (vlb_upload_matrix, re-layout on the host) of the same matrices."""
    import torch

    import vastloom_b200 as vb
    from vastloom_b200 import synth

    spec = synth.config(1)
    H, I = spec.hidden, spec.intermediate
    rng = np.random.default_rng(5)
    n_rec = 32
    t = vb.TYPE_IQ2_XXS
    shapes = ((I, H), (I, H), (H, I))
    recs = []
    for e in range(n_rec):
        parts = [np.asarray(synth.matrix(rng, t, r, c, synth.D_SCALE[t]), np.uint8).reshape(-1) for r, c in shapes]
        recs.append(np.concatenate(parts))
    nbytes = recs[0].nbytes
    tensors = []
    off = 0
    for r, c in shapes:
        nb = vb.matrix_bytes(t, r, c)
        tensors.append((r, c, off, nb))
        off += nb
    pins = [dev.host_buffer(nbytes) for _ in range(n_rec)]
    for p, rec in zip(pins, recs):
        p.array[:] = rec

    def ident(e, j):
        return ((e + 1) * 8 + j) * 2 + 1

    def record_pass():
        ups = [dev.upload_record(p.array, [(ident(e, j), t, r, c, o, nb) for j, (r, c, o, nb) in enumerate(tensors)])
               for e, p in enumerate(pins)]
        return [m for u in ups for m in u.finish()]

    for m in record_pass():  # warm: staging grown, stream created
        dev.release_matrix(m)
    times = []
    for _ in range(3):
        dev.synchronize()
        t0 = time.perf_counter()
        mats = record_pass()
        times.append(time.perf_counter() - t0)
        for m in mats:
            dev.release_matrix(m)
    rec_s = min(times)
    # the link: one copy of every record from page-locked memory into one device buffer
    src = [torch.from_numpy(p.array) for p in pins]
    dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    for s_ in src[:4]:
        dst.copy_(s_, non_blocking=True)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for s_ in src:
        dst.copy_(s_, non_blocking=True)
    ev1.record()
    ev1.synchronize()
    link_s = ev0.elapsed_time(ev1) / 1e3
    # the host path on the same records
    t0 = time.perf_counter()
    host_mats = []
    for e, rec in enumerate(recs[:8]):
        for j, (r, c, o, nb) in enumerate(tensors):
            host_mats.append(dev.upload_matrix(t, r, c, rec[o:o + nb], identity=ident(e, j)))
    host_s = (time.perf_counter() - t0) * n_rec / 8
    for m in host_mats:
        dev.release_matrix(m)
    for p in pins:
        p.free()
    del src, dst
    total = n_rec * nbytes
    return {
        "workload": f"{n_rec} config-1 expert records (IQ2_XXS, {nbytes} B each) from page-locked memory",
        "record_path": {"ms": round(rec_s * 1e3, 3), "gbs": round(total / rec_s / 1e9, 2),
                        "timing": "host wall clock, first start to last finish, best of 3"},
        "h2d_copy": {"ms": round(link_s * 1e3, 3), "gbs": round(total / link_s / 1e9, 2),
                     "timing": "CUDA events around plain copies of the same bytes"},
        "host_path": {"ms": round(host_s * 1e3, 3), "gbs": round(total / host_s / 1e9, 2),
                      "timing": "host wall clock of vlb_upload_matrix on 8 records, scaled to all"},
        "frac_of_link": round(link_s / rec_s, 4),
    }


def headline_config(spec, T, world):
    """The headline workload (configuration-1 decode), the same dict on both arms of the bench."""
    return {
        "workload": f"cfg1-v4flash-decode-T{T}",
        "hidden": spec.hidden, "intermediate": spec.intermediate, "experts": spec.experts,
        "top_k": spec.top_k, "shared_experts": 1, "tokens_per_gpu": T,
        "routed_type": "IQ2_XXS", "shared_type": "Q8_0", "routing": "sqrt_softplus+bias, renorm",
        "parallelism": "replicas" if world > 1 else "single",
        "l2": "flushed (256 MiB write) before every timed step",
    }


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU implementation of the same layer and batch."""
    from vastloom_b200 import synth
    from oracle.oracle import Reference

    if rank != 0:
        return None
    if not Reference.available():
        return {"impl": "reference", "unavailable": "oracle/_ref (reference compiled from source) is not built"}
    spec = synth.config(1)
    T = args.tokens
    W = synth.layer_weights(spec, seed=1)
    x, _, _ = synth.activations(spec, T, seed=2)
    ref = Reference()
    cores = os.cpu_count() or 1
    threads = max(1, cores // 2 + 1)
    per_step = max(1, args.ref_tokens_per_step)
    for i in range(args.warmup):
        ref.moe_forward(W, x[i % T: i % T + 1], threads=threads)
    times = []
    for i in range(args.steps):
        lo = (i * per_step) % T
        t0 = time.perf_counter()
        ref.moe_forward(W, x[lo: lo + per_step], threads=threads)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = per_step * args.steps / total
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * total / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (f64 accumulation)",
        "data": "synthetic (seeded; configuration distributions, no checkpoint)",
        "config": headline_config(spec, T, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads, "kind": "reference",
                         "sample": (f"{per_step} token(s) of the {T}-token batch per step through the "
                                    f"reference's layer loop on {threads} host threads (CPU: no L2 flush)")},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    # long enough timed regions for the clock sampler to see the load (~0.1 s of decode steps)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--ref-tokens-per-step", type=int, default=1)
    ap.add_argument("--no-prefill", action="store_true", help="skip the configuration-3 prefill object")
    ap.add_argument("--prefill-tokens", type=int, default=4096)
    ap.add_argument("--prefill-steps", type=int, default=20)
    ap.add_argument("--prefill-experts", type=int, default=256,
                    help="routed experts of the prefill case (smaller = a profiling-sized case)")
    ap.add_argument("--only-prefill", action="store_true", help="run the prefill object alone")
    ap.add_argument("--only-hc", action="store_true",
                    help="run the Hyper-Connection layer alone at T = --tokens (no plain-layer comparison)")
    ap.add_argument("--no-ep", action="store_true", help="skip the configuration-4 expert-parallel object")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the decode objects of configurations 0, 1 (T = 1, 8) and 2 (chain)")
    ap.add_argument("--ep-tokens", type=int, default=8192)
    ap.add_argument("--ep-steps", type=int, default=0, help="0: --steps")
    ap.add_argument("--ep-driver", default="native", choices=["native", "torch"],
                    help="expert-parallel host side: the library's C++ driver or the Python orchestration")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    res = run_ours(args, rank, world, local_rank)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
