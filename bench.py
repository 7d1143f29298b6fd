#!/usr/bin/env python
"""Benchmark of the fused FP8 block-scale DeepSeek-V3 MoE (main.py::fused_moe) on B200.

Workload (one "step" = one MoE layer call): BASELINE config 3 -- T = 8192 tokens,
all 256 experts, expert parallelism over N = --gpus ranks (E_local = 256/N,
local_expert_offset = rank * E_local).  Hidden states and routing logits are
replicated on every rank; rank r owns output tokens [r*T/N, (r+1)*T/N).  By
default GEMM2 stores each pair row into its token owner's buffer over peer memory
and the owner sums its tokens' rows; `--combine nccl` instead reduce-scatters
un-rounded fp32 partials.  At N = 1 the step is the plain fused_moe call.

value  = tokens/s of the whole job (T * steps / max-over-ranks device time).
e2e    = the same through the public API with the activations copied from pinned
         host memory and the rank's output rows copied back, inside the timing.
At N > 1 the line's `token_dispatch` object (inputs token-sharded: each rank holds
T/N tokens) carries its own `e2e`, in which each rank uploads only its tokens.
On N = 1 the line also carries the decode sweep (config 1: T = 1..64, 32 local
experts, HBM roofline) and prefill points (config 2: skewed routing, FP8 tensor
roofline), each measured with L2 flushed (cold and clean, L2Flush) between calls, after a 5 s idle pause
that lets the SM clock recover from the power-capped config-3 loop, and each with
its own `clocks` record.

`--impl reference` times the reference operator's own CPU algorithm (the oracle
restatement of run(), solution/triton/main.py:2430-2609) on a bounded sample of
the same workload on the host cores, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "flashinfer-bench-moe_b200")
sys.path.insert(0, PKG)

T_EP = 8192
E_TOTAL = 256
H = 7168
BYTES_PER_EXPERT = 29_360_128 + 14_680_064 + 7_168 + 3_584  # W1 + W2 fp8 + their fp32 scales
BYTES_PER_TOKEN = 7_168 + 224 + 1_024 + 14_336             # hidden fp8 + scales + logits + bf16 out
FLOPS_PER_PAIR = 2 * (4096 * 7168 + 7168 * 2048)
SWEEP_SETTLE_S = 5.0  # idle pause before the N=1 sweeps (SM clock recovery after the power-capped loop)
GEMM1_FLOPS_PER_PAIR = 2 * 4096 * 7168


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during the timed region.

    NVML is polled from a background thread every 2 ms (timed regions can be a few
    milliseconds long); if NVML is unavailable, nvidia-smi is sampled every 200 ms."""

    REASONS = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20), ("hw_thermal_slowdown", 0x40),
               ("hw_power_brake_slowdown", 0x80), ("sw_power_cap", 0x4))

    def __init__(self, device_index: int, interval_s: float = 0.002):
        self.dev = device_index
        self.interval_s = interval_s
        self.samples = []
        self.max_mhz = None
        self.source = "none"

    def __enter__(self):
        import threading
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.dev)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons

            def poll():
                while not self._stop.is_set():
                    try:
                        self.samples.append((float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),
                                             int(get_reasons(h))))
                    except Exception:
                        pass
                    self._stop.wait(self.interval_s)
            self.source = "nvml"
        except Exception:
            def poll():
                while not self._stop.is_set():
                    try:
                        out = subprocess.run(["nvidia-smi", "--query-gpu=clocks.sm,clocks.max.sm",
                                              "--format=csv,noheader,nounits", "-i", str(self.dev)],
                                             capture_output=True, text=True, timeout=5).stdout
                        mhz, mx = [float(x) for x in out.strip().split(",")[:2]]
                        self.max_mhz = mx
                        self.samples.append((mhz, 0))
                    except Exception:
                        pass
                    self._stop.wait(0.2)
            self.source = "nvidia-smi"
        self._thread = threading.Thread(target=poll, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thread.join(timeout=5)
        return False

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"], "samples": 0,
                    "source": self.source}
        mhz = [m for m, _ in self.samples]
        reasons = sorted({name for _, bits in self.samples for name, bit in self.REASONS if bits & bit})
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples), "source": self.source}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


METRIC = "tokens/s per MoE layer call (DS-V3 FP8 MoE, T=8192, 256 experts, EP over N GPUs)"


def workload_config(world):
    """The workload both arms report (identical dicts): what one step computes, not how."""
    E_local = E_TOTAL // world
    return {"workload": "config3_ep_T8192_E256", "T": T_EP, "E_total": E_TOTAL, "E_local": E_local,
            "parallelism": f"ep{world}",
            "l2": "inputs larger than L2 (weights %.1f GB per GPU)" % (E_local * BYTES_PER_EXPERT / 1e9)}


# --------------------------------------------------------------------------- our arm
def ep_inputs(world, rank):
    import fbmoe_ep
    import fbmoe_workloads as W
    E_local, off = fbmoe_ep.shard(rank, world)
    weights = W.make_weights(E_local, 1000 + rank, "cuda")
    inp = W.make_inputs(T_EP, seed=0, config="standard", device="cuda", E_local=E_local,
                        local_expert_offset=off, weights=weights)
    return inp, E_local, off


def make_step(inp, world, rank, exchange=None):
    """One timed step: the operator on this rank's experts plus the cross-rank combine, either the fused
    peer-memory scatter (``exchange``, a fbmoe_ep.PeerExchange) or fp32 partial + NCCL reduce-scatter."""
    import fbmoe_lib as L
    args = [inp[k] for k in ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale",
                             "gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale")]
    off, scale = inp["local_expert_offset"], inp["routed_scaling_factor"]
    T = T_EP
    if world == 1:
        out = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")

        def step():
            L.forward(*args, off, scale, out=out, check=False)
            return out
        return step, out
    if exchange is not None:
        out = torch.empty((T // world, H), dtype=torch.bfloat16, device="cuda")

        def step():
            return exchange.forward(*args, scale, out=out, check=False)
        return step, out
    import fbmoe_ep
    partial = torch.empty((T, H), dtype=torch.float32, device="cuda")
    shard = torch.empty((T // world, H), dtype=torch.float32, device="cuda")
    out = torch.empty((T // world, H), dtype=torch.bfloat16, device="cuda")

    def step():
        L.forward(*args, off, scale, out=partial, check=False, partial_f32=True)
        fbmoe_ep.combine(partial, out=out, scratch=shard)
        return out
    return step, out


def local_pairs(inp, E_local, off):
    import fbmoe_lib as L
    idx, _ = L.route(inp["routing_logits"], inp["routing_bias"], inp["routed_scaling_factor"])
    loc = (idx >= off) & (idx < off + E_local)
    return int(loc.sum().item()), int(torch.unique(idx[loc]).numel())


def run_ours(args, world, rank, local):
    import fbmoe_lib as L
    peaks = load_peaks()
    inp, E_local, off = ep_inputs(world, rank)
    exchange, fallback = None, None
    if world > 1 and args.combine == "p2p":
        import fbmoe_ep
        try:
            exchange = fbmoe_ep.PeerExchange(T_EP, dispatch=True)
        except RuntimeError as e:  # raised on every rank alike: all ranks take the NCCL combine
            fallback = str(e)[:300]
    step, out = make_step(inp, world, rank, exchange)
    for _ in range(args.warmup):
        step()
    barrier(world)

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    L.profile_begin(args.steps)
    with ClockSampler(local) as clk:
        barrier(world)
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        barrier(world)
    stage_ms, nfwd = L.profile_end()
    ms = max_over_ranks(start.elapsed_time(end), world)
    ms_per_step = ms / args.steps
    value = T_EP * args.steps / (ms / 1e3)

    # roofline of the dominant kernel (per launch, averaged over the timed region, this rank)
    pairs, active = local_pairs(inp, E_local, off)
    per_stage = {n: stage_ms[i] / max(nfwd, 1) for i, n in enumerate(L.STAGES)}
    dom = max(("gemm1", "gemm2"), key=lambda n: per_stage[n])
    if dom == "gemm1":
        flops = pairs * GEMM1_FLOPS_PER_PAIR
        peak = 2.0 * peaks["bf16_tflops_sustained"]
        peak_note = "fp8 dense = 2x the measured sustained bf16 cuBLAS figure"
    else:
        flops = pairs * 2 * 7168 * 2048
        peak = peaks["bf16_tflops_sustained"]
        peak_note = "f16 dense = the measured sustained bf16 cuBLAS figure"
    achieved = flops / (per_stage[dom] / 1e3) / 1e12
    traffic = None
    tpath = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get(f"{dom}_ep{world}_bytes_per_launch")
    roofline = {"bound": "tensor", "kernel": dom, "achieved": round(achieved, 1), "peak": round(peak, 1),
                "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                "peak_source": f"{peaks['source']} ({peak_note})", "algorithmic_flops_per_launch": flops,
                "stage_ms_per_step": {k: round(v, 4) for k, v in per_stage.items()}, "local_pairs": pairs,
                "active_local_experts": active}

    if world == 1:
        e2e = run_e2e(args, world, rank, inp, "single")
    elif exchange is None:
        e2e = run_e2e(args, world, rank, inp, "nccl")
    else:
        # replicated inputs from the host: every rank uploading all T tokens, or each rank its T/N tokens plus
        # an NVLink all-gather; the line reports the faster plan and keeps the other beside it
        plans = [run_e2e(args, world, rank, inp, m, exchange) for m in ("replicated_full", "replicated_sliced")]
        e2e = dict(min(plans, key=lambda r: r["ms_per_step"]))
        e2e["plans"] = {r["mode"]: {"ms_per_step": r["ms_per_step"], "h2d_bytes_per_step": r["h2d_bytes_per_step"]}
                        for r in plans}
    dispatch = run_dispatch(args, world, rank, inp, exchange) if exchange is not None else None
    if dispatch is not None:
        dispatch["e2e"] = run_e2e(args, world, rank, inp, "dispatch", exchange)
    if fallback is not None:
        dispatch = {"unavailable": fallback}
    if exchange is not None:
        exchange.close()
    combine = ("none" if world == 1 else "GEMM2 epilogue stores pair rows into the owner's buffer over NVLink "
               "(CUDA IPC), owner sums slots" if exchange is not None else "nccl reduce_scatter fp32")
    line = {
        "metric": METRIC,
        "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp8_e4m3 GEMM1 / f16 GEMM2, fp32 accumulate",
        "data": "synthetic (seeded N(0,1) activations/logits, N(0,0.02) weights, FP8 block-quantised)",
        "config": workload_config(world), "combine": combine,
        "roofline": roofline, "e2e": e2e,
        "gpu_launches": launches_per_forward(T_EP, E_local, world, exchange is not None) * args.steps,
        "clocks": clk.summary(),
    }
    if dispatch is not None:
        line["token_dispatch"] = dispatch
    if world == 1 and not args.no_sweep:
        # After the seconds-long config-3 loop under the power cap the SM clock stays
        # near 1430 MHz for a few seconds; latency-bound decode calls timed then run
        # up to 20 % slower.  Let the clock recover, and record it for every sweep.
        time.sleep(SWEEP_SETTLE_S)
        for key, fn in (("decode_sweep", decode_sweep), ("quantiser", quantiser_point), ("prefill", prefill_points),
                        ("prepack", prepack_points),
                        ("fp8_intermediate", lambda p: fp8_intermediate_points(p, inp))):
            with ClockSampler(local, interval_s=0.05) as sweep_clk:
                line[key] = fn(peaks)
            line[key]["clocks"] = sweep_clk.summary()
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline_ep(inp, E_local)
    return line


def run_dispatch(args, world, rank, inp, exchange):
    """The token-dispatch layer on the same workload: rank r holds only tokens [r*T/N, (r+1)*T/N) (their logits,
    fp8 rows and scales), routes them, ships rows to the experts' ranks and gets its tokens' output rows back
    (csrc/moe_ep.cu).  Same T and experts as the replicated-input line; device time, max over ranks."""
    import fbmoe_ep
    lo, hi = fbmoe_ep.row_range(rank, world, T_EP)
    loc = (inp["routing_logits"][lo:hi].contiguous(), inp["routing_bias"], inp["hidden_states"][lo:hi].contiguous(),
           inp["hidden_states_scale"][:, lo:hi].contiguous())
    w = [inp[k] for k in ("gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale")]
    out = torch.empty((hi - lo, H), dtype=torch.bfloat16, device="cuda")

    def step():
        exchange.forward_dispatch(*loc, *w, inp["routed_scaling_factor"], out=out)

    for _ in range(args.warmup):
        step()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    s.record()
    for _ in range(args.steps):
        step()
    e.record()
    barrier(world)
    ms = max_over_ranks(s.elapsed_time(e), world)
    status = exchange.status()
    return {"value": round(T_EP * args.steps / (ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(ms / args.steps, 4),
            "inputs": "token-sharded (each rank holds T/N tokens)", "status": status,
            "gpu_launches_per_step": launches_per_forward(T_EP, E_TOTAL // world, world, True) + 3}


class E2ELoop:
    """The pipelined host-buffer loop of the e2e measurements.  Every step copies its activations H2D from pinned
    memory, runs the layer and copies this rank's output rows D2H, the way a server would run it: two device
    buffer sets, uploads on one copy stream and downloads on another, overlapping the neighbouring steps' compute.

    mode: "single" (N = 1, fused_moe), "replicated_full" (every rank uploads all T tokens), "replicated_sliced"
    (each rank uploads its T/N tokens; fbmoe_ep.TokenReplicator rebuilds all T on the compute stream),
    "dispatch" (token-dispatch layer on the rank's T/N tokens) or "nccl" (fp32 partial + reduce-scatter).

    Host copies slow a concurrent NVLink exchange several-fold (measured at N = 4: the dispatch send 0.14 ->
    0.4-0.6 ms, the NCCL all-gather 0.19 -> 1.13 ms).  In the two modes that open a step with an exchange (the
    dispatch send, the all-gather) the copies are therefore ordered after it: step i+1's upload and step i-1's
    download start once step i's exchange is done and overlap the rest of its compute."""

    def __init__(self, world, rank, inp, exchange, mode):
        import fbmoe_ep
        import fbmoe_lib as L
        self.L, self.world, self.rank, self.inp, self.exchange, self.mode = L, world, rank, inp, exchange, mode
        self.names = ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale")
        self.T = T = inp["routing_logits"].size(0)
        if mode in ("replicated_sliced", "dispatch"):
            lo, hi = fbmoe_ep.row_range(rank, world, T)
            src = {"routing_logits": inp["routing_logits"][lo:hi], "routing_bias": inp["routing_bias"],
                   "hidden_states": inp["hidden_states"][lo:hi],
                   "hidden_states_scale": inp["hidden_states_scale"][:, lo:hi]}
        else:
            src = {k: inp[k] for k in self.names}
        self.host = {k: src[k].cpu().contiguous().pin_memory() for k in self.names}
        self.dev = [{k: torch.empty(v.shape, dtype=v.dtype, device="cuda") for k, v in self.host.items()}
                    for _ in range(2)]
        self.w = [inp[k] for k in ("gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale")]
        rows = T // world
        self.out_host = [torch.empty((rows, H), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        self.out_dev = [torch.empty((rows, H), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
        self.h2d = sum(v.numel() * v.element_size() for v in self.host.values())
        self.d2h = self.out_host[0].numel() * self.out_host[0].element_size()
        self.rep = self.full = None
        if mode == "replicated_sliced":
            self.rep = fbmoe_ep.TokenReplicator(T)
            self.full = {k: torch.empty(inp[k].shape, dtype=inp[k].dtype, device="cuda")
                         for k in self.names if k != "routing_bias"}
        if mode == "nccl":
            self.partial = torch.empty((T, H), dtype=torch.float32, device="cuda")
            self.shard = torch.empty((rows, H), dtype=torch.float32, device="cuda")
        self.gate = mode in ("replicated_sliced", "dispatch")
        self.main = torch.cuda.current_stream()
        self.up, self.down = torch.cuda.Stream(), torch.cuda.Stream()
        self.ev_in = [torch.cuda.Event() for _ in range(2)]    # the slot's inputs uploaded
        self.ev_used = [torch.cuda.Event() for _ in range(2)]  # compute done with the slot
        self.ev_out = [torch.cuda.Event() for _ in range(2)]   # the slot's output downloaded
        self.ev_x = [torch.cuda.Event() for _ in range(2)]     # the step's exchange phase done
        for i in range(2):
            self.ev_used[i].record(self.main)
            self.ev_out[i].record(self.main)
        self.pending = None  # (slot, marks) whose download waits for the next step's exchange

    def _download(self, b, marks, after_x=None):
        self.down.wait_event(self.ev_used[b])
        if after_x is not None:
            self.down.wait_event(after_x)
        with torch.cuda.stream(self.down):
            _mark(marks, "down0", self.down)
            self.out_host[b].copy_(self.out_dev[b], non_blocking=True)
            _mark(marks, "down1", self.down)
        self.ev_out[b].record(self.down)

    def step(self, i, marks=None):
        L, main, b = self.L, self.main, i & 1
        self.up.wait_event(self.ev_used[b])
        if self.gate and i > 0:
            self.up.wait_event(self.ev_x[(i - 1) & 1])
        with torch.cuda.stream(self.up):
            _mark(marks, "up0", self.up)
            for k in self.names:
                self.dev[b][k].copy_(self.host[k], non_blocking=True)
            _mark(marks, "up1", self.up)
        self.ev_in[b].record(self.up)
        main.wait_event(self.ev_in[b])
        main.wait_event(self.ev_out[b])
        _mark(marks, "c0", main)
        d, ex, scale = self.dev[b], self.exchange, self.inp["routed_scaling_factor"]
        epoch = ex._next_epoch() if ex is not None else 0
        if self.rep is not None:
            self.rep.gather(d["routing_logits"], d["hidden_states"], d["hidden_states_scale"],
                            self.full["routing_logits"], self.full["hidden_states"], self.full["hidden_states_scale"])
            d = dict(self.full, routing_bias=d["routing_bias"])
        if self.mode == "dispatch":
            L.ep_dispatch_send(d["routing_logits"], d["routing_bias"], d["hidden_states"], d["hidden_states_scale"],
                               self.T, ex.E_local, scale, self.rank, self.world, ex.dispatch_ptrs, epoch,
                               ex.workspace)
        self.ev_x[b].record(main)
        _mark(marks, "exchanged", main)
        if self.pending is not None:
            self._download(*self.pending, after_x=self.ev_x[b])
            self.pending = None
        if self.mode == "single":
            L.forward(d["routing_logits"], d["routing_bias"], d["hidden_states"], d["hidden_states_scale"], *self.w,
                      self.inp["local_expert_offset"], scale, out=self.out_dev[b], check=False)
            _mark(marks, "computed", main)
        elif self.mode == "nccl":
            import fbmoe_ep
            L.forward(d["routing_logits"], d["routing_bias"], d["hidden_states"], d["hidden_states_scale"], *self.w,
                      self.inp["local_expert_offset"], scale, out=self.partial, partial_f32=True, check=False)
            _mark(marks, "computed", main)
            fbmoe_ep.combine(self.partial, out=self.out_dev[b], scratch=self.shard)
        else:
            if self.mode == "dispatch":
                L.ep_dispatch_compute(*self.w, self.T, self.rank, self.world, ex.dispatch_local, ex.ptrs, epoch,
                                      ex.workspace)
            else:
                L.ep_send((d["routing_logits"], d["routing_bias"], d["hidden_states"], d["hidden_states_scale"],
                           *self.w, ex.offset, scale), self.rank, self.world, ex.ptrs, epoch, ex.workspace,
                          check=False)
            _mark(marks, "computed", main)
            L.ep_recv(ex.local, self.T, self.rank, self.world, epoch, self.out_dev[b], ex.workspace)
        _mark(marks, "c1", main)
        self.ev_used[b].record(main)
        if self.gate:
            self.pending = (b, marks)
        else:
            self._download(b, marks)

    def flush(self):
        if self.pending is not None:
            self._download(*self.pending)
            self.pending = None
        self.main.wait_stream(self.down)


def _mark(marks, key, stream):
    if marks is not None:
        marks[key].record(stream)


E2E_MARKS = ("up0", "up1", "c0", "exchanged", "computed", "c1", "down0", "down1")


def run_e2e(args, world, rank, inp, mode, exchange=None, steps=None, instrument=False):
    """e2e of the layer through the public API with host buffers (E2ELoop), timed on the compute stream from before
    the first upload to after the last download; max over ranks.  instrument: also per-step stream timelines."""
    loop = E2ELoop(world, rank, inp, exchange, mode)
    n = steps if steps is not None else max(3, min(args.steps, 10))
    for i in range(2):
        loop.step(i)
    loop.flush()
    torch.cuda.synchronize()
    barrier(world)
    marks = [{k: torch.cuda.Event(enable_timing=True) for k in E2E_MARKS} for _ in range(n)] if instrument else None
    host_ms = []
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(loop.main)
    for i in range(n):
        t0 = time.perf_counter()
        loop.step(2 + i, marks[i] if instrument else None)
        host_ms.append((time.perf_counter() - t0) * 1e3)
    loop.flush()
    e.record(loop.main)
    torch.cuda.synchronize()
    barrier(world)
    own = s.elapsed_time(e)
    ms = max_over_ranks(own, world)
    res = {"value": round(loop.T * n / (ms / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": loop.h2d,
           "d2h_bytes_per_step": loop.d2h, "steps": n, "ms_per_step": round(ms / n, 4), "mode": mode,
           "pipelining": "2 buffer sets; H2D and D2H on their own streams overlap the neighbouring steps' compute"
                         + ("; copies ordered after the step's NVLink exchange" if loop.gate else "")}
    if instrument:
        tl = [{k: s.elapsed_time(v) for k, v in m.items()} for m in marks]
        med = lambda v: round(statistics.median(v), 3)  # noqa: E731
        res["timeline"] = {
            "rank": rank, "own_ms_per_step": round(own / n, 3), "upload": med([t["up1"] - t["up0"] for t in tl]),
            "exchange": med([t["exchanged"] - t["c0"] for t in tl]),
            "experts": med([t["computed"] - t["exchanged"] for t in tl]),
            "owner_combine": med([t["c1"] - t["computed"] for t in tl]),
            "compute_step": med([t["c1"] - t["c0"] for t in tl]),
            "download": med([t["down1"] - t["down0"] for t in tl]),
            "gap_between_steps": med([tl[i]["c0"] - tl[i - 1]["c1"] for i in range(1, len(tl))]),
            "host_enqueue": med(host_ms)}
        if exchange is not None:
            res["timeline"]["status"] = exchange.status()
    return res


def launches_per_forward(T, E_local, world=1, p2p=False):
    """Our kernels per forward (mirrors forward_core in csrc/moe_capi.cu): T <= 16: router+permute (one CTA),
    decode kernel; T <= 64: router, permute, decode kernel; otherwise router, [per-chunk count], permute, gather,
    GEMM1, GEMM2 (two launches: the pairs kernel and the one-block kernel, one of which returns at once), combine.
    The peer-memory expert-parallel path (csrc/moe_ep.cu) always takes the second chain and replaces the combine
    with a flag-release kernel and the owner's combine."""
    import fbmoe_lib as L
    if p2p and world > 1:
        return 8 + (1 if T > 1024 else 0)
    if L.block_rows(T, E_local) == 16:
        return 2 if T <= 16 else 3
    return 7 + (1 if T > 1024 else 0)


class L2Flush:
    """Called between timed calls.  A 256 MB read-modify-write evicts everything the previous call left in the
    126 MB L2.  In the default "clean" mode a read of another 256 MB follows, so the write's own dirty lines go
    back to DRAM before the timed call starts (a cold, clean L2: the state ncu's cache control gives a profiled
    launch).  "dirty" skips that read: the timed call then starts by writing back up to ~126 MB of the flush's
    data, which a streaming kernel pays for in DRAM time as if it were its own traffic."""

    def __init__(self, mode="clean"):
        assert mode in ("clean", "dirty")
        self.mode = mode
        self.w = torch.zeros(64 * 1024 * 1024, dtype=torch.float32, device="cuda")
        self.r = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device="cuda") if mode == "clean" else None

    def __call__(self):
        self.w.add_(1)
        if self.r is not None:
            torch.amax(self.r)


def time_calls(fn, iters, flush):
    ts = []
    for _ in range(3):
        fn()
    for _ in range(iters):
        flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e))
    return statistics.median(ts)


def decode_sweep(peaks):
    import fbmoe_lib as L
    import fbmoe_workloads as W
    weights = W.make_weights(32, 4242, "cuda")
    flush, dirty = L2Flush(), L2Flush("dirty")
    res = []
    for T in (1, 2, 4, 8, 16, 32, 64):
        inp = W.make_inputs(T, seed=T, config="standard", device="cuda", weights=weights)
        args = W.as_args(inp)
        us = 1e3 * time_calls(lambda: L.forward(*args, check=False), 30, flush)
        us_dirty = 1e3 * time_calls(lambda: L.forward(*args, check=False), 30, dirty)
        # stage breakdown from a separate pass: the events between stages serialise the launches
        L.profile_begin(8)
        time_calls(lambda: L.forward(*args, check=False), 5, flush)
        stage_ms, nf = L.profile_end()
        pairs, active = local_pairs(inp, 32, 0)
        nbytes = active * BYTES_PER_EXPERT + BYTES_PER_TOKEN * T + 512
        gbs = nbytes / (us / 1e6) / 1e9
        res.append({"T": T, "us_per_call": round(us, 2), "active_experts": active, "local_pairs": pairs,
                    "algorithmic_bytes": nbytes, "hbm_gbs": round(gbs, 1),
                    "frac_hbm": round(gbs / peaks["hbm_gbs"], 4), "us_per_call_dirty_l2": round(us_dirty, 2),
                    "frac_hbm_dirty_l2": round(nbytes / (us_dirty / 1e6) / 1e9 / peaks["hbm_gbs"], 4),
                    "stage_us_profiled": {n: round(1e3 * stage_ms[i] / max(nf, 1), 1) for i, n in enumerate(L.STAGES)}})
    del weights
    del dirty
    return {"config": "config1 decode, 32 local experts, offset 0, L2 flushed between calls",
            "flush": "clean (L2Flush); *_dirty_l2: the same calls after a flush that leaves its dirty lines in L2",
            "peak_hbm_gbs": peaks["hbm_gbs"], "peak_source": peaks["source"], "points": res}


def quantiser_point(peaks, T=8192):
    """The activation quantiser (bf16 [T,7168] -> e4m3 + [56,T] scales) at T tokens, L2 flushed between calls.
    HBM roofline: 14,336 B read + 7,168 + 224 B written per token."""
    import fbmoe_lib as L
    x = (torch.randn((T, H), device="cuda") * 3).to(torch.bfloat16)
    flush, dirty = L2Flush(), L2Flush("dirty")
    ms = time_calls(lambda: L.quantize_act(x), 20, flush)
    ms_dirty = time_calls(lambda: L.quantize_act(x), 20, dirty)
    nbytes = T * (2 * H + H + 4 * (H // 128))
    gbs = nbytes / (ms / 1e3) / 1e9
    return {"T": T, "us_per_call": round(ms * 1e3, 2), "algorithmic_bytes": nbytes, "hbm_gbs": round(gbs, 1),
            "frac_hbm": round(gbs / peaks["hbm_gbs"], 4), "us_per_call_dirty_l2": round(ms_dirty * 1e3, 2),
            "frac_hbm_dirty_l2": round(nbytes / ms_dirty / 1e6 / peaks["hbm_gbs"], 4)}


def prefill_points(peaks):
    import fbmoe_lib as L
    import fbmoe_workloads as W
    weights = W.make_weights(32, 4242, "cuda")
    flush = L2Flush()
    res = []
    for T in (1024, 4096, 8192):
        inp = W.make_inputs(T, seed=T, config="skew", device="cuda", weights=weights)
        args = W.as_args(inp)
        ms = time_calls(lambda: L.forward(*args, check=False), 10, flush)
        pairs, active = local_pairs(inp, 32, 0)
        flops = pairs * FLOPS_PER_PAIR
        tf = flops / (ms / 1e3) / 1e12
        # mixed precision: GEMM1 (2/3 of FLOPs) at fp8 rate, GEMM2 at f16 rate
        peak_mixed = 1.0 / ((2 / 3) / (2 * peaks["bf16_tflops"]) + (1 / 3) / peaks["bf16_tflops"])
        res.append({"T": T, "us_per_call": round(ms * 1e3, 1), "local_pairs": pairs, "tflops": round(tf, 1),
                    "frac_tensor_mixed_peak": round(tf / peak_mixed, 4),
                    "frac_fp8_peak": round(tf / (2 * peaks["bf16_tflops"]), 4)})
    return {"config": "config2 prefill, +3.0 bias on 4 local experts, 32 local experts",
            "peak_note": "fp8 peak = 2x measured bf16 burst; mixed peak weights GEMM1 fp8 and GEMM2 f16 by FLOPs",
            "points": res}


def prepack_points(peaks):
    """Offline W1 pre-pack (fbmoe_prepack_w1): the same calls on raw and on pre-packed W1, timed alternately on the
    same inputs (config 1 decode at T = 1, 8, 64; config 2 prefill at T = 4096, 8192), L2 flushed between calls."""
    import fbmoe_lib as L
    import fbmoe_workloads as W
    weights = W.make_weights(32, 4242, "cuda")
    packed = L.prepack_w1(weights[0])
    flush = L2Flush()
    res = []
    for T, cfg, iters in ((1, "standard", 30), (8, "standard", 30), (64, "standard", 30), (4096, "skew", 10),
                          (8192, "skew", 10)):
        inp = W.make_inputs(T, seed=T, config=cfg, device="cuda", weights=weights)
        raw_args = W.as_args(inp)
        pk_args = list(raw_args)
        pk_args[4] = packed
        raw = time_calls(lambda: L.forward(*raw_args, check=False), iters, flush)
        pk = time_calls(lambda: L.forward(*pk_args, check=False, w1_packed=True), iters, flush)
        res.append({"T": T, "config": cfg, "raw_us": round(raw * 1e3, 2), "prepacked_us": round(pk * 1e3, 2),
                    "speedup": round(raw / pk, 4)})
    del packed, weights
    return {"what": "forward on raw W1 vs on fbmoe_prepack_w1 layout (one TMA box per GEMM1 tile)", "points": res}


def fp8_intermediate_points(peaks, inp_ep):
    """The fp8-intermediate mode (forward(intermediate="fp8"): the reference solution's re-quantised SwiGLU
    output and an fp8 GEMM2) against the default f16 intermediate on the same inputs, timed alternately with L2
    flushed between calls: config 2 at T = 4096 and 8192, and config 3 (the N = 1 benchmark step, T = 8192 over
    all 256 experts).  Its accuracy is measured by tests/test_gpu_fp8_inter.py, not here."""
    import fbmoe_lib as L
    import fbmoe_workloads as W
    weights = W.make_weights(32, 4242, "cuda")
    flush = L2Flush()
    cases = [(T, "config2_skew", W.as_args(W.make_inputs(T, seed=T, config="skew", device="cuda", weights=weights)))
             for T in (4096, 8192)]
    cases.append((T_EP, "config3_ep1", W.as_args(inp_ep)))
    res = []
    for T, name, args in cases:
        f16 = time_calls(lambda: L.forward(*args, check=False), 6, flush)
        fp8 = time_calls(lambda: L.forward(*args, check=False, intermediate="fp8"), 6, flush)
        E = args[4].size(0)
        idx, _ = L.route(args[0], args[1], args[9])
        pairs = int(((idx >= args[8]) & (idx < args[8] + E)).sum().item())
        tf = pairs * FLOPS_PER_PAIR / (fp8 / 1e3) / 1e12
        res.append({"T": T, "config": name, "f16_us": round(f16 * 1e3, 1), "fp8_us": round(fp8 * 1e3, 1),
                    "speedup": round(f16 / fp8, 4), "fp8_tflops": round(tf, 1),
                    "fp8_frac_fp8_peak": round(tf / (2 * peaks["bf16_tflops"]), 4)})
    del weights, cases
    return {"what": "fp8-intermediate mode vs the default f16 intermediate (same inputs, alternated)",
            "peak_note": "fp8 peak = 2x measured bf16 burst (both GEMMs fp8 in this mode)", "points": res}


# --------------------------------------------------------------------------- CPU baselines
CPU_EXPERTS_PER_STEP = 4


def cpu_sample_steps(logits, bias, hs, hs_scale, E_local, n_steps, n_exp=CPU_EXPERTS_PER_STEP, seed=1000):
    """The reference's algorithm (the oracle's restatement of run(), solution/triton/main.py:2430-2609) on the
    host cores, one bounded sample per step: n_exp of the shard's E_local experts with every token routed to
    them (their rows dequantised, then per expert: W13/W2 dequantisation, GEMM1, SwiGLU, GEMM2, weighted
    accumulation).  Each step stands for the fraction n_exp / E_local of the layer, i.e. T * n_exp / E_local
    tokens.  The routing of all T tokens (about 0.1 s per call, under 1 % of it) is computed once, outside the
    steps.  Returns (per-step seconds, tokens per step, description)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import fbmoe_workloads as W
    import oracle as O
    T = logits.shape[0]
    routing = O.route(logits, bias, 2.5)
    idx = routing[0]
    w1, s1, w2, s2 = W.make_weights(n_exp, seed, "cpu")  # the sample's experts (same distributions)
    times = []
    for i in range(n_steps):
        e0 = (i * 37 * n_exp) % (E_local - n_exp + 1)
        rows = np.nonzero(((idx >= e0) & (idx < e0 + n_exp)).any(axis=1))[0]
        t0 = time.perf_counter()
        O.run(logits, bias, hs, hs_scale, w1, s1, w2, s2, e0, 2.5, tokens=rows, routing=routing)
        times.append(time.perf_counter() - t0)
    desc = (f"each step: {n_exp} of {E_local} experts with all their routed tokens of T={T} "
            f"(= {T * n_exp / E_local:.0f} tokens of the layer's work), oracle restatement of the reference's "
            f"run() (torch fp32 CPU + C router); routing of all T tokens once outside the steps")
    return times, T * n_exp / E_local, desc


def cpu_baseline_ep(inp, E_local, n_steps=4):
    """cpu_baseline for the N=1 line: a few sample steps of the reference algorithm on the host cores."""
    keys = ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale")
    logits, bias, hs, hs_scale = (inp[k].cpu() for k in keys)
    times, tok, desc = cpu_sample_steps(logits, bias, hs, hs_scale, E_local, n_steps)
    step_s = statistics.median(times)
    return {"value": round(tok / step_s, 2), "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n_steps} steps; " + desc, "seconds_per_step": round(step_s, 3),
            "seconds_per_call_estimate": round(step_s * E_local / CPU_EXPERTS_PER_STEP, 1)}


def run_reference(args, world, rank):
    """The reference algorithm on the host cores (oracle restatement of run()), rank 0 only; same metric, unit
    and config as our arm.  Every step is a bounded sample of the workload (cpu_sample_steps); ms_per_step is the
    measured wall time of a step and value the tokens it stands for per second."""
    if rank != 0:
        return None
    import fbmoe_workloads as W
    torch.set_num_threads(os.cpu_count() or 1)
    E_local = E_TOTAL // world
    logits, bias, hs, hs_scale = W.make_activations(T_EP, seed=0, config="standard", device="cpu")
    times, tok, desc = cpu_sample_steps(logits, bias, hs, hs_scale, E_local, args.warmup + args.steps)
    timed = times[args.warmup:]
    total = sum(timed)
    value = tok * len(timed) / total
    return {
        "impl": "reference", "metric": METRIC,
        "value": round(value, 3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / len(timed), 1), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp32 (reference run(): fp32 dequantisation and matmul on CPU)",
        "data": "synthetic (seeded N(0,1) activations/logits, N(0,0.02) weights, FP8 block-quantised)",
        "config": workload_config(world),
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# --------------------------------------------------------------------------- EP timeline (diagnosis)
def copy_bandwidth(nbytes=64 << 20, reps=5):
    """GB/s of H2D, D2H and both at once on separate streams, fresh pinned buffers, CUDA events."""
    h_up = torch.ones(nbytes, dtype=torch.uint8).pin_memory()
    h_down = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d_up = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    d_down = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    res = {}
    for name in ("h2d", "d2h", "duplex"):
        t_up, t_down = [], []
        for _ in range(reps):
            torch.cuda.synchronize()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            if name != "d2h":
                with torch.cuda.stream(up):
                    ev[0].record()
                    d_up.copy_(h_up, non_blocking=True)
                    ev[1].record()
            if name != "h2d":
                with torch.cuda.stream(down):
                    ev[2].record()
                    h_down.copy_(d_down, non_blocking=True)
                    ev[3].record()
            torch.cuda.synchronize()
            if name != "d2h":
                t_up.append(ev[0].elapsed_time(ev[1]))
            if name != "h2d":
                t_down.append(ev[2].elapsed_time(ev[3]))
        if t_up:
            res[name + "_up_gbs"] = round(nbytes / (statistics.median(t_up) / 1e3) / 1e9, 1)
        if t_down:
            res[name + "_down_gbs"] = round(nbytes / (statistics.median(t_down) / 1e3) / 1e9, 1)
    return res


def run_ep_timeline(args):
    """--case ep-timeline under torchrun (N >= 2): device-only steps of both EP layers, host copy bandwidth per
    rank alone and all ranks at once, and the per-step stream timelines of the e2e loops (run_e2e with events
    on every stream of every step); one JSON line."""
    import torch.distributed as dist
    import fbmoe_ep
    world, rank, local = dist_setup()
    if world < 2:
        raise SystemExit("--case ep-timeline needs torchrun with 2 or more ranks")
    inp, E_local, off = ep_inputs(world, rank)
    exchange = fbmoe_ep.PeerExchange(T_EP, dispatch=True)
    line = {"case": "ep-timeline", "n_gpus": world, "workload": workload_config(world), "host_cpus": os.cpu_count()}
    lo, hi = fbmoe_ep.row_range(rank, world, T_EP)
    loc = (inp["routing_logits"][lo:hi].contiguous(), inp["routing_bias"], inp["hidden_states"][lo:hi].contiguous(),
           inp["hidden_states_scale"][:, lo:hi].contiguous())
    w = [inp[k] for k in ("gemm1_weights", "gemm1_weights_scale", "gemm2_weights", "gemm2_weights_scale")]
    full = [inp[k] for k in ("routing_logits", "routing_bias", "hidden_states", "hidden_states_scale")]
    out = torch.empty((hi - lo, H), dtype=torch.bfloat16, device="cuda")
    scale = inp["routed_scaling_factor"]
    for name, fn in (("dispatch", lambda: exchange.forward_dispatch(*loc, *w, scale, out=out)),
                     ("replicated", lambda: exchange.forward(*full, *w, scale, out=out, check=False))):
        for _ in range(args.warmup):
            fn()
        barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.steps):
            fn()
        e.record()
        barrier(world)
        line[f"device_{name}_ms_per_step"] = round(max_over_ranks(s.elapsed_time(e), world) / args.steps, 4)
    alone = None
    for r in range(world):
        barrier(world)
        if rank == r:
            alone = copy_bandwidth()
        barrier(world)
    together = copy_bandwidth()
    barrier(world)
    objs = [None] * world
    dist.all_gather_object(objs, {"rank": rank, "alone": alone, "all_ranks_at_once": together})
    line["copy_gbs"] = objs
    for mode in ("dispatch", "replicated_full", "replicated_sliced"):
        r = run_e2e(args, world, rank, inp, mode, exchange, instrument=True)
        objs = [None] * world
        dist.all_gather_object(objs, r["timeline"])
        line["e2e_" + mode] = {"ms_per_step": r["ms_per_step"], "h2d_bytes_per_step": r["h2d_bytes_per_step"],
                               "d2h_bytes_per_step": r["d2h_bytes_per_step"], "ranks": objs}
    exchange.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def run_case(args):
    """One config at one T on GPU 0 (used for profiling captures): decode = config 1,
    prefill = config 2 (skewed routing); 32 local experts, L2 flushed between calls.
    quant = the activation quantiser alone on T rows."""
    import fbmoe_lib as L
    import fbmoe_workloads as W
    torch.cuda.set_device(0)
    peaks = load_peaks()
    if args.case == "quant":
        x = (torch.randn((args.T, H), device="cuda") * 3).to(torch.bfloat16)
        flush = L2Flush()
        for _ in range(args.warmup):
            L.quantize_act(x)
        ms = time_calls(lambda: L.quantize_act(x), args.steps, flush)
        nbytes = args.T * (2 * H + H + 4 * (H // 128))
        print(json.dumps({"case": "quant", "T": args.T, "us_per_call": round(ms * 1e3, 2),
                          "hbm_gbs": round(nbytes / (ms / 1e3) / 1e9, 1), "peak_hbm_gbs": peaks["hbm_gbs"]}),
              flush=True)
        return
    weights = W.make_weights(32, 4242, "cuda")
    inp = W.make_inputs(args.T, seed=args.T, config="skew" if args.case == "prefill" else "standard",
                        device="cuda", weights=weights)
    fargs = W.as_args(inp)
    flush = L2Flush()
    for _ in range(args.warmup):
        L.forward(*fargs, check=False)
    ts = []
    for _ in range(args.steps):
        flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        L.forward(*fargs, check=False)
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e))
    pairs, active = local_pairs(inp, 32, 0)
    ms = statistics.median(ts)
    nbytes = active * BYTES_PER_EXPERT + BYTES_PER_TOKEN * args.T + 512
    print(json.dumps({"case": args.case, "T": args.T, "us_per_call": round(ms * 1e3, 2), "local_pairs": pairs,
                      "active_experts": active, "hbm_gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
                      "tflops": round(pairs * FLOPS_PER_PAIR / (ms / 1e3) / 1e12, 1),
                      "peak_hbm_gbs": peaks["hbm_gbs"]}), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("fbmoe", "reference"), default="fbmoe")
    ap.add_argument("--combine", choices=("p2p", "nccl"), default="p2p",
                    help="N>1: GEMM2 stores pair rows into the owners' buffers over NVLink (p2p), or fp32 partial + "
                         "NCCL reduce-scatter (nccl)")
    ap.add_argument("--no-sweep", action="store_true", help="skip the decode/prefill sweeps (N=1)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--case", choices=("ep", "decode", "prefill", "shard", "quant", "ep-timeline"), default="ep",
                    help="ep = the benchmark line (default); decode/prefill/shard/quant = one small config for "
                         "profiling (quant = the activation quantiser on T rows; "
                         "shard = uniform routing over 32 local experts: one rank's work at N=8 when T=8192); "
                         "ep-timeline = per-rank stream timelines of the e2e loops and host copy bandwidth "
                         "(torchrun, N >= 2)")
    ap.add_argument("--T", type=int, default=64, help="tokens for --case decode/prefill/shard/quant")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.case == "ep-timeline":
        run_ep_timeline(args)
        return
    if args.case != "ep":
        run_case(args)
        return

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    world, rank, local = dist_setup()
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    line = run_ours(args, world, rank, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
