"""Benchmark of the B200 Jakal-Net hot path (one JSON line on rank 0).

Workload: SparsePropagation with a causal window of 512 intersected
with top-k 32 (window-intersect-top-k), batch 8, N=2048 nodes, dim 384, score rank 64,
bf16 inputs with f32 accumulation, softsign edges, seed 1; synthetic inputs of that shape
(val, state ~ N(0,1), projection weights ~ N(0, 1/sqrt(384)), core weight ones).
One step = the projections (two tcgen05 GEMMs) + the fused score / top-k / aggregate
kernel over the whole batch. Metric: scored (target, visible source) pairs per second.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 2|5]

Under torchrun every rank runs its own batch (weak scaling, no collective on the data
path); timings are device-side CUDA events, max over ranks.

--config 5 (B4, N32768, D512, R64, causal window 4096, top-k 64, bf16,
seed 4) runs the query-row-block partition instead: inputs replicated on every rank, rank r
computes rows [r N/P, (r+1) N/P) (jakal_net_b200.sharding), then an NCCL all-gather
assembles the outputs (strong scaling: the total work is fixed).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "jakal-net_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

B, N, D, R, K_TOP, WINDOW, SEED = 8, 2048, 384, 64, 32, 512, 1
METRIC = "fused propagation Gpairs/s"
UNIT = "Gpairs/s"
WORKLOAD = "config2: SparsePropagation causal window 512 intersect top-k 32, B8 N2048 D384 R64, bf16, softsign"
# dram__bytes_read.sum + dram__bytes_write.sum of one fused-kernel launch on this workload,
# from an ncu capture of this bench's kernel (a recorded constant, not measured per run).
NCU_TRAFFIC_BYTES = 16975104  # 16.98 MB read + 0 B written (outputs stay in L2), one launch

# Kernels each C-ABI entry point launches (the library's own kernels only).
KERNELS_PER_CALL = {
    "jk_lowrank_project": 1, "jk_lowrank_project_pair": 1, "jk_propagation_topk_forward": 1,
    "jk_propagation_topk_forward_mh": 1, "jk_propagation_topk_rows_forward": 1,
    "jk_propagation_window_forward": 1, "jk_propagation_window_forward_mh": 1, "jk_select_aggregate_forward": 1,
    "jk_split3_bf16": 1, "jk_split2_bf16": 1, "jk_transition_pairwise_topk_routes": 1,
    "jk_transition_pairwise_topk_routes_mh": 1, "jk_transition_pairwise_topk_forward": 2,
    "jk_transition_pairwise_topk_forward_mh": 2, "jk_transition_query_topk_forward": 1,
    "jk_transition_query_topk_forward_mh": 1, "jk_transition_pairwise_dense_forward": 2,
    "jk_transition_pairwise_dense_forward_mh": 2, "jk_softmax_backward": 1, "jk_softsign_backward": 1,
    "jk_topk_reduce_backward_edges": 1, "jk_topk_to_dense": 1,
}


def count_launches(fn) -> int:
    """Runs fn once and counts the library kernels it launches, from the C-ABI calls it makes."""
    import jakal_net_b200 as jk

    lib = jk._LIBRARY
    counts = {}
    saved = {}
    for name in KERNELS_PER_CALL:
        f = getattr(lib, name)
        saved[name] = f

        def wrapped(*a, _f=f, _n=name):
            counts[_n] = counts.get(_n, 0) + 1
            return _f(*a)

        setattr(lib, name, wrapped)
    try:
        fn()
    finally:
        for name, f in saved.items():
            setattr(lib, name, f)
    return sum(KERNELS_PER_CALL[n] * c for n, c in counts.items())


def pairs_per_batch_item(n: int, window: int) -> int:
    """Visible (target, source) pairs of a causal window: sum_t min(t, window) + 1."""
    return sum(min(t, window) + 1 for t in range(n))


PAIRS_PER_STEP = B * pairs_per_batch_item(N, WINDOW)


def fused_kernel_bytes() -> int:
    """Algorithmic HBM bytes of one fused-kernel launch: per target row it reads its
    target projection row and one source projection row (2 * R * 2 B; every source row is
    needed once per launch), one value row and one state of the sources (each needed once),
    and writes its output value row and state: (2*R*2 + D*2 + 2) + (D*2 + 2) bytes per row."""
    per_row = 2 * R * 2 + D * 2 + 2 + D * 2 + 2
    return B * N * per_row


def make_inputs(device, seed):
    g = torch.Generator().manual_seed(seed)
    val = torch.randn(B, N, D, generator=g)
    state = torch.randn(B, N, generator=g)
    w_s = torch.randn(R, D, generator=g) / D ** 0.5
    w_t = torch.randn(R, D, generator=g) / D ** 0.5
    core = torch.ones(R)
    core_hat = core / core.norm()
    to = dict(device=device, dtype=torch.bfloat16)
    return dict(val=val.to(**to), state=state.to(**to), w_s=w_s.to(**to), w_t=w_t.to(**to),
                core=core_hat.to(**to), bias=torch.zeros((), device=device, dtype=torch.bfloat16))


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML from a thread (read-only)."""

    REASONS = {
        0x0000000000000004: "sw_power_cap",
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown",
    }

    def __init__(self, index: int):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001
            self._nvml = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self._nvml.nvmlDeviceGetClockInfo(self._h, self._nvml.NVML_CLOCK_SM)
                rs = self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, rs))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self._nvml is not None:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._nvml is not None:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = statistics.median(s[0] for s in self.samples)
        reasons = set()
        for _, rs in self.samples:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        return {"sm_mhz": mhz, "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons), "samples": len(self.samples)}


def measured_peak_hbm():
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, "fallback"


def cpu_port_time(seconds: float = 10.0):
    """Times the CPU port (oracle/cpu_port.py) on one batch item of the same workload,
    repeated for about `seconds`; returns (pairs/s in G, sample description, threads)."""
    from oracle import cpu_port

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(SEED)
    val = torch.randn(1, N, D, generator=g).bfloat16().float()
    state = torch.randn(1, N, generator=g).bfloat16().float()
    w_s = (torch.randn(R, D, generator=g) / D ** 0.5).bfloat16()
    w_t = (torch.randn(R, D, generator=g) / D ** 0.5).bfloat16()
    core = torch.full((R,), 1.0 / R ** 0.5)
    pt = cpu_port.lowrank_project_bf16(val, w_t)  # untimed warm-up: first-call overheads
    ps = cpu_port.lowrank_project_bf16(val, w_s, core)
    cpu_port.window_topk_propagation(pt, ps, state, val, K_TOP, WINDOW)
    reps = 0
    t0 = time.perf_counter()
    while True:
        pt = cpu_port.lowrank_project_bf16(val, w_t)
        ps = cpu_port.lowrank_project_bf16(val, w_s, core)
        cpu_port.window_topk_propagation(pt, ps, state, val, K_TOP, WINDOW)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    pairs = reps * pairs_per_batch_item(N, WINDOW)
    sample = f"{reps} runs of 1 of the 8 batch items (N=2048, window 512, k 32) in {el:.1f} s, torch CPU ops"
    return pairs / el / 1e9, sample, threads


def _median_rate(run, work, seconds: float, min_reps: int = 3, warmup: bool = True):
    """Times run() until `seconds` have passed and at least min_reps runs were made (after
    an untimed warm-up run unless warmup is False); returns (work / median run time, runs)."""
    if warmup:
        run()
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < min_reps:
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    return work / statistics.median(times), len(times)


def cpu_reference_config2(seconds: float = 10.0):
    """The reference's own CPU code on config 2 (one batch item per run, all host threads):
    window-intersect-top-k is not a single reference op, so it is composed from the
    reference's primitives exactly as its Python path would run them -- the
    LowRankBilinearPairwise scores (modules.py:93-100), causal_window_mask and build_topk_mask
    (kernel_common.py:433-456), _compress_edges (propagation.py:67-88) and the einsum
    aggregate (propagation.py:215-219) -- in f32 (the reference's CPU precision).
    Returns (Gpairs/s, sample text, threads) or None when the reference is not staged."""
    jn, _ = _import_reference_model()
    if jn is None:
        return None
    from jakal_net.kernel_common import build_topk_mask, causal_window_mask
    from jakal_net.propagation import _compress_edges
    from torch.nn import functional as F

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(SEED)
    val = torch.randn(1, N, D, generator=g)
    state = torch.randn(1, N, generator=g)
    torch.manual_seed(SEED)
    pw = jn.LowRankBilinearPairwise(dim=D, rank=R)
    win = causal_window_mask(0, N, 0, N, WINDOW).view(1, N, N)

    @torch.no_grad()
    def run():
        scores = pw(val, val)
        masked = scores.masked_fill(~win, float("-inf"))
        keep = build_topk_mask(masked, K_TOP) & win
        e = _compress_edges(scores, F.softsign, mask=keep)
        return torch.einsum("bij,bj->bi", e, state), torch.einsum("bij,bjd->bid", e, val)

    rate, reps = _median_rate(run, pairs_per_batch_item(N, WINDOW), seconds)
    sample = (f"median of {reps} runs of 1 of the 8 batch items (N=2048, window 512, k 32, f32) through the "
              f"reference's own primitives; torch threads {torch.get_num_threads()}, {_cpu_model()}")
    return rate / 1e9, sample, threads


def cpu_port_time(seconds: float = 10.0):
    """The CPU port (oracle/cpu_port.py, the reference's blocked algorithm restated in torch
    CPU ops) on one batch item; returns (Gpairs/s, sample text, threads)."""
    from oracle import cpu_port

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(SEED)
    val = torch.randn(1, N, D, generator=g).bfloat16().float()
    state = torch.randn(1, N, generator=g).bfloat16().float()
    w_s = (torch.randn(R, D, generator=g) / D ** 0.5).bfloat16()
    w_t = (torch.randn(R, D, generator=g) / D ** 0.5).bfloat16()
    core = torch.full((R,), 1.0 / R ** 0.5)

    def run():
        pt = cpu_port.lowrank_project_bf16(val, w_t)
        ps = cpu_port.lowrank_project_bf16(val, w_s, core)
        cpu_port.window_topk_propagation(pt, ps, state, val, K_TOP, WINDOW)

    rate, reps = _median_rate(run, pairs_per_batch_item(N, WINDOW), seconds)
    sample = (f"median of {reps} runs of 1 of the 8 batch items (N=2048, window 512, k 32), blocked torch CPU "
              f"port; torch threads {torch.get_num_threads()}, {_cpu_model()}")
    return rate / 1e9, sample, threads


def cpu_native_window(seconds: float = 3.0):
    """The reference's C++ CPU extension (built from its sources by oracle/build_ref.py) on the
    closest single reference op to config 2: propagation_window (window 512, no top-k, softsign,
    f32) on one batch item, all host threads. Returns (Gpairs/s, runs) or None."""
    from oracle import build_ref

    if not build_ref.available("cpu"):
        return None
    native = build_ref.load_built("cpu")
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(SEED)
    val = torch.randn(1, N, D, generator=g)
    state = torch.randn(1, N, generator=g)
    w_s = torch.randn(R, D, generator=g) / D ** 0.5
    w_t = torch.randn(R, D, generator=g) / D ** 0.5
    core = torch.full((R,), R ** -0.5)

    def run():
        native.propagation_window("low_rank_bilinear", core, None, w_s, None, w_t, None, "softsign", val, state, val,
                                  WINDOW, 128, 128)

    rate, reps = _median_rate(run, pairs_per_batch_item(N, WINDOW), seconds, min_reps=1, warmup=False)
    return rate / 1e9, reps


def cpu_baseline_config2(seconds: float = 10.0):
    """The reference's own code when staged (kind "reference"), else the port (kind "port")."""
    ref = cpu_reference_config2(seconds)
    if ref is not None:
        return (*ref, "reference")
    return (*cpu_port_time(seconds), "port")


def run_reference(args, rank):
    if rank != 0:
        return
    if args.config == 4:
        jn, _ = _import_reference_model()
        if jn is None:
            print(json.dumps({"impl": "reference", "unavailable": "reference model not staged (baseline/_ref)"}))
            return
        value, sample, threads = cpu_progressive_b(max(10.0, min(30.0, 0.1 * args.steps)))
        metric, unit, cfg, dtype = C4_METRIC, "tokens/s", C4_WORKLOAD, "bf16"
        ms = C4["P"] * 2 / value * 1e3
        kind = "reference"
    elif args.config == 2:
        value, sample, threads, kind = cpu_baseline_config2(max(5.0, min(30.0, 0.05 * args.steps)))
        metric, unit, cfg, dtype = METRIC, UNIT, WORKLOAD, "f32"
        ms = PAIRS_PER_STEP / (value * 1e9) * 1e3
    elif args.config == 3:
        cb = cpu_config3(max(5.0, min(30.0, 0.05 * args.steps)))
        if cb is None:
            print(json.dumps({"impl": "reference", "unavailable": "the reference's native CPU build is absent"}))
            return
        value, sample, threads = cb
        metric, unit, cfg, dtype, kind = C3_METRIC, UNIT, C3_WORKLOAD, "f32", "reference"
        ms = C3["B"] * C3["Q"] * C3["S"] / (value * 1e9) * 1e3
    else:
        print(json.dumps({"impl": "reference", "unavailable": "the reference arm covers configs 2, 3 and 4"}))
        return
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic (seeded inputs of the config shape)",
        "config": {"workload": cfg, "implementation": "the reference's own CPU code on the host cores" if
                   kind == "reference" else "CPU port of the reference blocked path (oracle/cpu_port.py)"},
        "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args, rank, world, device):
    import jakal_net_b200 as jk

    inp = make_inputs(device, SEED + rank)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)

    def api_step(val, state):
        return jk.propagation_window_topk("low_rank_bilinear", inp["core"], inp["bias"], inp["w_s"], None,
                                          inp["w_t"], None, "softsign", val, state, val, WINDOW, K_TOP, 128, 128)

    launches_per_step = count_launches(lambda: api_step(inp["val"], inp["state"]))
    # CUDA graph of one step (projections + fused kernel) on the resident inputs.
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for _ in range(2):
            api_step(inp["val"], inp["state"])
    torch.cuda.current_stream(device).wait_stream(stream)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        api_step(inp["val"], inp["state"])

    # Kernel-only graph for the roofline (projections precomputed).
    row_proj = jk.lowrank_project(inp["val"], inp["w_t"])
    col_proj = jk.lowrank_project(inp["val"], inp["w_s"], core=inp["core"])
    torch.cuda.synchronize(device)
    kgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(kgraph):
        jk.topk_aggregate(row_proj, col_proj, inp["state"], inp["val"], K_TOP, window=WINDOW)

    def timed(replay, steps):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for e0, e1 in evs:
            flush.add_(1)  # write 256 MiB: evicts the 126 MB L2 between steps
            e0.record()
            replay()
            e1.record()
        torch.cuda.synchronize(device)
        return sum(e0.elapsed_time(e1) for e0, e1 in evs)  # ms

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(device.index if device.index is not None else 0) as clk:
        total_ms = timed(graph.replay, args.steps)
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
        t = torch.tensor([total_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps

    for _ in range(3):
        kgraph.replay()
    kernel_ms = timed(kgraph.replay, args.steps) / args.steps

    # End to end through the public API with host buffers: every step copies its inputs in
    # from pinned host memory and its outputs back. Steps are pipelined over three streams
    # (host-to-device copy, compute, device-to-host copy) with two buffer sets, so step
    # i + 1's upload and step i - 1's download overlap step i's compute (PCIe is full duplex).
    h_val = inp["val"].cpu().pin_memory()
    h_state = inp["state"].cpu().pin_memory()
    nbuf = 2
    d_val = [torch.empty_like(inp["val"]) for _ in range(nbuf)]
    d_state = [torch.empty_like(inp["state"]) for _ in range(nbuf)]
    h_out_state = [torch.empty(B, N, dtype=torch.bfloat16).pin_memory() for _ in range(nbuf)]
    h_out_val = [torch.empty(B, N, D, dtype=torch.bfloat16).pin_memory() for _ in range(nbuf)]
    s_in, s_cmp, s_out = (torch.cuda.Stream(device) for _ in range(3))
    ev_in = [torch.cuda.Event() for _ in range(nbuf)]
    ev_cmp = [torch.cuda.Event() for _ in range(nbuf)]
    ev_out = [torch.cuda.Event() for _ in range(nbuf)]
    e2e_steps = max(3, min(args.steps, 50))

    def e2e_run(steps):
        for i in range(steps):
            j = i % nbuf
            with torch.cuda.stream(s_in):
                s_in.wait_event(ev_cmp[j])  # the compute that last read buffer set j is done
                d_val[j].copy_(h_val, non_blocking=True)
                d_state[j].copy_(h_state, non_blocking=True)
                ev_in[j].record(s_in)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(ev_in[j])
                s_cmp.wait_event(ev_out[j])  # the download of this buffer set's last outputs is done
                st, vv = api_step(d_val[j], d_state[j])
                ev_cmp[j].record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_cmp[j])
                h_out_state[j].copy_(st, non_blocking=True)
                h_out_val[j].copy_(vv, non_blocking=True)
                st.record_stream(s_out)
                vv.record_stream(s_out)
                ev_out[j].record(s_out)

    e2e_run(3)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    s_cmp.wait_event(e0)
    e2e_run(e2e_steps)
    s_in.wait_stream(s_out)
    e1.record(s_in)
    torch.cuda.synchronize(device)
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    e2e_wall_ms = (time.perf_counter() - t0) * 1e3 / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms, kernel_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms, kernel_ms = (float(x) for x in t.tolist())

    c5 = None
    if not args.no_config5:
        if world > 1:
            torch.distributed.barrier()
        c5 = measure_config5(5, 3, rank, world, device)
    if rank != 0:
        return
    value = world * PAIRS_PER_STEP / (ms_per_step * 1e-3) / 1e9
    e2e_value = world * PAIRS_PER_STEP / (e2e_ms * 1e-3) / 1e9
    peak, peak_kind = measured_peak_hbm()
    achieved = fused_kernel_bytes() / (kernel_ms * 1e-3) / 1e9
    traffic = None if NCU_TRAFFIC_BYTES is None else int(NCU_TRAFFIC_BYTES)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded N(0,1) inputs of the config shape, random-init weights)",
        "config": {"workload": WORKLOAD, "batch_per_gpu": B, "nodes": N, "dim": D, "rank": R, "topk": K_TOP,
                   "window": WINDOW, "pairs_per_step_per_gpu": PAIRS_PER_STEP,
                   "l2": "flushed between timed steps (256 MiB write, outside the timed events)",
                   "timing": "CUDA graph replay of the step, CUDA events per step, max over ranks",
                   "parallelism": f"batch-sharded x{world}, no collective on the data path"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": (h_val.numel() + h_state.numel()) * 2,
                "d2h_bytes_per_step": (h_out_val[0].numel() + h_out_state[0].numel()) * 2, "ms_per_step": e2e_ms,
                "wall_ms_per_step": e2e_wall_ms,
                "how": "public op per step, pinned host inputs copied in and outputs copied out every step; "
                       "steps pipelined over copy-in / compute / copy-out streams (2 buffer sets)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, burst)",
                     "kernel": "jk::topk::topk_kernel (fused score / top-k / aggregate)",
                     "kernel_ms": kernel_ms, "algorithmic_bytes": fused_kernel_bytes(), "traffic": traffic,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of this "
                                       "kernel on this workload (recorded constant, not measured in this run)"},
    }
    if c5 is not None:
        line["config5_row_sharded"] = {
            "what": "config 5 (B4 N32768 D512 R64, window 4096, top-k 64) split by query-row blocks over the "
                    f"{world} GPU(s) of this run: strong scaling, total work fixed",
            "compute": {"value": c5["pairs"] / (c5["compute_ms"] * 1e-3) / 1e9, "unit": UNIT,
                        "ms_per_step": c5["compute_ms"], "note": "outputs left row-sharded"},
            "with_allgather": {"value": c5["pairs"] / (c5["sharded_ms"] * 1e-3) / 1e9, "unit": UNIT,
                               "ms_per_step": c5["sharded_ms"], "note": "NCCL all-gather of the outputs"},
            "e2e": {"value": c5["pairs"] / (c5["e2e_ms"] * 1e-3) / 1e9, "unit": UNIT, "ms_per_step": c5["e2e_ms"]},
        }
    if world == 1 and not args.no_cpu_baseline:
        v, sample, threads, kind = cpu_baseline_config2(10.0)
        line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample}
        nat = cpu_native_window()
        if nat is not None:
            line["cpu_baseline"]["native_cpp_window512"] = {
                "value": nat[0], "unit": UNIT, "runs": nat[1],
                "what": "the reference's C++ CPU extension, propagation_window (window 512, no top-k), one batch "
                        "item, median run (no warm-up: it takes seconds per run)"}
    print(json.dumps(line), flush=True)


C5 = dict(B=4, N=32768, D=512, R=64, K=64, W=4096, SEED=4)
C5_WORKLOAD = "config5: causal window 4096 intersect top-k 64, B4 N32768 D512 R64, bf16, softsign, row-sharded"


def measure_config5(steps, warmup, rank, world, device):
    """Config 5 (B4 N32768 D512 R64, window 4096, top-k 64) partitioned by query-row blocks
    over the ranks: block compute alone (outputs left row-sharded) and with the all-gather
    that assembles them on every rank, plus the end-to-end time with host copies. Every
    time is the max over ranks. Returns a dict on every rank."""
    import jakal_net_b200 as jk
    from jakal_net_b200 import sharding

    b, n, d, r, k, w = C5["B"], C5["N"], C5["D"], C5["R"], C5["K"], C5["W"]
    pairs = b * pairs_per_batch_item(n, w)
    g = torch.Generator().manual_seed(C5["SEED"])
    to = dict(device=device, dtype=torch.bfloat16)
    h_val = torch.randn(b, n, d, generator=g).to(torch.bfloat16).pin_memory()
    h_state = torch.randn(b, n, generator=g).to(torch.bfloat16).pin_memory()
    w_s = (torch.randn(r, d, generator=g) / d ** 0.5).to(**to)
    w_t = (torch.randn(r, d, generator=g) / d ** 0.5).to(**to)
    core = torch.full((r,), r ** -0.5).to(**to)
    val = torch.empty(b, n, d, **to)
    state = torch.empty(b, n, **to)
    if rank == 0:
        val.copy_(h_val)
        state.copy_(h_state)
    if world > 1:  # inputs replicated once at setup
        sharding.replicate(val)
        sharding.replicate(state)
    blocks = sharding.row_blocks(n, world)
    begin, count = blocks[rank]
    out_state = torch.zeros(b, n, **to)
    out_val = torch.zeros(b, n, d, **to)

    def compute(v, s):
        rp = jk.lowrank_project(v, w_t)
        cp = jk.lowrank_project(v, w_s, core=core)
        sharding._kernel_block(rp, cp, s, v, k, w, begin, count, out_state, out_val)

    def gather():
        if world > 1:
            sharding.gather_row_blocks(out_state, out_val, blocks)

    def timed(fn, steps):
        ms = []
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize(device)
            ms.append(e0.elapsed_time(e1))
        return sum(ms) / len(ms)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    launches_per_step = count_launches(lambda: compute(val, state))
    for _ in range(warmup):
        compute(val, state)
        gather()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    with ClockSampler(device.index if device.index is not None else 0) as clk:
        compute_ms = max_over_ranks(timed(lambda: compute(val, state), steps))
        if world > 1:
            torch.distributed.barrier()
        sharded_ms = max_over_ranks(timed(lambda: (compute(val, state), gather()), steps))
    h_out_val = torch.empty(b, count, d, dtype=torch.bfloat16).pin_memory()

    def e2e():
        val.copy_(h_val, non_blocking=True)
        state.copy_(h_state, non_blocking=True)
        compute(val, state)
        gather()
        h_out_val.copy_(out_val[:, begin:begin + count], non_blocking=True)

    if world > 1:
        torch.distributed.barrier()
    e2e_ms = max_over_ranks(timed(e2e, max(3, min(steps, 20))))
    return dict(pairs=pairs, compute_ms=compute_ms, sharded_ms=sharded_ms, e2e_ms=e2e_ms,
                launches_per_step=launches_per_step, clocks=clk.summary(),
                h2d=(h_val.numel() + h_state.numel()) * 2, d2h=h_out_val.numel() * 2)


def run_config5(args, rank, world, device):
    m = measure_config5(args.steps, args.warmup, rank, world, device)
    b, n, d, r, k, w = C5["B"], C5["N"], C5["D"], C5["R"], C5["K"], C5["W"]
    pairs, compute_ms, sharded_ms, e2e_ms = m["pairs"], m["compute_ms"], m["sharded_ms"], m["e2e_ms"]
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": pairs / (compute_ms * 1e-3) / 1e9, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": compute_ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) inputs of the config shape, random-init weights)",
        "config": {"workload": C5_WORKLOAD, "batch": b, "nodes": n, "dim": d, "rank": r, "topk": k, "window": w,
                   "pairs_per_step": pairs, "l2": "inputs (134 MB values) larger than L2",
                   "timing": "CUDA events per step, max over ranks",
                   "parallelism": f"query-row blocks x{world}; value = block compute, outputs left row-sharded"},
        "gpu_launches": m["launches_per_step"] * args.steps,
        "clocks": m["clocks"],
        "with_allgather": {"ms_per_step": sharded_ms, "value": pairs / (sharded_ms * 1e-3) / 1e9, "unit": UNIT},
        "e2e": {"value": pairs / (e2e_ms * 1e-3) / 1e9, "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": m["h2d"], "d2h_bytes_per_step": m["d2h"]},
    }
    print(json.dumps(line), flush=True)


C3 = dict(B=16, S=4096, Q=512, D=512, R=64, K=16, SEED=2)
C3_METRIC = "per-query transition Gpairs/s"
C3_WORKLOAD = ("config3: transition S -> expanded B query-top-k routing, B16 S4096 Q512 D512 R64 k16, bf16, "
               "softmax routes, sender-weighted")


def _config3_inputs(batch, device=None, dtype=torch.bfloat16):
    """Config 3's inputs (S val ~ N(0,1), B slots ~ N(0, 0.02), projection weights ~ N(0,
    1/sqrt(D)), seed 2); `batch` items of the B16 batch. The sender strength is softplus of the
    source state, as the reference's SparseTransition forms it from Layer.state."""
    c = C3
    g = torch.Generator().manual_seed(c["SEED"])
    to = dict(dtype=dtype) if device is None else dict(device=device, dtype=dtype)
    src = torch.randn(c["B"], c["S"], c["D"], generator=g)[:batch]
    slots = (0.02 * torch.randn(c["B"], c["Q"], c["D"], generator=g))[:batch]
    state = torch.randn(c["B"], c["S"], generator=g)[:batch]
    w_s = torch.randn(c["R"], c["D"], generator=g) / c["D"] ** 0.5
    w_t = torch.randn(c["R"], c["D"], generator=g) / c["D"] ** 0.5
    core = torch.full((c["R"],), c["R"] ** -0.5)
    sender = torch.nn.functional.softplus(state)
    return [t.to(**to) for t in (src, slots, state, sender, w_s, w_t, core)]


def _config3_call(mod, src, slots, state, sender, w_s, w_t, core):
    """One per-query transition through a module's reference-facing op (this backend or the
    reference's native extension): rows = query slots, columns = sources."""
    return mod.transition_query_topk("low_rank_bilinear_route", w_s, None, w_t, None, core, None, None, None, None,
                                     None, 1.0, sender, src, slots, state, src, C3["K"], 128, 128, False)


def cpu_config3(seconds: float = 10.0):
    """The reference's C++ CPU extension (oracle/build_ref.py, from its own sources) on one
    batch item of config 3 in f32, all host threads: (Gpairs/s, sample, threads) or None."""
    from oracle import build_ref

    if not build_ref.available("cpu"):
        return None
    native = build_ref.load_built("cpu")
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    args = _config3_inputs(1, dtype=torch.float32)
    pairs = C3["Q"] * C3["S"]
    rate, reps = _median_rate(lambda: _config3_call(native, *args), pairs, seconds, min_reps=3)
    sample = (f"median of {reps} runs of 1 of the 16 batch items (S4096 Q512 D512 k16, f32) through the reference's "
              f"native CPU transition_query_topk; torch threads {torch.get_num_threads()}, {_cpu_model()}")
    return rate / 1e9, sample, threads


def run_config3(args, rank, world, device):
    """Config 3 on this backend: batch-sharded (weak scaling), every rank its own B16 batch."""
    import jakal_net_b200 as jk

    c = C3
    src, slots, state, sender, w_s, w_t, core = _config3_inputs(c["B"], device)
    pairs = c["B"] * c["Q"] * c["S"]

    def step():
        return _config3_call(jk, src, slots, state, sender, w_s, w_t, core)

    launches = count_launches(step)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    steps = max(1, args.steps)
    ms = []
    with ClockSampler(device.index if device.index is not None else 0) as clk:
        for _ in range(steps):
            flush.add_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            step()
            e1.record()
            torch.cuda.synchronize(device)
            ms.append(e0.elapsed_time(e1))
    step_ms = sum(ms) / len(ms)
    # end to end: host (pinned) sources and slots in, outputs back, every step
    h_src, h_slots = src.cpu().pin_memory(), slots.cpu().pin_memory()
    h_state = state.cpu().pin_memory()
    st0, vv0 = step()
    h_out_s = torch.empty(st0.shape, dtype=st0.dtype).pin_memory()
    h_out_v = torch.empty(vv0.shape, dtype=vv0.dtype).pin_memory()

    def e2e():
        d_src = h_src.to(device, non_blocking=True)
        d_slots = h_slots.to(device, non_blocking=True)
        d_state = h_state.to(device, non_blocking=True)
        snd = torch.nn.functional.softplus(d_state.float()).to(d_state.dtype)
        st, vv = _config3_call(jk, d_src, d_slots, d_state, snd, w_s, w_t, core)
        h_out_s.copy_(st, non_blocking=True)
        h_out_v.copy_(vv, non_blocking=True)

    e2e()
    torch.cuda.synchronize(device)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record()
    for _ in range(steps):
        e2e()
    g1.record()
    torch.cuda.synchronize(device)
    e2e_ms = g0.elapsed_time(g1) / steps
    if world > 1:
        t = torch.tensor([step_ms, e2e_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        step_ms, e2e_ms = (float(x) for x in t.tolist())
    if rank != 0:
        return
    line = {
        "metric": C3_METRIC, "value": world * pairs / (step_ms * 1e-3) / 1e9, "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded inputs of the config-3 shapes and distributions, random-init weights)",
        "config": {"workload": C3_WORKLOAD, "pairs_per_step": pairs, "l2": "256 MiB write between timed steps",
                   "timing": "CUDA events per step (public op: projections + fused kernel), max over ranks",
                   "parallelism": f"batch-sharded x{world}, no collective"},
        "gpu_launches": launches * steps, "clocks": clk.summary(),
        "e2e": {"value": world * pairs / (e2e_ms * 1e-3) / 1e9, "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": (h_src.numel() + h_slots.numel() + h_state.numel()) * 2,
                "d2h_bytes_per_step": (h_out_s.numel() + h_out_v.numel()) * h_out_v.element_size()},
    }
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_config3()
        if cb is not None:
            line["cpu_baseline"] = {"value": cb[0], "unit": UNIT, "cores": cb[2], "kind": "reference",
                                    "sample": cb[1]}
    print(json.dumps(line), flush=True)


C4 = dict(B=32, P=1024, D=512, VOCAB=16384, LAYERS=6, EXPAND=256, COMPRESS=64, WINDOW=512, TOPK=32, HIDDEN=64,
          TARGET=128, SEED=3)
C4_METRIC = "Progressive-B fwd tokens/s"
C4_WORKLOAD = ("config4: ProgressiveBExampleLM.forward_query_block, B32 prefix 1024 dim 512 vocab 16384, 6 joint "
               "blocks (expanded 256 / compressed 64), s_window 512, top-k 32, rank 64, 128 query slots, bf16 autocast")
C4_OPS = ("propagation_window", "propagation_topk", "transition_pairwise_topk", "propagation_dense",
          "transition_pairwise_dense", "propagation_query_dense", "transition_query_topk",
          "low_rank_pairwise_topk_forward_cuda")


def _progressive_b(pb, implementation, batch_hint=None):
    c = C4
    torch.manual_seed(c["SEED"])
    specs = pb.build_progressive_b_stage_specs(c["P"], lite_layers=c["LAYERS"], mid_layers=0, full_layers=0,
                                               lite_expand_ratio=c["EXPAND"] / c["P"],
                                               lite_compress_ratio=c["COMPRESS"] / c["P"])
    return pb.ProgressiveBExampleLM(
        vocab_size=c["VOCAB"], dim=c["D"], seq_nodes=c["P"], stage_specs=specs, s_window=c["WINDOW"],
        route_topk=c["TOPK"], expanded_topk=c["TOPK"], compressed_topk=c["TOPK"], query_topk=c["TOPK"],
        route_kind="low_rank_bilinear", pairwise_kind="low_rank_bilinear", route_hidden_dim=c["HIDDEN"],
        pairwise_hidden_dim=c["HIDDEN"], implementation=implementation).eval()


def _import_reference_model():
    """The reference's Progressive-B model script and package, staged by
    baseline/stage_reference.py (None when not staged)."""
    sys.path.insert(0, str(ROOT / "baseline"))
    import reference_shim

    if not reference_shim.available():
        return None, None
    os.environ["JAKAL_NET_NATIVE_MODULE"] = "jakal_net_b200"
    jn = reference_shim.import_reference()
    return jn, reference_shim.import_progressive_b()


def cpu_progressive_b(seconds: float = 15.0, batch: int = 2):
    """The reference's own CPU forward (implementation="reference", the Python/ATen path on
    all host threads) of config 4's model on a bounded batch; tokens/s, sample text, threads."""
    jn, pb = _import_reference_model()
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    model = _progressive_b(pb, "reference")
    ids = torch.randint(0, C4["VOCAB"], (batch, C4["P"]), generator=torch.Generator().manual_seed(C4["SEED"]))
    times = []
    with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16):
        model.forward_query_block(ids, target_len=C4["TARGET"])  # untimed warm-up
        t_end = time.perf_counter() + seconds
        while time.perf_counter() < t_end or len(times) < 3:
            t0 = time.perf_counter()
            model.forward_query_block(ids, target_len=C4["TARGET"])
            times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    sample = (f"median of {len(times)} forwards of batch {batch} (prefix 1024, config-4 model), "
              f"implementation=reference, bf16 CPU autocast, torch threads {torch.get_num_threads()}, {_cpu_model()}")
    return batch * C4["P"] / med, sample, threads


def _time_wrapped(obj, names, fn, device):
    """Runs fn once with obj.<name> (every name) bracketed by CUDA events; returns
    ({name: device ms}, {name: calls}, total device ms of fn)."""
    per = {}
    saved = {n: getattr(obj, n) for n in names if hasattr(obj, n)}

    def wrap(name, f):
        def timed(*a, **kw):
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            out = f(*a, **kw)
            s1.record()
            per.setdefault(name, []).append((s0, s1))
            return out
        return timed

    for n, f in saved.items():
        setattr(obj, n, wrap(n, f))
    try:
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        fn()
        f1.record()
        torch.cuda.synchronize(device)
    finally:
        for n, f in saved.items():
            setattr(obj, n, f)
    ms = {n: sum(a.elapsed_time(z) for a, z in evs) for n, evs in per.items()}
    return ms, {n: len(evs) for n, evs in per.items()}, f0.elapsed_time(f1)


def _operator_classes(jn, pb):
    """(class, method) pairs whose device time the config-4 breakdown reports: the
    reference's operator classes and Progressive-B's query propagation."""
    return [(jn.SparsePropagation, "compute_delta"), (jn.Propagation, "compute_delta"),
            (jn.SparseTransition, "compute_delta"), (jn.Transition, "compute_delta"),
            (pb.ProgressiveBExampleLM, "apply_query_propagation")]


def _time_wrapped_methods(targets, fn, device):
    """_time_wrapped over class methods (outermost calls only: a method called from inside
    another timed method is not counted twice)."""
    per, depth = {}, [0]
    saved = [(cls, name, cls.__dict__[name]) for cls, name in targets if name in cls.__dict__]

    def wrap(label, f):
        def timed(*a, **kw):
            if depth[0]:
                return f(*a, **kw)
            depth[0] += 1
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            try:
                out = f(*a, **kw)
            finally:
                depth[0] -= 1
            s1.record()
            per.setdefault(label, []).append((s0, s1))
            return out
        return timed

    for cls, name, f in saved:
        setattr(cls, name, wrap(f"{cls.__name__}.{name}", f))
    try:
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        fn()
        f1.record()
        torch.cuda.synchronize(device)
    finally:
        for cls, name, f in saved:
            setattr(cls, name, f)
    ms = {n: sum(a.elapsed_time(z) for a, z in evs) for n, evs in per.items()}
    return ms, {n: len(evs) for n, evs in per.items()}, f0.elapsed_time(f1)


def run_config4(args, rank, world, device):
    jn, pb = _import_reference_model()
    if pb is None:
        if rank == 0:
            print(json.dumps({"metric": C4_METRIC, "unavailable": "reference model not staged (baseline/_ref)"}))
        return
    import jakal_net_b200 as jk

    status = jn.native_status(force_reload=True)
    assert status.available and status.backend_name == jk.backend_name(), status
    model = _progressive_b(pb, "native").to(device)
    b, p = C4["B"], C4["P"]
    h_ids = torch.randint(0, C4["VOCAB"], (b, p), generator=torch.Generator().manual_seed(C4["SEED"] + rank))
    ids = h_ids.to(device)
    h_ids = h_ids.pin_memory()

    def forward(x):
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            return model.forward_query_block(x, target_len=C4["TARGET"])

    for _ in range(args.warmup):
        forward(ids)
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    steps = max(1, min(args.steps, 20))
    with ClockSampler(device.index if device.index is not None else 0) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            forward(ids)
        e1.record()
        torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / steps

    # per-op device time: every backend op the model calls, bracketed by CUDA events
    op_ms, calls, fwd_ms = _time_wrapped(jk, C4_OPS, lambda: forward(ids), device)
    # per-operator-class device time of the whole model step (the reference's Layer API
    # classes and the query propagation), for this backend and for the reference's torch path
    cls_targets = _operator_classes(jn, pb)
    cls_ms, cls_calls, _ = _time_wrapped_methods(cls_targets, lambda: forward(ids), device)

    # end to end: token ids from pinned host memory in, logits back to pinned host memory
    h_logits = torch.empty((b, C4["TARGET"], C4["VOCAB"]), dtype=torch.bfloat16).pin_memory()

    def e2e():
        d = h_ids.to(device, non_blocking=True)
        h_logits.copy_(forward(d), non_blocking=True)

    e2e()
    torch.cuda.synchronize(device)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, min(steps, 5))
    g0.record()
    for _ in range(e2e_steps):
        e2e()
    g1.record()
    torch.cuda.synchronize(device)
    e2e_ms = g0.elapsed_time(g1) / e2e_steps

    # the reference's own torch implementation of the same model on this GPU (informative)
    ref_ms = None
    if not args.no_reference_gpu:
        ref_model = _progressive_b(pb, "reference").to(device)
        ref_model.load_state_dict(model.state_dict())

        def ref_forward():
            with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
                return ref_model.forward_query_block(ids, target_len=C4["TARGET"])

        ref_forward()
        torch.cuda.synchronize(device)
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record()
        for _ in range(3):
            ref_forward()
        r1.record()
        torch.cuda.synchronize(device)
        ref_ms = r0.elapsed_time(r1) / 3
        ref_cls_ms, ref_cls_calls, _ = _time_wrapped_methods(cls_targets, ref_forward, device)
        del ref_model

    def max_over_ranks(x):
        if world == 1 or x is None:
            return x
        t = torch.tensor([x], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    ms, e2e_ms, ref_ms = max_over_ranks(ms), max_over_ranks(e2e_ms), max_over_ranks(ref_ms)
    if rank != 0:
        return
    tokens = world * b * p
    line = {
        "metric": C4_METRIC, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (uniform token ids, random-init weights of the config-4 architecture)",
        "config": {"workload": C4_WORKLOAD, "batch_per_gpu": b, "prefix": p, "dim": C4["D"],
                   "backend": "JAKAL_NET_NATIVE_MODULE=jakal_net_b200, implementation=native",
                   "l2": "per-step working set (weights + activations) far above L2",
                   "timing": "eager forward (the reference forces its torch path under graph capture), "
                             "CUDA events, max over ranks",
                   "parallelism": f"batch-sharded x{world}, no collective on the data path"},
        "clocks": clk.summary(),
        "per_op": {"forward_ms": fwd_ms, "ops_ms": op_ms, "calls": calls,
                   "ops_share": {n: v / fwd_ms for n, v in op_ms.items()},
                   "operator_classes_ms": cls_ms, "operator_classes_calls": cls_calls},
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h_ids.numel() * 8, "d2h_bytes_per_step": h_logits.numel() * 2},
    }
    if ref_ms is not None:
        line["reference_torch_gpu"] = {"value": tokens / (ref_ms * 1e-3), "unit": "tokens/s", "ms_per_step": ref_ms,
                                       "what": "the same model with implementation=reference on this GPU",
                                       "operator_classes_ms": ref_cls_ms}
    if world == 1 and not args.no_cpu_baseline:
        v, sample, threads = cpu_progressive_b()
        line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "reference",
                                "sample": sample}
    print(json.dumps(line), flush=True)


def _cpu_model() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown CPU"


MICRO = {
    # config 4's operator shapes (B32, dim 512, rank 64, bf16): the S window propagation,
    # the expanded-B top-k propagation and the S -> query per-source transition
    "window": dict(B=32, N=1024, D=512, R=64, W=512),
    "topk": dict(B=32, N=256, D=512, R=64, K=32),
    "transition": dict(B=32, S=1024, Q=128, D=512, R=64, K=32),
    # the same top-k propagation through the select-aggregate kernel (path comparison)
    "topk_select": dict(B=32, N=256, D=512, R=64, K=32),
    # one batch item of config 5 (window 4096 intersect top-k 64): the small case of the
    # fused kernel's long-window form for profiling
    "window_topk": dict(B=1, N=32768, D=512, R=64, K=64, W=4096),
}


def run_micro(args, device):
    """Times one reference-facing op of the module at a config-4 shape (device time per call,
    CUDA events, inputs resident): the per-operator view of the Progressive-B forward."""
    import jakal_net_b200 as jk

    c = MICRO[args.micro]
    g = torch.Generator().manual_seed(5)
    to = dict(device=device, dtype=torch.bfloat16)
    R, D = c["R"], c["D"]
    w_s = (torch.randn(R, D, generator=g) / D ** 0.5).to(**to)
    w_t = (torch.randn(R, D, generator=g) / D ** 0.5).to(**to)
    core = torch.full((R,), R ** -0.5).to(**to)
    if args.micro == "transition":
        src = torch.randn(c["B"], c["S"], D, generator=g).to(**to)
        dst = torch.randn(c["B"], c["Q"], D, generator=g).to(**to)
        st = torch.randn(c["B"], c["S"], generator=g).to(**to)
        snd = torch.nn.functional.softplus(st.float()).to(torch.bfloat16)

        def op():
            return jk.transition_pairwise_topk("low_rank_bilinear_route", w_s, None, w_t, None, core, None, None, None,
                                               None, None, 1.0, snd, src, dst, st, src, c["K"], 128, 128)
    else:
        val = torch.randn(c["B"], c["N"], D, generator=g).to(**to)
        st = torch.randn(c["B"], c["N"], generator=g).to(**to)
        if args.micro == "window":
            def op():
                return jk.propagation_window("low_rank_bilinear", core, None, w_s, None, w_t, None, "softsign", val,
                                             st, val, c["W"], 128, 128)
        elif args.micro == "window_topk":
            def op():
                return jk.propagation_window_topk("low_rank_bilinear", core, None, w_s, None, w_t, None, "softsign",
                                                  val, st, val, c["W"], c["K"], 128, 128)
        elif args.micro == "topk_select":
            def op():
                rp, cp = jk.lowrank_project_pair(val, w_t, w_s, core=core)
                return jk.select_aggregate(rp, cp, st, val, c["K"])
        else:
            def op():
                return jk.propagation_topk("low_rank_bilinear", core, None, w_s, None, w_t, None, "softsign", val,
                                           st, val, c["K"], 128, 128)
    for _ in range(args.warmup):
        op()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        op()
    e1.record()
    torch.cuda.synchronize(device)
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    print(json.dumps({"micro": args.micro, "shape": c, "us_per_call": us,
                      "launches_per_call": count_launches(op)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", type=int, choices=[2, 3, 4, 5], default=2)
    ap.add_argument("--no-reference-gpu", action="store_true")
    ap.add_argument("--no-config5", action="store_true", help="skip the config-5 row-sharded record of the default run")
    ap.add_argument("--micro", choices=sorted(MICRO), help="time one module op at a config-4 shape instead")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.micro:
        run_micro(args, device)
        return
    if world > 1:
        torch.distributed.init_process_group("nccl", device_id=device)
    try:
        {2: run_b200, 3: run_config3, 4: run_config4, 5: run_config5}[args.config](args, rank, world, device)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
