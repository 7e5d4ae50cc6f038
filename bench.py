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
# from the ncu capture summarised in profiles/topk_kernel_config2.md.
NCU_TRAFFIC_BYTES = 16975104  # 16.98 MB read + 0 B written (outputs stay in L2), one launch


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


def run_reference(args, rank):
    if rank != 0:
        return
    value, sample, threads = cpu_port_time(max(5.0, min(30.0, 0.05 * args.steps)))
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": PAIRS_PER_STEP / (value * 1e9) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) inputs of the config shape)",
        "config": {"workload": WORKLOAD, "implementation": "CPU port of the reference blocked path (oracle/cpu_port.py)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args, rank, world, device):
    import jakal_net_b200 as jk

    inp = make_inputs(device, SEED + rank)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)

    def api_step(val, state):
        return jk.propagation_window_topk("low_rank_bilinear", inp["core"], inp["bias"], inp["w_s"], None,
                                          inp["w_t"], None, "softsign", val, state, val, WINDOW, K_TOP, 128, 128)

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

    # End to end through the public API with host buffers (H2D inputs, D2H outputs).
    h_val = inp["val"].cpu().pin_memory()
    h_state = inp["state"].cpu().pin_memory()
    d_val = torch.empty_like(inp["val"])
    d_state = torch.empty_like(inp["state"])
    h_out_state = torch.empty(B, N, dtype=torch.bfloat16).pin_memory()
    h_out_val = torch.empty(B, N, D, dtype=torch.bfloat16).pin_memory()
    e2e_steps = max(3, min(args.steps, 50))

    def e2e_once():
        d_val.copy_(h_val, non_blocking=True)
        d_state.copy_(h_state, non_blocking=True)
        st, vv = api_step(d_val, d_state)
        h_out_state.copy_(st, non_blocking=True)
        h_out_val.copy_(vv, non_blocking=True)

    for _ in range(3):
        e2e_once()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        e2e_once()
    e1.record()
    torch.cuda.synchronize(device)
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms, kernel_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms, kernel_ms = (float(x) for x in t.tolist())

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
        "gpu_launches": 3 * args.steps,
        "clocks": clk.summary(),
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": (h_val.numel() + h_state.numel()) * 2,
                "d2h_bytes_per_step": (h_out_val.numel() + h_out_state.numel()) * 2, "ms_per_step": e2e_ms},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, burst)",
                     "kernel": "jk::topk::topk_kernel (fused score / top-k / aggregate)",
                     "kernel_ms": kernel_ms, "algorithmic_bytes": fused_kernel_bytes(), "traffic": traffic},
    }
    if world == 1 and not args.no_cpu_baseline:
        v, sample, threads = cpu_port_time(10.0)
        line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}
    print(json.dumps(line), flush=True)


C5 = dict(B=4, N=32768, D=512, R=64, K=64, W=4096, SEED=4)
C5_WORKLOAD = "config5: causal window 4096 intersect top-k 64, B4 N32768 D512 R64, bf16, softsign, row-sharded"


def run_config5(args, rank, world, device):
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

    for _ in range(args.warmup):
        compute(val, state)
        gather()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    with ClockSampler(device.index if device.index is not None else 0) as clk:
        compute_ms = max_over_ranks(timed(lambda: compute(val, state), args.steps))
        if world > 1:
            torch.distributed.barrier()
        sharded_ms = max_over_ranks(timed(lambda: (compute(val, state), gather()), args.steps))
    h_out_val = torch.empty(b, count, d, dtype=torch.bfloat16).pin_memory()

    def e2e():
        val.copy_(h_val, non_blocking=True)
        state.copy_(h_state, non_blocking=True)
        compute(val, state)
        gather()
        h_out_val.copy_(out_val[:, begin:begin + count], non_blocking=True)

    if world > 1:
        torch.distributed.barrier()
    e2e_ms = max_over_ranks(timed(e2e, max(3, min(args.steps, 20))))
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
        "gpu_launches": 3 * args.steps,
        "clocks": clk.summary(),
        "with_allgather": {"ms_per_step": sharded_ms, "value": pairs / (sharded_ms * 1e-3) / 1e9, "unit": UNIT},
        "e2e": {"value": pairs / (e2e_ms * 1e-3) / 1e9, "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": (h_val.numel() + h_state.numel()) * 2,
                "d2h_bytes_per_step": h_out_val.numel() * 2},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", type=int, choices=[2, 5], default=2)
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
    if world > 1:
        torch.distributed.init_process_group("nccl", device_id=device)
    try:
        (run_config5 if args.config == 5 else run_b200)(args, rank, world, device)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
