"""Per-CTA phase timeline of the fused top-k kernel (developer tool).

    python jakal-net_b200/phase_trace.py --build     # compile the traced library (no GPU needed)
    python jakal-net_b200/phase_trace.py             # run on cuda:0, print the timeline

The traced library is the normal one compiled with -DJK_PHASE_PROFILE into
jakal-net_b200/_build/: one thread of every CTA stores clock64() at each phase boundary
(plain stores, no atomics, so the timeline is not perturbed) and jk_debug_trace copies the
stamps out. Workload: the benchmark's configuration 2 (B8 N2048 D384 R64, window 512,
top-k 32, bf16), L2 flushed before the traced launch. Cycles are SM clocks (1.965 GHz at
boost) from the CTA's start; only differences within one CTA are meaningful.
"""
from __future__ import annotations

import argparse
import ctypes
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
TRACE_LIB = HERE / "_build" / "libjakal_b200_trace.so"

# slot -> phase end (stamped by thread 0 of the CTA unless noted)
PHASES = [(10, "first score MMA (MMA warp)"), (1, "pass A"), (2, "pass B"), (3, "pass C"), (4, "select"),
          (16, "compress: bias"), (17, "compress: edges"), (18, "compress: state"), (5, "compress done"),
          (14, "loader: score tiles issued"), (11, "aggregate MMAs start (MMA warp)"), (7, "edge tiles built"),
          (12, "aggregate MMAs issued (MMA warp)"), (13, "aggregate MMAs done (MMA warp)"), (6, "epilogue"),
          (9, "end")]


def build() -> None:
    sys.path.insert(0, str(HERE))
    import build as b  # noqa: E402

    TRACE_LIB.parent.mkdir(exist_ok=True)
    cmd = [b.nvcc_path(), *b.NVCC_FLAGS, "-DJK_PHASE_PROFILE", "-I", str(b.INCLUDE), str(b.CSRC / "jk_lib.cu"),
           "-o", str(TRACE_LIB), "-lcudart"]
    subprocess.run(cmd, check=True)
    print(TRACE_LIB)


def run() -> None:
    os.environ["JAKAL_B200_LIB"] = str(TRACE_LIB)
    sys.path.insert(0, str(HERE))
    import numpy as np
    import torch
    import jakal_net_b200 as jk

    lib = jk._LIBRARY
    lib.jk_debug_trace.argtypes = [ctypes.c_void_p, ctypes.c_int]
    B, N, D, R, K, W = 8, 2048, 384, 64, 32, 512
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(1)
    val = torch.randn(B, N, D, generator=g).to(dev, torch.bfloat16)
    state = torch.randn(B, N, generator=g).to(dev, torch.bfloat16)
    ws = (torch.randn(R, D, generator=g) / D ** 0.5).to(dev, torch.bfloat16)
    wt = (torch.randn(R, D, generator=g) / D ** 0.5).to(dev, torch.bfloat16)
    core = torch.full((R,), R ** -0.5).to(dev, torch.bfloat16)
    rp, cp = jk.lowrank_project_pair(val, wt, ws, core=core)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    for _ in range(3):
        jk.topk_aggregate(rp, cp, state, val, K, window=W)
    flush.add_(1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    jk.topk_aggregate(rp, cp, state, val, K, window=W)
    e1.record()
    torch.cuda.synchronize()
    n = B * N // 128
    buf = (ctypes.c_longlong * (32 * n))()
    lib.jk_debug_trace(buf, n)
    t = np.array(buf, dtype=np.int64).reshape(n, 32)
    rel = t - t[:, :1]
    print(f"traced launch {e0.elapsed_time(e1) * 1e3:.1f} us, {n} CTAs on {len(set(t[:, 15]))} SMs")
    print(f"{'phase end':36s} {'median':>9s} {'max':>9s}  (cycles from CTA start)")
    for slot, name in PHASES:
        print(f"{name:36s} {np.median(rel[:, slot]):9.0f} {np.max(rel[:, slot]):9.0f}")
    print(f"select, warp 0 over its 16 rows: rank loop {np.median(t[:, 19]):.0f}, tail {np.median(t[:, 20]):.0f}, "
          f"candidates {np.median(t[:, 21]):.0f}")
    for h, o in ((0, 24), (1, 27)):
        print(f"edge builder, half {h} (thread 0 of its first warp): waits {np.median(t[:, o]):.0f}, entries "
              f"{np.median(t[:, o + 1]):.0f}, TMEM store {np.median(t[:, o + 2]):.0f}")
    print(f"MMA warp waits: edge tiles {np.median(t[:, 22]):.0f}, value slices {np.median(t[:, 23]):.0f}")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--build", action="store_true")
    a = ap.parse_args()
    build() if a.build else run()
