#!/usr/bin/env python
"""Benchmark: W4A8 GEMV weight-stream throughput on B200 (libkernelsmith).

Workload (the W4A8 GEMV configuration of the headline metric):
  W int4 [11008, 4096] packed low nibble first, group 32 along K with f16
  scales, x int8 [4096] with per-token f32 scale 0.02, f32 output.
  One step = 64 such GEMVs over 64 distinct resident weight matrices (the
  gate and up projections of a 32-layer 7B-class model for one decode
  token), each with its own activation vector: 1.63 GB of weights and
  scales, far larger than the 126 MB L2, so no flush is needed.

  N > 1 GPUs (weak scaling): each rank holds an 11008-row shard of each of
  the 64 matrices ([N*11008, 4096] globally), runs the same per-GPU work as
  N = 1, and the output slices are gathered to every rank over NVLink: by
  default the GEMV kernel itself stores each output into every rank's
  gathered buffer (CUDA IPC peer pointers) and one arrival wait per step
  closes it; `--gather nccl` uses NCCL all-gathers on a second stream
  instead.

Numbers:
  value      algorithmic bytes of all GEMVs of all ranks / device time (TB/s),
             weights already resident in HBM, CUDA events on the launching
             stream, max over ranks.
  e2e        same metric through the public synchronous C ABI
             (ks_b200_matvec_w4a8_f16) with pinned HOST buffers: every GEMV
             copies its weights, scales and x host->device and its output
             back inside the timed region.
  roofline   achieved GB/s of the GEMV kernel (bytes per launch / average
             launch time over the timed region) against the measured HBM peak.
  cpu_baseline  the reference's own C implementation (ks_matvec_w4a8 built
             from the reference sources, f32 scales) on this host's cores,
             rows split across threads.

--impl reference runs only the reference CPU path on rank 0 and prints its
line; other ranks exit without work.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import datetime
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
for _p in (ROOT / "ulir-kernels_b200", ROOT / "oracle"):
    sys.path.insert(0, str(_p))

METRIC = "INT8/W4A8 GEMV weight-stream TB/s & % HBM peak at 1/2/4/8 B200"
ROWS, COLS, GROUP = 11008, 4096, 32
SX = 0.02
MATS = 64
SEED = 20261201
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
# dram__bytes_read.sum + dram__bytes_write.sum of the batched W4A8 kernel on
# this workload, per GEMV (one ncu launch = 64 GEMVs: 1,623,528,704 +
# 6,081,792 bytes), from the capture summarised under profiles/.
NCU_TRAFFIC_PER_GEMV = (1_623_528_704 + 6_081_792) // 64


def gemv_bytes(rows=ROWS, cols=COLS, group=GROUP, scale_bytes=2) -> int:
    """Algorithmic bytes of one GEMV: packed weights + scales + x + y."""
    return rows * (cols // 2) + rows * (cols // group) * scale_bytes + cols + rows * 4


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--e2e-steps", type=int, default=None, help="steps of the host-buffer e2e loop")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the INT8 GEMV and skinny GEMM secondary measurements")
    ap.add_argument("--only", choices=["gemm", "gemm_w4a8", "int8", "decode", "import"], default=None,
                    help="run only this secondary measurement on one GPU and print it (small device "
                         "footprint, for profiling); the headline line is not produced")
    ap.add_argument("--decode-layers", type=int, default=32,
                    help="secondary measurement: a chain of this many fused W4A8 decode layers (0: skip)")
    ap.add_argument("--gemvs-per-launch", type=int, default=0,
                    help="GEMVs per batched launch (default 64; 16 with --gather nccl)")
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                    help="N > 1: output gather by peer stores from the GEMV kernel (default) or NCCL")
    return ap.parse_args()


_JSON_OUT = sys.stdout  # replaced in main() by a private copy of the original stdout


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def measured_hbm_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


# ------------------------------------------------------------ CPU baseline --
def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def make_host_inputs(seed=SEED):
    import oracle as O

    x = O.rng(seed, 0).integers(-127, 128, COLS, dtype=np.int8)
    w = O.rng(seed, 1).integers(0, 256, (ROWS, COLS // 2), dtype=np.uint8)
    s16 = O.rng(seed, 2).uniform(1e-3, 1e-2, (ROWS, COLS // GROUP)).astype(np.float16)
    return x, w, s16


def cpu_reference_runner():
    """(run_one_gemv, kind, threads): the reference C on row slices across threads."""
    import oracle as O

    x, w, s16 = make_host_inputs()
    s32 = s16.astype(np.float32)
    y = np.zeros(ROWS, np.float32)
    if O.ref_available("generic"):
        impl, kind = O.RefLib("generic"), "reference"
        fn = impl.lib.ks_matvec_w4a8
        call = lambda r0, n: fn(x.ctypes.data, w.ctypes.data + r0 * w.strides[0], w.strides[0],  # noqa: E731
                                s32.ctypes.data + r0 * s32.strides[0], s32.shape[1], y.ctypes.data + 4 * r0,
                                n, COLS, GROUP, SX, 0, 0, None, 0)
    else:
        impl, kind = O.Oracle(), "port"
        fn = impl.lib.kso_matvec_w4a8
        call = lambda r0, n: fn(x.ctypes.data, w.ctypes.data + r0 * w.strides[0], w.strides[0],  # noqa: E731
                                s32.ctypes.data + r0 * s32.strides[0], s32.shape[1], y.ctypes.data + 4 * r0,
                                n, COLS, GROUP, SX, 0, 0)
    T = host_threads()
    bounds = [(ROWS * i // T, ROWS * (i + 1) // T) for i in range(T)]
    bounds = [(a, b - a) for a, b in bounds if b > a]
    pool = cf.ThreadPoolExecutor(max_workers=len(bounds))

    def one():
        rcs = list(pool.map(lambda ab: call(*ab), bounds))
        assert all(rc == 0 for rc in rcs), rcs

    return one, kind, len(bounds), pool


def time_cpu_reference(n_gemvs: int, warmup: int = 1):
    one, kind, threads, pool = cpu_reference_runner()
    for _ in range(warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(n_gemvs):
        one()
    dt = time.perf_counter() - t0
    pool.shutdown()
    return dt, kind, threads


def run_reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    one, kind, threads, pool = cpu_reference_runner()
    for _ in range(args.warmup):
        one()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    pool.shutdown()
    total = sum(times)
    value = gemv_bytes() * args.steps / total / 1e12
    sample = (f"1 GEMV {ROWS}x{COLS} G{GROUP} per step (f32 scales widened from the f16 set), rows split over "
              f"{threads} threads, reference ks_matvec_w4a8 ({'oracle/_ref generic -O3' if kind == 'reference' else 'oracle port'})")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "w4a8-f32acc",
        "data": "synthetic (seeded)", "config": workload_config(world),
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), file=_JSON_OUT, flush=True)
    return 0


def workload_config(world, gather="peer"):
    return {
        "workload": f"w4a8_gemv rows={ROWS} cols={COLS} group={GROUP} f16 scales; {MATS} resident matrices per step",
        "rows_per_gpu": ROWS, "cols": COLS, "group": GROUP, "scale_dtype": "f16", "gemvs_per_step": MATS,
        "global_rows": ROWS * world,
        "parallelism": ("row-shard + gather by peer stores (NVLink, CUDA IPC)" if gather == "peer" else
                        "row-shard + NCCL all-gather") if world > 1 else "single GPU",
        "l2": f"inputs {MATS * gemv_bytes() / 1e9:.2f} GB per GPU > 126 MB L2; no flush",
        "bytes_per_gemv": gemv_bytes(),
    }


# ------------------------------------------------------------ clocks (NVML) --
REASON_BITS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
    0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler:
    """Polls SM clock and clock-event reasons of this rank's GPU via NVML."""

    def __init__(self, torch_device):
        self.samples = []
        self.ok = False
        self._stop = threading.Event()
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(torch_device).uuid)
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.ok = True
        except Exception as e:  # pragma: no cover - NVML missing
            self.err = repr(e)

    def _run(self):
        while not self._stop.is_set():
            try:
                sm = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = int(self._reasons(self.h))
                self.samples.append((sm, rs))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": getattr(self, "max_mhz", None), "reasons": [],
                    "samples": 0, "note": getattr(self, "err", "no samples")}
        mhz = [s for s, _ in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= r
        reasons = [name for bit, name in REASON_BITS.items() if bits & bit and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples), "source": "NVML (same counters as nvidia-smi)"}


# ---------------------------------------------------------------- B200 arm --
def run_b200_arm(args):
    import torch
    import torch.distributed as dist

    import kernelsmith_b200 as K

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.only:
        if world > 1:
            raise SystemExit("--only runs on one GPU")
        fn = {"gemm": lambda: run_gemm(K, torch, dev), "int8": lambda: run_int8_gemv(K, torch, dev),
              "decode": lambda: run_decode_layers(K, torch, dev, args),
              "import": lambda: run_import(K, torch, dev),
              "gemm_w4a8": lambda: run_gemm_w4a8(K, torch, dev)}[args.only]
        print(json.dumps({"only": args.only, "result": fn()}), file=_JSON_OUT, flush=True)
        return 0
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    L = K.lib()
    # launches per step: one batched launch of all 64 GEMVs, except with the
    # NCCL gather, whose all-gathers overlap the next launch of 16
    per_launch = args.gemvs_per_launch or (16 if world > 1 and args.gather == "nccl" else MATS)
    if MATS % per_launch:
        raise SystemExit(f"--gemvs-per-launch must divide {MATS}")
    CHUNKS = MATS // per_launch

    # ---- resident inputs: 64 shards of [ROWS, COLS] (this rank's rows) ----
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED + 7919 * rank)
    W = torch.randint(0, 256, (MATS, ROWS, COLS // 2), dtype=torch.uint8, device=dev, generator=gen)
    S = (torch.rand((MATS, ROWS, COLS // GROUP), device=dev, generator=gen) * 9e-3 + 1e-3).to(torch.float16)
    X = torch.randint(-127, 128, (MATS, COLS), dtype=torch.int8, device=dev, generator=gen)
    Yfull = torch.zeros((CHUNKS, world, MATS // CHUNKS, ROWS), dtype=torch.float32, device=dev)
    Yloc = torch.zeros((CHUNKS, MATS // CHUNKS, ROWS), dtype=torch.float32, device=dev)
    status = torch.zeros(K.STATUS_WORDS, dtype=torch.int32, device=dev)
    assert L.ks_b200_w4a8_kernel_path(X.data_ptr(), W.data_ptr(), COLS // 2, S.data_ptr(), K.SCALE_F16,
                                      COLS // GROUP, ROWS, COLS, GROUP) == 1

    main = torch.cuda.Stream(device=dev)
    comm = torch.cuda.Stream(device=dev)
    main.wait_stream(torch.cuda.current_stream(dev))  # inputs and zero-filled outputs first
    comm.wait_stream(torch.cuda.current_stream(dev))
    per_chunk = MATS // CHUNKS
    peer = world > 1 and args.gather == "peer"
    pgw = None
    if peer:
        from kernelsmith_b200.sharded import PeerGatherW4A8

        pgw = PeerGatherW4A8(MATS, ROWS, dev)
    signals = [0] * CHUNKS

    def gemv_chunk(c):
        # one batched launch: per_chunk independent GEMVs streamed back to back
        ms = range(c * per_chunk, (c + 1) * per_chunk)
        if peer:
            signals[c] = pgw.run([X[m] for m in ms], [W[m] for m in ms], [S[m] for m in ms], COLS, GROUP, SX,
                                 K.SCALE_F16, stream=main, wait=False, m0=c * per_chunk)
        else:
            K.matvec_w4a8_batch_async([X[m] for m in ms], [W[m] for m in ms], [S[m] for m in ms],
                                      [Yloc[c, j] for j in range(per_chunk)], COLS // 2, COLS // GROUP, ROWS,
                                      COLS, GROUP, SX, scale_type=K.SCALE_F16, status=status, stream=main)

    def gemv_single_chain():
        # the same 64 GEMVs as 64 single launches (programmatic dependent launch chain)
        for m in range(MATS):
            K.matvec_w4a8_async(X[m], W[m], COLS // 2, S[m], COLS // GROUP, Yloc[m // per_chunk, m % per_chunk],
                                ROWS, COLS, GROUP, SX, scale_type=K.SCALE_F16, status=status, stream=main)

    # one CUDA graph per batched launch
    graphs = []
    with torch.cuda.stream(main):
        for c in range(CHUNKS):
            gemv_chunk(c)  # warm-up / attribute setup outside capture
        if peer:
            pgw.wait(sum(signals), stream=main)
    main.synchronize()
    for c in range(CHUNKS):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=main):
            gemv_chunk(c)
        graphs.append(g)
    wait_graph = None
    if peer:
        wait_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(wait_graph, stream=main):
            pgw.wait(sum(signals), stream=main)

    def step():
        for c in range(CHUNKS):
            graphs[c].replay()
            if world > 1 and not peer:
                ev = torch.cuda.Event()
                ev.record(main)
                comm.wait_event(ev)
                with torch.cuda.stream(comm):
                    dist.all_gather_into_tensor(Yfull[c], Yloc[c])
        if peer:
            wait_graph.replay()
        elif world > 1:
            main.wait_stream(comm)

    with torch.cuda.stream(main):
        for _ in range(max(3, args.warmup)):
            step()
    torch.cuda.synchronize()
    # NVML set-up and the sampling thread start before the ranks line up, so
    # no rank enters the timed region late
    clocks = ClockSampler(dev)
    clocks.__enter__()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    try:
        with torch.cuda.stream(main):
            start.record(main)
            for _ in range(args.steps):
                step()
            end.record(main)
            end.synchronize()
    finally:
        clocks.__exit__(None, None, None)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    rank_ms = [ms]
    if world > 1:
        t = torch.zeros(world, device=dev)
        t[rank] = ms
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        rank_ms = t.cpu().tolist()
        ms = max(rank_ms)
        dist.barrier()
    st = status.cpu().tolist()
    assert st == [0, 0], f"device status {st}"
    if peer:
        pst = pgw.status.cpu().tolist()
        assert pst == [0, 0], f"peer-gather status {pst}"

    # secondary: the single-GEMV launch chain (what a dependent decode chain of
    # ks_* calls costs per GEMV), timed the same way on this rank
    chain = torch.cuda.CUDAGraph()
    with torch.cuda.stream(main):
        gemv_single_chain()
    main.synchronize()
    with torch.cuda.graph(chain, stream=main):
        gemv_single_chain()
    with torch.cuda.stream(main):
        for _ in range(3):
            chain.replay()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(main)
        n_chain = max(3, min(args.steps, 50))
        for _ in range(n_chain):
            chain.replay()
        c1.record(main)
        c1.synchronize()
    chain_us = c0.elapsed_time(c1) * 1e3 / (n_chain * MATS)
    del chain

    total_bytes = gemv_bytes() * MATS * args.steps * world
    value = total_bytes / (ms * 1e-3) / 1e12
    per_launch_s = ms * 1e-3 / (MATS * args.steps)  # per GEMV
    peak, peak_kind = measured_hbm_peak()
    achieved = gemv_bytes() / per_launch_s / 1e9

    # ---- e2e: public synchronous C ABI with pinned host buffers ----------
    e2e_steps = args.e2e_steps if args.e2e_steps is not None else max(1, min(args.steps, 5))
    e2e = run_e2e(L, K, torch, dist, dev, world, rank, e2e_steps) if e2e_steps > 0 else None

    layer = run_decode_layers(K, torch, dev, args) if args.decode_layers > 0 else None
    # the other configurations, single GPU only (per-GPU numbers)
    i8 = run_int8_gemv(K, torch, dev) if world == 1 and not args.no_secondary else None
    gemm = run_gemm(K, torch, dev) if world == 1 and not args.no_secondary else None
    imp = run_import(K, torch, dev) if world == 1 and not args.no_secondary else None
    gw4 = run_gemm_w4a8(K, torch, dev) if world == 1 and not args.no_secondary else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n = MATS
        dt, kind, threads = time_cpu_reference(n)
        cpu = {"value": gemv_bytes() * n / dt / 1e12, "unit": "TB/s", "cores": threads, "kind": kind,
               "sample": f"{n} GEMVs {ROWS}x{COLS} G{GROUP} (one step), f32 scales, rows split over {threads} "
                         f"threads, {dt:.2f} s wall"}

    for g in graphs:
        del g
    graphs.clear()
    wait_graph = None
    if peer:
        dist.barrier()
        torch.cuda.synchronize()
        pgw.close()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms / args.steps,
            "ms_per_step_by_rank": [round(v / args.steps, 5) for v in rank_ms], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "w4a8-i32acc-f32out",
            "data": "synthetic (seeded uniform int4 / int8, f16 scales U[1e-3,1e-2])",
            "config": workload_config(world, args.gather),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": NCU_TRAFFIC_PER_GEMV, "traffic_per": "GEMV (ncu capture)",
                         "kernel": f"gemv_stream_kernel<W4A8Op<__half,4,false>,16> (batched, {MATS // CHUNKS} GEMVs per launch)",
                         "bytes_per_gemv": gemv_bytes(), "us_per_gemv": per_launch_s * 1e6,
                         "gemvs_per_launch": MATS // CHUNKS},
            "single_launch_chain": {"us_per_gemv": chain_us, "GB_s": gemv_bytes() / chain_us / 1e3,
                                    "frac": gemv_bytes() / chain_us / 1e3 / peak,
                                    "note": "64 single-GEMV launches, PDL chain, per GPU"},
            "decode_layer": layer,
            "int8_gemv": i8,
            "gemm_i8": gemm,
            "q4_0_import": imp,
            "gemm_w4a8": gw4,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": CHUNKS * args.steps * world,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), file=_JSON_OUT, flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


LAYER_H, LAYER_I = 4096, 11008


def layer_bytes(h=LAYER_H, i=LAYER_I, group=GROUP):
    """Weights + f16 scales of one decode layer (QKV, O, gate, up, down)."""
    mats = [(3 * h, h), (h, h), (i, h), (i, h), (h, i)]
    return sum(r * c // 2 + r * (c // group) * 2 for r, c in mats)


def run_decode_layers(K, torch, dev, args):
    """A chain of fused W4A8 decode layers (hidden 4096, inter 11008, G 32,
    distinct random weights per layer), graph-captured; per-layer time."""
    import ctypes

    L = K.lib()
    n = args.decode_layers
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED + 17)
    h, i = LAYER_H, LAYER_I
    shapes = [(3 * h, h), (h, h), (i, h), (i, h), (h, i)]
    Ws = [[torch.randint(0, 256, (r, c // 2), dtype=torch.uint8, device=dev, generator=gen) for r, c in shapes]
          for _ in range(n)]
    Ss = [[(torch.rand((r, c // GROUP), device=dev, generator=gen) * 9e-3 + 1e-3).to(torch.float16)
           for r, c in shapes] for _ in range(n)]
    norms = torch.rand((2, h), device=dev, generator=gen) + 0.5
    acts = torch.zeros((n + 1, h), dtype=torch.float32, device=dev)
    acts[0].uniform_(-1, 1, generator=gen)
    ws_bytes = L.ks_b200_decode_layer_workspace(h, i)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    status = torch.zeros(K.STATUS_WORDS, dtype=torch.int32, device=dev)
    wp = [(ctypes.c_void_p * 5)(*[t.data_ptr() for t in W]) for W in Ws]
    sp = [(ctypes.c_void_p * 5)(*[t.data_ptr() for t in S]) for S in Ss]
    stream = torch.cuda.Stream(device=dev)
    # the zero-filled workspace and the inputs are written on the current
    # stream; the layers run on `stream`
    stream.wait_stream(torch.cuda.current_stream(dev))

    def chain():
        for l in range(n):
            K.check(L.ks_b200_decode_layer_w4a8_async(acts[l].data_ptr(), acts[l + 1].data_ptr(),
                                                      norms[0].data_ptr(), norms[1].data_ptr(), 1e-5, wp[l], sp[l],
                                                      h, i, GROUP, ws.data_ptr(), ws_bytes, status.data_ptr(),
                                                      K.stream_handle(stream)))

    with torch.cuda.stream(stream):
        chain()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        chain()
    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * n)
    del g
    assert status.cpu().tolist() == [0, 0]
    peak, _ = measured_hbm_peak()
    b = layer_bytes()
    return {"layers": n, "us_per_layer": us, "weight_bytes_per_layer": b, "GB_s": b / us / 1e3,
            "frac": b / us / 1e3 / peak, "launches_per_layer": L.ks_b200_decode_layer_launches(h, i, GROUP),
            "shape": "hidden 4096, inter 11008, W4A8 G32 f16 scales, batch 1, fused RMSNorm/quantise/SiLU/residual"}


def _graph_us(torch, stream, fn, units, reps=10):
    """Device time per unit of `fn` (graph-captured, CUDA events on `stream`)."""
    with torch.cuda.stream(stream):
        fn()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * units)
    del g
    return us


I8_N, I8_K, I8_SA = 4096, 4096, 0.02


def run_int8_gemv(K, torch, dev):
    """INT8 GEMV with per-channel dequant, y = (f32(acc) * ws) * sa, 4096 x 4096
    (the reference's CPU-runnable configuration): 64 distinct resident matrices
    (1.08 GB > L2), as 4 batched launches of 16 and as 64 single launches."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED + 31)
    n = 64
    W = [torch.randint(-127, 128, (I8_N, I8_K), dtype=torch.int8, device=dev, generator=gen) for _ in range(n)]
    WS = [torch.rand(I8_N, device=dev, generator=gen) * 9e-3 + 1e-3 for _ in range(n)]
    x = torch.randint(-127, 128, (I8_K,), dtype=torch.int8, device=dev, generator=gen)
    Y = torch.zeros((n, I8_N), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))

    def batched():
        for c in range(0, n, 16):
            K.matvec_i8_batch_async([x] * 16, W[c:c + 16], [Y[j] for j in range(c, c + 16)], I8_K, I8_N, I8_K,
                                    w_scales=WS[c:c + 16], sa=I8_SA, stream=stream)

    def single():
        for j in range(n):
            K.matvec_i8_dequant_async(x, W[j], I8_K, WS[j], I8_SA, Y[j], I8_N, I8_K, stream=stream)

    b = I8_N * I8_K + I8_K + 8 * I8_N  # weights, x, dequant scales, f32 outputs
    peak, _ = measured_hbm_peak()
    out = {"shape": f"{I8_N}x{I8_K} int8, per-channel f32 dequant", "bytes_per_gemv": b}
    for name, fn in (("batched_16", batched), ("single_launch_chain", single)):
        us = _graph_us(torch, stream, fn, n)
        out[name] = {"us_per_gemv": us, "GB_s": b / us / 1e3, "frac": b / us / 1e3 / peak}
    return out


def run_gemm(K, torch, dev):
    """Skinny INT8 GEMM with requantisation, M x 4096 x 14336 (M = 8, 16, 32, 64),
    output scale 0.05: a graph of 32 launches over 8 distinct weight copies
    (470 MB > L2) per M."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED + 47)
    N, Kd, copies = 14336, 4096, 8
    W = [torch.randint(-127, 128, (N, Kd), dtype=torch.int8, device=dev, generator=gen) for _ in range(copies)]
    ws = torch.rand(N, device=dev, generator=gen) * 9e-3 + 1e-3
    stream = torch.cuda.Stream(device=dev)
    peak, _ = measured_hbm_peak()
    out = {"shape": "M x 4096 x 14336 int8 -> int8, per-token / per-channel f32 scales, out scale 0.05",
           "kernel": "gemm_i8_tc_kernel (tcgen05.mma kind::i8, TMEM accumulators)"}
    for M in (8, 16, 32, 64):
        A = torch.randint(-127, 128, (M, Kd), dtype=torch.int8, device=dev, generator=gen)
        sa = torch.rand(M, device=dev, generator=gen) * 9e-3 + 1e-3
        o = torch.zeros((M, N), dtype=torch.int8, device=dev)
        status = torch.zeros(K.STATUS_WORDS, dtype=torch.int32, device=dev)
        stream.wait_stream(torch.cuda.current_stream(dev))

        def fn():
            for i in range(32):
                K.gemm_i8_requant_async(A, sa, W[i % copies], ws, 0.05, o, M, N, Kd, status=status, stream=stream)

        outs = [torch.zeros((M, N), dtype=torch.int8, device=dev) for _ in range(16)]

        def fn_batched():
            # the same 32 GEMMs as two batched launches of 16
            for c in range(2):
                ids = range(16 * c, 16 * c + 16)
                K.gemm_i8_requant_batch_async([A] * 16, [sa] * 16, [W[i % copies] for i in ids], [ws] * 16, 0.05,
                                              outs, M, N, Kd, status=status, stream=stream)

        us = _graph_us(torch, stream, fn, 32, reps=5)
        us_b = _graph_us(torch, stream, fn_batched, 32, reps=5)
        assert status.cpu().tolist() == [0, 0]
        b = N * Kd + M * Kd + M * N + 4 * (M + N)
        out[f"M{M}"] = {"us": us, "TB_s": b / us / 1e6, "frac": b / us / 1e3 / peak,
                        "batched_16": {"us": us_b, "TB_s": b / us_b / 1e6, "frac": b / us_b / 1e3 / peak}}
    out["note"] = ("M<n>: one launch per GEMM (graph of 32, programmatic dependent launch); batched_16: the same "
                   "32 GEMMs as two launches of ks_b200_gemm_i8_requant_batch_async")
    return out


def run_gemm_w4a8(K, torch, dev):
    """Batched W4A8 GEMM on the tensor cores, M x 4096 x 14336 (M = 8, 16, 32,
    64), G 32, f16 scales: a graph of 32 launches over 8 distinct weight copies
    (264 MB > L2) per M; bytes = packed weights + scales + activations + f32 out."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED + 71)
    N, Kd, G, copies = 14336, 4096, 32, 8
    W = [torch.randint(0, 256, (N, Kd // 2), dtype=torch.uint8, device=dev, generator=gen) for _ in range(copies)]
    S = [(torch.rand((N, Kd // G), device=dev, generator=gen) * 9e-3 + 1e-3).to(torch.float16) for _ in range(copies)]
    stream = torch.cuda.Stream(device=dev)
    peak, _ = measured_hbm_peak()
    out = {"shape": "M x 4096 x 14336 int8 x W4A8 (G 32, f16 scales) -> f32",
           "kernel": "gemm_w4a8_tc_kernel (int4 unpacked to int8 in shared memory, tcgen05.mma kind::i8)"}
    for M in (8, 16, 32, 64):
        A = torch.randint(-127, 128, (M, Kd), dtype=torch.int8, device=dev, generator=gen)
        sx = torch.rand(M, device=dev, generator=gen) * 0.02 + 0.01
        y = torch.zeros((M, N), dtype=torch.float32, device=dev)
        status = torch.zeros(K.STATUS_WORDS, dtype=torch.int32, device=dev)
        stream.wait_stream(torch.cuda.current_stream(dev))

        def fn():
            for i in range(32):
                K.gemm_w4a8_async(A, sx, W[i % copies], S[i % copies], y, M, N, Kd, G, status=status, stream=stream)

        us = _graph_us(torch, stream, fn, 32, reps=5)
        assert status.cpu().tolist() == [0, 0]
        b = N * Kd // 2 + N * (Kd // G) * 2 + M * Kd + 4 * M + 4 * M * N
        out[f"M{M}"] = {"us": us, "TB_s": b / us / 1e6, "frac": b / us / 1e3 / peak}
    return out


def run_import(K, torch, dev):
    """GGML Q4_0 -> native W4A8 G32 f16 for an 11008 x 4096 matrix (the bench
    matrix shape), 8 distinct inputs per graph (200 MB read > L2): bytes moved
    per matrix = Q4_0 blocks read + packed int4 and f16 scales written."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED + 59)
    rows, cols, group, n = ROWS, COLS, GROUP, 8
    src = [torch.randint(0, 256, (rows, cols // 32 * 18), dtype=torch.uint8, device=dev, generator=gen)
           for _ in range(n)]
    for t in src:  # finite f16 d in every block
        t.view(rows, cols // 32, 18)[:, :, 1] = 0x20
    packed = torch.zeros((n, rows, cols // 2), dtype=torch.uint8, device=dev)
    scales = torch.zeros((n, rows, cols // group), dtype=torch.float16, device=dev)
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))

    def fn():
        for i in range(n):
            K.import_ggml_q4_0_async(src[i], cols // 32 * 18, rows, cols, group, packed[i], cols // 2, scales[i],
                                     scale_type=K.SCALE_F16, stream=stream)

    us = _graph_us(torch, stream, fn, n)
    b = rows * (cols // 32) * 18 + rows * cols // 2 + rows * (cols // group) * 2
    peak, _ = measured_hbm_peak()
    return {"shape": f"{rows}x{cols} Q4_0 -> W4A8 G{group} f16", "bytes_per_matrix": b, "us_per_matrix": us,
            "GB_s": b / us / 1e3, "frac": b / us / 1e3 / peak,
            "kernel": "import_q4_0_kernel (one thread per group, 16-byte packed stores)"}


def run_e2e(L, K, torch, dist, dev, world, rank, steps):
    """Host buffers through ks_b200_matvec_w4a8_f16: H2D + kernel + D2H per GEMV."""
    nbuf = 4
    x, w, s16 = make_host_inputs(SEED + rank)
    hw = [torch.from_numpy(w).pin_memory() for _ in range(nbuf)]
    hs = [torch.from_numpy(s16.view(np.uint16)).pin_memory() for _ in range(nbuf)]
    hx = torch.from_numpy(x).pin_memory()
    hy = torch.zeros((MATS, ROWS), dtype=torch.float32).pin_memory()
    gathered = torch.zeros((world, ROWS), dtype=torch.float32, device=dev) if world > 1 else None

    def one_step():
        for m in range(MATS):
            rc = L.ks_b200_matvec_w4a8_f16(hx.data_ptr(), hw[m % nbuf].data_ptr(), COLS // 2,
                                           hs[m % nbuf].data_ptr(), COLS // GROUP, hy[m].data_ptr(), ROWS, COLS,
                                           GROUP, SX, 0, 0)
            K.check(rc)
        if world > 1:  # the step's output slices, exchanged (device round trip)
            dist.all_gather_into_tensor(gathered, hy[MATS - 1].to(dev, non_blocking=False))
            torch.cuda.synchronize()

    one_step()  # warm-up (staging buffers)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        one_step()
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([dt], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    h2d = MATS * (w.nbytes + s16.nbytes + x.nbytes)
    d2h = MATS * ROWS * 4
    return {"value": gemv_bytes() * MATS * steps * world / dt / 1e12, "unit": "TB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps,
            "api": "ks_b200_matvec_w4a8_f16 (synchronous C ABI), pinned host buffers"}


def main():
    global _JSON_OUT
    args = parse_args()
    # The one JSON line is the only thing on stdout: anything libraries write to
    # file descriptor 1 (NCCL's version banner, for one) goes to stderr.
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_b200_arm(args)


if __name__ == "__main__":
    sys.exit(main())
