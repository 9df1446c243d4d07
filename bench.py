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
# this workload, per GEMV (one ncu launch = 64 GEMVs: 1,623,533,056 +
# 5,308,672 bytes), from the capture summarised under profiles/.
NCU_TRAFFIC_PER_GEMV = (1_623_533_056 + 5_308_672) // 64


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


REF_BUILDS = ("generic", "avx2")  # the reference's generic and x86_avx2 profiles, compiled by oracle/Makefile


class RowSlicedCPU:
    """The reference's C on contiguous row slices across host threads (legal:
    its functions are reentrant, include/kernelsmith/ks_quantized.h:12, and
    rows are independent, so the result is bit-identical to one call)."""

    def __init__(self, threads=None):
        self.threads = threads or host_threads()
        self.pool = cf.ThreadPoolExecutor(max_workers=self.threads)

    def run(self, rows, call):
        T = min(self.threads, rows)
        bounds = [(rows * i // T, rows * (i + 1) // T - rows * i // T) for i in range(T)]
        rcs = list(self.pool.map(lambda ab: call(*ab), bounds))
        assert all(rc == 0 for rc in rcs), rcs

    def seconds(self, fn, reps):
        fn()  # warm-up
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t0) / reps

    def close(self):
        self.pool.shutdown()


def ref_libs():
    """{build: ctypes lib} of the reference builds present (else the oracle port as 'port')."""
    import oracle as O

    libs = {b: O.RefLib(b).lib for b in REF_BUILDS if O.ref_available(b)}
    return libs


def w4a8_rows_call(lib, x, w, s32, y, cols, group, sx=SX):
    """call(r0, n): the reference ks_matvec_w4a8 on rows [r0, r0 + n)."""
    fn = lib.ks_matvec_w4a8
    return lambda r0, n: fn(x.ctypes.data, w.ctypes.data + r0 * w.strides[0], w.strides[0],  # noqa: E731
                            s32.ctypes.data + r0 * s32.strides[0], s32.shape[1], y.ctypes.data + 4 * r0, n, cols,
                            group, sx, 0, 0, None, 0)


def i8_rows_call(lib, x, w, y, cols):
    """call(r0, n): the reference ks_matvec_i8 on rows [r0, r0 + n)."""
    fn = lib.ks_matvec_i8
    return lambda r0, n: fn(x.ctypes.data, w.ctypes.data + r0 * w.strides[0], w.strides[0],  # noqa: E731
                            y.ctypes.data + 4 * r0, n, cols, 0, 0, None, 0)


def port_w4a8_rows_call(x, w, s32, y, cols, group, sx=SX):
    """The oracle port (only when the reference builds are absent)."""
    import oracle as O

    fn = O.Oracle().lib.kso_matvec_w4a8
    return lambda r0, n: fn(x.ctypes.data, w.ctypes.data + r0 * w.strides[0], w.strides[0],  # noqa: E731
                            s32.ctypes.data + r0 * s32.strides[0], s32.shape[1], y.ctypes.data + 4 * r0, n, cols,
                            group, sx, 0, 0)


def w4a8_host_matrix(seed, rows, cols, group):
    import oracle as O

    x = O.rng(seed, 0).integers(-127, 128, cols, dtype=np.int8)
    w = O.rng(seed, 1).integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    s16 = O.rng(seed, 2).uniform(1e-3, 1e-2, (rows, cols // group)).astype(np.float16)
    return x, w, s16


def cpu_reference_runner(build=None):
    """(run_one_gemv, kind, threads, runner, build) for the headline GEMV:
    the reference ks_matvec_w4a8 (f32 scales widened from the f16 set) on row
    slices across all host threads."""
    x, w, s16 = make_host_inputs()
    s32 = s16.astype(np.float32)
    y = np.zeros(ROWS, np.float32)
    libs = ref_libs()
    cpu = RowSlicedCPU()
    if libs:
        build = build if build in libs else ("avx2" if "avx2" in libs else next(iter(libs)))
        call, kind = w4a8_rows_call(libs[build], x, w, s32, y, COLS, GROUP), "reference"
    else:
        build, call, kind = "oracle port", port_w4a8_rows_call(x, w, s32, y, COLS, GROUP), "port"
    return (lambda: cpu.run(ROWS, call)), kind, cpu.threads, cpu, build


def cpu_baseline_headline():
    """The headline configuration on every reference build present; the
    faster build is the line's value, the others are listed beside it."""
    libs = ref_libs() or {"oracle port": None}
    per_build = {}
    for b in libs:
        one, kind, threads, cpu, build = cpu_reference_runner(b if b in REF_BUILDS else None)
        reps = 16
        dt = cpu.seconds(one, reps)
        cpu.close()
        per_build[build] = {"us_per_gemv": dt * 1e6, "TB_s": gemv_bytes() / dt / 1e12, "kind": kind}
    best = max(per_build, key=lambda b: per_build[b]["TB_s"])
    return {"value": per_build[best]["TB_s"], "unit": "TB/s", "cores": host_threads(),
            "kind": per_build[best]["kind"], "build": best, "builds": per_build,
            "sample": f"16 GEMVs {ROWS}x{COLS} G{GROUP} per build (f32 scales widened from the f16 set), "
                      f"rows split over {host_threads()} threads"}


def attach_cpu_baselines(i8, gemm, layer, cfg5):
    """Beside each secondary configuration: the reference's own C for that
    configuration on this host's cores (both builds), rows split over all
    threads.  The f32 / int8 epilogues (a few multiplies per output) and the
    decode layer's RMSNorm / SiLU / quantisation are not timed; the GEMV work
    that dominates them is."""
    libs = ref_libs()
    if not libs:
        return
    import oracle as O

    peak, _ = measured_hbm_peak()
    cpu = RowSlicedCPU()
    T = cpu.threads
    try:
        if i8 is not None:  # configuration 1: ks_matvec_i8 4096 x 4096
            x = O.rng(SEED + 31, 0).integers(-127, 128, I8_K, dtype=np.int8)
            w = O.rng(SEED + 31, 1).integers(-127, 128, (I8_N, I8_K), dtype=np.int8)
            y = np.zeros(I8_N, np.int32)
            b = I8_N * I8_K + I8_K + 8 * I8_N
            builds = {}
            for name, lib in libs.items():
                call = i8_rows_call(lib, x, w, y, I8_K)
                dt = cpu.seconds(lambda: cpu.run(I8_N, call), 64)
                builds[name] = {"us_per_gemv": dt * 1e6, "TB_s": b / dt / 1e12}
            best = max(builds, key=lambda k: builds[k]["TB_s"])
            i8["cpu_baseline"] = {"value": builds[best]["TB_s"], "unit": "TB/s", "cores": T, "kind": "reference",
                                  "build": best, "builds": builds,
                                  "sample": f"64 x ks_matvec_i8 {I8_N}x{I8_K} per build (int32 accumulate; the "
                                            f"per-channel f32 epilogue not timed), rows over {T} threads"}
        if gemm is not None:  # configuration 3: per token, ks_matvec_i8 over W [14336, 4096]
            N, Kd = 14336, 4096
            w = O.rng(SEED + 47, 1).integers(-127, 128, (N, Kd), dtype=np.int8)
            y = np.zeros(N, np.int32)
            res = {}
            for M in (8, 16, 32, 64):
                A = O.rng(SEED + 47, 2 + M).integers(-127, 128, (M, Kd), dtype=np.int8)
                b = N * Kd + M * Kd + M * N + 4 * (M + N)
                builds = {}
                for name, lib in libs.items():
                    calls = [i8_rows_call(lib, A[m], w, y, Kd) for m in range(M)]

                    def one_gemm():
                        for c in calls:
                            cpu.run(N, c)

                    dt = cpu.seconds(one_gemm, 1)
                    builds[name] = {"us": dt * 1e6, "TB_s": b / dt / 1e12}
                best = max(builds, key=lambda k: builds[k]["TB_s"])
                res[f"M{M}"] = {"value": builds[best]["TB_s"], "build": best, "builds": builds}
            gemm["cpu_baseline"] = {"unit": "TB/s", "cores": T, "kind": "reference", "per_m": res,
                                    "sample": "one M x 4096 x 14336 GEMM per M and build as M calls of the "
                                              "reference ks_matvec_i8 (int32 rows per token; the requantising "
                                              f"epilogue not timed), rows over {T} threads"}
        if layer is not None:  # configuration 4: the five W4A8 GEMVs of a layer
            h, i = LAYER_H, LAYER_I
            shapes = [(3 * h, h), (h, h), (i, h), (i, h), (h, i)]
            mats = []
            for k, (r, c) in enumerate(shapes):
                x, w, s16 = w4a8_host_matrix(SEED + 400 + k, r, c, GROUP)
                mats.append((r, c, x, w, s16.astype(np.float32), np.zeros(r, np.float32)))
            builds = {}
            for name, lib in libs.items():
                calls = [(r, w4a8_rows_call(lib, x, w, s, y, c, GROUP)) for r, c, x, w, s, y in mats]

                def one_layer():
                    for r, call in calls:
                        cpu.run(r, call)

                dt = cpu.seconds(one_layer, 1)
                builds[name] = {"us_per_layer": dt * 1e6, "GB_s": layer_bytes() / dt / 1e9}
            best = max(builds, key=lambda k: builds[k]["GB_s"])
            layer["cpu_baseline"] = {"value": builds[best]["GB_s"] / 1e3, "unit": "TB/s", "cores": T,
                                     "kind": "reference", "build": best, "builds": builds,
                                     "sample": "one layer = the five W4A8 GEMVs (QKV, O, gate, up, down; G32, f32 "
                                               "scales) through the reference ks_matvec_w4a8; RMSNorm, SiLU, "
                                               f"residuals and quantisation not timed; rows over {T} threads"}
        if cfg5 is not None:  # configuration 5: the two large shapes
            res = {}
            for name, rows, _ in CFG5_SHAPES:
                sample_rows = min(rows, 32064)  # a bounded sample of the LM head's rows
                x, w, s16 = w4a8_host_matrix(SEED + 500 + rows, sample_rows, CFG5_COLS, CFG5_GROUP)
                s = s16.astype(np.float32)
                y = np.zeros(sample_rows, np.float32)
                builds = {}
                for bname, lib in libs.items():
                    call = w4a8_rows_call(lib, x, w, s, y, CFG5_COLS, CFG5_GROUP)
                    dt = cpu.seconds(lambda: cpu.run(sample_rows, call), 1)
                    dt_full = dt * rows / sample_rows
                    builds[bname] = {"us_per_gemv": dt_full * 1e6, "TB_s": cfg5_bytes(rows) / dt_full / 1e12}
                best = max(builds, key=lambda k: builds[k]["TB_s"])
                res[name] = {"value": builds[best]["TB_s"], "build": best, "builds": builds,
                             "rows_timed": sample_rows}
            cfg5["cpu_baseline"] = {"unit": "TB/s", "cores": T, "kind": "reference", "per_shape": res,
                                    "sample": "one GEMV per shape and build through the reference ks_matvec_w4a8 "
                                              "(f32 scales), the LM head on its first 32064 rows and scaled by "
                                              f"rows; rows over {T} threads"}
    finally:
        cpu.close()


def run_reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    # the faster of the reference's builds on this host (two GEMVs each)
    probe = {}
    for b in ref_libs() or [None]:
        one, kind, threads, cpu, build = cpu_reference_runner(b)
        probe[build] = cpu.seconds(one, 2)
        cpu.close()
    one, kind, threads, cpu, build = cpu_reference_runner(min(probe, key=probe.get))
    for _ in range(args.warmup):
        one()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    cpu.close()
    total = sum(times)
    value = gemv_bytes() * args.steps / total / 1e12
    sample = (f"1 GEMV {ROWS}x{COLS} G{GROUP} per step (f32 scales widened from the f16 set), rows split over "
              f"{threads} threads, reference ks_matvec_w4a8 "
              f"({'oracle/_ref ' + build + ' build, -O3' if kind == 'reference' else 'oracle port'})")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "w4a8-f32acc",
        "data": "synthetic (seeded)", "config": workload_config(world),
        "cpu_baseline": {"value": value, "unit": "TB/s", "cores": threads, "kind": kind, "build": build,
                         "sample": sample},
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

    # NVML sampling runs from before the warm-up to the end of the run, so the
    # line's clock record covers the GPU under load, not one sample
    clocks = ClockSampler(dev)
    clocks.__enter__()
    # ---- resident inputs: 64 shards of [ROWS, COLS] (this rank's rows) ----
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED + 7919 * rank)
    W = torch.randint(0, 256, (MATS, ROWS, COLS // 2), dtype=torch.uint8, device=dev, generator=gen)
    S = (torch.rand((MATS, ROWS, COLS // GROUP), device=dev, generator=gen) * 9e-3 + 1e-3).to(torch.float16)
    # x is replicated: the same activation vectors on every rank
    genx = torch.Generator(device=dev)
    genx.manual_seed(SEED + 1)
    X = torch.randint(-127, 128, (MATS, COLS), dtype=torch.int8, device=dev, generator=genx)
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

        pgw = PeerGatherW4A8(MATS, ROWS, dev, timeout_ns=5_000_000_000)
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
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    n_before = len(clocks.samples)
    with torch.cuda.stream(main):
        start.record(main)
        for _ in range(args.steps):
            step()
        end.record(main)
        end.synchronize()
    n_timed = len(clocks.samples) - n_before
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
    gathered_check = None
    if world > 1:
        # values, not only status words: the gathered outputs of the first and
        # last matrix of the last step against the single-GPU result of the
        # full matrix on this GPU (its row blocks all-gathered from the ranks)
        def full_out(m):
            if peer:
                return pgw.y[m]
            return Yfull[m // per_chunk][:, m % per_chunk, :].reshape(-1)

        ok = True
        for m in (0, MATS - 1):
            wf = torch.empty((world * ROWS, COLS // 2), dtype=torch.uint8, device=dev)
            sf = torch.empty((world * ROWS, COLS // GROUP), dtype=torch.float16, device=dev)
            dist.all_gather_into_tensor(wf, W[m].contiguous())
            dist.all_gather_into_tensor(sf, S[m].contiguous())
            y1 = torch.zeros(world * ROWS, dtype=torch.float32, device=dev)
            K.matvec_w4a8_async(X[m], wf, COLS // 2, sf, COLS // GROUP, y1, world * ROWS, COLS, GROUP, SX,
                                scale_type=K.SCALE_F16, status=status)
            torch.cuda.synchronize()
            ok = ok and bool(torch.equal(y1, full_out(m)))
            del wf, sf
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        gathered_check = {"matrices": [0, MATS - 1], "bitwise_equal_single_gpu_on_every_rank": bool(flag.item()),
                          "reference": "full matrix on one GPU (row blocks all-gathered), same kernel family"}

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

    for g in graphs:
        del g
    graphs.clear()
    wait_graph = None
    if peer:
        dist.barrier()
        torch.cuda.synchronize()
        pgw.close()
    del W, S, Yfull, Yloc
    torch.cuda.empty_cache()

    # the sharded large-matrix configuration, at every N (strong scaling)
    cfg5 = run_sharded_cfg5(K, torch, dist, dev, world, rank) if not args.no_secondary else None
    layer = run_decode_layers(K, torch, dev, args) if args.decode_layers > 0 else None
    # the other configurations, single GPU only (per-GPU numbers)
    i8 = run_int8_gemv(K, torch, dev) if world == 1 and not args.no_secondary else None
    gemm = run_gemm(K, torch, dev) if world == 1 and not args.no_secondary else None
    imp = run_import(K, torch, dev) if world == 1 and not args.no_secondary else None
    gw4 = run_gemm_w4a8(K, torch, dev) if world == 1 and not args.no_secondary else None
    clocks.__exit__(None, None, None)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_headline()
        attach_cpu_baselines(i8, gemm, layer, cfg5)

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
            "gathered_check": gathered_check,
            "sharded_cfg5": cfg5,
            "decode_layer": layer,
            "int8_gemv": i8,
            "gemm_i8": gemm,
            "q4_0_import": imp,
            "gemm_w4a8": gw4,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": CHUNKS * args.steps * world,
            "clocks": dict(clocks.summary(), samples_in_timed_region=n_timed,
                           window="from before the warm-up to the end of the secondary measurements"),
        }
        print(json.dumps(line), file=_JSON_OUT, flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if gathered_check is not None and not gathered_check["bitwise_equal_single_gpu_on_every_rank"]:
        raise SystemExit("gathered outputs differ from the single-GPU result")
    if cfg5 is not None and cfg5.get("gathered_equal_single_gpu") is False:
        raise SystemExit("sharded configuration: gathered outputs differ from the single-GPU result")
    return 0


LAYER_H, LAYER_I = 4096, 11008


def layer_bytes(h=LAYER_H, i=LAYER_I, group=GROUP):
    """Weights + f16 scales of one decode layer (QKV, O, gate, up, down)."""
    mats = [(3 * h, h), (h, h), (i, h), (i, h), (h, i)]
    return sum(r * c // 2 + r * (c // group) * 2 for r, c in mats)


def run_decode_layers(K, torch, dev, args):
    """A chain of fused W4A8 decode layers (hidden 4096, inter 11008, G 32,
    distinct random weights per layer), graph-captured; per-layer time.  The
    headline form is ks_b200_decode_layers_w4a8_async (the whole chain in one
    call: one persistent launch per 32 layers); one_launch_per_layer is the
    same chain as one ks_b200_decode_layer_w4a8_async call per layer."""
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
    out = torch.zeros(h, dtype=torch.float32, device=dev)
    ws_bytes = L.ks_b200_decode_layers_workspace(h, i)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    status = torch.zeros(K.STATUS_WORDS, dtype=torch.int32, device=dev)
    wp = [(ctypes.c_void_p * 5)(*[t.data_ptr() for t in W]) for W in Ws]
    sp = [(ctypes.c_void_p * 5)(*[t.data_ptr() for t in S]) for S in Ss]
    w_all = (ctypes.c_void_p * (5 * n))(*[t.data_ptr() for W in Ws for t in W])
    s_all = (ctypes.c_void_p * (5 * n))(*[t.data_ptr() for S in Ss for t in S])
    n1 = (ctypes.c_void_p * n)(*([norms[0].data_ptr()] * n))
    n2 = (ctypes.c_void_p * n)(*([norms[1].data_ptr()] * n))
    stream = torch.cuda.Stream(device=dev)
    # the zero-filled workspace and the inputs are written on the current
    # stream; the layers run on `stream`
    stream.wait_stream(torch.cuda.current_stream(dev))

    def chain_one_call():
        K.check(L.ks_b200_decode_layers_w4a8_async(n, acts[0].data_ptr(), out.data_ptr(), n1, n2, 1e-5, w_all, s_all,
                                                    h, i, GROUP, ws.data_ptr(), ws_bytes, status.data_ptr(),
                                                    K.stream_handle(stream)))

    def chain_per_layer():
        for l in range(n):
            K.check(L.ks_b200_decode_layer_w4a8_async(acts[l].data_ptr(), acts[l + 1].data_ptr(),
                                                      norms[0].data_ptr(), norms[1].data_ptr(), 1e-5, wp[l], sp[l],
                                                      h, i, GROUP, ws.data_ptr(), ws_bytes, status.data_ptr(),
                                                      K.stream_handle(stream)))

    us = _graph_us(torch, stream, chain_one_call, n)
    us_per = _graph_us(torch, stream, chain_per_layer, n)
    same = bool(torch.equal(out, acts[n]))
    assert status.cpu().tolist() == [0, 0]
    peak, _ = measured_hbm_peak()
    b = layer_bytes()
    return {"layers": n, "us_per_layer": us, "weight_bytes_per_layer": b, "GB_s": b / us / 1e3,
            "frac": b / us / 1e3 / peak, "launches": -(-n // 32),
            "one_launch_per_layer": {"us_per_layer": us_per, "frac": b / us_per / 1e3 / peak,
                                     "launches_per_layer": L.ks_b200_decode_layer_launches(h, i, GROUP)},
            "chain_equals_per_layer_calls": same,
            "shape": "hidden 4096, inter 11008, W4A8 G32 f16 scales, batch 1, fused RMSNorm/quantise/SiLU/residual",
            "api": "ks_b200_decode_layers_w4a8_async (32 layers per persistent launch)"}


def _graph_us(torch, stream, fn, units, reps=10, before_timing=None):
    """Device time per unit of `fn` (graph-captured, CUDA events on `stream`).
    before_timing() runs after the warm-up replays (a barrier across ranks)."""
    with torch.cuda.stream(stream):
        fn()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
        if before_timing is not None:
            stream.synchronize()
            before_timing()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * units)
    del g
    return us


CFG5_COLS, CFG5_GROUP = 8192, 128
# (name, rows, distinct matrices per step): 16 x 121 MB and 4 x 542 MB of
# weights per step on one GPU, both above the 126 MB L2 at every N
CFG5_SHAPES = [("up_28672x8192", 28672, 16), ("lm_head_128256x8192", 128256, 4)]


def cfg5_bytes(rows, cols=CFG5_COLS, group=CFG5_GROUP):
    """Algorithmic bytes of one sharded-configuration GEMV over `rows` rows."""
    return rows * (cols // 2) + rows * (cols // group) * 2 + cols + rows * 4


def _reduce(torch, dist, dev, world, v, op):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=op)
    return float(t.item())


def run_sharded_cfg5(K, torch, dist, dev, world, rank, reps=10):
    """W4A8 K=8192, N=28672 and N=128256, G128, f16 scales, split along N over
    the ranks (strong scaling: the matrices are the same at every N).  Per GEMV,
    max over ranks, CUDA events:
      t_gemv   this rank's row block only, local outputs (one batched launch
               of the step's matrices);
      t_peer   the same launch with the gather fused into it (peer stores,
               arrival wait);
      t_nccl   the same launch with local outputs, then an NCCL all-gather
               of the step's output slices (serialised after it);
      t_peer_chain  one matrix per launch, each followed by its arrival wait
               (a dependent chain: the next GEMV may use the gathered output);
      t1, t1_chain  the full matrices on one GPU (measured on every rank,
               the fastest taken), batched and one launch per matrix.
    Efficiency(P) = t1 / (P * t(P)) for each.  After the timing every rank
    compares the gathered outputs of two matrices bitwise with its own
    single-GPU result."""
    from kernelsmith_b200.sharded import NcclGatherW4A8, PeerGatherW4A8

    peak, _ = measured_hbm_peak()
    main = torch.cuda.Stream(device=dev)
    out = {"cols": CFG5_COLS, "group": CFG5_GROUP, "scale_dtype": "f16", "n_gpus": world, "shapes": {},
           "method": "per GEMV, CUDA events on the launching stream, max over ranks (t1: fastest rank)"}
    all_equal = True
    for si, (name, rows, C) in enumerate(CFG5_SHAPES):
        R = rows // world
        gen = torch.Generator(device=dev)
        gen.manual_seed(SEED + 101 * (si + 1) + 7919 * rank)
        W = torch.randint(0, 256, (C, R, CFG5_COLS // 2), dtype=torch.uint8, device=dev, generator=gen)
        S = (torch.rand((C, R, CFG5_COLS // CFG5_GROUP), device=dev, generator=gen) * 9e-3 + 1e-3).to(torch.float16)
        genx = torch.Generator(device=dev)
        genx.manual_seed(SEED + 202 * (si + 1))
        X = torch.randint(-127, 128, (C, CFG5_COLS), dtype=torch.int8, device=dev, generator=genx)
        Yl = torch.zeros((C, R), dtype=torch.float32, device=dev)
        status = torch.zeros(K.STATUS_WORDS, dtype=torch.int32, device=dev)
        main.wait_stream(torch.cuda.current_stream(dev))
        xs, ws, ss = [X[m] for m in range(C)], [W[m] for m in range(C)], [S[m] for m in range(C)]
        wst, sst = CFG5_COLS // 2, CFG5_COLS // CFG5_GROUP

        def local():
            K.matvec_w4a8_batch_async(xs, ws, ss, [Yl[m] for m in range(C)], wst, sst, R, CFG5_COLS, CFG5_GROUP, SX,
                                      scale_type=K.SCALE_F16, status=status, stream=main)

        rec = {"rows": rows, "rows_per_rank": R, "matrices_per_step": C,
               "bytes_per_gemv_full": cfg5_bytes(rows), "bytes_per_gemv_per_rank": cfg5_bytes(R)}
        line_up = dist.barrier if world > 1 else None
        t_gemv = _reduce(torch, dist, dev, world, _graph_us(torch, main, local, C, reps, line_up),
                         dist.ReduceOp.MAX)
        rec["t_gemv_us"] = t_gemv
        rec["gemv_frac_per_rank"] = cfg5_bytes(R) / t_gemv / 1e3 / peak
        peer_out = nccl_out = None
        if world > 1:
            pg = PeerGatherW4A8(C, R, dev, timeout_ns=5_000_000_000)
            rec["t_peer_us"] = _reduce(torch, dist, dev, world, _graph_us(
                torch, main, lambda: pg.run(xs, ws, ss, CFG5_COLS, CFG5_GROUP, SX, K.SCALE_F16, stream=main), C,
                reps, line_up), dist.ReduceOp.MAX)

            def chain():
                for m in range(C):
                    pg.run([xs[m]], [ws[m]], [ss[m]], CFG5_COLS, CFG5_GROUP, SX, K.SCALE_F16, stream=main, m0=m)

            rec["t_peer_chain_us"] = _reduce(torch, dist, dev, world, _graph_us(torch, main, chain, C, reps, line_up),
                                             dist.ReduceOp.MAX)
            # NCCL: the launch is graph-captured, the all-gather issued after each replay
            ng = NcclGatherW4A8(C, R, dev)

            def nccl_launch():
                K.matvec_w4a8_batch_async(xs, ws, ss, [ng.y_local[m] for m in range(C)], wst, sst, R, CFG5_COLS,
                                          CFG5_GROUP, SX, scale_type=K.SCALE_F16, status=status, stream=main)

            with torch.cuda.stream(main):
                nccl_launch()
            main.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=main):
                nccl_launch()

            def nccl_step():
                g.replay()
                dist.all_gather_into_tensor(ng.y_all, ng.y_local)

            with torch.cuda.stream(main):
                for _ in range(3):
                    nccl_step()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(main):
                e0.record(main)
                for _ in range(reps):
                    nccl_step()
                e1.record(main)
                e1.synchronize()
            rec["t_nccl_us"] = _reduce(torch, dist, dev, world, e0.elapsed_time(e1) * 1e3 / (reps * C),
                                       dist.ReduceOp.MAX)
            del g
            peer_out, nccl_out = pg, ng
        # single GPU: the full matrices, row blocks all-gathered from the ranks
        if world > 1:
            Wf = torch.empty((C, rows, CFG5_COLS // 2), dtype=torch.uint8, device=dev)
            Sf = torch.empty((C, rows, CFG5_COLS // CFG5_GROUP), dtype=torch.float16, device=dev)
            for m in range(C):
                dist.all_gather_into_tensor(Wf[m], W[m])
                dist.all_gather_into_tensor(Sf[m], S[m])
        else:
            Wf, Sf = W, S
        Y1 = torch.zeros((C, rows), dtype=torch.float32, device=dev)

        def full_batched():
            K.matvec_w4a8_batch_async(xs, [Wf[m] for m in range(C)], [Sf[m] for m in range(C)],
                                      [Y1[m] for m in range(C)], wst, sst, rows, CFG5_COLS, CFG5_GROUP, SX,
                                      scale_type=K.SCALE_F16, status=status, stream=main)

        def full_chain():
            for m in range(C):
                K.matvec_w4a8_async(xs[m], Wf[m], wst, Sf[m], sst, Y1[m], rows, CFG5_COLS, CFG5_GROUP, SX,
                                    scale_type=K.SCALE_F16, status=status, stream=main)

        main.wait_stream(torch.cuda.current_stream(dev))
        t1 = _reduce(torch, dist, dev, world, _graph_us(torch, main, full_batched, C, reps), dist.ReduceOp.MIN)
        t1c = _reduce(torch, dist, dev, world, _graph_us(torch, main, full_chain, C, reps), dist.ReduceOp.MIN)
        full_batched()  # Y1 for the value check
        main.synchronize()
        rec["t1_us"], rec["t1_chain_us"] = t1, t1c
        rec["t1_frac"] = cfg5_bytes(rows) / t1 / 1e3 / peak
        rec["efficiency_gemv_only"] = t1 / (world * t_gemv)
        if world > 1:
            rec["efficiency_gemv_peer_gather"] = t1 / (world * rec["t_peer_us"])
            rec["efficiency_gemv_nccl_gather"] = t1 / (world * rec["t_nccl_us"])
            rec["efficiency_chain_peer_gather"] = t1c / (world * rec["t_peer_chain_us"])
            ok = True
            for m in (0, C - 1):
                ok = ok and bool(torch.equal(peer_out.y[m], Y1[m])) and bool(torch.equal(nccl_out.full(m), Y1[m]))
            flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            rec["gathered_equal_single_gpu"] = bool(flag.item())
            all_equal = all_equal and rec["gathered_equal_single_gpu"]
            assert peer_out.status.cpu().tolist() == [0, 0], "peer-gather status"
            dist.barrier()
            torch.cuda.synchronize()
            peer_out.close()
            del Wf, Sf
        assert status.cpu().tolist() == [0, 0], f"device status {status.cpu().tolist()}"
        out["shapes"][name] = rec
        del W, S, X, Yl, Y1, peer_out, nccl_out
        torch.cuda.empty_cache()
    if world > 1:
        out["gathered_equal_single_gpu"] = all_equal
    out["note"] = ("t1 and the efficiencies come from this run (the full matrices all-gathered to every rank and "
                   "timed on one GPU each); GEMV-only efficiency excludes any gather")
    return out


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
           "kernel": "gemm_w4a8_tc_kernel (int4 widened to int8 into tensor memory, tcgen05.mma kind::i8 with the A operand in TMEM)"}
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
