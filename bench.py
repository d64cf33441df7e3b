"""Benchmark: exact KNN-graph build of 1M x 128 (integer-valued), k=10, L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 3]

A step is one whole build of the graph over the configuration's synthetic
dataset (pack + fused tensor-core KNN + exact fallback; for N > 1 also the
NCCL exchange of packed rows and the gather of the graph rows). Prints one
JSON line on rank 0. Under torchrun every rank builds its query shard and
the time is the max over ranks.

* ``value``: algorithmic distance throughput 2*n*n*d / build time, inputs
  resident in HBM (each rank holds its slice of the fp32 rows), TOP/s.
* ``e2e``: the same metric through the public host API: pinned host rows ->
  device, build, graph rows -> pinned host memory, every step.
* ``roofline``: the fused kernel against the dense int8 tensor peak (twice
  the measured bf16 cuBLAS figure of MEASURED_PEAKS.json).
* ``cpu_baseline``: the reference's own OpenMP builder
  (knng::cpu::brute_force_knn_l2_omp, src/cpu/brute_force_omp.cpp:32-105,
  compiled unmodified into oracle/_ref) on a seeded prefix of the same
  dataset, scaled by pair count.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC_NAME = "KNNG build time & distance TFLOP/s, 1M×128 k=10, 1/2/4/8 B200; recall vs ref"
UNIT = "TOP/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--n", type=int, default=0, help="override n (debug only)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ------------------------------------------------------------------ CPU arms
def ref_lib():
    import ctypes

    so = ROOT / "oracle" / "_ref" / "libknng_ref.so"
    if not so.exists():
        return None
    lib = ctypes.CDLL(str(so))
    lib.ref_brute_force_knn_omp.restype = ctypes.c_int
    lib.ref_brute_force_knn_omp.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                                            ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    return lib


def time_reference_omp(x: np.ndarray, n_prefix: int, k: int, threads: int) -> float:
    lib = ref_lib()
    xs = np.ascontiguousarray(x[:n_prefix])
    ids = np.empty(n_prefix * k, np.uint32)
    dists = np.empty(n_prefix * k, np.float32)
    t0 = time.perf_counter()
    rc = lib.ref_brute_force_knn_omp(xs.ctypes.data, n_prefix, xs.shape[1], k, threads, ids.ctypes.data,
                                     dists.ctypes.data)
    t = time.perf_counter() - t0
    if rc != 0:
        raise RuntimeError("reference builder failed")
    return t


def cpu_baseline(x: np.ndarray, k: int, target_s: float) -> dict:
    """The reference's all-core builder on a prefix sized to ~target_s."""
    threads = os.cpu_count() or 1
    d = x.shape[1]
    probe = min(4000, x.shape[0])
    t = time_reference_omp(x, probe, k, threads)
    rate = probe * probe / max(t, 1e-9)  # pairs / s
    n_prefix = int(min(x.shape[0], max(probe, (rate * target_s) ** 0.5)))
    t = time_reference_omp(x, n_prefix, k, threads)
    tops = 2.0 * n_prefix * n_prefix * d / t / 1e12
    return {
        "value": tops,
        "unit": UNIT,
        "cores": threads,
        "kind": "reference",
        "sample": f"knng::cpu::brute_force_knn_l2_omp on the first {n_prefix} rows of the dataset "
                  f"({n_prefix * n_prefix:.3g} pairs, {t:.1f} s); throughput = 2*pairs*d/time, "
                  f"full 1M build extrapolated by pair count = {t * (x.shape[0] / n_prefix) ** 2:.0f} s",
        "seconds": t,
        "full_build_seconds_extrapolated": t * (x.shape[0] / n_prefix) ** 2,
    }


def run_reference_arm(args, cfg, x) -> None:
    world, rank, _ = dist_env()
    if rank != 0:
        return
    if ref_lib() is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libknng_ref.so was not built"}))
        return
    threads = os.cpu_count() or 1
    n_prefix = min(cfg.n, 20000)
    for _ in range(args.warmup):
        time_reference_omp(x, 2000, cfg.k, threads)
    times = [time_reference_omp(x, n_prefix, cfg.k, threads) for _ in range(args.steps)]
    t = float(np.mean(times))
    tops = 2.0 * n_prefix * n_prefix * cfg.d / t / 1e12
    sample = (f"each step: knng::cpu::brute_force_knn_l2_omp (unmodified reference, oracle/_ref) on the first "
              f"{n_prefix} rows of the {cfg.name} dataset with {threads} threads; scaled by pair count")
    print(json.dumps({
        "impl": "reference", "metric": METRIC_NAME, "value": tops, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": cfg.name, "n": cfg.n, "d": cfg.d, "k": cfg.k, "metric": "L2Squared",
                   "sample_rows": n_prefix},
        "cpu_baseline": {"value": tops, "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": tops, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "full_build_seconds_extrapolated": t * (cfg.n / n_prefix) ** 2,
    }))


# ------------------------------------------------------------------ clocks
class ClockSampler:
    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = ROOT / "gpurun_out" / f"clocks_{index}.csv"

    def __enter__(self):
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait()
            self.f.close()

    def summary(self) -> dict:
        try:
            rows = [r.split(", ") for r in self.path.read_text().strip().splitlines() if r.strip()]
        except Exception:
            rows = []
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for nm, v in zip(names, r[5:9]):
                if v.strip() == "Active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(rows[0][2]), "reasons": sorted(reasons),
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows)}


# ------------------------------------------------------------------ GPU arm
def main() -> None:
    args = parse()
    world, rank, local = dist_env()
    from knng_gpu_b200 import synthetic as syn

    cfg = syn.CONFIGS[args.config]
    n = args.n or cfg.n
    if args.impl == "reference":
        x = syn.generate_config(cfg, n if n < cfg.n else None) if rank == 0 else None
        run_reference_arm(args, cfg, x)
        return

    import torch
    import torch.distributed as dist

    import knng_gpu_b200 as kg
    from knng_gpu_b200.distributed import ShardedBuilder

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    x_host = torch.from_numpy(syn.generate_config(cfg, n)).pin_memory()
    d, k = cfg.d, cfg.k
    builder = ShardedBuilder(n, d, k, cfg.metric)
    lo, hi = builder.slice_bounds
    x_slice = x_host[lo:hi].to(dev)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-resident steps (clock sampling spans warm-up and timed steps)
    knn_ms = []
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        for _ in range(args.warmup):
            builder.build(x_slice)
        barrier()
        ev0.record(stream)
        for _ in range(args.steps):
            ids, dists = builder.build(x_slice)
            knn_ms.append(builder.last_stats.get("knn_ms", 0.0))
        ev1.record(stream)
        barrier()
    step_ms = ev0.elapsed_time(ev1) / args.steps
    # one extra, separately timed build: where the time of a step goes
    builder.timing = True
    builder.build(x_slice)
    phases = builder.phase_ms()
    builder.timing = False
    launches_per_step = int(builder.last_stats.get("kernel_launches", 0)) + 2  # + pack and augmentation
    t = torch.tensor([step_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms = float(t.item())
    ops = 2.0 * n * n * d
    value = ops / (step_ms * 1e-3) / 1e12

    # ---- roofline of the fused kernel on this rank's shard
    kms = float(np.mean(knn_ms))
    shard_ops = 2.0 * builder.shard.count * n * d
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        int8_peak = 2.0 * float(peaks["bf16_tflops"])
        peak_src = "2x measured bf16 cuBLAS burst (MEASURED_PEAKS.json): dense int8 rate is twice bf16 on B200"
    except Exception:
        int8_peak = 2.0 * 1590.0
        peak_src = "2x fallback 1.59 PFLOP/s bf16"
    achieved = shard_ops / (kms * 1e-3) / 1e12
    traffic = None
    try:
        tj = json.loads((ROOT / "profiles" / "knn_tc_u8_cfg3_traffic.json").read_text())
        traffic = float(tj["dram_bytes_per_launch_full_cfg3"]) * builder.shard.count / n
    except Exception:
        pass
    roofline = {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOP/s",
                "frac": achieved / int8_peak, "traffic": traffic, "kernel": "knn_tc_kernel<ElemU8,...>",
                "kernel_ms": kms, "peak_basis": peak_src}

    # ---- parity spot check: 4 rows recomputed in float64 with torch (exact
    # for integer-valued rows), ordered by (distance, id) like knng::TopK
    recall_info = None
    if rank == 0:
        xx = x_host.to(dev, dtype=torch.float64)
        q = torch.tensor([0, 1, n // 2, n - 1], device=dev)
        if cfg.metric == 1:
            dd = -(xx[q] @ xx.T)
        else:
            dd = (xx * xx).sum(1)[None, :] + (xx[q] * xx[q]).sum(1)[:, None] - 2.0 * (xx[q] @ xx.T)
        dd[torch.arange(4, device=dev), q] = float("inf")
        order = torch.sort(dd, dim=1, stable=True).indices[:, :k]
        ref_d = torch.gather(dd, 1, order).float()
        got_ids = ids[q].long()
        recall_info = {"rows_checked": 4,
                       "ids_equal": bool(torch.equal(order, got_ids)),
                       "dists_equal": bool(torch.equal(ref_d, dists[q]))}
        del xx, dd

    # ---- end to end through the public API (host buffers every step)
    e2e = None
    if not args.no_e2e:
        out_ids = torch.empty((n, k), dtype=torch.int32).pin_memory()
        out_d = torch.empty((n, k), dtype=torch.float32).pin_memory()
        if world == 1:
            xnp = x_host.numpy()
            for _ in range(max(1, args.warmup // 2)):
                kg.brute_force_knn(xnp, k, cfg.metric)
            barrier()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                g = kg.brute_force_knn(xnp, k, cfg.metric)
            e2e_s = (time.perf_counter() - t0) / args.steps
            h2d = n * d * 4
            d2h = n * k * 8
        else:
            xh = x_host[lo:hi]
            for _ in range(max(1, args.warmup // 2)):
                xs = xh.to(dev, non_blocking=True)
                i2, d2 = builder.build(xs)
            barrier()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                xs = xh.to(dev, non_blocking=True)
                i2, d2 = builder.build(xs)
                if rank == 0:
                    out_ids.copy_(i2, non_blocking=True)
                    out_d.copy_(d2, non_blocking=True)
                torch.cuda.synchronize()
            e2e_local = (time.perf_counter() - t0) / args.steps
            tt = torch.tensor([e2e_local], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e2e_s = float(tt.item())
            h2d = n * d * 4
            d2h = n * k * 8
        e2e = {"value": ops / e2e_s / 1e12, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "seconds_per_build": e2e_s,
               "api": "knng_gpu_brute_force (C ABI, host buffers)" if world == 1 else
               "ShardedBuilder.build (pinned H2D of each rank's slice + NCCL + gather to rank 0 + D2H)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and ref_lib() is not None:
        cpu = cpu_baseline(x_host.numpy(), k, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC_NAME, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "build_seconds": step_ms / 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic (seeded XorShift64 integers in [0,255] stored as fp32)",
            "config": {"workload": cfg.name, "n": n, "d": d, "k": k, "metric": "L2Squared",
                       "parallelism": f"query-shard x{world}, base all-gathered (NCCL)",
                       "l2": "inputs larger than L2 (512 MB fp32 rows)"},
            "roofline": roofline, "e2e": e2e, "cpu_baseline": cpu, "clocks": clk.summary(),
            "gpu_launches": launches_per_step * args.steps, "parity_spot_check": recall_info,
            "path": builder.last_stats.get("path"), "fallback_rows": builder.last_stats.get("fallback_rows"),
            "phase_ms_rank0": phases,
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
