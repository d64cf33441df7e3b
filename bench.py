"""Benchmark: exact all-points KNN-graph build of a configuration of BASELINE.json.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 1..5]

Default: configuration 3 (n = 1M, d = 128, integer-valued fp32 rows, k = 10,
L2Squared) -- the workload the headline metric is quoted on. A step is one
whole build of the graph over the configuration's synthetic dataset: pack +
integer check, the fused tensor-core KNN, the exact fallback, and for N > 1
the NCCL exchange of packed rows and the gather of the graph rows to rank 0.
Prints one JSON line on rank 0; under torchrun every rank builds its query
shard and the time is the max over ranks.

* ``value``: algorithmic distance throughput 2*n*n*d / build time (TOP/s),
  inputs resident in HBM.
* ``e2e``: the same metric through the public host API (host rows in, graph
  rows out, copies inside the timed region).
* ``roofline``: the dominant tensor-core kernel, timed with CUDA events on its
  stream, against the measured peak of its precision.
* ``parity``: after the timed region, rank 0 recomputes >= 256 seeded query
  rows with the reference's own brute-force loop (the unmodified reference
  sources compiled into oracle/_ref; include/knng/cpu/brute_force.hpp:355-374)
  and compares ids and fp32 distance bits with the assembled graph.
* ``cpu_baseline`` (N = 1): the time of that reference run (all host cores,
  the seeded query subset against the full base), scaled to the full build.

``--impl reference`` times the same reference loop on a seeded query subset
against the full base, every step, and prints the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC_NAME = "KNNG build time & distance TFLOP/s, 1M×128 k=10, 1/2/4/8 B200; recall vs ref"
UNIT = "TOP/s"
PARITY_SEED = 0x5EED
# Query rows per reference-arm step, sized so that a step takes a few seconds
# on 16 host cores (the canonical loop runs at ~1 ns per coordinate per core).
REF_QUERIES = {1: 10_000, 2: 2048, 3: 512, 4: 64, 5: 16}
# Seeded query rows of the one-GPU parity check, which also times the CPU
# baseline: ~10-30 s of reference work on 16 host cores (all of config 1).
CPU_SAMPLE = {1: 10_000, 2: 8192, 3: 2048, 4: 256, 5: 256}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=3)
    # --rows is the spelling to use under torch.distributed.run, whose own
    # parser takes a bare --n for an abbreviation of its --nnodes/--nproc-per-node.
    ap.add_argument("--n", "--rows", dest="n", type=int, default=0,
                    help="override n (smaller runs of the same recipe)")
    ap.add_argument("--parity-rows", type=int, default=256)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), int(
        os.environ.get("LOCAL_RANK", "0"))


def describe(cfg) -> dict:
    """Fields of the JSON line that depend on the configuration."""
    from knng_gpu_b200 import synthetic as syn

    integer = cfg.kind in (syn.KIND_UNIFORM_INT, syn.KIND_SPARSE_INT)
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        bf16 = float(peaks["bf16_tflops"])
        src = "measured bf16 cuBLAS burst of MEASURED_PEAKS.json"
    except Exception:
        bf16 = 1590.0
        src = "fallback 1.59 PFLOP/s bf16 burst"
    if integer and cfg.d <= 1024:
        # The library's selection: the CTA-pair kernel for rows longer than
        # 256 bytes with k <= 64, the single-CTA kernel otherwise.
        kernel = "knn_pair_kernel" if (cfg.d > 256 and cfg.k <= 64) else "knn_tc_kernel<ElemU8>"
        peak = 2.0 * bf16
        basis = f"2 x {src} ({bf16} TFLOP/s): the dense int8 tensor rate of B200 is twice its bf16 rate"
        dtype = "u8"
    else:
        kernel = "knn_tc_kernel<ElemBf16x3>"
        peak = bf16 / 3.0
        basis = (f"{src} ({bf16} TFLOP/s) / 3: the fp32 path executes three bf16 UMMAs (hi.hi + hi.lo + lo.hi) "
                 "per fp32-equivalent multiply-add, so its ceiling is a third of the bf16 rate")
        dtype = "f32"
    return {"integer": integer, "dtype": dtype, "kernel": kernel, "peak": peak, "peak_basis": basis,
            "metric_name": "L2Squared" if cfg.metric == 0 else "NegativeInnerProduct",
            "data": ("synthetic (seeded XorShift64 recipe of the configuration, "
                     + ("integer values stored as fp32)" if integer else "fp32 values)"))}


# ------------------------------------------------------------------ the reference on the host cores
def ref_lib():
    import ctypes

    so = ROOT / "oracle" / "_ref" / "libknng_ref.so"
    if not so.exists():
        return None
    lib = ctypes.CDLL(str(so))
    c = ctypes
    lib.ref_subset_knn.restype = c.c_int
    lib.ref_subset_knn.argtypes = [c.c_void_p, c.c_uint64, c.c_uint64, c.c_uint64, c.c_int, c.c_void_p, c.c_uint64,
                                   c.c_int, c.c_void_p, c.c_void_p]
    lib.ref_brute_force_knn.restype = c.c_int
    lib.ref_brute_force_knn.argtypes = [c.c_void_p, c.c_uint64, c.c_uint64, c.c_uint64, c.c_int, c.c_void_p,
                                        c.c_void_p]
    return lib


def ref_subset(lib, x: np.ndarray, k: int, metric: int, q: np.ndarray, threads: int):
    """The reference's loop body (brute_force.hpp:355-374) for query rows q
    against all rows of x; returns (ids, dists, seconds)."""
    n, d = x.shape
    q = np.ascontiguousarray(q, dtype=np.uint64)
    ids = np.zeros((len(q), k), np.uint32)
    dists = np.zeros((len(q), k), np.float32)
    t0 = time.perf_counter()
    rc = lib.ref_subset_knn(x.ctypes.data, n, d, k, metric, q.ctypes.data, len(q), threads, ids.ctypes.data,
                            dists.ctypes.data)
    t = time.perf_counter() - t0
    if rc != 0:
        raise RuntimeError("reference subset harness failed")
    return ids, dists, t


def run_reference_arm(args, cfg, n) -> None:
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from knng_gpu_b200 import synthetic as syn

    lib = ref_lib()
    if lib is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libknng_ref.so was not built"}))
        return
    x = syn.generate_config(cfg, n)
    threads = os.cpu_count() or 1
    m = min(REF_QUERIES.get(args.config, 256), n)
    q = syn.sample_ids(cfg.seed ^ PARITY_SEED, n, m)
    for _ in range(args.warmup):
        ref_subset(lib, x, cfg.k, cfg.metric, q[: max(1, m // 8)], threads)
    times = [ref_subset(lib, x, cfg.k, cfg.metric, q, threads)[2] for _ in range(args.steps)]
    t = float(np.mean(times))
    tops = 2.0 * m * n * cfg.d / t / 1e12
    full_s = t * n / m
    f = describe(cfg)
    extra = {}
    if args.config == 3 and world == 1:
        # The canonical single-thread builder (the oracle itself) on config 1.
        c1 = syn.CONFIGS[1]
        x1 = syn.generate_config(c1)
        ids = np.empty(c1.n * c1.k, np.uint32)
        dd = np.empty(c1.n * c1.k, np.float32)
        t0 = time.perf_counter()
        lib.ref_brute_force_knn(x1.ctypes.data, c1.n, c1.d, c1.k, c1.metric, ids.ctypes.data, dd.ctypes.data)
        extra["canonical_single_thread_cfg1_s"] = time.perf_counter() - t0
    sample = (f"each step: the reference's canonical brute-force loop (knng::cpu::brute_force_knn body, "
              f"brute_force.hpp:355-374, unmodified sources in oracle/_ref) for {m} seeded query rows against "
              f"all {n} rows, OpenMP over queries on {threads} threads; rate = 2*m*n*d/time, full build "
              f"= time x n/m")
    print(json.dumps({
        "impl": "reference", "metric": METRIC_NAME, "value": tops, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": f["data"],
        "config": {"workload": cfg.name, "n": n, "d": cfg.d, "k": cfg.k, "metric": f["metric_name"],
                   "query_sample": m},
        "cpu_baseline": {"value": tops, "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": tops, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "full_build_seconds_extrapolated": full_s, **extra,
    }))


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples of one GPU's clocks and throttle reasons, written to
    a temporary file while the timed region runs."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=f"_clocks_{index}.csv", delete=False)
        self.path = Path(self.tmp.name)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait()
        self.tmp.close()

    def summary(self) -> dict:
        try:
            rows = [r.split(", ") for r in self.path.read_text().strip().splitlines() if r.strip()]
            self.path.unlink()
        except Exception:
            rows = []
        rows = [r for r in rows if len(r) >= 9]
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


def traffic_for(kernel: str, workload: str, shard_frac: float):
    """DRAM bytes per launch of `kernel` on `workload` from the committed ncu
    summary (profiles/*_traffic.json), scaled to this rank's share of the
    query rows; None when no capture of this kernel exists."""
    for p in sorted((ROOT / "profiles").glob("*_traffic.json")):
        try:
            tj = json.loads(p.read_text())
        except Exception:
            continue
        if tj.get("kernel", "").startswith(kernel) and tj.get("workload_name") == workload:
            return float(tj["dram_bytes_per_launch_full"]) * shard_frac
    return None


# ------------------------------------------------------------------ GPU arm
def main() -> None:
    args = parse()
    world, rank, local = dist_env()
    from knng_gpu_b200 import synthetic as syn

    cfg = syn.CONFIGS[args.config]
    n = args.n or cfg.n
    if args.impl == "reference":
        run_reference_arm(args, cfg, n)
        return

    import torch
    import torch.distributed as dist

    import knng_gpu_b200 as kg
    from knng_gpu_b200.distributed import make_builder

    f = describe(cfg)
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    d, k = cfg.d, cfg.k
    builder = make_builder(n, d, k, cfg.metric, ring=(args.config == 5 and world > 1))
    lo, hi = builder.slice_bounds
    x_local_host = torch.from_numpy(syn.generate_config_rows(cfg, lo, hi - lo)).pin_memory()
    x_local = x_local_host.to(dev)
    stream = torch.cuda.current_stream()
    # Inputs smaller than L2 (126 MB) are flushed from it between steps.
    flush = None if n * d * 4 > (256 << 20) else torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-resident steps
    tc_ms, knn_ms = [], []
    step_ms_list = []
    with ClockSampler(local) as clk:
        for _ in range(args.warmup):
            builder.build(x_local)
        barrier()
        if flush is None:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
            for _ in range(args.steps):
                out = builder.build(x_local)
                tc_ms.append(builder.last_stats.get("tc_ms", 0.0))
                knn_ms.append(builder.last_stats.get("knn_ms", 0.0))
            ev1.record(stream)
            barrier()
            step_ms = ev0.elapsed_time(ev1) / args.steps
        else:
            for _ in range(args.steps):
                flush.fill_(1)
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ev0.record(stream)
                out = builder.build(x_local)
                ev1.record(stream)
                torch.cuda.synchronize()
                step_ms_list.append(ev0.elapsed_time(ev1))
                tc_ms.append(builder.last_stats.get("tc_ms", 0.0))
                knn_ms.append(builder.last_stats.get("knn_ms", 0.0))
            barrier()
            step_ms = float(np.mean(step_ms_list))
    t = torch.tensor([step_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms = float(t.item())
    ops = 2.0 * n * n * d
    value = ops / (step_ms * 1e-3) / 1e12
    launches_per_step = int(builder.last_stats.get("kernel_launches", 0))

    # ---- roofline of the dominant kernel on this rank's shard
    kms = float(np.mean(tc_ms))
    shard_ops = 2.0 * builder.shard.count * n * d
    achieved = shard_ops / (kms * 1e-3) / 1e12 if kms > 0 else None
    roofline = {"bound": "tensor", "achieved": achieved, "peak": f["peak"], "unit": "TOP/s",
                "frac": (achieved / f["peak"]) if achieved else None,
                "traffic": traffic_for(f["kernel"], cfg.name, builder.shard.count / n),
                "kernel": f["kernel"], "kernel_ms": kms, "peak_basis": f["peak_basis"],
                "note": "achieved = algorithmic 2*q*n*d ops of this rank's query shard / the kernel's CUDA-event time"}

    # ---- end to end through the public API (host buffers every step)
    e2e = None
    if not args.no_e2e:
        e2e = builder.time_e2e(x_local_host, args.steps, max(1, args.warmup // 2))
        if e2e is not None:
            e2e["value"] = ops / e2e.pop("seconds_per_build") / 1e12
            e2e["unit"] = UNIT

    # ---- parity against the reference's own loop (+ the CPU baseline)
    parity, cpu = None, None
    if rank == 0 and not args.no_parity:
        lib = ref_lib()
        if lib is None:
            parity = {"unavailable": "oracle/_ref/libknng_ref.so was not built"}
        else:
            g_ids, g_d = out
            x_full = syn.generate_config(cfg, n)
            rows = max(args.parity_rows, CPU_SAMPLE.get(args.config, 0)) if world == 1 else args.parity_rows
            q = syn.sample_ids(cfg.seed ^ PARITY_SEED, n, min(rows, n))
            threads = os.cpu_count() or 1
            r_ids, r_d, secs = ref_subset(lib, x_full, k, cfg.metric, q, threads)
            qi = torch.from_numpy(q.astype(np.int64)).to(g_ids.device)
            gi = g_ids.index_select(0, qi).cpu().numpy().view(np.uint32)
            gd = g_d.index_select(0, qi).cpu().numpy()
            parity = {"rows_checked": int(len(q)), "ids_equal": bool(np.array_equal(gi, r_ids)),
                      "dists_bitequal": bool(np.array_equal(gd.view(np.uint32), r_d.view(np.uint32))),
                      "checker": "reference brute-force loop (oracle/_ref ref_subset_knn), seeded rows",
                      "cpu_seconds": secs}
            if not f["integer"]:
                rel = np.abs(gd - r_d) / np.maximum(np.abs(r_d), 1e-30)
                parity["max_rel_dist_err"] = float(rel.max())
            if world == 1:
                rate = 2.0 * len(q) * n * d / secs / 1e12
                cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "reference",
                       "sample": (f"the reference's canonical loop (oracle/_ref ref_subset_knn) for {len(q)} seeded "
                                  f"query rows against all {n} rows on {threads} threads, {secs:.1f} s; "
                                  f"full build = time x n/{len(q)} = {secs * n / len(q):.0f} s"),
                       "full_build_seconds_extrapolated": secs * n / len(q)}
            del x_full

    if rank == 0:
        line = {
            "metric": METRIC_NAME, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "build_seconds": step_ms / 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": f["dtype"],
            "data": f["data"],
            "config": {"workload": cfg.name, "n": n, "d": d, "k": k, "metric": f["metric_name"],
                       "parallelism": builder.describe(),
                       "l2": ("inputs larger than L2" if flush is None else "L2 flushed between steps")},
            "roofline": roofline, "e2e": e2e, "cpu_baseline": cpu, "parity": parity, "clocks": clk.summary(),
            "gpu_launches": launches_per_step * args.steps,
            "path": builder.last_stats.get("path"), "fallback_rows": builder.last_stats.get("fallback_rows"),
            "phase_ms_rank0": builder.last_phase_ms(),
        }
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
