"""python -m knng_gpu_b200.cli -- build_knng with ``--gpus N``.

The flags, messages and output of the reference's ``build_knng``
(tools/build_knng.cpp:35-60, 196-244): ``--dataset PATH --k N [--metric
l2|inner_product] [--algorithm brute_force_gpu|brute_force] [--output PATH]
[--ground-truth PATH]``, plus ``--gpus N``. One GPU calls the C ABI directly
(``.bvecs`` bytes go to the u8 entry point without a float copy). With N > 1
this process drives GPUs 0..N-1 through knng_gpu_brute_force_multi (NCCL
inside the library). Started under torchrun instead (``relaunch_command``
gives that command line), every rank reads the dataset, packs and searches
its query shard with :class:`~knng_gpu_b200.distributed.ShardedBuilder`, and
rank 0 writes the ``.knng`` file (and the ground-truth cache).
"""
from __future__ import annotations

import argparse
import os
import socket
import subprocess
import sys

import numpy as np

USAGE_ERROR = 2


class CliError(ValueError):
    pass


class _Parser(argparse.ArgumentParser):
    def error(self, message):  # usage errors raise instead of exiting
        raise CliError(message)


def parse_args(argv: list[str]) -> argparse.Namespace:
    ap = _Parser(prog="python -m knng_gpu_b200.cli")
    ap.add_argument("--dataset", required=True, help="Path to a .fvecs or .bvecs dataset.")
    ap.add_argument("--k", required=True, help="Neighbors per point. Must satisfy 1 <= k <= n-1.")
    ap.add_argument("--metric", default="l2", help="l2 (default) | inner_product")
    ap.add_argument("--algorithm", default="brute_force_gpu",
                    help="brute_force_gpu (default) | brute_force (same graph, algorithm_id 0)")
    ap.add_argument("--output", default=None, help="Output .knng path (default: <dataset>.knng)")
    ap.add_argument("--ground-truth", default=None, help="Also write a ground-truth cache file")
    ap.add_argument("--gpus", default="1", help="GPUs of this node to use (default 1)")
    a = ap.parse_args(argv)
    try:
        a.k = int(a.k, 10)
        a.gpus = int(a.gpus, 10)
    except ValueError as e:
        raise CliError(f"bad integer value: {e}") from None
    if a.k <= 0:
        raise CliError("--k must be > 0")
    if a.gpus <= 0:
        raise CliError("--gpus must be > 0")
    if a.metric not in ("l2", "inner_product"):
        raise CliError(f"--metric must be 'l2' or 'inner_product', got '{a.metric}'")
    if a.algorithm not in ("brute_force_gpu", "brute_force"):
        raise CliError(f"--algorithm must be 'brute_force_gpu' or 'brute_force', got '{a.algorithm}'")
    if a.output is None:
        a.output = a.dataset + ".knng"
    return a


def relaunch_command(argv: list[str], gpus: int, port: int) -> list[str]:
    """The torch.distributed.run command line that runs this CLI on ``gpus``
    processes of one node."""
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
            "--master-addr=127.0.0.1", f"--master-port={port}", "-m", "knng_gpu_b200.cli", *argv]


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _log(msg: str) -> None:
    print(f"build_knng_gpu: {msg}", file=sys.stderr, flush=True)


def _write_outputs(a, x, ids, dists, metric: int) -> None:
    from knng_gpu_b200 import io as kio

    _log(f"writing {a.output}")
    alg = kio.ALGORITHM_BRUTE_FORCE if a.algorithm == "brute_force" else kio.ALGORITHM_BRUTE_FORCE_GPU
    kio.write_knng(a.output, ids, dists, metric, alg)
    if a.ground_truth:
        kio.save_ground_truth(a.ground_truth, ids, dists, kio.dataset_hash(x), metric)
        _log(f"wrote ground truth {a.ground_truth}")


def run_single(a) -> int:
    import knng_gpu_b200 as kg
    from knng_gpu_b200 import io as kio

    _log(f"loading {a.dataset}")
    x = kio.read_vecs(a.dataset)
    n, d = x.shape
    _log(f"loaded n={n} d={d}")
    metric = 0 if a.metric == "l2" else 1
    _log(f"building k={a.k} metric={a.metric} algorithm={a.algorithm}")
    if a.gpus > 1:
        # One process drives the GPUs (NCCL inside the library).
        g = kg.brute_force_knn_multi(np.asarray(x, np.float32), a.k, metric, num_gpus=a.gpus)
    elif x.dtype == np.uint8:
        g = kg.brute_force_knn_u8(x, a.k, metric)
    else:
        g = kg.brute_force_knn(x, a.k, metric)
    _write_outputs(a, x, g.neighbors.reshape(n, a.k), g.distances.reshape(n, a.k), metric)
    _log("done")
    return 0


def run_rank(a) -> int:
    import torch
    import torch.distributed as dist

    from knng_gpu_b200 import io as kio
    from knng_gpu_b200.distributed import ShardedBuilder

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    rank = dist.get_rank()
    try:
        if rank == 0:
            _log(f"loading {a.dataset} on {dist.get_world_size()} GPUs")
        x = kio.read_vecs(a.dataset)
        n, d = x.shape
        metric = 0 if a.metric == "l2" else 1
        if a.k > n - 1:
            raise CliError(f"knng::gpu::brute_force_knn: k ({a.k}) must be <= ds.n - 1 ({n - 1})")
        b = ShardedBuilder(n, d, a.k, metric)
        lo, hi = b.slice_bounds
        xs = torch.from_numpy(np.ascontiguousarray(x[lo:hi], np.float32)).cuda()
        ids, dists = b.build(xs)
        if rank == 0:
            _write_outputs(a, x, ids.cpu().numpy().view(np.uint32), dists.cpu().numpy(), metric)
            _log("done")
        dist.barrier()
    finally:
        dist.destroy_process_group()
    return 0


def main(argv: list[str] | None = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    try:
        a = parse_args(argv)
    except CliError as e:
        print(f"build_knng_gpu: {e}", file=sys.stderr)
        return USAGE_ERROR
    try:
        if "RANK" in os.environ and int(os.environ.get("WORLD_SIZE", "1")) > 1:
            return run_rank(a)
        return run_single(a)
    except Exception as e:  # the reference prints the message and exits 1
        print(f"build_knng_gpu: {e}", file=sys.stderr)
        return 1


if __name__ == "__main__":
    sys.exit(main())
