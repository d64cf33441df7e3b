"""File formats around the path, against the reference's own code compiled
here (oracle/_ref): vecs readers, the .knng v1 writer (byte-compared with
the reference's build_knng), the ground-truth cache and recall_at_k."""
from __future__ import annotations

import ctypes
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from knng_gpu_b200 import io as kio
from knng_gpu_b200 import synthetic as syn
from refs import REF_SO, ROOT, oracle_knn, reference

REF_CLI = ROOT / "oracle" / "_ref" / "build_knng"
CLI = ROOT / "knng_gpu_b200" / "bin" / "build_knng_gpu"


def _ref_load(path, kind):
    lib = reference()
    lib.ref_load_vecs.restype = ctypes.c_int
    lib.ref_load_vecs.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    n = ctypes.c_uint64()
    d = ctypes.c_uint64()
    rc = lib.ref_load_vecs(str(path).encode(), kind, None, ctypes.byref(n), ctypes.byref(d))
    if rc:
        return None, lib.ref_last_error().decode()
    dt = [np.float32, np.int32, np.uint8][kind]
    out = np.empty((n.value, d.value), dt)
    lib.ref_load_vecs(str(path).encode(), kind, out.ctypes.data, ctypes.byref(n), ctypes.byref(d))
    return out, ""


needs_ref = pytest.mark.skipif(not REF_SO.exists(), reason="reference library not built")


@needs_ref
@pytest.mark.parametrize("suffix,kind", [(".fvecs", 0), (".ivecs", 1), (".bvecs", 2)])
def test_vecs_roundtrip_matches_reference_loader(tmp_path, suffix, kind):
    rng = np.random.default_rng(kind)
    x = (rng.integers(0, 255, (37, 19)) if kind else rng.standard_normal((37, 19))).astype(kio._DTYPES[suffix])
    p = tmp_path / f"x{suffix}"
    kio.write_vecs(p, x)
    ref, err = _ref_load(p, kind)
    assert err == ""
    got = kio.read_vecs(p)
    assert np.array_equal(got, ref) and np.array_equal(got, x)


@needs_ref
def test_vecs_errors_match_reference(tmp_path):
    x = np.ones((4, 3), np.float32)
    p = tmp_path / "bad.fvecs"
    kio.write_vecs(p, x)
    raw = bytearray(p.read_bytes())
    raw[16] = 7  # second record's dim prefix
    p.write_bytes(bytes(raw))
    _, err = _ref_load(p, 0)
    with pytest.raises(RuntimeError) as e:
        kio.read_vecs(p)
    assert "record 1 has dim 7" in err and "record 1 has dim 7" in str(e.value)
    p.write_bytes(bytes(raw[:-2]))
    _, err = _ref_load(p, 0)
    with pytest.raises(RuntimeError) as e:
        kio.read_vecs(p)
    assert "is not a multiple of record size" in err and "is not a multiple of record size" in str(e.value)


@needs_ref
@pytest.mark.parametrize("metric", [0, 1])
def test_knng_writer_bytes_match_reference_cli(tmp_path, metric):
    x = syn.generate(syn.KIND_UNIFORM_INT, 3, 300, 24)
    p = tmp_path / "d.fvecs"
    kio.write_vecs(p, x)
    out = tmp_path / "ref.knng"
    r = subprocess.run([str(REF_CLI), "--dataset", str(p), "--k", "7", "--metric",
                        ["l2", "inner_product"][metric], "--output", str(out)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    ids, dists = oracle_knn(x, 7, metric)
    mine = tmp_path / "mine.knng"
    kio.write_knng(mine, ids, dists, metric, algorithm=kio.ALGORITHM_BRUTE_FORCE)
    assert mine.read_bytes() == out.read_bytes()
    gi, gd, m, a = kio.read_knng(out)
    assert np.array_equal(gi, ids) and np.array_equal(gd, dists) and m == metric and a == 0


@needs_ref
def test_ground_truth_cache_matches_reference(tmp_path):
    x = syn.generate(syn.KIND_UNIFORM_PM1, 5, 200, 16)
    ids, dists = oracle_knn(x, 6, 0)
    h = kio.dataset_hash(x)
    lib = reference()
    assert h == lib.ref_dataset_hash(x.ctypes.data, 200, 16)
    lib.ref_save_ground_truth.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64,
                                          ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int]
    ref_path = tmp_path / "ref.gt"
    assert lib.ref_save_ground_truth(str(ref_path).encode(), ids.ctypes.data, dists.ctypes.data, 200, 6, h, 0) == 0
    mine = tmp_path / "mine.gt"
    kio.save_ground_truth(mine, ids, dists, h, 0)
    assert mine.read_bytes() == ref_path.read_bytes()
    got = kio.load_ground_truth(mine, x, 6, 0)
    assert got is not None and np.array_equal(got[0], ids)
    assert kio.load_ground_truth(mine, x, 5, 0) is None  # wrong k
    assert kio.load_ground_truth(mine, x, 6, 1) is None  # wrong metric
    y = x.copy()
    y[0, 0] += 1
    assert kio.load_ground_truth(mine, y, 6, 0) is None  # dataset changed
    mine.write_bytes(mine.read_bytes() + b"\0")
    assert kio.load_ground_truth(mine, x, 6, 0) is None  # trailing garbage


@needs_ref
def test_recall_matches_reference():
    rng = np.random.default_rng(1)
    truth = np.stack([rng.permutation(50)[:8] for _ in range(40)]).astype(np.uint32)
    approx = truth.copy()
    approx[::3, 2] = approx[::3, 1]  # duplicates count once
    approx[1::4, 5] = 49
    ref = reference().ref_recall_at_k(approx.ctypes.data, truth.ctypes.data, 40, 8)
    assert abs(kio.recall_at_k(approx, truth) - ref) < 1e-12


@pytest.mark.gpu
def test_gpu_cli_output_equals_reference_cli(cuda_ok, tmp_path):
    """build_knng_gpu writes the reference build_knng's file byte for byte,
    apart from the algorithm id field (1 = brute_force_gpu)."""
    if not REF_CLI.exists():
        pytest.skip("reference CLI not built")
    for suffix, kind, metric, k in [(".fvecs", syn.KIND_UNIFORM_INT, "l2", 10),
                                     (".fvecs", syn.KIND_UNIFORM_PM1, "l2", 5),
                                     (".fvecs", syn.KIND_SPARSE_INT, "inner_product", 8)]:
        x = syn.generate(kind, 21, 900, 48, p_zero=0.6)
        p = tmp_path / f"d{suffix}"
        kio.write_vecs(p, x)
        a, b = tmp_path / "ref.knng", tmp_path / "gpu.knng"
        r1 = subprocess.run([str(REF_CLI), "--dataset", str(p), "--k", str(k), "--metric", metric, "--output",
                             str(a)], capture_output=True, text=True)
        r2 = subprocess.run([str(CLI), "--dataset", str(p), "--k", str(k), "--metric", metric, "--output", str(b),
                             "--ground-truth", str(tmp_path / "g.gt")], capture_output=True, text=True)
        assert r1.returncode == 0 and r2.returncode == 0, r2.stderr
        ra, rb = bytearray(a.read_bytes()), bytearray(b.read_bytes())
        assert rb[24:28] == (1).to_bytes(4, "little")
        rb[24:28] = ra[24:28]
        assert ra == rb
        assert kio.load_ground_truth(tmp_path / "g.gt", x, k, 0 if metric == "l2" else 1) is not None


@pytest.mark.gpu
def test_gpu_cli_reads_bvecs(cuda_ok, tmp_path):
    x = syn.generate(syn.KIND_UNIFORM_INT, 8, 700, 40)
    p = tmp_path / "d.bvecs"
    kio.write_vecs(p, x.astype(np.uint8))
    out = tmp_path / "o.knng"
    r = subprocess.run([str(CLI), "--dataset", str(p), "--k", "6", "--output", str(out)], capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stderr
    ids, dists, m, a = kio.read_knng(out)
    oi, od = oracle_knn(x, 6, 0)
    assert np.array_equal(ids, oi) and np.array_equal(dists, od) and a == 1


def test_cli_rejects_bad_flags():
    if not CLI.exists():
        pytest.skip("CLI not built")
    r = subprocess.run([str(CLI), "--dataset", "x.fvecs", "--k", "3", "--metric", "cosine"], capture_output=True,
                       text=True)
    assert r.returncode == 2 and "--metric must be" in r.stderr
    r = subprocess.run([str(CLI), "--k", "3"], capture_output=True, text=True)
    assert r.returncode == 2 and "missing required flag --dataset" in r.stderr


def test_python_cli_arguments_and_relaunch():
    from knng_gpu_b200.cli.__main__ import CliError, main, parse_args, relaunch_command

    a = parse_args(["--dataset", "d.fvecs", "--k", "4"])
    assert a.output == "d.fvecs.knng" and a.metric == "l2" and a.gpus == 1 and a.algorithm == "brute_force_gpu"
    for bad in (["--dataset", "d.fvecs", "--k", "0"], ["--dataset", "d.fvecs", "--k", "3", "--metric", "cosine"],
                ["--dataset", "d.fvecs", "--k", "3", "--gpus", "0"], ["--dataset", "d.fvecs", "--k", "x"],
                ["--k", "3"]):
        with pytest.raises(CliError):
            parse_args(bad)
    assert main(["--dataset", "d.fvecs", "--k", "3", "--metric", "cosine"]) == 2
    cmd = relaunch_command(["--dataset", "d.fvecs", "--k", "3", "--gpus", "2"], 2, 29555)
    assert cmd[1:3] == ["-m", "torch.distributed.run"] and "--nproc-per-node=2" in cmd
    assert "--master-addr=127.0.0.1" in cmd and cmd[-6:] == ["--dataset", "d.fvecs", "--k", "3", "--gpus", "2"]


@pytest.mark.gpu
def test_python_cli_single_gpu(cuda_ok, tmp_path):
    x = syn.generate(syn.KIND_UNIFORM_INT, 9, 600, 36)
    for suffix, data in ((".bvecs", x.astype(np.uint8)), (".fvecs", x)):
        p = tmp_path / f"d{suffix}"
        kio.write_vecs(p, data)
        out, gt = tmp_path / f"o{suffix}.knng", tmp_path / f"g{suffix}.gt"
        r = subprocess.run([sys.executable, "-m", "knng_gpu_b200.cli", "--dataset", str(p), "--k", "7", "--output",
                            str(out), "--ground-truth", str(gt)], capture_output=True, text=True, cwd=ROOT)
        assert r.returncode == 0, r.stderr
        ids, dists, m, a = kio.read_knng(out)
        oi, od = oracle_knn(x, 7, 0)
        assert np.array_equal(ids, oi) and np.array_equal(dists, od) and a == 1 and m == 0
        assert kio.load_ground_truth(gt, x, 7, 0) is not None
