"""Cross-set KNN (query rows against a separate base, global ids) and GPU
recall@k -- the batched query != base search and the recall of the
reference's bench harness (src/bench/recall.cpp:52-96), on the GPU.

Cross-set results are compared bit for bit with the oracle's cross-set loop
(the reference's brute-force loop body with global ids and self exclusion by
id, as src/dist/brute_force_mpi.cpp:76-82 does); recall with the reference's
own recall_at_k compiled into oracle/_ref."""
from __future__ import annotations

import numpy as np
import pytest

from refs import oracle_knn_sets, reference

from knng_gpu_b200 import api
from knng_gpu_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("metric,kind,d,k", [(0, syn.KIND_GAUSSIAN_MIXTURE, 128, 32), (1, syn.KIND_UNIFORM_PM1, 96, 10),
                                             (0, syn.KIND_UNIT_ROWS, 960, 100)])
def test_f32_cross_set_against_oracle(cuda_ok, metric, kind, d, k):
    import torch

    b = syn.generate(kind, 5, 3000, d, components=20, sigma=0.1)
    q = syn.generate(kind, 6, 700, d, components=20, sigma=0.1)
    dev = torch.device("cuda", 0)
    qt, bt = torch.from_numpy(q).to(dev), torch.from_numpy(b).to(dev)
    ids = torch.empty((q.shape[0], k), dtype=torch.int32, device=dev)
    dists = torch.empty((q.shape[0], k), dtype=torch.float32, device=dev)
    st = api.knn_f32_sets(qt, 1_000_000, bt, 5000, k, metric, False, ids, dists)
    oi, od = oracle_knn_sets(q, 1_000_000, b, 5000, k, metric, False)
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), oi)
    assert np.array_equal(dists.cpu().numpy().view(np.uint32), od.view(np.uint32))
    assert st["f32_err_ratio"] < 1.0


def test_f32_sets_with_self_exclusion_equal_self_graph_rows(cuda_ok):
    import torch

    x = syn.generate(syn.KIND_UNIFORM_PM1, 9, 2500, 64)
    dev = torch.device("cuda", 0)
    xt = torch.from_numpy(x).to(dev)
    q0, nq, k = 300, 400, 12
    ids = torch.empty((nq, k), dtype=torch.int32, device=dev)
    dists = torch.empty((nq, k), dtype=torch.float32, device=dev)
    api.knn_f32_sets(xt[q0:q0 + nq].contiguous(), q0, xt, 0, k, 0, True, ids, dists)
    oi, od = oracle_knn_sets(x[q0:q0 + nq], q0, x, 0, k, 0, True)
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), oi)
    assert np.array_equal(dists.cpu().numpy(), od)


@pytest.mark.parametrize("metric", [0, 1])
def test_u8_cross_set_against_oracle(cuda_ok, metric):
    import torch

    d, k = 200, 16
    b = syn.generate(syn.KIND_UNIFORM_INT, 15, 5000, d)
    q = syn.generate(syn.KIND_UNIFORM_INT, 16, 900, d)
    dev = torch.device("cuda", 0)
    pitch = api.padded_dim(d)
    pk = {}
    for name, arr in (("q", q), ("b", b)):
        t = torch.from_numpy(arr).to(dev)
        packed = torch.empty((arr.shape[0], pitch), dtype=torch.uint8, device=dev)
        norms = torch.empty(arr.shape[0], dtype=torch.int32, device=dev)
        flag = torch.zeros(1, dtype=torch.int32, device=dev)
        api.pack_u8(t, packed, norms, flag)
        assert int(flag.item()) == 0
        pk[name] = (packed, norms)
    ids = torch.empty((q.shape[0], k), dtype=torch.int32, device=dev)
    dists = torch.empty((q.shape[0], k), dtype=torch.float32, device=dev)
    scratch = torch.empty(api.knn_scratch_bytes(q.shape[0], k), dtype=torch.uint8, device=dev)
    api.knn_u8_sets(pk["q"][0], pk["q"][1], 20_000, pk["b"][0], pk["b"][1], 7, d, k, metric, False, ids, dists, scratch)
    oi, od = oracle_knn_sets(q, 20_000, b, 7, k, metric, False)
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), oi)
    assert np.array_equal(dists.cpu().numpy(), od)
    # Base key offsets that are not 16-byte aligned are refused, not misread.
    with pytest.raises(api.InvalidArgument):
        api.knn_u8_sets(pk["q"][0], pk["q"][1], 20_000, pk["b"][0][1:], pk["b"][1][1:], 8, d, k, metric, False, ids,
                        dists, scratch)


def test_gpu_recall_matches_reference(cuda_ok):
    import torch

    lib = reference()
    if lib is None:
        pytest.skip("oracle/_ref not built")
    rng = np.random.RandomState(3)
    n, k = 2000, 10
    truth = np.stack([rng.permutation(500)[:k] for _ in range(n)]).astype(np.uint32)
    approx = truth.copy()
    # wrong ids, repeated ids (count once) and a fully correct row
    approx[::3, ::2] = rng.randint(0, 500, size=approx[::3, ::2].shape)
    approx[1::5, 1:] = approx[1::5, :1]
    ref = lib.ref_recall_at_k(approx.ctypes.data, truth.ctypes.data, n, k)
    dev = torch.device("cuda", 0)
    got = api.recall_at_k(torch.from_numpy(approx.view(np.int32)).to(dev), torch.from_numpy(truth.view(np.int32)).to(dev))
    assert abs(got - ref) < 1e-12
    assert api.recall_at_k(torch.from_numpy(truth.view(np.int32)).to(dev),
                           torch.from_numpy(truth.view(np.int32)).to(dev)) == 1.0
