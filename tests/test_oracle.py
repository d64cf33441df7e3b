"""The CPU oracle, pinned against the reference's own known answers and
against golden vectors produced by the reference's compiled sources."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from cases import CASES
from refs import eight_points, oracle, oracle_knn

GOLD = Path(__file__).resolve().parent / "golden"


def test_xorshift_matches_reference_stream():
    g = np.load(GOLD / "xorshift.npz")
    lib = oracle()
    for i, s in enumerate(g["seeds"]):
        out = np.zeros(64, np.uint64)
        lib.oracle_xorshift64_stream(int(s), 64, out.ctypes.data)
        assert np.array_equal(out, g["u64"][i])
        st = np.array([s], np.uint64)
        f = [lib.oracle_next_float01(st.ctypes.data) for _ in range(64)]
        assert np.array_equal(np.array(f, np.float32), g["float01"][i])
        st = np.array([s], np.uint64)
        b = [lib.oracle_next_below(st.ctypes.data, 256) for _ in range(64)]
        assert np.array_equal(np.array(b, np.uint64), g["below256"][i])


def test_package_generator_matches_reference_stream():
    from knng_gpu_b200 import synthetic as syn

    g = np.load(GOLD / "xorshift.npz")
    for i, s in enumerate(g["seeds"]):
        x = syn.generate(syn.KIND_UNIFORM_INT, int(s), 1, 64)
        assert np.array_equal(x[0], g["below256"][i].astype(np.float32))
        y = syn.generate(syn.KIND_UNIFORM_PM1, int(s), 1, 64)
        assert np.array_equal(y[0], 2.0 * g["float01"][i] - 1.0)


def test_topk_matches_reference():
    g = np.load(GOLD / "topk.npz")
    lib = oracle()
    ids, dists = g["push_ids"], g["push_dists"]
    for k in (0, 1, 2, 5, 17, 200, 250):
        oi = np.zeros(max(k, 1), np.uint32)
        od = np.zeros(max(k, 1), np.float32)
        m = lib.oracle_topk_run(k, len(ids), ids.ctypes.data, dists.ctypes.data, oi.ctypes.data, od.ctypes.data)
        assert np.array_equal(oi[:m], g[f"ids_{k}"])
        assert np.array_equal(od[:m], g[f"dists_{k}"])


def test_topk_tie_break_known_answer():
    # tests/top_k_test.cpp:82-97: three candidates at 1.0, k=2 keeps ids 2 and 5.
    ids = np.array([7, 2, 5], np.uint32)
    dists = np.ones(3, np.float32)
    oi = np.zeros(2, np.uint32)
    od = np.zeros(2, np.float32)
    m = oracle().oracle_topk_run(2, 3, ids.ctypes.data, dists.ctypes.data, oi.ctypes.data, od.ctypes.data)
    assert m == 2 and list(oi) == [2, 5] and list(od) == [1.0, 1.0]


def test_squared_l2_hand_values():
    # tests/core_test.cpp:38-62 and :93
    lib = oracle()
    a = np.array([0, 0, 0], np.float32)
    b = np.array([3, 4, 0], np.float32)
    assert lib.oracle_squared_l2(a.ctypes.data, b.ctypes.data, 3) == 25.0
    assert lib.oracle_squared_l2(a.ctypes.data, b.ctypes.data, 0) == 0.0
    c = np.array([1, 2, 3], np.float32)
    e = np.array([4, 5, 6], np.float32)
    assert lib.oracle_negative_inner_product(c.ctypes.data, e.ctypes.data, 3) == -32.0


def test_eight_point_known_answers():
    # tests/brute_force_test.cpp:67-111 and :139-150
    x = eight_points()
    ids, dists = oracle_knn(x, 3)
    assert list(ids[0]) == [1, 2, 3] and list(dists[0]) == [1, 1, 2]
    assert list(ids[7]) == [5, 6, 4] and list(dists[7]) == [1, 1, 2]
    assert list(ids[4]) == [5, 6, 7] and list(dists[4]) == [1, 1, 2]
    ids1, _ = oracle_knn(x, 1)
    assert ids1[0, 0] == 1 and ids1[3, 0] == 1 and ids1[7, 0] == 5
    ids5, d5 = oracle_knn(x, 5)
    for q in range(8):
        assert q not in ids5[q]
        assert np.all(np.diff(d5[q]) >= 0)


def test_argument_errors():
    # tests/brute_force_test.cpp:166-189
    x = eight_points()
    for k in (0, 8):
        with pytest.raises(ValueError):
            oracle_knn(x, k)
    with pytest.raises(ValueError):
        oracle_knn(np.zeros((0, 0), np.float32), 1)


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_oracle_matches_reference_golden(case):
    g = np.load(GOLD / f"knn_{case.name}.npz")
    x = np.ascontiguousarray(case.make(), np.float32)
    assert oracle().oracle_dataset_hash(x.ctypes.data, x.shape[0], x.shape[1]) == int(g["data_hash"])
    ids, dists = oracle_knn(x, case.k, case.metric)
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(dists.view(np.uint32), g["dists"].view(np.uint32))


def test_subset_harness_equals_full_rows():
    case = next(c for c in CASES if c.name == "cfg1_u8_n2000_d128_k10_l2")
    g = np.load(GOLD / f"knn_{case.name}.npz")
    x = case.make()
    q = np.array([0, 17, 999, 1999], np.uint64)
    ids, dists = oracle_knn(x, case.k, 0, queries=q)
    assert np.array_equal(ids, g["ids"][q.astype(np.int64)])
    assert np.array_equal(dists, g["dists"][q.astype(np.int64)])


def test_recall_at_k():
    # src/bench/recall.cpp:79-96; duplicates in the approximate row count once.
    lib = oracle()
    truth = np.array([[1, 2, 3], [0, 2, 3]], np.uint32)
    approx = np.array([[1, 1, 9], [0, 2, 3]], np.uint32)
    assert abs(lib.oracle_recall_at_k(approx.ctypes.data, truth.ctypes.data, 2, 3) - 4 / 6) < 1e-12


def test_cross_set_oracle_equals_reference_subset_loop():
    """oracle_knn_sets with self exclusion equals the reference's own loop
    body run for the same query rows (ref_subset_knn)."""
    from refs import oracle_knn_sets, ref_subset_knn, reference

    if reference() is None:
        pytest.skip("oracle/_ref not built")
    from knng_gpu_b200 import synthetic as syn

    x = syn.generate(syn.KIND_GAUSSIAN_MIXTURE, 7, 900, 24, components=5, sigma=0.2)
    q = np.arange(100, 250, dtype=np.uint64)
    for metric in (0, 1):
        oi, od = oracle_knn_sets(x[100:250], 100, x, 0, 9, metric, True)
        ri, rd = ref_subset_knn(x, 9, metric, q)
        assert np.array_equal(oi, ri) and np.array_equal(od.view(np.uint32), rd.view(np.uint32))
