"""The outside bound of the ring build, checked on the host.

From the second block on, the ring build (sharded.cuh, ring_bound_kernel)
lets a block's search admit only keys at or below the running k-th key of
the blocks already searched, so a block may return fewer than k entries,
padded with (0xFFFFFFFF, +inf), before the (distance, id) merge. This test
restates that rule with exact integer arithmetic on integer rows (ties
everywhere on {0, 1} rows) and checks that it yields the oracle's graph --
ids and fp32 distance bits -- for both metrics and for ring sizes 2-8 with
the blocks of compute_shard (include/knng/dist/sharded_dataset.hpp:145-155).
"""
from __future__ import annotations

import numpy as np
import pytest

from refs import oracle_knn

from knng_gpu_b200.distributed import compute_shard

SENT_ID = np.uint32(0xFFFFFFFF)


def _dists(x, q, metric):
    xi = x.astype(np.int64)
    if metric == 0:
        diff = xi[None, :, :] - xi[q][:, None, :]
        return (diff * diff).sum(-1)
    return -(xi[q] @ xi.T)


def _topk(d_row, ids, k):
    """k best (distance, id) of one row; fewer if fewer are given, padded."""
    order = np.lexsort((ids, d_row))[:k]
    out_d = np.full(k, np.inf)
    out_i = np.full(k, SENT_ID, dtype=np.uint32)
    out_d[: order.size] = d_row[order]
    out_i[: order.size] = ids[order]
    return out_i, out_d


def _merge(ai, ad, bi, bd, k):
    ids = np.concatenate([ai, bi])
    ds = np.concatenate([ad, bd])
    order = np.lexsort((ids, ds))[:k]
    return ids[order], ds[order]


@pytest.mark.parametrize("metric", [0, 1])
@pytest.mark.parametrize("values", ["bits", "bytes"])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_bounded_ring_blocks_give_the_oracle_graph(metric, values, world):
    rng = np.random.default_rng(100 * metric + world + (7 if values == "bits" else 0))
    n, d, k = 403, 12, 10
    hi = 2 if values == "bits" else 256
    x = rng.integers(0, hi, size=(n, d)).astype(np.float32)
    q = np.arange(n)
    full = _dists(x, q, metric)  # exact integers, all below 2^24
    assert np.abs(full).max() < (1 << 24)
    blocks = [compute_shard(n, world, b) for b in range(world)]
    oi, od = oracle_knn(x, k, metric)
    for r in range(world):
        rows = np.arange(blocks[r].start, blocks[r].start + blocks[r].count)
        for qi in rows:
            run_i = run_d = None
            for step in range(world):
                b = blocks[(r - step) % world]
                ids = np.arange(b.start, b.start + b.count, dtype=np.uint32)
                dr = full[qi, ids.astype(np.int64)].astype(np.float64)
                keep = ids != qi  # self excluded by id
                if step > 0:
                    # the running k-th distance is exact: admit keys <= it
                    keep &= dr <= run_d[k - 1]
                bi, bd = _topk(dr[keep], ids[keep], k)
                run_i, run_d = (bi, bd) if step == 0 else _merge(run_i, run_d, bi, bd, k)
            assert np.array_equal(run_i, oi[qi]), (r, qi)
            assert np.array_equal(run_d.astype(np.float32).view(np.uint32), od[qi].view(np.uint32))
