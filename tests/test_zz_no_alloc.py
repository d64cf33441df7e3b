"""knng_gpu_knn_u8_noalloc: the allocation-free variant of knng_gpu_knn_u8.

Some callers cannot hand the library any scratch buffer -- they run inside a
host process that owns all device memory through its own pool, or they are
plugins that only receive device pointers and are not allowed to call
cudaMalloc. This variant keeps its scratch in a fixed device array inside the
library. These tests call it through the C ABI and require its output to be
bit-identical (the tolerance every parity test here uses) to the regular
entry point's, on two calls in a row, so that stale contents left in the
shared array by the first call cannot leak into the second.

This file is named so that pytest collects it last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from knng_gpu_b200 import _native, api
from knng_gpu_b200 import synthetic as syn

MAX_Q = 1 << 20


def _noalloc(packed, norms, n, d, q_begin, q_count, k, metric, ids, dists, stream):
    stats = _native.KnngGpuStats()
    st = _native.gpu_lib().knng_gpu_knn_u8_noalloc(
        packed.data_ptr(), norms.data_ptr(), n, d, q_begin, q_count, k, metric, ids.data_ptr(),
        dists.data_ptr(), stream, ctypes.byref(stats))
    api.check(st)
    return stats


def test_rejects_more_queries_than_the_array_holds():
    lib = _native.gpu_lib()
    st = lib.knng_gpu_knn_u8_noalloc(None, None, MAX_Q + 10, 128, 0, MAX_Q + 1, 10, 0, None, None, None, None)
    assert st == 1
    assert b"at most" in lib.knng_gpu_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("metric,k,n,d,seed", [(0, 10, 3000, 128, 5), (1, 20, 2500, 300, 6), (0, 5, 500, 1024, 7)])
def test_noalloc_matches_regular_entry_twice(cuda_ok, metric, k, n, d, seed):
    import torch

    if d == 1024:  # {0,255} rows: every row goes through the fallback list
        x = (syn.generate(syn.KIND_UNIFORM_INT, seed, n, d) >= 128).astype(np.float32) * 255.0
    else:
        x = syn.generate(syn.KIND_UNIFORM_INT, seed, n, d)
    dev = torch.device("cuda", 0)
    xt = torch.from_numpy(x).to(dev)
    pitch = api.padded_dim(d)
    packed = torch.empty((n, pitch), dtype=torch.uint8, device=dev)
    norms = torch.empty(n, dtype=torch.int32, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    api.pack_u8(xt, packed, norms, flag)
    assert int(flag.item()) == 0
    stream = torch.cuda.current_stream().cuda_stream

    q_begin, q_count = 7, n - 19
    ref_ids = torch.empty((q_count, k), dtype=torch.int32, device=dev)
    ref_d = torch.empty((q_count, k), dtype=torch.float32, device=dev)
    scratch = torch.empty(api.knn_scratch_bytes(q_count, k), dtype=torch.uint8, device=dev)
    ref_stats = api.knn_u8(packed, norms, n, d, q_begin, q_count, k, metric, ref_ids, ref_d, scratch)

    for call in range(2):
        ids = torch.full((q_count, k), -1, dtype=torch.int32, device=dev)
        dists = torch.full((q_count, k), -1.0, dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info(dev)[0]
        stats = _noalloc(packed, norms, n, d, q_begin, q_count, k, metric, ids, dists, stream)
        torch.cuda.synchronize()
        if call == 1:
            # The point of the entry point: once the library is loaded and the
            # array's address resolved, a call takes no device memory.
            assert torch.cuda.mem_get_info(dev)[0] == free_before
        assert torch.equal(ids, ref_ids)
        assert torch.equal(dists.view(torch.int32), ref_d.view(torch.int32))
        assert stats.fallback_rows == ref_stats["fallback_rows"]
