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


def _driver():
    lib = ctypes.CDLL("libcuda.so.1")
    c = ctypes
    for name, args in [("cuInit", [c.c_uint]), ("cuDeviceGet", [c.c_void_p, c.c_int]),
                       ("cuCtxCreate_v2", [c.c_void_p, c.c_uint, c.c_int]), ("cuCtxDestroy_v2", [c.c_void_p]),
                       ("cuCtxPushCurrent_v2", [c.c_void_p]), ("cuCtxPopCurrent_v2", [c.c_void_p]),
                       ("cuCtxSynchronize", []), ("cuMemAlloc_v2", [c.c_void_p, c.c_size_t]),
                       ("cuMemFree_v2", [c.c_uint64]), ("cuMemcpyHtoD_v2", [c.c_uint64, c.c_void_p, c.c_size_t]),
                       ("cuMemcpyDtoH_v2", [c.c_void_p, c.c_uint64, c.c_size_t])]:
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = c.c_int
    return lib


@pytest.mark.gpu
def test_noalloc_in_a_second_context_then_the_primary_again(cuda_ok):
    """A host that makes its own (non-primary) context current: the array's
    address is resolved in that context, and afterwards in the primary one
    again. Every buffer of the second context is allocated in it through the
    driver API."""
    import torch

    n, d, k, metric = 2000, 128, 10, 0
    x = syn.generate(syn.KIND_UNIFORM_INT, 11, n, d)
    dev = torch.device("cuda", 0)
    pitch = api.padded_dim(d)
    packed = torch.empty((n, pitch), dtype=torch.uint8, device=dev)
    norms = torch.empty(n, dtype=torch.int32, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    api.pack_u8(torch.from_numpy(x).to(dev), packed, norms, flag)
    ref_ids = torch.empty((n, k), dtype=torch.int32, device=dev)
    ref_d = torch.empty((n, k), dtype=torch.float32, device=dev)
    scratch = torch.empty(api.knn_scratch_bytes(n, k), dtype=torch.uint8, device=dev)
    api.knn_u8(packed, norms, n, d, 0, n, k, metric, ref_ids, ref_d, scratch)
    torch.cuda.synchronize()
    h_packed = packed.cpu().numpy()
    h_norms = norms.cpu().numpy()

    cu = _driver()
    assert cu.cuInit(0) == 0
    cudev = ctypes.c_int()
    assert cu.cuDeviceGet(ctypes.byref(cudev), torch.cuda.current_device()) == 0
    ctx = ctypes.c_void_p()
    assert cu.cuCtxCreate_v2(ctypes.byref(ctx), 0, cudev.value) == 0  # now current
    bufs = []
    try:
        def alloc(nbytes):
            p = ctypes.c_uint64()
            assert cu.cuMemAlloc_v2(ctypes.byref(p), nbytes) == 0
            bufs.append(p.value)
            return p.value

        d_packed, d_norms = alloc(h_packed.nbytes), alloc(h_norms.nbytes)
        d_ids, d_dists = alloc(n * k * 4), alloc(n * k * 4)
        assert cu.cuMemcpyHtoD_v2(d_packed, h_packed.ctypes.data, h_packed.nbytes) == 0
        assert cu.cuMemcpyHtoD_v2(d_norms, h_norms.ctypes.data, h_norms.nbytes) == 0
        st = _native.gpu_lib().knng_gpu_knn_u8_noalloc(d_packed, d_norms, n, d, 0, n, k, metric, d_ids, d_dists,
                                                         None, None)
        api.check(st)
        assert cu.cuCtxSynchronize() == 0
        ids = np.empty((n, k), np.int32)
        dists = np.empty((n, k), np.float32)
        assert cu.cuMemcpyDtoH_v2(ids.ctypes.data, d_ids, ids.nbytes) == 0
        assert cu.cuMemcpyDtoH_v2(dists.ctypes.data, d_dists, dists.nbytes) == 0
    finally:
        for p in bufs:
            cu.cuMemFree_v2(p)
        popped = ctypes.c_void_p()
        cu.cuCtxPopCurrent_v2(ctypes.byref(popped))
        cu.cuCtxDestroy_v2(ctx)
    assert np.array_equal(ids, ref_ids.cpu().numpy())
    assert np.array_equal(dists.view(np.int32), ref_d.cpu().numpy().view(np.int32))

    # The primary context again (torch's): same results.
    ids2 = torch.full((n, k), -1, dtype=torch.int32, device=dev)
    dists2 = torch.full((n, k), -1.0, dtype=torch.float32, device=dev)
    _noalloc(packed, norms, n, d, 0, n, k, metric, ids2, dists2, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(ids2, ref_ids) and torch.equal(dists2.view(torch.int32), ref_d.view(torch.int32))
