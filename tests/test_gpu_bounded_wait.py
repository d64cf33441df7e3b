"""Failure path of the bounded device-side waits, without a GPU fault.

Every wait in the kernels gives up after a bounded number of clock cycles,
sets an error word, raises an abort flag for the other roles of its CTA pair,
frees its TMEM and returns; the host maps the error word to
KNNG_GPU_TIMEOUT (the reference's convention of returning errors instead of
aborting, docs/STYLE.md:118-128). knng_gpu_selftest_bounded_wait runs a small
build with a short wait bound while the producer withholds one arrival on
purpose, so a wait must run out. Afterwards a normal build on the same device
must still match the oracle: the context survived.
"""
from __future__ import annotations

import numpy as np
import pytest

import knng_gpu_b200 as kg
from knng_gpu_b200 import _native
from knng_gpu_b200 import synthetic as syn
from refs import oracle_knn


@pytest.mark.gpu
def test_withheld_arrival_times_out_and_context_stays_usable(cuda_ok):
    lib = _native.gpu_lib()
    st = lib.knng_gpu_selftest_bounded_wait(20_000_000)  # ~10 ms of SM clock
    assert st == 3, (st, lib.knng_gpu_last_error())
    assert b"bounded device wait" in lib.knng_gpu_last_error()
    x = syn.generate(syn.KIND_UNIFORM_INT, 11, 1500, 128)
    g = kg.brute_force_knn(x, 10, kg.L2Squared())
    oi, od = oracle_knn(x, 10, 0)
    assert np.array_equal(g.neighbors.reshape(-1, 10), oi)
    assert np.array_equal(g.distances.reshape(-1, 10), od)
