"""bench.py reports, for every configuration of BASELINE.json, the metric,
dtype, tensor-core kernel and peak that the library actually uses (no GPU
needed: only the description is checked)."""
from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("cfg_id,metric,dtype,kernel", [
    (1, "L2Squared", "u8", "knn_tc_kernel<ElemU8>"),
    (2, "L2Squared", "f32", "knn_tc_kernel<ElemBf16x3>"),
    (3, "L2Squared", "u8", "knn_tc_kernel<ElemU8>"),
    (4, "L2Squared", "f32", "knn_tc_kernel<ElemBf16x3>"),
    (5, "NegativeInnerProduct", "u8", "knn_pair_kernel"),
])
def test_describe_matches_the_configuration(cfg_id, metric, dtype, kernel):
    from knng_gpu_b200 import synthetic as syn

    f = _bench().describe(syn.CONFIGS[cfg_id])
    assert f["metric_name"] == metric
    assert f["dtype"] == dtype
    assert f["kernel"] == kernel
    # int8 peak is twice the bf16 figure; the fp32 path's is a third of it
    ratio = 6.0 if dtype == "u8" else 1.0
    f_other = _bench().describe(syn.CONFIGS[2 if dtype == "u8" else 3])
    assert f["peak"] == pytest.approx(f_other["peak"] * (ratio if dtype == "u8" else 1 / 6.0))
