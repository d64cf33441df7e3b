"""Parity cases shared by the golden-fixture generator and the tests.

Each case is a small seeded dataset (regenerated at test time by the
package's generator and pinned by the reference's FNV-1a dataset hash), a k
and a metric. Together they cover the five benchmark shapes scaled down to
sizes the CPU oracle finishes in seconds, plus the edge cases the reference
tests (tiny n, k = n - 1, ragged d, ties, duplicates) and the paths of the GPU
library (u8 tensor-core path with both tile layouts, heap top-k, rows routed
to the exact kernel, the fp32 exact path).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import numpy as np

from knng_gpu_b200 import synthetic as syn

from refs import eight_points


@dataclass(frozen=True)
class Case:
    name: str
    make: Callable[[], np.ndarray]
    k: int
    metric: int  # 0 L2Squared, 1 NegativeInnerProduct


def _gen(kind, seed, n, d, **kw):
    return lambda: syn.generate(kind, seed, n, d, **kw)


def _bimodal(seed, n, d):
    # integers {0, 255}: distances and dots above 2^24 at d = 1024
    return lambda: (syn.generate(syn.KIND_UNIFORM_INT, seed, n, d) >= 128).astype(np.float32) * 255.0


def _binary(seed, n, d):
    # integers {0, 1}: massive distance ties and duplicate rows
    return lambda: (syn.generate(syn.KIND_UNIFORM_INT, seed, n, d) >= 128).astype(np.float32)


U8, GMM, UNIT, SPARSE, PM1 = (syn.KIND_UNIFORM_INT, syn.KIND_GAUSSIAN_MIXTURE, syn.KIND_UNIT_ROWS,
                              syn.KIND_SPARSE_INT, syn.KIND_UNIFORM_PM1)

CASES = [
    Case("eight_l2_k1", eight_points, 1, 0),
    Case("eight_l2_k3", eight_points, 3, 0),
    Case("eight_l2_k7", eight_points, 7, 0),
    Case("eight_negip_k3", eight_points, 3, 1),
    Case("u8_n2_d1_k1_l2", _gen(U8, 3, 2, 1), 1, 0),
    Case("u8_n33_d3_k32_l2", _gen(U8, 11, 33, 3), 32, 0),
    Case("u8_n300_d17_k32_l2", _gen(U8, 13, 300, 17), 32, 0),
    Case("cfg1_u8_n2000_d128_k10_l2", _gen(U8, 42, 2000, 128), 10, 0),
    Case("u8_n1537_d128_k16_l2", _gen(U8, 5, 1537, 128), 16, 0),
    Case("u8_n1000_d128_k10_negip", _gen(U8, 6, 1000, 128), 10, 1),
    Case("u8_n700_d300_k10_l2", _gen(U8, 21, 700, 300), 10, 0),
    Case("u8_n600_d960_k100_l2", _gen(U8, 22, 600, 960), 100, 0),
    Case("u8_n300_d1100_k5_l2", _gen(U8, 23, 300, 1100), 5, 0),
    Case("binary_n512_d16_k20_l2", _binary(24, 512, 16), 20, 0),
    Case("binary_n512_d16_k20_negip", _binary(25, 512, 16), 20, 1),
    Case("bimodal_n500_d1024_k5_l2", _bimodal(26, 500, 1024), 5, 0),
    Case("bimodal_n400_d1024_k5_negip", _bimodal(27, 400, 1024), 5, 1),
    Case("cfg5_sparse_n1500_d784_k64_negip", _gen(SPARSE, 2024, 1500, 784, p_zero=0.6), 64, 1),
    Case("cfg2_gmm_n2000_d128_k32_l2", _gen(GMM, 7, 2000, 128, components=100, sigma=0.1), 32, 0),
    Case("cfg4_unit_n800_d960_k100_l2", _gen(UNIT, 99, 800, 960), 100, 0),
    Case("pm1_n1024_d128_k10_l2", _gen(PM1, 42, 1024, 128), 10, 0),
    Case("pm1_n500_d64_k10_negip", _gen(PM1, 43, 500, 64), 10, 1),
    Case("u8_n1000_d128_k200_l2", _gen(U8, 31, 1000, 128), 200, 0),
]

BY_NAME = {c.name: c for c in CASES}
