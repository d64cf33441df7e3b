"""knng_gpu_b200 -- exact brute-force KNN-graph construction on NVIDIA B200.

A drop-in GPU counterpart of ``knng::cpu::brute_force_knn`` from the
reference project (include/knng/cpu/brute_force.hpp:336-376): hand-written
sm_100a kernels behind the C ABI of ``include/knng_gpu.h``.
"""
from .api import (  # noqa: F401
    Dataset,
    InvalidArgument,
    Knng,
    KnngGpuError,
    L2Squared,
    NegativeInnerProduct,
    brute_force_knn,
    brute_force_knn_device,
    brute_force_knn_multi,
    brute_force_knn_u8,
    device_count,
    knn_f32,
    knn_f32_scratch_bytes,
    knn_f32_sets,
    knn_f32_sets_scratch_bytes,
    knn_scratch_bytes,
    knn_u8,
    knn_u8_sets,
    merge_topk,
    pack_u8,
    pack_u8_bytes,
    padded_dim,
    recall_at_k,
    workspace_bytes,
)
