/// @file
/// @brief knng::gpu::brute_force_knn -- header-only drop-in for
///        knng::cpu::brute_force_knn (include/knng/cpu/brute_force.hpp:336-376)
///        that builds the graph on an NVIDIA B200 through libknng_gpu.so.
///
/// Same signature, output layout and errors as the CPU template:
///   template <Distance D> Knng brute_force_knn(const Dataset&, std::size_t k, D = D{});
/// instantiable for L2Squared and NegativeInnerProduct (the two metrics the
/// reference instantiates, src/cpu/brute_force.cpp:39-43). Rows are sorted
/// ascending by (distance, id), self excluded by index. Throws
/// std::invalid_argument for n == 0, k == 0, k > n - 1 (brute_force.hpp:339-352)
/// and std::runtime_error for device failures. Include paths: the reference's
/// include/ (knng/core/...) and this repository's include/ (knng_gpu.h);
/// link with -lknng_gpu.
#pragma once

#include <cstddef>
#include <stdexcept>
#include <string>
#include <type_traits>

#include "knng/core/dataset.hpp"
#include "knng/core/distance.hpp"
#include "knng/core/graph.hpp"
#include "knng_gpu.h"

namespace knng::gpu {

namespace detail {
template <class D>
constexpr int metric_id()
{
    if constexpr (std::is_same_v<D, L2Squared>) {
        return KNNG_METRIC_L2_SQUARED;
    } else {
        static_assert(std::is_same_v<D, NegativeInnerProduct>,
                      "knng::gpu::brute_force_knn supports L2Squared and NegativeInnerProduct");
        return KNNG_METRIC_NEGATIVE_INNER_PRODUCT;
    }
}

inline void throw_on(knng_gpu_status st)
{
    if (st == KNNG_GPU_OK) return;
    const std::string msg = knng_gpu_last_error();
    if (st == KNNG_GPU_INVALID_ARGUMENT) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}
}  // namespace detail

/// How to spread one build over the GPUs of this node (no counterpart in
/// the reference, whose multi-node builder is src/dist/brute_force_mpi.cpp).
struct Options {
    int num_gpus = 1;   ///< devices 0..num_gpus-1, NCCL between them
    bool ring = false;  ///< pass base blocks around a ring instead of replicating the base
};

template <Distance D>
Knng brute_force_knn(const Dataset& ds, std::size_t k, D distance, const Options& opt)
{
    (void)distance;
    if (ds.n == 0) {
        throw std::invalid_argument("knng::gpu::brute_force_knn: dataset is empty");
    }
    if (k == 0) {
        throw std::invalid_argument("knng::gpu::brute_force_knn: k must be > 0");
    }
    if (k > ds.n - 1) {
        throw std::invalid_argument("knng::gpu::brute_force_knn: k (" + std::to_string(k) +
                                    ") must be <= ds.n - 1 (" + std::to_string(ds.n - 1) + ")");
    }
    Knng out(ds.n, k);
    if (opt.num_gpus > 1 || opt.ring) {
        detail::throw_on(knng_gpu_brute_force_multi(ds.data_ptr(), ds.n, ds.d, k, detail::metric_id<D>(),
                                                    opt.num_gpus, opt.ring ? 1 : 0, out.neighbors.data(),
                                                    out.distances.data(), nullptr));
    } else {
        detail::throw_on(knng_gpu_brute_force(ds.data_ptr(), ds.n, ds.d, k, detail::metric_id<D>(),
                                              out.neighbors.data(), out.distances.data(), nullptr));
    }
    return out;
}

/// The reference's signature: one GPU (the current device).
template <Distance D>
Knng brute_force_knn(const Dataset& ds, std::size_t k, D distance = D{})
{
    return brute_force_knn(ds, k, distance, Options{});
}

}  // namespace knng::gpu
