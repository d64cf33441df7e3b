// ref_shim.cpp -- TEST INFRASTRUCTURE. A thin extern "C" layer over the
// reference's own, unmodified C++ sources (compiled where they lie by
// oracle/Makefile into oracle/_ref/libknng_ref.so). It lets the Python tests
// and bench.py's reference arm call knng::cpu::brute_force_knn and friends
// through ctypes. Nothing in the product links this.
//
// Entry points and the reference code each one reaches:
//   ref_brute_force_knn      -> knng::cpu::brute_force_knn<D>   (include/knng/cpu/brute_force.hpp:336-376)
//   ref_brute_force_knn_omp  -> knng::cpu::brute_force_knn_l2_omp (src/cpu/brute_force_omp.cpp:32-105)
//   ref_subset_knn           -> the loop body of brute_force.hpp:355-374, run
//                               for a list of query rows with the reference's
//                               own TopK and distance functors, OpenMP over rows
//   ref_xorshift_*           -> knng::random::XorShift64 (include/knng/random.hpp:48-144)
//   ref_dataset_hash         -> knng::bench::dataset_hash (src/bench/ground_truth.cpp:90-101)
//   ref_recall_at_k          -> knng::bench::recall_at_k (src/bench/recall.cpp:79-96)
//   ref_topk_run             -> knng::TopK push/extract_sorted (include/knng/top_k.hpp:56-91)
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include <omp.h>

#include "knng/bench/ground_truth.hpp"
#include "knng/bench/recall.hpp"
#include "knng/core/dataset.hpp"
#include "knng/core/distance.hpp"
#include "knng/core/graph.hpp"
#include "knng/cpu/brute_force.hpp"
#include "knng/random.hpp"
#include "knng/top_k.hpp"

namespace {
thread_local std::string g_err;

knng::Dataset make_ds(const float* x, uint64_t n, uint64_t d)
{
    knng::Dataset ds(n, d);
    if (n * d) std::memcpy(ds.data.data(), x, n * d * sizeof(float));
    return ds;
}

void copy_out(const knng::Knng& g, uint32_t* ids, float* dists)
{
    std::memcpy(ids, g.neighbors.data(), g.neighbors.size() * sizeof(uint32_t));
    std::memcpy(dists, g.distances.data(), g.distances.size() * sizeof(float));
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

// 0 ok, 1 invalid_argument (message in ref_last_error), 2 other exception.
int ref_brute_force_knn(const float* x, uint64_t n, uint64_t d, uint64_t k, int metric,
                        uint32_t* ids, float* dists)
{
    try {
        const knng::Dataset ds = make_ds(x, n, d);
        knng::Knng g = metric == 0 ? knng::cpu::brute_force_knn(ds, k, knng::L2Squared{})
                                   : knng::cpu::brute_force_knn(ds, k, knng::NegativeInnerProduct{});
        copy_out(g, ids, dists);
        return 0;
    } catch (const std::invalid_argument& e) {
        g_err = e.what();
        return 1;
    } catch (const std::exception& e) {
        g_err = e.what();
        return 2;
    }
}

int ref_brute_force_knn_omp(const float* x, uint64_t n, uint64_t d, uint64_t k, int threads,
                            uint32_t* ids, float* dists)
{
    try {
        const knng::Dataset ds = make_ds(x, n, d);
        knng::Knng g = knng::cpu::brute_force_knn_l2_omp(ds, k, threads);
        copy_out(g, ids, dists);
        return 0;
    } catch (const std::invalid_argument& e) {
        g_err = e.what();
        return 1;
    } catch (const std::exception& e) {
        g_err = e.what();
        return 2;
    }
}

// Subset harness: the canonical loop body for the listed query rows against
// the full base, with the reference's TopK and functors. Borrowed input (no
// copy), so it can run on multi-GB datasets.
int ref_subset_knn(const float* x, uint64_t n, uint64_t d, uint64_t k, int metric,
                   const uint64_t* queries, uint64_t nq, int threads, uint32_t* ids, float* dists)
{
    if (n == 0 || k == 0 || k > n - 1) {
        g_err = "ref_subset_knn: invalid n/k";
        return 1;
    }
    if (threads > 0) omp_set_num_threads(threads);
    const knng::L2Squared l2{};
    const knng::NegativeInnerProduct ip{};
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t qi = 0; qi < static_cast<int64_t>(nq); ++qi) {
        const uint64_t q = queries[qi];
        knng::TopK heap(k);
        const std::span<const float> query{x + q * d, d};
        for (uint64_t r = 0; r < n; ++r) {
            if (r == q) continue;
            const std::span<const float> row{x + r * d, d};
            const float dd = metric == 0 ? l2(query, row) : ip(query, row);
            heap.push(static_cast<knng::index_t>(r), dd);
        }
        const auto sorted = heap.extract_sorted();
        for (std::size_t j = 0; j < sorted.size(); ++j) {
            ids[qi * k + j] = sorted[j].first;
            dists[qi * k + j] = sorted[j].second;
        }
    }
    return 0;
}

void ref_xorshift_u64(uint64_t seed, uint64_t count, uint64_t* out)
{
    knng::random::XorShift64 rng(seed);
    for (uint64_t i = 0; i < count; ++i) out[i] = rng();
}

void ref_xorshift_float01(uint64_t seed, uint64_t count, float* out)
{
    knng::random::XorShift64 rng(seed);
    for (uint64_t i = 0; i < count; ++i) out[i] = rng.next_float01();
}

void ref_xorshift_below(uint64_t seed, uint64_t bound, uint64_t count, uint64_t* out)
{
    knng::random::XorShift64 rng(seed);
    for (uint64_t i = 0; i < count; ++i) out[i] = rng.next_below(bound);
}

uint64_t ref_dataset_hash(const float* x, uint64_t n, uint64_t d)
{
    const knng::Dataset ds = make_ds(x, n, d);
    return knng::bench::dataset_hash(ds);
}

double ref_recall_at_k(const uint32_t* approx, const uint32_t* truth, uint64_t n, uint64_t k)
{
    knng::Knng a(n, k), t(n, k);
    std::memcpy(a.neighbors.data(), approx, n * k * sizeof(uint32_t));
    std::memcpy(t.neighbors.data(), truth, n * k * sizeof(uint32_t));
    return knng::bench::recall_at_k(a, t);
}

uint64_t ref_topk_run(uint64_t k, uint64_t count, const uint32_t* ids, const float* dists,
                      uint32_t* out_ids, float* out_dists)
{
    knng::TopK heap(k);
    for (uint64_t i = 0; i < count; ++i) heap.push(ids[i], dists[i]);
    const auto s = heap.extract_sorted();
    for (std::size_t j = 0; j < s.size(); ++j) {
        out_ids[j] = s[j].first;
        out_dists[j] = s[j].second;
    }
    return s.size();
}

}  // extern "C"

// File-format hooks: the reference's loaders and ground-truth writer.
#include "knng/io/fvecs.hpp"
extern "C" {
// kind 0 fvecs, 1 ivecs, 2 bvecs. Returns 0 and fills n/d (and out when
// non-NULL, sized n*d elements); 1 with the message in ref_last_error.
int ref_load_vecs(const char* path, int kind, void* out, uint64_t* n, uint64_t* d)
{
    try {
        if (kind == 0) {
            const knng::Dataset ds = knng::io::load_fvecs(path);
            *n = ds.n; *d = ds.d;
            if (out) std::memcpy(out, ds.data.data(), ds.data.size() * 4);
        } else if (kind == 1) {
            const auto ds = knng::io::load_ivecs(path);
            *n = ds.n; *d = ds.d;
            if (out) std::memcpy(out, ds.data.data(), ds.data.size() * 4);
        } else {
            const auto ds = knng::io::load_bvecs(path);
            *n = ds.n; *d = ds.d;
            if (out) std::memcpy(out, ds.data.data(), ds.data.size());
        }
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return 1;
    }
}

int ref_save_ground_truth(const char* path, const uint32_t* ids, const float* dists, uint64_t n, uint64_t k,
                          uint64_t hash, int metric)
{
    try {
        knng::Knng g(n, k);
        std::memcpy(g.neighbors.data(), ids, n * k * 4);
        std::memcpy(g.distances.data(), dists, n * k * 4);
        knng::bench::save_ground_truth(path, g, hash, static_cast<knng::bench::MetricId>(metric));
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return 1;
    }
}
}  // extern "C"
