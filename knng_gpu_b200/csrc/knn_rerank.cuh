// knn_rerank.cuh -- the fp32 path around the bf16x3 tensor-core filter:
// column means and the hi/lo bf16 split before it, and after it the exact
// re-rank of each row's C candidates with a proof that no excluded row could
// belong to the top k.
//
// Exactness: a candidate's distance is recomputed with the reference's own
// arithmetic (sequential fp32, each step rounded: knng::squared_l2 /
// NegativeInnerProduct, include/knng/core/distance.hpp:52-116) and the k
// best are ranked by (distance, id) like knng::TopK (include/knng/top_k.hpp:
// 56-72). Let A be the largest approximate distance among the candidates
// (every excluded row's approximate distance is >= A) and eps a bound on
// |approximate - reference| for any pair. If A - eps > D_k (the k-th exact
// distance), every excluded row is strictly worse than the k-th: the row is
// exact. Otherwise the row goes to the exact kernel.
//
// Error bound (per pair, L2 on centred rows q' = q - mu, r' = r - mu):
//   bf16 hi/lo split leaves < 2^-16 |x| per coordinate, so the three-pass
//   products miss at most 2^-14 sum|q'_i r'_i|; the fp32 accumulator is
//   rounded once per UMMA instruction (K = 16 exact bf16 products each; see
//   the measured error ratio below), 3d/16 roundings of < 2^-22 relative
//   (a 4x allowance over round-to-nearest), i.e. (3d/16 + 3) 2^-22
//   sum|q'_i r'_i|; the norms, the key arithmetic and centring add
//   < 2^-19 (|q'| + |r'|)^2; the reference's own sequential sum differs from
//   the real distance by < (d+3) 2^-24 dist. With sum|q'_i r'_i| <= |q'||r'|
//   and dist <= (|q'| + |r'|)^2:
//     eps <= [2 (2^-14 + (3d/16 + 3) 2^-22) + 2^-19 + (d+3) 2^-24] (|q'| + R)^2,
//   R = max |r'|. Inner product (no centring): eps <= [2^-14 + (3d/16 + 3)
//   2^-22 + 2^-21 + (d+3) 2^-24] |q| R. Every call also records the largest
//   observed |approximate - exact| / eps over all candidates
//   (knng_gpu_stats.f32_err_ratio); it must stay well below 1.
#pragma once
#include <cuda_bf16.h>

#include <climits>
#include <cstdint>

#include "topk.cuh"

namespace knng_b200 {

// Column sums in fp64 (one pass over the rows); mean = sum / n.
__global__ void __launch_bounds__(256) column_sum_kernel(const float* __restrict__ x, uint64_t n, uint32_t d,
                                                         double* __restrict__ sums)
{
    const uint64_t rows_per_block = 256;
    const uint64_t r0 = static_cast<uint64_t>(blockIdx.x) * rows_per_block;
    const uint64_t r1 = r0 + rows_per_block < n ? r0 + rows_per_block : n;
    for (uint32_t c = threadIdx.x; c < d; c += blockDim.x) {
        double acc = 0.0;
        for (uint64_t r = r0; r < r1; ++r) acc += static_cast<double>(x[r * d + c]);
        atomicAdd(sums + c, acc);
    }
}

__global__ void column_mean_kernel(const double* __restrict__ sums, uint64_t n, uint32_t d, float* __restrict__ mu)
{
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < d) mu[c] = static_cast<float>(sums[c] / static_cast<double>(n));
}

// One warp per row: x' = x - mu (fp32), hi = bf16(x'), lo = bf16(x' - hi),
// rows padded with zeros to `pitch` elements; |x'|^2 (fp64 sum, rounded to
// fp32) and max |x'| (rounded up) over all rows.
__global__ void __launch_bounds__(256) split_bf16_kernel(const float* __restrict__ x, uint64_t rows, uint32_t d,
                                                         uint32_t pitch, const float* __restrict__ mu,
                                                         __nv_bfloat16* __restrict__ hi,
                                                         __nv_bfloat16* __restrict__ lo, float* __restrict__ norms,
                                                         unsigned int* __restrict__ max_norm_bits)
{
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t warp0 = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
    float local_max = 0.0f;
    for (uint64_t r = warp0; r < rows; r += nwarps) {
        const float* xr = x + r * d;
        double sum = 0.0;
        for (uint32_t c = lane; c < pitch; c += 32) {
            float v = 0.0f;
            if (c < d) v = mu ? __fsub_rn(xr[c], mu[c]) : xr[c];
            const __nv_bfloat16 h = __float2bfloat16_rn(v);
            const __nv_bfloat16 l = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(h)));
            hi[r * pitch + c] = h;
            lo[r * pitch + c] = l;
            sum += static_cast<double>(v) * static_cast<double>(v);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) {
            norms[r] = static_cast<float>(sum);
            local_max = fmaxf(local_max, __double2float_ru(sqrt(sum)));
        }
    }
    if (lane == 0) atomicMax(max_norm_bits, __float_as_uint(local_max));
}

struct RerankParams {
    const float* x;            // base rows (the reference's data); base row r has id base_id0 + r
    const float* qx;           // query rows; query i has id query_id0 + i
    uint64_t d;
    uint64_t n_b;              // base rows
    uint32_t base_id0;
    uint32_t query_id0;
    uint32_t exclude_self;
    uint32_t n_queries;
    uint32_t c;                // candidates per row
    uint32_t k;
    const uint32_t* cand_ids;  // n_queries x c, ascending approximate key
    const int32_t* cand_keys;  // ordered approximate keys
    const float* q_norms;      // |q'|^2 per query row (centred for L2)
    const unsigned int* max_norm_bits;
    double gamma;              // eps = gamma * (|q'| + R)^2 (L2) or gamma * |q| R (IP)
    uint32_t* out_ids;         // n_queries x k
    float* out_dists;
    uint32_t* fallback_rows;
    uint32_t* fallback_count;
    unsigned int* err_ratio_bits;  // max over candidates of |approx - exact| / eps (diagnostic)
};

constexpr int kRerankWarps = 8;

// One warp per query row; lane l owns candidates l, l+32, ... (CPL per lane).
// Candidate rows are read 32 rows x 32 coordinates at a time, coalesced, into
// shared memory; each lane then continues its own candidate's sequential sum.
template <int METRIC, int CPL>
__global__ void __launch_bounds__(32 * kRerankWarps) rerank_kernel(const RerankParams p)
{
    __shared__ float tile[kRerankWarps][32][33];
    __shared__ float qtile[kRerankWarps][32];
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t wib = threadIdx.x >> 5;
    const uint64_t warp0 = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
    for (uint64_t qi = warp0; qi < p.n_queries; qi += nwarps) {
        const float* qr = p.qx + qi * p.d;
        const uint32_t qid = p.query_id0 + static_cast<uint32_t>(qi);
        // Base rows this query can see: all, minus itself when excluded.
        const uint64_t eligible =
            p.n_b - ((p.exclude_self && qid >= p.base_id0 && qid - p.base_id0 < p.n_b) ? 1 : 0);
        int32_t key[CPL];
        uint32_t id[CPL];
        float dist[CPL];
#pragma unroll
        for (int t = 0; t < CPL; ++t) {
            const uint32_t j = t * 32 + lane;
            id[t] = j < p.c ? p.cand_ids[qi * p.c + j] : UINT32_MAX;
            float acc = 0.0f;
            if (t * 32 < p.c) {
                for (uint64_t d0 = 0; d0 < p.d; d0 += 32) {
                    __syncwarp();
                    const uint64_t col = d0 + lane;
                    qtile[wib][lane] = col < p.d ? qr[col] : 0.0f;
                    for (int r = 0; r < 32; ++r) {
                        const uint32_t rid = __shfl_sync(0xffffffffu, id[t], r);
                        tile[wib][r][lane] = (rid != UINT32_MAX && col < p.d)
                                                 ? p.x[static_cast<uint64_t>(rid - p.base_id0) * p.d + col]
                                                 : 0.0f;
                    }
                    __syncwarp();
                    const int cnt = p.d - d0 < 32 ? static_cast<int>(p.d - d0) : 32;
                    for (int i = 0; i < cnt; ++i) {
                        const float qv = qtile[wib][i];
                        const float rv = tile[wib][lane][i];
                        if (METRIC == 0) {
                            const float df = __fsub_rn(qv, rv);
                            acc = __fadd_rn(acc, __fmul_rn(df, df));
                        } else {
                            acc = __fadd_rn(acc, __fmul_rn(qv, rv));
                        }
                    }
                }
            }
            dist[t] = METRIC == 0 ? acc : -acc;
            key[t] = j < p.c ? ordered_key(dist[t]) : INT_MAX;
        }
        // Rank of each candidate under (distance, id): how many precede it.
        int rank[CPL];
#pragma unroll
        for (int t = 0; t < CPL; ++t) rank[t] = 0;
#pragma unroll
        for (int u = 0; u < CPL; ++u) {
            for (int s = 0; s < 32; ++s) {
                const int32_t ok_ = __shfl_sync(0xffffffffu, key[u], s);
                const uint32_t oi = __shfl_sync(0xffffffffu, id[u], s);
#pragma unroll
                for (int t = 0; t < CPL; ++t) rank[t] += key_gt(key[t], id[t], ok_, oi) ? 1 : 0;
            }
        }
        // Diagnostic: how close the observed filter error comes to eps.
        {
            const float qn = p.q_norms[qi];
            const double R = static_cast<double>(__uint_as_float(*p.max_norm_bits));
            const double sq = sqrt(static_cast<double>(qn));
            const double eps = METRIC == 0 ? p.gamma * (sq + R) * (sq + R) : p.gamma * sq * R;
            float worst = 0.0f;
#pragma unroll
            for (int t = 0; t < CPL; ++t) {
                const uint32_t j = t * 32 + lane;
                if (j < p.c) {
                    const double a = static_cast<double>(key_to_float(p.cand_keys[qi * p.c + j])) +
                                     (METRIC == 0 ? static_cast<double>(qn) : 0.0);
                    const double e = fabs(a - static_cast<double>(dist[t])) / (eps > 0.0 ? eps : 1e-300);
                    worst = fmaxf(worst, static_cast<float>(e));
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) worst = fmaxf(worst, __shfl_xor_sync(0xffffffffu, worst, o));
            if (lane == 0) atomicMax(p.err_ratio_bits, __float_as_uint(worst));
        }
        int32_t kth = INT_MIN;
#pragma unroll
        for (int t = 0; t < CPL; ++t) {
            const uint32_t j = t * 32 + lane;
            if (j < p.c && rank[t] < static_cast<int>(p.k)) {
                float f = dist[t];
                // -(+0.0f) is -0.0f in the reference (an fp32 sum is never -0.0).
                if (METRIC == 1 && f == 0.0f) f = -0.0f;
                p.out_ids[qi * p.k + rank[t]] = id[t];
                p.out_dists[qi * p.k + rank[t]] = f;
                if (rank[t] == static_cast<int>(p.k) - 1) kth = key[t];
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) kth = max(kth, __shfl_xor_sync(0xffffffffu, kth, o));
        if (lane == 0 && p.c < eligible) {
            // Proof that the excluded rows cannot enter the top k.
            const float qn = p.q_norms[qi];
            const double R = static_cast<double>(__uint_as_float(*p.max_norm_bits));
            const double a_c = static_cast<double>(key_to_float(p.cand_keys[qi * p.c + p.c - 1]));
            double approx_bound, eps;
            if (METRIC == 0) {
                approx_bound = static_cast<double>(qn) + a_c;
                const double s = sqrt(static_cast<double>(qn)) + R;
                eps = p.gamma * s * s;
            } else {
                approx_bound = a_c;
                eps = p.gamma * sqrt(static_cast<double>(qn)) * R;
            }
            const double dk = static_cast<double>(key_to_float(kth));
            if (!(approx_bound - eps > dk)) {
                const uint32_t slot = atomicAdd(p.fallback_count, 1u);
                p.fallback_rows[slot] = static_cast<uint32_t>(qi);
            }
        }
    }
}

}  // namespace knng_b200
