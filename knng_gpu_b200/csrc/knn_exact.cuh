// knn_exact.cuh -- exact fp32 brute-force KNN on CUDA cores, bit-identical to
// the reference's arithmetic: for every (query, base) pair the distance is the
// sequential left-to-right fp32 sum of knng::squared_l2
// (include/knng/core/distance.hpp:52-62) or knng::NegativeInnerProduct
// (distance.hpp:105-116), each step rounded separately (no FMA contraction),
// followed by the TopK admission rule (include/knng/top_k.hpp:56-72).
//
// Used for data that is not integer-valued in [0, 255], for dimensions above
// the tensor-core path's limit, and for the rare rows of the u8 path whose
// fp32 sums reach 2^24 (row_list mode). T is the element type of the input
// rows: float, or uint8_t for rows already packed by the u8 path (every u8
// value is an exact fp32 integer, so the sums are the same).
#pragma once
#include <climits>
#include <cstdint>

#include "topk.cuh"

namespace knng_b200 {

constexpr int kExactThreads = 128;  // queries per CTA, one per thread
constexpr int kExactBaseRows = 32;  // base rows per smem tile
constexpr int kExactDims = 32;      // dimensions per smem chunk

template <class T>
struct KnnExactParams {
    const T* base;
    uint64_t base_stride;  // elements between base rows
    uint64_t n_base;
    uint32_t base_id0;
    const T* queries;      // query row r lives at queries + r * query_stride
    uint64_t query_stride;
    uint32_t n_queries;
    uint32_t query_id0;
    uint32_t exclude_self;
    uint32_t d;
    uint32_t k;
    const uint32_t* row_list;   // optional: only these query rows
    const uint32_t* row_count;  // device count for row_list
    uint32_t* out_ids;
    float* out_dists;
};

template <class T>
__device__ __forceinline__ float load_as_float(const T* p)
{
    return static_cast<float>(*p);
}

template <int METRIC, class TopK, class T>
__global__ void __launch_bounds__(kExactThreads)
    knn_exact_kernel(const KnnExactParams<T> p)
{
    __shared__ float sQ[kExactDims * kExactThreads];         // [dim][query]
    __shared__ float4 sB[kExactBaseRows * kExactDims / 4];   // [row][dim/4]
    __shared__ uint32_t sRow[kExactThreads];

    const int t = threadIdx.x;
    const uint32_t nrows = p.row_list ? *p.row_count : p.n_queries;
    const uint32_t first = blockIdx.x * kExactThreads;
    if (first >= nrows) return;  // uniform across the block
    const uint32_t slot = first + t;
    const bool valid = slot < nrows;
    const uint32_t qlocal = valid ? (p.row_list ? p.row_list[slot] : slot) : 0u;
    sRow[t] = qlocal;
    const uint32_t self_id = p.exclude_self ? p.query_id0 + qlocal : UINT32_MAX;
    __syncthreads();

    TopK tk;
    tk.init(p.k);
    int32_t thr = tk.thr();
    const uint64_t n_btiles = (p.n_base + kExactBaseRows - 1) / kExactBaseRows;
    for (uint64_t bt = 0; bt < n_btiles; ++bt) {
        float acc[kExactBaseRows];
#pragma unroll
        for (int b = 0; b < kExactBaseRows; ++b) acc[b] = 0.0f;
        for (uint32_t dc = 0; dc < p.d; dc += kExactDims) {
            __syncthreads();
            for (int e = t; e < kExactDims * kExactThreads; e += kExactThreads) {
                const int qq = e / kExactDims, ii = e % kExactDims;
                float v = 0.0f;
                if (first + qq < nrows && dc + ii < p.d)
                    v = load_as_float(p.queries + static_cast<uint64_t>(sRow[qq]) * p.query_stride + dc + ii);
                sQ[ii * kExactThreads + qq] = v;
            }
            float* sBf = reinterpret_cast<float*>(sB);
            for (int e = t; e < kExactBaseRows * kExactDims; e += kExactThreads) {
                const int bb = e / kExactDims, ii = e % kExactDims;
                const uint64_t r = bt * kExactBaseRows + bb;
                float v = 0.0f;
                if (r < p.n_base && dc + ii < p.d) v = load_as_float(p.base + r * p.base_stride + dc + ii);
                sBf[bb * kExactDims + ii] = v;
            }
            __syncthreads();
            // Zero padding past d adds +0.0 at the end of each sum, which
            // leaves an fp32 sum that is never -0.0 unchanged.
#pragma unroll
            for (int i4 = 0; i4 < kExactDims / 4; ++i4) {
                const float q0 = sQ[(4 * i4 + 0) * kExactThreads + t];
                const float q1 = sQ[(4 * i4 + 1) * kExactThreads + t];
                const float q2 = sQ[(4 * i4 + 2) * kExactThreads + t];
                const float q3 = sQ[(4 * i4 + 3) * kExactThreads + t];
#pragma unroll
                for (int b = 0; b < kExactBaseRows; ++b) {
                    const float4 bv = sB[b * (kExactDims / 4) + i4];
                    float a = acc[b];
                    if (METRIC == 0) {
                        float df;
                        df = __fsub_rn(q0, bv.x); a = __fadd_rn(a, __fmul_rn(df, df));
                        df = __fsub_rn(q1, bv.y); a = __fadd_rn(a, __fmul_rn(df, df));
                        df = __fsub_rn(q2, bv.z); a = __fadd_rn(a, __fmul_rn(df, df));
                        df = __fsub_rn(q3, bv.w); a = __fadd_rn(a, __fmul_rn(df, df));
                    } else {
                        a = __fadd_rn(a, __fmul_rn(q0, bv.x));
                        a = __fadd_rn(a, __fmul_rn(q1, bv.y));
                        a = __fadd_rn(a, __fmul_rn(q2, bv.z));
                        a = __fadd_rn(a, __fmul_rn(q3, bv.w));
                    }
                    acc[b] = a;
                }
            }
        }
#pragma unroll
        for (int b = 0; b < kExactBaseRows; ++b) {
            const uint64_t r = bt * kExactBaseRows + b;
            const uint32_t id = p.base_id0 + static_cast<uint32_t>(r);
            const float dist = METRIC == 0 ? acc[b] : -acc[b];
            const int32_t key = ordered_key(dist);
            if (r < p.n_base && id != self_id && key < thr) {
                tk.insert_increasing(key, id);
                thr = tk.thr();
            }
        }
    }
    if (!valid) return;
    uint32_t* oid = p.out_ids + static_cast<uint64_t>(qlocal) * p.k;
    float* odist = p.out_dists + static_cast<uint64_t>(qlocal) * p.k;
    tk.for_each(p.k, [&](int j, int32_t key, uint32_t id) {
        float f = key_to_float(key);
        // -(+0.0f) is -0.0f in the reference (an fp32 sum is never -0.0).
        if (METRIC == 1 && f == 0.0f) f = -0.0f;
        oid[j] = id;
        odist[j] = f;
    });
}

}  // namespace knng_b200
