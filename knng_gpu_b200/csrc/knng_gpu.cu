// knng_gpu.cu -- C-ABI entry points (include/knng_gpu.h) and the host-side
// orchestration of the kernels: integer check + u8 pack + row norms, the
// fused tensor-core KNN, and the exact fp32 kernel.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "knn_exact.cuh"
#include "knn_pair.cuh"
#include "knn_rerank.cuh"
#include "knn_tc.cuh"
#include "knng_gpu.h"

using namespace knng_b200;

namespace {

thread_local std::string g_last_error;

knng_gpu_status fail(knng_gpu_status s, const std::string& msg)
{
    g_last_error = msg;
    return s;
}

#define KNNG_CUDA(call)                                                                                     \
    do {                                                                                                    \
        cudaError_t e_ = (call);                                                                            \
        if (e_ != cudaSuccess)                                                                              \
            return fail(e_ == cudaErrorMemoryAllocation ? KNNG_GPU_OUT_OF_MEMORY : KNNG_GPU_CUDA_ERROR,     \
                        std::string("knng::gpu: ") + #call + ": " + cudaGetErrorString(e_));                \
    } while (0)

#define KNNG_TRY(expr)                                    \
    do {                                                  \
        knng_gpu_status s_ = (expr);                      \
        if (s_ != KNNG_GPU_OK) return s_;                 \
    } while (0)

constexpr uint64_t align_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }

#ifdef KNNG_GPU_EXPERIMENTS
constexpr bool kExperiments = true;
#else
constexpr bool kExperiments = false;
#endif

// Tuning knobs for kernel experiments (grid size, stages, tile shape,
// profiling modes). Only a build compiled with -DKNNG_GPU_EXPERIMENTS reads
// them; the shipped library never looks at the environment, so no variable
// can change what a build computes.
const char* experiment_knob(const char* name)
{
#ifdef KNNG_GPU_EXPERIMENTS
    return std::getenv(name);
#else
    (void)name;
    return nullptr;
#endif
}

// Argument checks and messages of brute_force.hpp:339-352.
knng_gpu_status validate(uint64_t n, uint64_t d, uint64_t k, int metric)
{
    if (n == 0) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu::brute_force_knn: dataset is empty");
    if (k == 0) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu::brute_force_knn: k must be > 0");
    if (k > n - 1)
        return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu::brute_force_knn: k (" + std::to_string(k) +
                                                   ") must be <= ds.n - 1 (" + std::to_string(n - 1) + ")");
    if (metric != KNNG_METRIC_L2_SQUARED && metric != KNNG_METRIC_NEGATIVE_INNER_PRODUCT)
        return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu::brute_force_knn: unknown metric id " +
                                                   std::to_string(metric));
    if (k > KNNG_GPU_MAX_K)
        return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu::brute_force_knn: k (" + std::to_string(k) +
                                                ") exceeds the GPU limit " + std::to_string(KNNG_GPU_MAX_K));
    if (n > 0xFFFFFFFFull)
        return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu::brute_force_knn: n exceeds the 32-bit index_t range");
    if (d == 0 || d > (1u << 20))
        return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu::brute_force_knn: d must be in [1, 2^20]");
    return KNNG_GPU_OK;
}

// ------------------------------------------------------------------ pack
// One warp per row: read fp32 (128-bit loads when rows are 16-byte aligned),
// check integer-in-[0,255], write u8 rows with zero padding to the pitch,
// and the exact int32 squared norm (compute_norms_squared,
// src/cpu/distance.cpp:17-38, exact for such data).
__global__ void __launch_bounds__(256) pack_u8_kernel(const float* __restrict__ x, uint64_t rows, uint32_t d,
                                                      uint32_t data_bytes, uint32_t pitch, uint8_t* __restrict__ packed,
                                                      int32_t* __restrict__ norms, int32_t* nonint)
{
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t warp0 = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
    const bool vec = (d % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    bool bad = false;
    for (uint64_t r = warp0; r < rows; r += nwarps) {
        const float* xr = x + r * d;
        int32_t sum = 0;
        for (uint32_t c0 = lane * 4; c0 < data_bytes; c0 += 128) {
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (vec && c0 + 3 < d) {
                const float4 f = __ldcs(reinterpret_cast<const float4*>(xr + c0));
                v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (c0 + e < d) v[e] = xr[c0 + e];
            }
            uint32_t word = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float f = v[e];
                const bool ok = f >= 0.0f && f <= 255.0f && f == truncf(f);  // NaN fails
                bad |= !ok;
                const uint32_t u = ok ? static_cast<uint32_t>(f) : 0u;
                sum += static_cast<int32_t>(u * u);
                word |= u << (8 * e);
            }
            *reinterpret_cast<uint32_t*>(packed + r * pitch + c0) = word;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) norms[r] = sum;
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(nonint, 1);
}

// u8 ingest: rows that are already bytes (a .bvecs file's records, any row
// stride and byte offset) -> the packed layout + exact int32 |x|^2, with no
// float round trip. One warp per row; lane l handles bytes 4l..4l+3 of every
// 128-byte chunk.
__global__ void __launch_bounds__(256) pack_u8_bytes_kernel(const uint8_t* __restrict__ src, uint64_t rows,
                                                            uint32_t d, uint64_t row_stride, uint32_t data_bytes,
                                                            uint32_t pitch, uint8_t* __restrict__ packed,
                                                            int32_t* __restrict__ norms)
{
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t warp0 = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
    for (uint64_t r = warp0; r < rows; r += nwarps) {
        const uint8_t* xr = src + r * row_stride;
        int32_t sum = 0;
        for (uint32_t c0 = lane * 4; c0 < data_bytes; c0 += 128) {
            uint32_t word = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t u = c0 + e < d ? static_cast<uint32_t>(xr[c0 + e]) : 0u;
                sum += static_cast<int32_t>(u * u);
                word |= u << (8 * e);
            }
            *reinterpret_cast<uint32_t*>(packed + r * pitch + c0) = word;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) norms[r] = sum;
    }
}

// Augmentation of the packed rows for the tensor-core L2 filter. For each
// 128-row tile of this pack call, C = max over its rows of ceil(|r|^2 / 2)
// and S(r) = min(8160, (C - ceil(|r|^2 / 2)) / 255); the row's 32
// augmentation bytes hold S(r) as min(255, max(0, S - 255 j)), j = 0..31, so
// that a query side of 32 bytes of 255 adds 255 * S(r) to q.r. The norm is
// replaced by the key offset keyoff(r) = |r|^2 + 510 * S(r): then
// |r|^2 - 2 q.r = keyoff(r) - 2 (q.r + 255 S(r)), and within a tile keyoff
// varies by at most 509 unless the tile's norms spread over more than
// 2 * 255 * 8160 (rows past that keep S = 8160; every key stays exact).
__global__ void __launch_bounds__(128) pack_aug_kernel(uint64_t rows, uint32_t data_bytes, uint32_t pitch,
                                                       uint8_t* __restrict__ packed, int32_t* __restrict__ norms)
{
    __shared__ int32_t s_max[4];
    const uint64_t r = static_cast<uint64_t>(blockIdx.x) * 128 + threadIdx.x;
    const bool valid = r < rows;
    const int32_t nr = valid ? norms[r] : 0;
    const int32_t half = static_cast<int32_t>((static_cast<uint32_t>(nr) + 1u) >> 1);
    int32_t m = __reduce_max_sync(0xffffffffu, valid ? half : 0);
    if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = m;
    __syncthreads();
    m = max(max(s_max[0], s_max[1]), max(s_max[2], s_max[3]));
    if (!valid) return;
    const int32_t sv = min(8160, (m - half) / 255);
    uint32_t w[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        uint32_t word = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int32_t b = min(255, max(0, sv - 255 * (4 * q + e)));
            word |= static_cast<uint32_t>(b) << (8 * e);
        }
        w[q] = word;
    }
    uint4* dst = reinterpret_cast<uint4*>(packed + r * pitch + data_bytes);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    norms[r] = nr + 510 * sv;
}

// ------------------------------------------------------------------ TMA maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

knng_gpu_status get_encode_fn(EncodeTiledFn* out)
{
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
            return fail(KNNG_GPU_CUDA_ERROR, "knng::gpu: cuTensorMapEncodeTiled entry point not available");
        fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    *out = fn;
    return KNNG_GPU_OK;
}

// rows x width elements with a row stride of stride_bytes; box of 128 rows x
// box_bytes (128 with 128-byte swizzle, or 32 with 32-byte swizzle); rows past
// the end read as zeros.
knng_gpu_status make_map(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t elem_bytes, const void* base,
                         uint64_t rows, uint64_t width_elems, uint64_t stride_bytes, uint32_t box_bytes = kChunkBytes)
{
    EncodeTiledFn enc;
    KNNG_TRY(get_encode_fn(&enc));
    const cuuint64_t dims[2] = {width_elems, rows};
    const cuuint64_t strides[1] = {stride_bytes};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_bytes / elem_bytes), static_cast<cuuint32_t>(kTileRows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapSwizzle sw = box_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_128B;
    CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(KNNG_GPU_CUDA_ERROR, "knng::gpu: cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return KNNG_GPU_OK;
}

// 1-D map over n int32 values, boxes of `box` elements (zero fill past n).
knng_gpu_status make_map_1d_i32(CUtensorMap* map, const void* base, uint64_t n, uint32_t box)
{
    EncodeTiledFn enc;
    KNNG_TRY(get_encode_fn(&enc));
    const cuuint64_t dims[1] = {n};
    const cuuint64_t strides[1] = {4};
    const cuuint32_t boxd[1] = {box};
    const cuuint32_t estr[1] = {1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_INT32, 1, const_cast<void*>(base), dims, strides, boxd, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(KNNG_GPU_CUDA_ERROR, "knng::gpu: cuTensorMapEncodeTiled (1-D) failed (" + std::to_string(int(r)) + ")");
    return KNNG_GPU_OK;
}

// Packed u8 row: the data (d rounded up to 128 bytes), then kAugBytes of
// augmentation.
uint64_t u8_data_bytes(uint64_t d) { return align_up(d == 0 ? 1 : d, kChunkBytes); }

int sm_count()
{
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms > 0 ? sms : 148;
}

// ------------------------------------------------------------------ launch helpers
// Scratch of a u8 search: the fallback-row list (one entry per query), two
// counters (fallback count, error word), the seeded bounds (one per query),
// then the partial (key, id) lists of tail query tiles cut between units
// (two lists of up to 256 rows x k per unit). Without the partial region the
// single-CTA kernel searches whole query tiles only and the pair kernel is
// not used.
struct ScratchU8 {
    uint32_t* fallback_rows;
    uint32_t* counters;  // [0] fallback count, [1] error flag
    int32_t* seeds;      // per query: seeded bound on its k-th key (pair kernel)
    int32_t* part_keys;
    uint32_t* part_ids;
    uint32_t part_units;  // units (CTAs or CTA pairs) whose partial lists fit (0: none)
};

// Seeding pass of the pair kernel: the first kSeedRows base rows, used when
// the base holds at least kSeedMinBase rows.
constexpr uint64_t kSeedRows = 16384;
constexpr uint64_t kSeedMinBase = 8 * kSeedRows;

// Units of a persistent launch: at most one CTA per SM.
uint32_t max_units() { return static_cast<uint32_t>(std::max(1, sm_count())); }

// Two partial lists of one 256-row query tile per unit.
uint64_t partial_bytes_per_unit(uint64_t k) { return 2ull * 256 * k * 8; }

uint64_t scratch_u8_base_bytes(uint64_t q_count) { return align_up(q_count * 4, 256) + 256; }

uint64_t scratch_u8_bytes(uint64_t q_count, uint64_t k)
{
    return scratch_u8_base_bytes(q_count) + align_up(q_count * 4, 256) +
           align_up(max_units() * partial_bytes_per_unit(k), 256);
}

ScratchU8 carve_scratch_u8(void* p, uint64_t q_count, uint64_t k, uint64_t bytes)
{
    ScratchU8 s{};
    uint8_t* b = static_cast<uint8_t*>(p);
    s.fallback_rows = reinterpret_cast<uint32_t*>(b);
    s.counters = reinterpret_cast<uint32_t*>(b + align_up(q_count * 4, 256));
    s.seeds = reinterpret_cast<int32_t*>(b + scratch_u8_base_bytes(q_count));
    const uint64_t base = scratch_u8_base_bytes(q_count) + align_up(q_count * 4, 256);
    const uint64_t rest = bytes > base ? bytes - base : 0;
    const uint64_t per_unit = partial_bytes_per_unit(k);
    s.part_units = static_cast<uint32_t>(std::min<uint64_t>(rest / per_unit, 1u << 16));
    s.part_keys = reinterpret_cast<int32_t*>(b + base);
    s.part_ids = reinterpret_cast<uint32_t*>(b + base + s.part_units * per_unit / 2);
    return s;
}

struct TcMaps {
    CUtensorMap q0, q1, b0, b1;
};

// Persistent launch, one CTA per SM. u8 with register lists and partial-list
// scratch: whole query tiles in full waves, the last partial wave cut into
// equal ranges and merged afterwards (schedule.cuh); otherwise whole query
// tiles round-robin.
template <class Elem, int MT, int NBUF, bool A_STREAM, int METRIC, class TopK, int SPLIT = 1>
knng_gpu_status launch_tc_t(const TcMaps& m, KnnTcParams p, cudaStream_t st)
{
    const SmemLayoutTc L = smem_layout_tc(Elem::kPlanes, MT, A_STREAM, p.kchunks, p.stages, SPLIT,
                                          SPLIT > 1 ? TopK::kRegs / 2 : 0, !Elem::kFloat && METRIC == 0);
    const uint32_t smem = L.total + 1024;
    auto kern = knn_tc_kernel<Elem, MT, NBUF, A_STREAM, METRIC, TopK, SPLIT>;
    KNNG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const uint32_t n_qtiles = (p.n_queries + MT * kTileRows - 1) / (MT * kTileRows);
    const uint32_t n_btiles = static_cast<uint32_t>((p.n_base + kTileRows - 1) / kTileRows);
    uint32_t units = static_cast<uint32_t>(sm_count());
    if (const char* gv = experiment_knob("KNNG_GPU_GRID")) units = std::min<uint32_t>(units, std::max(1, std::atoi(gv)));
    bool tail = !Elem::kFloat && TopK::kCap > 0 && p.part_keys != nullptr && p.part_units >= units;
    if (const char* tv = experiment_knob("KNNG_GPU_TAIL_SPLIT")) tail = tail && std::atoi(tv) != 0;
    if (tail) {
        if (n_qtiles < units) units = static_cast<uint32_t>(std::min<uint64_t>(units, uint64_t(n_qtiles) * n_btiles));
    } else {
        units = std::min<uint32_t>(units, n_qtiles);
    }
    p.sched = make_schedule(units, n_qtiles, n_btiles, !tail);
    kern<<<units, 64 + 128 * MT * SPLIT, smem, st>>>(m.q0, m.q1, m.b0, m.b1, p);
    KNNG_CUDA(cudaGetLastError());
    if constexpr (!Elem::kFloat && TopK::kCap > 0) {
        if (tail && units > 1 && p.sched.tail_total > 0) {
            MergeParams mp{};
            mp.s = p.sched;
            mp.qtile_rows = MT * kTileRows;
            mp.k = p.k;
            mp.n_queries = p.n_queries;
            mp.part_keys = p.part_keys;
            mp.part_ids = p.part_ids;
            mp.out_ids = p.out_ids;
            mp.out_dists = p.out_dists;
            mp.query_norms = p.query_norms;
            mp.query_packed = p.query_packed;
            mp.pitch = p.pitch;
            mp.data_bytes = p.data_bytes;
            mp.fallback_rows = p.fallback_rows;
            mp.fallback_count = p.fallback_count;
            mp.skip_flag = p.skip_flag;
            merge_partials<METRIC, TopK::kCap><<<units - 1, MT * kTileRows, 0, st>>>(mp);
            KNNG_CUDA(cudaGetLastError());
        }
    }
    return KNNG_GPU_OK;
}

// Stages that fit the shared-memory budget for a tile configuration.
uint32_t pick_stages(int planes, int mt, bool a_stream, uint32_t kchunks, int split = 1, int kcap = 0,
                     bool aug = false)
{
    const SmemLayoutTc L0 = smem_layout_tc(planes, mt, a_stream, kchunks, 0, split, kcap, aug);
    const uint32_t budget = 227u * 1024u - 1024u;
    if (L0.total >= budget) return 0;
    uint32_t s = std::min<uint32_t>(16, (budget - L0.total) / L0.stage_bytes);
    if (const char* sv = experiment_knob("KNNG_GPU_STAGES")) s = std::min<uint32_t>(s, std::atoi(sv));
    return s;
}

template <int MT, int METRIC>
knng_gpu_status launch_u8_k(const TcMaps& m, const KnnTcParams& p, cudaStream_t st, int split)
{
    if constexpr (MT == 2) {
        if (split == 2 && p.k <= 10) return launch_tc_t<ElemU8, MT, 2, false, METRIC, RegTopK<10>, 2>(m, p, st);
        if (split == 2 && p.k <= 16) return launch_tc_t<ElemU8, MT, 2, false, METRIC, RegTopK<16>, 2>(m, p, st);
    }
    if (p.k <= 10) return launch_tc_t<ElemU8, MT, 2, false, METRIC, RegTopK<10>>(m, p, st);
    if (p.k <= 16) return launch_tc_t<ElemU8, MT, 2, false, METRIC, RegTopK<16>>(m, p, st);
    if (p.k <= 32) return launch_tc_t<ElemU8, MT, 2, false, METRIC, RegTopK<32>>(m, p, st);
    if constexpr (MT == 1) {
        if (p.k <= 64) return launch_tc_t<ElemU8, MT, 2, false, METRIC, RegTopK<64>>(m, p, st);
    }
    if (p.k <= 128) return launch_tc_t<ElemU8, MT, 2, false, METRIC, HeapTopK<128>>(m, p, st);
    return launch_tc_t<ElemU8, MT, 2, false, METRIC, HeapTopK<KNNG_GPU_MAX_K>>(m, p, st);
}

template <bool A_STREAM, int METRIC>
knng_gpu_status launch_bf16_k(const TcMaps& m, const KnnTcParams& p, cudaStream_t st)
{
    if (p.k <= 32) return launch_tc_t<ElemBf16x3, 1, 2, A_STREAM, METRIC, RegTopK<32>>(m, p, st);
    if (p.k <= 64) return launch_tc_t<ElemBf16x3, 1, 2, A_STREAM, METRIC, RegTopK<64>>(m, p, st);
    if (p.k <= 256) return launch_tc_t<ElemBf16x3, 1, 2, A_STREAM, METRIC, HeapTopK<256>>(m, p, st);
    return launch_tc_t<ElemBf16x3, 1, 2, A_STREAM, METRIC, HeapTopK<KNNG_GPU_MAX_K + 64>>(m, p, st);
}

template <int METRIC, class TopK, class T>
knng_gpu_status launch_exact_t(const KnnExactParams<T>& p, uint32_t max_rows, cudaStream_t st)
{
    if (max_rows == 0) return KNNG_GPU_OK;
    const uint32_t grid = (max_rows + kExactThreads - 1) / kExactThreads;
    knn_exact_kernel<METRIC, TopK, T><<<grid, kExactThreads, 0, st>>>(p);
    KNNG_CUDA(cudaGetLastError());
    return KNNG_GPU_OK;
}

template <int METRIC, class T>
knng_gpu_status launch_exact_k(const KnnExactParams<T>& p, uint32_t max_rows, cudaStream_t st)
{
    if (p.k <= 16) return launch_exact_t<METRIC, RegTopK<16>, T>(p, max_rows, st);
    if (p.k <= 32) return launch_exact_t<METRIC, RegTopK<32>, T>(p, max_rows, st);
    if (p.k <= 128) return launch_exact_t<METRIC, HeapTopK<128>, T>(p, max_rows, st);
    return launch_exact_t<METRIC, HeapTopK<KNNG_GPU_MAX_K>, T>(p, max_rows, st);
}

template <class T>
knng_gpu_status launch_exact(const KnnExactParams<T>& p, int metric, uint32_t max_rows, cudaStream_t st)
{
    return metric == 0 ? launch_exact_k<0, T>(p, max_rows, st) : launch_exact_k<1, T>(p, max_rows, st);
}

// Integer-valued data up to d = 1024 goes to the tensor cores; wider rows use
// the exact kernel on the packed bytes.
constexpr uint64_t kMaxTensorDim = 1024;

constexpr int kMaxDevices = 64;

// Timing events, created once per (host thread, device) and reused by every
// later call, so a call that fills stats creates no CUDA objects after the
// first one on its thread.
cudaEvent_t timing_event(int slot)
{
    thread_local cudaEvent_t ev[kMaxDevices][10] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices || slot < 0 || slot >= 10) return nullptr;
    if (!ev[dev][slot] && cudaEventCreate(&ev[dev][slot]) != cudaSuccess) ev[dev][slot] = nullptr;
    return ev[dev][slot];
}

// Device interval timer on the cached events of timer index `id` (0..4);
// ms() is 0 unless both ends were recorded (an elapsed-time query on an
// unrecorded event would leave a sticky error).
struct EventTimer {
    cudaEvent_t a = nullptr, b = nullptr;
    bool on, started = false, stopped = false;
    EventTimer(bool enable, int id) : on(enable)
    {
        if (on) {
            a = timing_event(2 * id);
            b = timing_event(2 * id + 1);
            on = a && b;
        }
    }
    void start(cudaStream_t s)
    {
        if (on) started = cudaEventRecord(a, s) == cudaSuccess;
    }
    void stop(cudaStream_t s)
    {
        if (on) stopped = cudaEventRecord(b, s) == cudaSuccess;
    }
    float ms()
    {
        float m = 0.f;
        if (on && started && stopped) {
            cudaEventSynchronize(b);
            cudaEventElapsedTime(&m, a, b);
        }
        return m;
    }
};

knng_gpu_status read_counters(const uint32_t* d_counters, uint32_t* host, cudaStream_t st)
{
    KNNG_CUDA(cudaMemcpyAsync(host, d_counters, 8, cudaMemcpyDeviceToHost, st));
    KNNG_CUDA(cudaStreamSynchronize(st));
    if (host[1] != 0)
        return fail(KNNG_GPU_TIMEOUT, "knng::gpu: a bounded device wait gave up (code " + std::to_string(host[1]) + ")");
    return KNNG_GPU_OK;
}

// Query rows and base rows as separate packed sets (they may be the same
// buffer). Ids are global: base row r is id b_id0 + r, query row i is
// q_id0 + i, and with exclude_self a query never returns its own id.
struct U8Sets {
    const uint8_t* q_packed;
    const int32_t* q_norms;
    uint64_t n_q;
    uint64_t q_id0;
    const uint8_t* b_packed;
    const int32_t* b_norms;
    uint64_t n_b;
    uint64_t b_id0;
    int exclude_self;
    // Optional, per query row: an exact upper bound on the keys worth
    // keeping (the running k-th key of a ring build). The pair kernel then
    // admits only keys at or below it, and its lists may hold fewer than k
    // entries; the single-CTA kernel ignores it (full lists are still right).
    const int32_t* seed = nullptr;
};

// Query tiles per CTA of the fused u8 kernel: two need k <= 32 (register
// budget of 320 threads) and at most two K chunks of resident A.
int u8_query_tiles_per_cta(uint64_t d, uint64_t k)
{
    int mt = (u8_data_bytes(d) / kChunkBytes <= 2 && k <= 32) ? 2 : 1;
    if (const char* mv = experiment_knob("KNNG_GPU_MT")) mt = std::atoi(mv) == 1 ? 1 : mt;  // experiments only
    return mt;
}

// Launch the u8 search of one (query set, base set) pair on `st`: the fused
// tensor-core kernel, then the exact kernel for the rows it flags (device-side
// count), or the exact kernel alone for d > kMaxTensorDim. No host sync; the
// caller zeroes sc.counters before and reads them after. tf (optional) times
// the exact pass.
knng_gpu_status launch_u8_sets(const U8Sets& z, uint64_t d, uint64_t k, int metric, uint32_t* ids, float* dists,
                               const ScratchU8& sc, cudaStream_t st, uint32_t* launches, EventTimer* tf,
                               const int* skip_flag = nullptr)
{
    const uint64_t q_count = z.n_q;
    const uint64_t pitch = knng_gpu_padded_dim(d);
    KnnExactParams<uint8_t> e{};
    e.base = z.b_packed;
    e.base_stride = pitch;
    e.n_base = z.n_b;
    e.base_id0 = static_cast<uint32_t>(z.b_id0);
    e.queries = z.q_packed;
    e.query_stride = pitch;
    e.n_queries = static_cast<uint32_t>(q_count);
    e.query_id0 = static_cast<uint32_t>(z.q_id0);
    e.exclude_self = z.exclude_self;
    e.d = static_cast<uint32_t>(d);
    e.k = static_cast<uint32_t>(k);
    e.out_ids = ids;
    e.out_dists = dists;
    if (d <= kMaxTensorDim) {
        const uint64_t data_bytes = u8_data_bytes(d);
        TcMaps m;
        KNNG_TRY(make_map(&m.q0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, z.q_packed, q_count, data_bytes, pitch));
        KNNG_TRY(make_map(&m.b0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, z.b_packed, z.n_b, data_bytes, pitch));
        m.q1 = m.q0;
        // L2: the base rows' augmentation bytes (32-byte boxes after the data)
        if (metric == 0)
            KNNG_TRY(make_map(&m.b1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, z.b_packed + data_bytes, z.n_b, kAugBytes,
                              pitch, kAugBytes));
        else
            m.b1 = m.b0;
        KnnTcParams p{};
        p.base_norms = z.b_norms;
        p.query_norms = z.q_norms;
        p.query_packed = z.q_packed;
        p.pitch = static_cast<uint32_t>(pitch);
        p.data_bytes = static_cast<uint32_t>(data_bytes);
        p.n_base = z.n_b;
        p.base_id0 = static_cast<uint32_t>(z.b_id0);
        p.n_queries = static_cast<uint32_t>(q_count);
        p.query_row0 = 0;
        p.query_id0 = static_cast<uint32_t>(z.q_id0);
        p.exclude_self = z.exclude_self;
        p.k = static_cast<uint32_t>(k);
        p.kchunks = static_cast<uint32_t>(data_bytes / kChunkBytes);
        p.out_ids = ids;
        p.out_dists = dists;
        p.fallback_rows = sc.fallback_rows;
        p.fallback_count = sc.counters;
        p.error = reinterpret_cast<int*>(sc.counters + 1);
        p.part_keys = sc.part_keys;
        p.part_ids = sc.part_ids;
        p.part_units = sc.part_units;
        p.skip_flag = skip_flag;
        if (const char* dbg = experiment_knob("KNNG_GPU_DEBUG_FLAGS")) p.debug_flags = static_cast<uint32_t>(std::atoi(dbg));
        int mt = u8_query_tiles_per_cta(d, k);
        // Optional column-split epilogue (four epilogue warps per SM
        // sub-partition, each on half of a 256-column tile), KNNG_GPU_SPLIT=2.
        // Measured slower than one warp per 32 rows at n=1M d=128 k=10 on B200
        // (305 ms vs 263 ms: the 96-register budget spills), so off by default.
        int split = 1;
        if (const char* sv = experiment_knob("KNNG_GPU_SPLIT")) split = (std::atoi(sv) == 2 && mt == 2 && k <= 16) ? 2 : 1;
        const bool aug = metric == 0;
        p.stages = pick_stages(1, mt, false, p.kchunks, split, split > 1 ? (k <= 10 ? 10 : 16) : 0, aug);
        if (split > 1 && p.stages < 3) {
            split = 1;
            p.stages = pick_stages(1, mt, false, p.kchunks, 1, 0, aug);
        }
        if (p.stages < 2 || (mt > 1 && p.stages < p.kchunks))
            return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: shared memory budget exceeded");
        unsigned long long* dbg_clk = nullptr;
        if (kExperiments && (p.debug_flags & 512u)) {  // profiling only
            cudaMalloc(&dbg_clk, 8 * sizeof(unsigned long long));
            cudaMemsetAsync(dbg_clk, 0, 8 * sizeof(unsigned long long), st);
            p.debug_clocks = dbg_clk;
        }
        knng_gpu_status s;
        if (mt == 2)
            s = metric == 0 ? launch_u8_k<2, 0>(m, p, st, split) : launch_u8_k<2, 1>(m, p, st, split);
        else
            s = metric == 0 ? launch_u8_k<1, 0>(m, p, st, split) : launch_u8_k<1, 1>(m, p, st, split);
        KNNG_TRY(s);
        if (dbg_clk) {
            unsigned long long h[8];
            cudaMemcpyAsync(h, dbg_clk, sizeof(h), cudaMemcpyDeviceToHost, st);
            cudaStreamSynchronize(st);
            std::fprintf(stderr,
                         "knng debug clocks (sum over CTAs): mma wait_tempty %llu wait_full %llu total %llu | "
                         "epi0 wait_tfull %llu total %llu | producer wait_stage %llu total %llu\n",
                         h[0], h[1], h[2], h[3], h[4], h[5], h[6]);
            cudaFree(dbg_clk);
        }
        // Rows whose fp32 sums may round: recompute exactly (device-side
        // count; CTAs past it exit at once).
        if (tf) tf->start(st);
        e.row_list = sc.fallback_rows;
        e.row_count = sc.counters;
        KNNG_TRY(launch_exact(e, metric, static_cast<uint32_t>(q_count), st));
        if (tf) tf->stop(st);
        *launches += 2;
    } else {
        KNNG_TRY(launch_exact(e, metric, static_cast<uint32_t>(q_count), st));
        *launches += 1;
    }
    return KNNG_GPU_OK;
}

// Options of one u8 search that only internal callers set.
struct U8RunOptions {
    bool allow_pair = true;                  // CTA-pair kernel where it applies
    long long wait_limit = kSpinLimitCycles;  // bound of every device-side wait
    uint32_t test_mode = 0;                  // 1: the pair kernel withholds one arrival
    bool timing = true;                      // fill the *_ms fields of stats
    const int* skip_flag = nullptr;          // pair kernel: device flag, non-zero = data not integer-valued
};

struct PairMaps {
    CUtensorMap q, b, baug, norm;
};

template <int METRIC, int KC, int EPI>
knng_gpu_status launch_pair_t(const PairMaps& m, PairParams& pp, uint32_t max_pairs_fit, cudaStream_t st,
                              uint32_t* launches, EventTimer* tt)
{
    const SmemLayoutPair L = smem_layout_pair(pp.kchunks, pp.stages, METRIC == 0, EPI > 4 ? KC : 0);
    const uint32_t smem = L.total + 1024;
    auto kern = knn_pair_kernel<METRIC, RegTopK<KC>, EPI>;
    KNNG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(pair_threads(EPI));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(2 * (max_units() / 2));
    int clusters = 0;
    KNNG_CUDA(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg));
    uint64_t np = std::min<uint64_t>(static_cast<uint64_t>(std::max(clusters, 0)), max_pairs_fit);
    if (const char* gv = experiment_knob("KNNG_GPU_PAIRS")) np = std::min<uint64_t>(np, std::max(1, std::atoi(gv)));
    // Whole query tiles in full waves over all pairs, the last partial wave
    // cut into equal ranges (few queries: only that).
    const uint64_t nqt = pp.sched.n_qtiles, nbt = pp.sched.n_btiles;
    if (nqt < np) np = std::min<uint64_t>(np, nqt * nbt);
    if (np == 0) return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: no CTA pair fits on this device");
    pp.sched = make_schedule(static_cast<uint32_t>(np), static_cast<uint32_t>(nqt), static_cast<uint32_t>(nbt), false);
    unsigned long long* dbg_clk = nullptr;
    if (kExperiments && (pp.debug_flags & 512u)) {  // profiling only
        cudaMalloc(&dbg_clk, 16 * sizeof(unsigned long long));
        cudaMemsetAsync(dbg_clk, 0, 16 * sizeof(unsigned long long), st);
        pp.debug_clocks = dbg_clk;
    }
    if (tt) tt->start(st);
    KNNG_CUDA(cudaLaunchKernelEx(&cfg, kern, m.q, m.b, m.baug, m.norm, pp));
    if (tt) tt->stop(st);
    ++*launches;
    if (dbg_clk) {
        unsigned long long h[16];
        cudaMemcpyAsync(h, dbg_clk, sizeof(h), cudaMemcpyDeviceToHost, st);
        cudaStreamSynchronize(st);
        const double warps = 2.0 * pp.sched.n_units * EPI;
        std::fprintf(stderr,
                     "pair clocks per epilogue warp: wait_tfull %.3g slow %.3g n_slow %.3g n_slow_calls %.3g total %.3g | "
                     "per MMA thread: wait_tempty %.3g wait_full %.3g total %.3g | tiles per pair %.3g\n",
                     h[0] / warps, h[1] / warps, h[2] / warps, h[7] / warps, h[3] / warps,
                     h[4] / double(pp.sched.n_units), h[5] / double(pp.sched.n_units),
                     h[6] / double(pp.sched.n_units),
                     double(pp.sched.n_qtiles) * pp.sched.n_btiles / pp.sched.n_units);
        cudaFree(dbg_clk);
    }
    if (pp.sched.n_units > 1 && pp.sched.tail_total > 0) {
        MergeParams mp{};
        mp.s = pp.sched;
        mp.qtile_rows = kPairTile;
        mp.k = pp.k;
        mp.n_queries = pp.n_queries;
        mp.part_keys = pp.part_keys;
        mp.part_ids = pp.part_ids;
        mp.out_ids = pp.out_ids;
        mp.out_dists = pp.out_dists;
        mp.seed_out = pp.seed_out;
        mp.seed_in = pp.seed_in;
        mp.query_norms = pp.query_norms;
        mp.query_packed = pp.query_packed;
        mp.pitch = pp.pitch;
        mp.data_bytes = pp.data_bytes;
        mp.fallback_rows = pp.fallback_rows;
        mp.fallback_count = pp.fallback_count;
        mp.skip_flag = pp.skip_flag;
        merge_partials<METRIC, KC><<<pp.sched.n_units - 1, kPairTile, 0, st>>>(mp);
        KNNG_CUDA(cudaGetLastError());
        ++*launches;
    }
    return KNNG_GPU_OK;
}

// Sixteen epilogue warps (four 64-column slices per lane quarter) for short
// tiles (d <= 256, where the tensor core finishes a tile in ~1000 cycles)
// and small lists; four otherwise.
int pair_epi_warps(uint32_t kchunks, uint64_t k)
{
    int epi = (kchunks <= 2 && k <= 16) ? 16 : 4;
    if (const char* ev = experiment_knob("KNNG_GPU_EPI")) {
        const int e = std::atoi(ev);
        if (e == 4 || e == 8) epi = e;
    }
    return epi;
}

template <int METRIC>
knng_gpu_status launch_pair_k(const PairMaps& m, PairParams& pp, uint32_t fit, cudaStream_t st, uint32_t* launches,
                              EventTimer* tt)
{
    const int epi = pair_epi_warps(pp.kchunks, pp.k);
    if (epi == 16) {
        if (pp.k <= 10) return launch_pair_t<METRIC, 10, 16>(m, pp, fit, st, launches, tt);
        return launch_pair_t<METRIC, 16, 16>(m, pp, fit, st, launches, tt);
    }
    if (kExperiments && epi == 8) {
        if (pp.k <= 10) return launch_pair_t<METRIC, 10, 8>(m, pp, fit, st, launches, tt);
        return launch_pair_t<METRIC, 16, 8>(m, pp, fit, st, launches, tt);
    }
    if (pp.k <= 10) return launch_pair_t<METRIC, 10, 4>(m, pp, fit, st, launches, tt);
    if (pp.k <= 16) return launch_pair_t<METRIC, 16, 4>(m, pp, fit, st, launches, tt);
    if (pp.k <= 32) return launch_pair_t<METRIC, 32, 4>(m, pp, fit, st, launches, tt);
    return launch_pair_t<METRIC, 64, 4>(m, pp, fit, st, launches, tt);
}

// Stages of the pair kernel that fit the shared-memory budget (0: none).
uint32_t pick_pair_stages(uint32_t kchunks, bool l2, uint64_t k)
{
    const uint32_t merge_cap = (pair_epi_warps(kchunks, k) > 4 && k <= 16) ? (k <= 10 ? 10 : 16) : 0;
    const SmemLayoutPair L0 = smem_layout_pair(kchunks, 0, l2, merge_cap);
    const uint32_t budget = 227u * 1024u - 1024u;
    if (L0.total >= budget) return 0;
    uint32_t s = std::min<uint32_t>(16, (budget - L0.total) / L0.stage_bytes);
    if (const char* sv = experiment_knob("KNNG_GPU_STAGES")) s = std::min<uint32_t>(s, std::atoi(sv));
    return s >= 2 ? s : 0;
}

// The pair kernel: base and query rows in 256-row tiles on CTA pairs,
// stream-K split, then the exact kernel on the rows it flags.
knng_gpu_status launch_u8_pair(const U8Sets& z, uint64_t d, uint64_t k, int metric, uint32_t* ids, float* dists,
                               const ScratchU8& sc, const U8RunOptions& opt, cudaStream_t st, uint32_t* launches,
                               EventTimer* tt)
{
    const uint64_t pitch = knng_gpu_padded_dim(d);
    const uint64_t data_bytes = u8_data_bytes(d);
    PairMaps m;
    KNNG_TRY(make_map(&m.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, z.q_packed, z.n_q, data_bytes, pitch));
    KNNG_TRY(make_map(&m.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, z.b_packed, z.n_b, data_bytes, pitch));
    if (metric == 0) {
        KNNG_TRY(make_map(&m.baug, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, z.b_packed + data_bytes, z.n_b, kAugBytes, pitch,
                          kAugBytes));
        KNNG_TRY(make_map_1d_i32(&m.norm, z.b_norms, z.n_b, kPairTile));
    } else {
        m.baug = m.b;
        m.norm = m.b;
    }
    PairParams pp{};
    pp.query_norms = z.q_norms;
    pp.query_packed = z.q_packed;
    pp.pitch = static_cast<uint32_t>(pitch);
    pp.data_bytes = static_cast<uint32_t>(data_bytes);
    pp.n_base = z.n_b;
    pp.base_id0 = static_cast<uint32_t>(z.b_id0);
    pp.n_queries = static_cast<uint32_t>(z.n_q);
    pp.query_id0 = static_cast<uint32_t>(z.q_id0);
    pp.exclude_self = z.exclude_self;
    pp.k = static_cast<uint32_t>(k);
    pp.kchunks = static_cast<uint32_t>(data_bytes / kChunkBytes);
    pp.stages = pick_pair_stages(pp.kchunks, metric == 0, k);
    pp.sched = make_schedule(1, static_cast<uint32_t>((z.n_q + kPairTile - 1) / kPairTile),
                             static_cast<uint32_t>((z.n_b + kPairTile - 1) / kPairTile), false);
    pp.out_ids = ids;
    pp.out_dists = dists;
    pp.part_keys = sc.part_keys;
    pp.part_ids = sc.part_ids;
    pp.fallback_rows = sc.fallback_rows;
    pp.fallback_count = sc.counters;
    pp.error = reinterpret_cast<int*>(sc.counters + 1);
    pp.wait_limit = opt.wait_limit;
    pp.test_mode = opt.test_mode;
    pp.skip_flag = opt.skip_flag;
    if (const char* dbg = experiment_knob("KNNG_GPU_DEBUG_FLAGS")) pp.debug_flags = static_cast<uint32_t>(std::atoi(dbg));
    if (tt) tt->start(st);
    // Seeding pass: the queries against the first kSeedRows base rows give
    // each query an exact upper bound on its k-th key over the whole base
    // (its k-th key among a subset of the rows). The main pass then admits
    // only keys at or below that bound, so the top-k lists see far fewer
    // insertions; the result is unchanged.
    bool seeded = z.n_b >= kSeedMinBase && k + 1 <= kSeedRows && opt.test_mode == 0;
    if (const char* sv = experiment_knob("KNNG_GPU_SEED")) seeded = seeded && std::atoi(sv) != 0;
    if (seeded) {
        PairMaps ms = m;
        KNNG_TRY(make_map(&ms.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, z.b_packed, kSeedRows, data_bytes, pitch));
        if (metric == 0) {
            KNNG_TRY(make_map(&ms.baug, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, z.b_packed + data_bytes, kSeedRows,
                              kAugBytes, pitch, kAugBytes));
            KNNG_TRY(make_map_1d_i32(&ms.norm, z.b_norms, kSeedRows, kPairTile));
        } else {
            ms.baug = ms.b;
            ms.norm = ms.b;
        }
        PairParams ps = pp;
        ps.n_base = kSeedRows;
        ps.sched.n_btiles = static_cast<uint32_t>(kSeedRows / kPairTile);
        ps.seed_in = z.seed;  // an outside bound caps the seeded one
        ps.seed_out = sc.seeds;
        ps.debug_flags = 0;
        KNNG_TRY(metric == 0 ? launch_pair_k<0>(ms, ps, sc.part_units, st, launches, nullptr)
                             : launch_pair_k<1>(ms, ps, sc.part_units, st, launches, nullptr));
        pp.seed_in = sc.seeds;
    } else {
        pp.seed_in = z.seed;
    }
    KNNG_TRY(metric == 0 ? launch_pair_k<0>(m, pp, sc.part_units, st, launches, nullptr)
                         : launch_pair_k<1>(m, pp, sc.part_units, st, launches, nullptr));
    if (tt) tt->stop(st);
    // Rows whose fp32 sums may round: recompute exactly (device-side count).
    KnnExactParams<uint8_t> e{};
    e.base = z.b_packed;
    e.base_stride = pitch;
    e.n_base = z.n_b;
    e.base_id0 = static_cast<uint32_t>(z.b_id0);
    e.queries = z.q_packed;
    e.query_stride = pitch;
    e.n_queries = static_cast<uint32_t>(z.n_q);
    e.query_id0 = static_cast<uint32_t>(z.q_id0);
    e.exclude_self = z.exclude_self;
    e.d = static_cast<uint32_t>(d);
    e.k = static_cast<uint32_t>(k);
    e.out_ids = ids;
    e.out_dists = dists;
    e.row_list = sc.fallback_rows;
    e.row_count = sc.counters;
    KNNG_TRY(launch_exact(e, metric, static_cast<uint32_t>(z.n_q), st));
    ++*launches;
    return KNNG_GPU_OK;
}

// Whether the pair kernel applies: rows longer than 256 bytes (the pair
// tile's hand-off costs more than a d <= 256 tile's tensor work; measured on
// B200: d = 128 searches run faster on the single-CTA kernel at every size,
// d = 784 ones faster on the pair kernel), d <= 1024 with a stage budget,
// k <= 64 (register lists), partial-list scratch present, and 16-byte aligned
// key offsets (TMA source).
bool pair_applies(const U8Sets& z, uint64_t d, uint64_t k, int metric, const ScratchU8& sc, const U8RunOptions& opt)
{
    if (!opt.allow_pair || d > kMaxTensorDim || k > 64 || sc.part_units == 0) return false;
    const uint32_t kchunks = static_cast<uint32_t>(u8_data_bytes(d) / kChunkBytes);
    bool want = kchunks >= 3 || opt.test_mode != 0;
    if (const char* pv = experiment_knob("KNNG_GPU_PAIR")) want = std::atoi(pv) != 0;
    if (!want) return false;
    if (metric == 0 && (reinterpret_cast<uintptr_t>(z.b_norms) & 15)) return false;
    return pick_pair_stages(kchunks, metric == 0, k) >= 2;
}

// u8 search of a query set against a base set: the pair kernel where it
// applies, else the single-CTA kernel; then the exact kernel for flagged rows.
// One host synchronisation at the end reads the fallback count and the error
// word.
knng_gpu_status knn_u8_sets_impl(const U8Sets& z, uint64_t d, uint64_t k, int metric, uint32_t* ids, float* dists,
                                 void* scratch, uint64_t scratch_bytes, cudaStream_t st, knng_gpu_stats* stats,
                                 const U8RunOptions& opt = U8RunOptions())
{
    const uint64_t q_count = z.n_q;
    if (scratch_bytes < scratch_u8_base_bytes(q_count))
        return fail(KNNG_GPU_WORKSPACE_TOO_SMALL, "knng::gpu: scratch smaller than knng_gpu_knn_scratch_bytes");
    if (q_count == 0) return KNNG_GPU_OK;
    if (z.n_b < k + (z.exclude_self ? 1 : 0))
        return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: fewer base rows than k");
    // TMA sources and the 16-byte copies of the base key offsets.
    if ((reinterpret_cast<uintptr_t>(z.q_packed) | reinterpret_cast<uintptr_t>(z.b_packed) |
         reinterpret_cast<uintptr_t>(z.b_norms)) & 15)
        return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: packed rows and base key offsets must be 16-byte aligned");
    const ScratchU8 sc = carve_scratch_u8(scratch, q_count, k, scratch_bytes);
    KNNG_CUDA(cudaMemsetAsync(sc.counters, 0, 8, st));
    uint32_t launches = 0;
    const bool timing = stats != nullptr && opt.timing;
    EventTimer tk(timing, 2), tf(timing, 3), tt(timing, 4);
    tk.start(st);
    if (pair_applies(z, d, k, metric, sc, opt)) {
        KNNG_TRY(launch_u8_pair(z, d, k, metric, ids, dists, sc, opt, st, &launches, &tt));
        tk.stop(st);
    } else {
        tt.start(st);
        KNNG_TRY(launch_u8_sets(z, d, k, metric, ids, dists, sc, st, &launches, &tf, opt.skip_flag));
        tt.stop(st);
        tk.stop(st);
    }
    uint32_t host_counters[2] = {0, 0};
    KNNG_TRY(read_counters(sc.counters, host_counters, st));
    if (stats) {
        stats->path = KNNG_PATH_U8_TENSOR;
        stats->fallback_rows = host_counters[0];
        stats->knn_ms = tk.ms();
        stats->fallback_ms = tf.ms();
        stats->tc_ms = tt.ms();
        stats->kernel_launches += launches;
    }
    return KNNG_GPU_OK;
}

knng_gpu_status knn_u8_impl(const uint8_t* packed, const int32_t* norms, uint64_t n, uint64_t d, uint64_t q_begin,
                            uint64_t q_count, uint64_t k, int metric, uint32_t* ids, float* dists, void* scratch,
                            uint64_t scratch_bytes, cudaStream_t st, knng_gpu_stats* stats,
                            const U8RunOptions& opt = U8RunOptions())
{
    if (q_begin + q_count > n) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: query range exceeds the base");
    const uint64_t pitch = knng_gpu_padded_dim(d);
    const U8Sets z{packed + q_begin * pitch, norms + q_begin, q_count, q_begin, packed, norms, n, 0, 1};
    return knn_u8_sets_impl(z, d, k, metric, ids, dists, scratch, scratch_bytes, st, stats, opt);
}

// Merge two row-wise sorted k-lists into the k best by (distance, id) -- the
// TopK order of include/knng/top_k.hpp:56-72 -- one thread per row.
__global__ void merge_topk_kernel(const uint32_t* __restrict__ a_ids, const float* __restrict__ a_d,
                                  const uint32_t* __restrict__ b_ids, const float* __restrict__ b_d, uint64_t rows,
                                  uint32_t k, uint32_t* __restrict__ o_ids, float* __restrict__ o_d)
{
    const uint64_t r = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const uint64_t base = r * k;
    uint32_t i = 0, j = 0;
    for (uint32_t o = 0; o < k; ++o) {
        bool take_a;
        if (i >= k) {
            take_a = false;
        } else if (j >= k) {
            take_a = true;
        } else {
            const int32_t ka = ordered_key(a_d[base + i]), kb = ordered_key(b_d[base + j]);
            take_a = !key_gt(ka, a_ids[base + i], kb, b_ids[base + j]);
        }
        if (take_a) {
            o_ids[base + o] = a_ids[base + i];
            o_d[base + o] = a_d[base + i];
            ++i;
        } else {
            o_ids[base + o] = b_ids[base + j];
            o_d[base + o] = b_d[base + j];
            ++j;
        }
    }
}

// ------------------------------------------------------------------ fp32 path
// Candidates kept per query row by the bf16x3 filter: k plus a margin, at
// most the rows a query can see (n_b, minus itself when excluded).
uint64_t f32_candidates_sets(uint64_t n_b, int exclude_self, uint64_t k)
{
    return std::min<uint64_t>(n_b - (exclude_self ? 1 : 0), k + 32);
}

uint64_t f32_pitch_elems(uint64_t d) { return align_up(d, kChunkBytes / 2); }

struct ScratchF32 {
    double* sums;
    float* mu;
    unsigned int* max_norm_bits;
    __nv_bfloat16* hi;  // base planes
    __nv_bfloat16* lo;
    float* norms;
    __nv_bfloat16* q_hi;  // query planes (separate query set only)
    __nv_bfloat16* q_lo;
    float* q_norms;
    uint32_t* cand_ids;
    int32_t* cand_keys;
    uint32_t* fallback_rows;
    uint32_t* counters;  // [0] fallback count, [1] error flag, [2] observed error ratio (fp32 bits)
    uint64_t total;
};

ScratchF32 layout_scratch_f32_sets(void* base, uint64_t n_b, uint64_t n_q, uint64_t d, uint64_t k, int exclude_self,
                                   bool separate_q)
{
    ScratchF32 s{};
    uint8_t* p = static_cast<uint8_t*>(base);
    uint64_t off = 0;
    auto take = [&](uint64_t bytes) {
        uint8_t* r = p ? p + off : nullptr;
        off = align_up(off + bytes, 256);
        return r;
    };
    const uint64_t pitch = f32_pitch_elems(d);
    const uint64_t c = f32_candidates_sets(n_b, exclude_self, k);
    s.sums = reinterpret_cast<double*>(take(d * 8));
    s.mu = reinterpret_cast<float*>(take(d * 4));
    s.max_norm_bits = reinterpret_cast<unsigned int*>(take(4));
    s.hi = reinterpret_cast<__nv_bfloat16*>(take(n_b * pitch * 2));
    s.lo = reinterpret_cast<__nv_bfloat16*>(take(n_b * pitch * 2));
    s.norms = reinterpret_cast<float*>(take(n_b * 4));
    if (separate_q) {
        s.q_hi = reinterpret_cast<__nv_bfloat16*>(take(n_q * pitch * 2));
        s.q_lo = reinterpret_cast<__nv_bfloat16*>(take(n_q * pitch * 2));
        s.q_norms = reinterpret_cast<float*>(take(n_q * 4));
    }
    s.cand_ids = reinterpret_cast<uint32_t*>(take(n_q * c * 4));
    s.cand_keys = reinterpret_cast<int32_t*>(take(n_q * c * 4));
    s.fallback_rows = reinterpret_cast<uint32_t*>(take(n_q * 4));
    s.counters = reinterpret_cast<uint32_t*>(take(16));
    s.total = off;
    return s;
}

// Self graph: queries are rows of the base (planes shared).
ScratchF32 layout_scratch_f32(void* base, uint64_t n, uint64_t d, uint64_t q_count, uint64_t k)
{
    return layout_scratch_f32_sets(base, n, q_count, d, k, 1, false);
}

// eps coefficient of the re-rank proof (knn_rerank.cuh).
double f32_gamma(uint64_t d, int metric)
{
    const double dd = static_cast<double>(d);
    const double split = std::ldexp(1.0, -14), acc = (3.0 * dd / 16.0 + 3.0) * std::ldexp(1.0, -22);
    const double ref = (dd + 3.0) * std::ldexp(1.0, -24);
    return metric == 0 ? 2.0 * (split + acc) + std::ldexp(1.0, -19) + ref : split + acc + std::ldexp(1.0, -21) + ref;
}

// fp32 query rows against fp32 base rows. Ids are global (base row r is
// b_id0 + r, query i is q_id0 + i); with exclude_self a query never returns
// its own id. q_row_in_b >= 0: the queries are rows [q_row_in_b, +n_q) of the
// base itself, whose hi/lo planes then serve both sides.
struct F32Sets {
    const float* q;
    uint64_t n_q, q_id0;
    const float* b;
    uint64_t n_b, b_id0;
    int exclude_self;
    int64_t q_row_in_b;
};

knng_gpu_status knn_f32_sets_impl(const F32Sets& z, uint64_t d, uint64_t k, int metric, uint32_t* ids, float* dists,
                                  void* scratch, uint64_t scratch_bytes, cudaStream_t st, knng_gpu_stats* stats)
{
    const bool separate = z.q_row_in_b < 0;
    const ScratchF32 sc = layout_scratch_f32_sets(scratch, z.n_b, z.n_q, d, k, z.exclude_self, separate);
    if (scratch_bytes < sc.total || (reinterpret_cast<uintptr_t>(scratch) & 255))
        return fail(KNNG_GPU_WORKSPACE_TOO_SMALL, "knng::gpu: fp32 scratch smaller than knng_gpu_knn_f32_scratch_bytes");
    if (z.n_q == 0) return KNNG_GPU_OK;
    if (z.n_b < k + (z.exclude_self ? 1 : 0)) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: fewer base rows than k");
    const uint64_t pitch = f32_pitch_elems(d);
    const uint64_t c = f32_candidates_sets(z.n_b, z.exclude_self, k);
    const uint32_t kchunks = static_cast<uint32_t>(pitch * 2 / kChunkBytes);
    EventTimer tk(stats != nullptr, 2), tf(stats != nullptr, 3);
    tk.start(st);
    KNNG_CUDA(cudaMemsetAsync(sc.counters, 0, 16, st));
    KNNG_CUDA(cudaMemsetAsync(sc.max_norm_bits, 0, 4, st));
    uint32_t launches = 0;
    if (metric == 0) {
        // L2 is translation invariant: centre both sets on the base's mean to
        // shrink the error bound.
        KNNG_CUDA(cudaMemsetAsync(sc.sums, 0, d * 8, st));
        column_sum_kernel<<<static_cast<uint32_t>((z.n_b + 255) / 256), 256, 0, st>>>(z.b, z.n_b,
                                                                                     static_cast<uint32_t>(d), sc.sums);
        column_mean_kernel<<<static_cast<uint32_t>((d + 255) / 256), 256, 0, st>>>(sc.sums, z.n_b,
                                                                                  static_cast<uint32_t>(d), sc.mu);
        launches += 2;
    }
    {
        // R = max |r'| over the base rows only (the proof's bound).
        const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((z.n_b + 7) / 8, 148ull * 16));
        split_bf16_kernel<<<blocks, 256, 0, st>>>(z.b, z.n_b, static_cast<uint32_t>(d), static_cast<uint32_t>(pitch),
                                                  metric == 0 ? sc.mu : nullptr, sc.hi, sc.lo, sc.norms,
                                                  sc.max_norm_bits);
        KNNG_CUDA(cudaGetLastError());
        launches += 1;
        if (separate) {
            // The queries' planes; their maximum norm goes to a throwaway slot.
            const uint32_t qb = static_cast<uint32_t>(std::min<uint64_t>((z.n_q + 7) / 8, 148ull * 16));
            split_bf16_kernel<<<qb, 256, 0, st>>>(z.q, z.n_q, static_cast<uint32_t>(d), static_cast<uint32_t>(pitch),
                                                  metric == 0 ? sc.mu : nullptr, sc.q_hi, sc.q_lo, sc.q_norms,
                                                  sc.counters + 3);
            KNNG_CUDA(cudaGetLastError());
            launches += 1;
        }
    }
    // Candidate filter on the tensor cores.
    TcMaps m;
    KNNG_TRY(make_map(&m.b0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, sc.hi, z.n_b, pitch, pitch * 2));
    KNNG_TRY(make_map(&m.b1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, sc.lo, z.n_b, pitch, pitch * 2));
    if (separate) {
        KNNG_TRY(make_map(&m.q0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, sc.q_hi, z.n_q, pitch, pitch * 2));
        KNNG_TRY(make_map(&m.q1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, sc.q_lo, z.n_q, pitch, pitch * 2));
    } else {
        m.q0 = m.b0;
        m.q1 = m.b1;
    }
    KnnTcParams p{};
    p.base_norms = sc.norms;
    p.n_base = z.n_b;
    p.base_id0 = static_cast<uint32_t>(z.b_id0);
    p.n_queries = static_cast<uint32_t>(z.n_q);
    p.query_row0 = separate ? 0u : static_cast<uint32_t>(z.q_row_in_b);
    p.query_id0 = static_cast<uint32_t>(z.q_id0);
    p.exclude_self = z.exclude_self;
    p.k = static_cast<uint32_t>(c);
    p.kchunks = kchunks;
    p.out_ids = sc.cand_ids;
    p.out_keys = sc.cand_keys;
    p.error = reinterpret_cast<int*>(sc.counters + 1);
    if (const char* dbg = experiment_knob("KNNG_GPU_DEBUG_FLAGS")) p.debug_flags = static_cast<uint32_t>(std::atoi(dbg));
    bool a_stream = false;
    p.stages = pick_stages(2, 1, false, kchunks);
    if (p.stages < 2) {
        a_stream = true;
        p.stages = pick_stages(2, 1, true, kchunks);
    }
    if (p.stages < 2) return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: shared memory budget exceeded");
    knng_gpu_status s;
    EventTimer tt(stats != nullptr, 4);
    tt.start(st);
    if (a_stream)
        s = metric == 0 ? launch_bf16_k<true, 0>(m, p, st) : launch_bf16_k<true, 1>(m, p, st);
    else
        s = metric == 0 ? launch_bf16_k<false, 0>(m, p, st) : launch_bf16_k<false, 1>(m, p, st);
    tt.stop(st);
    KNNG_TRY(s);
    // Exact re-rank of the candidates with the proof of exactness.
    RerankParams r{};
    r.x = z.b;
    r.qx = z.q;
    r.d = d;
    r.n_b = z.n_b;
    r.base_id0 = static_cast<uint32_t>(z.b_id0);
    r.query_id0 = static_cast<uint32_t>(z.q_id0);
    r.exclude_self = z.exclude_self;
    r.n_queries = static_cast<uint32_t>(z.n_q);
    r.c = static_cast<uint32_t>(c);
    r.k = static_cast<uint32_t>(k);
    r.cand_ids = sc.cand_ids;
    r.cand_keys = sc.cand_keys;
    r.q_norms = separate ? sc.q_norms : sc.norms + z.q_row_in_b;
    r.max_norm_bits = sc.max_norm_bits;
    r.gamma = f32_gamma(d, metric);
    r.out_ids = ids;
    r.out_dists = dists;
    r.fallback_rows = sc.fallback_rows;
    r.fallback_count = sc.counters;
    r.err_ratio_bits = sc.counters + 2;
    {
        const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((z.n_q + kRerankWarps - 1) / kRerankWarps,
                                                                         148ull * 8));
        const uint32_t cpl = static_cast<uint32_t>((c + 31) / 32);
        if (cpl <= 2)
            metric == 0 ? rerank_kernel<0, 2><<<blocks, 32 * kRerankWarps, 0, st>>>(r)
                        : rerank_kernel<1, 2><<<blocks, 32 * kRerankWarps, 0, st>>>(r);
        else if (cpl <= 8)
            metric == 0 ? rerank_kernel<0, 8><<<blocks, 32 * kRerankWarps, 0, st>>>(r)
                        : rerank_kernel<1, 8><<<blocks, 32 * kRerankWarps, 0, st>>>(r);
        else
            metric == 0 ? rerank_kernel<0, 34><<<blocks, 32 * kRerankWarps, 0, st>>>(r)
                        : rerank_kernel<1, 34><<<blocks, 32 * kRerankWarps, 0, st>>>(r);
        KNNG_CUDA(cudaGetLastError());
        launches += 2;
    }
    tk.stop(st);
    // Rows the proof could not certify: exact kernel on the original rows.
    tf.start(st);
    KnnExactParams<float> e{};
    e.base = z.b;
    e.base_stride = d;
    e.n_base = z.n_b;
    e.base_id0 = static_cast<uint32_t>(z.b_id0);
    e.queries = z.q;
    e.query_stride = d;
    e.n_queries = static_cast<uint32_t>(z.n_q);
    e.query_id0 = static_cast<uint32_t>(z.q_id0);
    e.exclude_self = z.exclude_self;
    e.d = static_cast<uint32_t>(d);
    e.k = static_cast<uint32_t>(k);
    e.row_list = sc.fallback_rows;
    e.row_count = sc.counters;
    e.out_ids = ids;
    e.out_dists = dists;
    KNNG_TRY(launch_exact(e, metric, static_cast<uint32_t>(z.n_q), st));
    tf.stop(st);
    launches += 1;
    uint32_t host_counters[3] = {0, 0, 0};
    KNNG_CUDA(cudaMemcpyAsync(host_counters, sc.counters, 12, cudaMemcpyDeviceToHost, st));
    KNNG_CUDA(cudaStreamSynchronize(st));
    if (host_counters[1] != 0)
        return fail(KNNG_GPU_TIMEOUT, "knng::gpu: a bounded device wait gave up (code " +
                                          std::to_string(host_counters[1]) + ")");
    if (stats) {
        float ratio;
        std::memcpy(&ratio, &host_counters[2], 4);
        stats->f32_err_ratio = ratio;
        stats->tc_ms = tt.ms();
        stats->path = KNNG_PATH_F32_TENSOR;
        stats->fallback_rows = host_counters[0];
        stats->knn_ms = tk.ms();
        stats->fallback_ms = tf.ms();
        stats->kernel_launches += launches;
    }
    return KNNG_GPU_OK;
}

knng_gpu_status knn_f32_impl(const float* x, uint64_t n, uint64_t d, uint64_t q_begin, uint64_t q_count, uint64_t k,
                             int metric, uint32_t* ids, float* dists, void* scratch, uint64_t scratch_bytes,
                             cudaStream_t st, knng_gpu_stats* stats)
{
    if (q_begin + q_count > n) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: query range exceeds the base");
    const F32Sets z{x + q_begin * d, q_count, q_begin, x, n, 0, 1, static_cast<int64_t>(q_begin)};
    return knn_f32_sets_impl(z, d, k, metric, ids, dists, scratch, scratch_bytes, st, stats);
}

// Recall of an approximate graph against the true one
// (src/bench/recall.cpp:52-96): per row, the distinct ids of the approximate
// row that also appear in the true row; a repeated approximate id counts
// once. One warp per row; lane l looks at entries l, l + 32, ...
__global__ void __launch_bounds__(256) recall_hits_kernel(const uint32_t* __restrict__ approx,
                                                          const uint32_t* __restrict__ truth, uint64_t n, uint32_t k,
                                                          unsigned long long* __restrict__ hits)
{
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t warp0 = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (static_cast<uint64_t>(gridDim.x) * blockDim.x) >> 5;
    unsigned long long local = 0;
    for (uint64_t r = warp0; r < n; r += nwarps) {
        const uint32_t* a = approx + r * k;
        const uint32_t* t = truth + r * k;
        for (uint32_t j = lane; j < k; j += 32) {
            const uint32_t id = a[j];
            bool first = true;
            for (uint32_t i = 0; i < j && first; ++i) first = a[i] != id;
            if (!first) continue;
            bool found = false;
            for (uint32_t i = 0; i < k && !found; ++i) found = t[i] == id;
            local += found ? 1ull : 0ull;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
    if (lane == 0 && local) atomicAdd(hits, local);
}

struct WorkspaceLayout {
    uint64_t packed, norms, flag, scratch, total;
};

// The u8 path and the fp32 path share one workspace (only one of them runs).
WorkspaceLayout workspace_layout(uint64_t n, uint64_t d, uint64_t k)
{
    WorkspaceLayout w;
    const uint64_t pitch = knng_gpu_padded_dim(d);
    w.packed = 0;
    w.norms = align_up(w.packed + n * pitch, 256);
    w.flag = align_up(w.norms + n * 4, 256);
    w.scratch = w.flag + 256;
    const uint64_t u8_total = w.scratch + scratch_u8_bytes(n, k);
    const uint64_t f32_total = w.scratch + layout_scratch_f32(nullptr, n, d, n, k).total;
    w.total = std::max(u8_total, f32_total);
    return w;
}

knng_gpu_status pack_impl(const float* x, uint64_t rows, uint64_t d, uint8_t* packed, int32_t* norms,
                          int32_t* nonint, cudaStream_t st)
{
    if (rows == 0) return KNNG_GPU_OK;
    const uint64_t pitch = knng_gpu_padded_dim(d);
    const uint64_t data_bytes = u8_data_bytes(d);
    const uint64_t warps_needed = rows;
    const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((warps_needed + 7) / 8, 148ull * 16));
    pack_u8_kernel<<<blocks, 256, 0, st>>>(x, rows, static_cast<uint32_t>(d), static_cast<uint32_t>(data_bytes),
                                          static_cast<uint32_t>(pitch), packed, norms, nonint);
    KNNG_CUDA(cudaGetLastError());
    pack_aug_kernel<<<static_cast<uint32_t>((rows + 127) / 128), 128, 0, st>>>(
        rows, static_cast<uint32_t>(data_bytes), static_cast<uint32_t>(pitch), packed, norms);
    KNNG_CUDA(cudaGetLastError());
    return KNNG_GPU_OK;
}

knng_gpu_status pack_bytes_impl(const uint8_t* rows_u8, uint64_t rows, uint64_t d, uint64_t row_stride,
                                uint8_t* packed, int32_t* norms, cudaStream_t st)
{
    if (rows == 0) return KNNG_GPU_OK;
    const uint64_t pitch = knng_gpu_padded_dim(d);
    const uint64_t data_bytes = u8_data_bytes(d);
    const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((rows + 7) / 8, 148ull * 16));
    pack_u8_bytes_kernel<<<blocks, 256, 0, st>>>(rows_u8, rows, static_cast<uint32_t>(d), row_stride,
                                                static_cast<uint32_t>(data_bytes), static_cast<uint32_t>(pitch),
                                                packed, norms);
    KNNG_CUDA(cudaGetLastError());
    pack_aug_kernel<<<static_cast<uint32_t>((rows + 127) / 128), 128, 0, st>>>(
        rows, static_cast<uint32_t>(data_bytes), static_cast<uint32_t>(pitch), packed, norms);
    KNNG_CUDA(cudaGetLastError());
    return KNNG_GPU_OK;
}

// Build from u8 rows already on the device (row_stride bytes apart).
knng_gpu_status device_pipeline_u8(const uint8_t* rows_u8, uint64_t n, uint64_t d, uint64_t row_stride, uint64_t k,
                                   int metric, uint32_t* ids, float* dists, void* ws, uint64_t ws_bytes,
                                   cudaStream_t st, knng_gpu_stats* stats)
{
    KNNG_TRY(validate(n, d, k, metric));
    if (row_stride < d) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: row_stride must be >= d");
    const WorkspaceLayout w = workspace_layout(n, d, k);
    if (ws_bytes < w.total || (reinterpret_cast<uintptr_t>(ws) & 255))
        return fail(KNNG_GPU_WORKSPACE_TOO_SMALL, "knng::gpu: workspace smaller than knng_gpu_workspace_bytes or "
                                                  "not 256-byte aligned");
    uint8_t* base = static_cast<uint8_t*>(ws);
    uint8_t* packed = base + w.packed;
    int32_t* norms = reinterpret_cast<int32_t*>(base + w.norms);
    EventTimer tall(stats != nullptr, 0), tp(stats != nullptr, 1);
    tall.start(st);
    tp.start(st);
    KNNG_TRY(pack_bytes_impl(rows_u8, n, d, row_stride, packed, norms, st));
    tp.stop(st);
    if (stats) {
        std::memset(stats, 0, sizeof(*stats));
        stats->kernel_launches = 2;  // pack + augmentation
    }
    KNNG_TRY(knn_u8_impl(packed, norms, n, d, 0, n, k, metric, ids, dists, base + w.scratch, w.total - w.scratch, st,
                         stats));
    tall.stop(st);
    if (stats) {
        stats->pack_ms = tp.ms();
        stats->total_ms = tall.ms();
    }
    return KNNG_GPU_OK;
}

knng_gpu_status device_pipeline(const float* x, uint64_t n, uint64_t d, uint64_t k, int metric, uint32_t* ids,
                                float* dists, void* ws, uint64_t ws_bytes, cudaStream_t st, knng_gpu_stats* stats)
{
    KNNG_TRY(validate(n, d, k, metric));
    const WorkspaceLayout w = workspace_layout(n, d, k);
    if (ws_bytes < w.total || (reinterpret_cast<uintptr_t>(ws) & 255))
        return fail(KNNG_GPU_WORKSPACE_TOO_SMALL, "knng::gpu: workspace smaller than knng_gpu_workspace_bytes or "
                                                  "not 256-byte aligned");
    uint8_t* base = static_cast<uint8_t*>(ws);
    uint8_t* packed = base + w.packed;
    int32_t* norms = reinterpret_cast<int32_t*>(base + w.norms);
    int32_t* flag = reinterpret_cast<int32_t*>(base + w.flag);
    EventTimer tall(stats != nullptr, 0), tp(stats != nullptr, 1);
    tall.start(st);
    tp.start(st);
    KNNG_CUDA(cudaMemsetAsync(flag, 0, 4, st));
    KNNG_TRY(pack_impl(x, n, d, packed, norms, flag, st));
    tp.stop(st);
    if (stats) {
        std::memset(stats, 0, sizeof(*stats));
        stats->kernel_launches = 2;  // pack + augmentation
    }
    U8RunOptions opt;
    opt.skip_flag = flag;
    // The tensor-core kernels read the flag and return at once for data that
    // is not integer-valued; the exact-only path (d > 1024) cannot skip.
    const bool pair = d <= kMaxTensorDim;
    int32_t nonint = 0;
    if (!pair) {
        KNNG_CUDA(cudaMemcpyAsync(&nonint, flag, 4, cudaMemcpyDeviceToHost, st));
        KNNG_CUDA(cudaStreamSynchronize(st));
    }
    if (nonint == 0) {
        // The pair kernel returns at once when the flag is set; the flag is
        // read after it, together with its counters.
        KNNG_TRY(knn_u8_impl(packed, norms, n, d, 0, n, k, metric, ids, dists, base + w.scratch, w.total - w.scratch,
                             st, stats, opt));
        if (pair) {
            KNNG_CUDA(cudaMemcpyAsync(&nonint, flag, 4, cudaMemcpyDeviceToHost, st));
            KNNG_CUDA(cudaStreamSynchronize(st));
        }
    }
    if (nonint != 0) {
        // The packed bytes are meaningless for such data; the fp32 path
        // reuses the whole workspace.
        if (stats) stats->kernel_launches = 2;
        KNNG_TRY(knn_f32_impl(x, n, d, 0, n, k, metric, ids, dists, base, w.total, st, stats));
    }
    tall.stop(st);
    if (stats) {
        stats->pack_ms = tp.ms();
        stats->total_ms = tall.ms();
    }
    return KNNG_GPU_OK;
}

}  // namespace

// ------------------------------------------------------------------ no-alloc scratch
// Scratch of knng_gpu_knn_u8_noalloc: the fallback-row list for up to
// KNNG_GPU_NOALLOC_MAX_QUERIES queries plus the counters. Host code must not
// pass `g_noalloc_scratch` itself to a kernel (on the host it names a host
// stand-in); noalloc_scratch_ptr() resolves the device address.
constexpr uint64_t kNoAllocScratchBytes = (static_cast<uint64_t>(KNNG_GPU_NOALLOC_MAX_QUERIES) * 4 + 255) / 256 * 256 + 256;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
// The address of a __device__ array belongs to a CUDA context, not to a
// device number, and a host may make a non-primary context current (or
// destroy one and get a new context with a recycled handle). So the address
// is resolved on every call, in whatever context is current; once the module
// is loaded in that context this is a table lookup and allocates nothing.
knng_gpu_status noalloc_scratch_ptr(void** out)
{
    KNNG_CUDA(cudaGetSymbolAddress(out, g_noalloc_scratch));
    return KNNG_GPU_OK;
}
}  // namespace

// ------------------------------------------------------------------ host-API buffer cache
// knng_gpu_brute_force keeps its device buffers and stream per device between
// calls (grown on demand, freed by knng_gpu_release_cached_buffers), so a
// build pays no cudaMalloc/cudaFree once the sizes have been seen.
namespace {
// Host buffers the caller did not pin (plain malloc / numpy / std::vector
// memory) go through a ring of pinned chunks: the DMA engine moves chunk i
// while host threads copy chunk i +- 1 between the caller's memory and the
// ring. A device-to-host copy straight into freshly allocated pageable memory
// runs at the page-fault rate of one thread (~4 GB/s measured on the B200
// hosts, against ~55 GB/s pinned); the threads fault the pages in parallel.
constexpr uint64_t kStageChunk = 32ull << 20;
constexpr int kStageSlots = 4;

struct HostStage {
    uint8_t* ring = nullptr;  // kStageSlots x kStageChunk pinned bytes
    cudaEvent_t ev[kStageSlots] = {};
};

bool host_is_pinned(const void* p)
{
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

// memcpy of `bytes` split over up to 8 host threads (the calling thread
// takes the first share).
void parallel_memcpy(void* dst, const void* src, uint64_t bytes)
{
    const unsigned hw = std::thread::hardware_concurrency();
    const uint64_t parts = std::max<uint64_t>(1, std::min<uint64_t>({8, hw ? hw : 1, bytes >> 20}));
    const uint64_t per = (bytes + parts - 1) / parts;
    auto piece = [&](uint64_t i) {
        const uint64_t lo = i * per, hi = std::min(bytes, lo + per);
        if (lo < hi) std::memcpy(static_cast<uint8_t*>(dst) + lo, static_cast<const uint8_t*>(src) + lo, hi - lo);
    };
    std::vector<std::thread> th;
    th.reserve(parts - 1);
    for (uint64_t i = 1; i < parts; ++i) th.emplace_back(piece, i);
    piece(0);
    for (auto& t : th) t.join();
}

knng_gpu_status stage_ready(HostStage& s)
{
    if (!s.ring) {
        KNNG_CUDA(cudaMallocHost(reinterpret_cast<void**>(&s.ring), kStageSlots * kStageChunk));
        for (auto& e : s.ev) KNNG_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    // A previous call's DMAs may still read or fill the ring.
    for (auto& e : s.ev) KNNG_CUDA(cudaEventSynchronize(e));
    return KNNG_GPU_OK;
}

void stage_release(HostStage& s)
{
    if (!s.ring) return;
    for (auto& e : s.ev) {
        cudaEventSynchronize(e);
        cudaEventDestroy(e);
        e = nullptr;
    }
    cudaFreeHost(s.ring);
    s.ring = nullptr;
}

// Host -> device on `st`. Pinned (or small) sources are copied directly.
knng_gpu_status copy_to_device(HostStage& s, void* dst, const void* src, uint64_t bytes, cudaStream_t st)
{
    if (bytes == 0) return KNNG_GPU_OK;
    if (bytes < (4ull << 20) || host_is_pinned(src)) {
        KNNG_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, st));
        return KNNG_GPU_OK;
    }
    KNNG_TRY(stage_ready(s));
    const uint64_t nch = (bytes + kStageChunk - 1) / kStageChunk;
    for (uint64_t i = 0; i < nch; ++i) {
        const int slot = static_cast<int>(i % kStageSlots);
        const uint64_t off = i * kStageChunk, len = std::min(kStageChunk, bytes - off);
        if (i >= kStageSlots) KNNG_CUDA(cudaEventSynchronize(s.ev[slot]));  // chunk i - slots has left the slot
        parallel_memcpy(s.ring + slot * kStageChunk, static_cast<const uint8_t*>(src) + off, len);
        KNNG_CUDA(cudaMemcpyAsync(static_cast<uint8_t*>(dst) + off, s.ring + slot * kStageChunk, len,
                                  cudaMemcpyHostToDevice, st));
        KNNG_CUDA(cudaEventRecord(s.ev[slot], st));
    }
    return KNNG_GPU_OK;
}

// Device -> host after the work queued on `st`; the data is in `dst` when
// this returns (pinned destinations: once `st` is synchronised).
knng_gpu_status copy_to_host(HostStage& s, void* dst, const void* src, uint64_t bytes, cudaStream_t st)
{
    if (bytes == 0) return KNNG_GPU_OK;
    if (bytes < (4ull << 20) || host_is_pinned(dst)) {
        KNNG_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, st));
        return KNNG_GPU_OK;
    }
    KNNG_TRY(stage_ready(s));
    const uint64_t nch = (bytes + kStageChunk - 1) / kStageChunk;
    auto issue = [&](uint64_t i) -> knng_gpu_status {
        const int slot = static_cast<int>(i % kStageSlots);
        const uint64_t off = i * kStageChunk, len = std::min(kStageChunk, bytes - off);
        KNNG_CUDA(cudaMemcpyAsync(s.ring + slot * kStageChunk, static_cast<const uint8_t*>(src) + off, len,
                                  cudaMemcpyDeviceToHost, st));
        KNNG_CUDA(cudaEventRecord(s.ev[slot], st));
        return KNNG_GPU_OK;
    };
    for (uint64_t i = 0; i < nch && i < kStageSlots; ++i) KNNG_TRY(issue(i));
    for (uint64_t i = 0; i < nch; ++i) {
        const int slot = static_cast<int>(i % kStageSlots);
        const uint64_t off = i * kStageChunk, len = std::min(kStageChunk, bytes - off);
        KNNG_CUDA(cudaEventSynchronize(s.ev[slot]));
        parallel_memcpy(static_cast<uint8_t*>(dst) + off, s.ring + slot * kStageChunk, len);
        if (i + kStageSlots < nch) KNNG_TRY(issue(i + kStageSlots));
    }
    return KNNG_GPU_OK;
}

struct HostCache {
    std::mutex mutex;
    int device = 0;
    cudaStream_t stream = nullptr;
    void *x = nullptr, *ids = nullptr, *dists = nullptr, *ws = nullptr;
    uint64_t x_cap = 0, ids_cap = 0, dists_cap = 0, ws_cap = 0;
    HostStage stage;
};
HostCache g_host_cache[kMaxDevices];

knng_gpu_status grow(void** ptr, uint64_t* cap, uint64_t need)
{
    if (*cap >= need && *ptr) return KNNG_GPU_OK;
    if (*ptr) cudaFree(*ptr);
    *ptr = nullptr;
    *cap = 0;
    KNNG_CUDA(cudaMalloc(ptr, need > 0 ? need : 256));
    *cap = need;
    return KNNG_GPU_OK;
}
}  // namespace

extern "C" {

const char* knng_gpu_last_error(void) { return g_last_error.c_str(); }

int knng_gpu_device_count(void)
{
    int c = 0;
    if (cudaGetDeviceCount(&c) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return c;
}

uint64_t knng_gpu_padded_dim(uint64_t d) { return u8_data_bytes(d) + kAugBytes; }

uint64_t knng_gpu_workspace_bytes(uint64_t n, uint64_t d, uint64_t k) { return workspace_layout(n, d, k).total; }

uint64_t knng_gpu_knn_f32_scratch_bytes(uint64_t n, uint64_t d, uint64_t q_count, uint64_t k)
{
    return layout_scratch_f32(nullptr, n, d, q_count, k).total;
}

uint64_t knng_gpu_knn_scratch_bytes(uint64_t q_count, uint64_t k) { return scratch_u8_bytes(q_count, k); }

knng_gpu_status knng_gpu_pack_u8(const float* d_x, uint64_t rows, uint64_t d, uint8_t* d_packed, int32_t* d_norms,
                                 int32_t* d_nonint, void* stream)
{
    g_last_error.clear();
    if (d == 0) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: d must be > 0");
    return pack_impl(d_x, rows, d, d_packed, d_norms, d_nonint, static_cast<cudaStream_t>(stream));
}

knng_gpu_status knng_gpu_knn_u8(const uint8_t* d_packed, const int32_t* d_norms, uint64_t n, uint64_t d,
                                uint64_t q_begin, uint64_t q_count, uint64_t k, int metric, uint32_t* d_ids,
                                float* d_dists, void* d_scratch, uint64_t scratch_bytes, void* stream,
                                knng_gpu_stats* stats)
{
    g_last_error.clear();
    KNNG_TRY(validate(n, d, k, metric));
    return knn_u8_impl(d_packed, d_norms, n, d, q_begin, q_count, k, metric, d_ids, d_dists, d_scratch,
                       scratch_bytes, static_cast<cudaStream_t>(stream), stats);
}

knng_gpu_status knng_gpu_knn_f32(const float* d_x, uint64_t n, uint64_t d, uint64_t q_begin, uint64_t q_count,
                                 uint64_t k, int metric, uint32_t* d_ids, float* d_dists, void* d_scratch,
                                 uint64_t scratch_bytes, void* stream, knng_gpu_stats* stats)
{
    g_last_error.clear();
    KNNG_TRY(validate(n, d, k, metric));
    return knn_f32_impl(d_x, n, d, q_begin, q_count, k, metric, d_ids, d_dists, d_scratch, scratch_bytes,
                        static_cast<cudaStream_t>(stream), stats);
}

knng_gpu_status knng_gpu_brute_force_device(const float* d_data, uint64_t n, uint64_t d, uint64_t k, int metric,
                                            uint32_t* d_ids, float* d_dists, void* d_workspace,
                                            uint64_t workspace_bytes, void* stream, knng_gpu_stats* stats)
{
    g_last_error.clear();
    return device_pipeline(d_data, n, d, k, metric, d_ids, d_dists, d_workspace, workspace_bytes,
                           static_cast<cudaStream_t>(stream), stats);
}

knng_gpu_status knng_gpu_brute_force(const float* data, uint64_t n, uint64_t d, uint64_t k, int metric,
                                     uint32_t* ids, float* dists, knng_gpu_stats* stats)
{
    g_last_error.clear();
    KNNG_TRY(validate(n, d, k, metric));
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(KNNG_GPU_CUDA_ERROR, "knng::gpu::brute_force_knn: no CUDA device available");
    }
    int dev = 0;
    KNNG_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: device index out of range");
    HostCache& c = g_host_cache[dev];
    std::lock_guard<std::mutex> lock(c.mutex);
    c.device = dev;
    if (!c.stream) KNNG_CUDA(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
    cudaStream_t st = c.stream;
    const uint64_t ws_bytes = knng_gpu_workspace_bytes(n, d, k);
    KNNG_TRY(grow(&c.x, &c.x_cap, n * d * sizeof(float)));
    KNNG_TRY(grow(&c.ids, &c.ids_cap, n * k * sizeof(uint32_t)));
    KNNG_TRY(grow(&c.dists, &c.dists_cap, n * k * sizeof(float)));
    KNNG_TRY(grow(&c.ws, &c.ws_cap, ws_bytes));
    float* dx = static_cast<float*>(c.x);
    uint32_t* dids = static_cast<uint32_t*>(c.ids);
    float* ddist = static_cast<float*>(c.dists);
    KNNG_TRY(copy_to_device(c.stage, dx, data, n * d * sizeof(float), st));
    KNNG_TRY(device_pipeline(dx, n, d, k, metric, dids, ddist, c.ws, c.ws_cap, st, stats));
    KNNG_TRY(copy_to_host(c.stage, ids, dids, n * k * sizeof(uint32_t), st));
    KNNG_TRY(copy_to_host(c.stage, dists, ddist, n * k * sizeof(float), st));
    KNNG_CUDA(cudaStreamSynchronize(st));
    return KNNG_GPU_OK;
}

knng_gpu_status knng_gpu_pack_u8_bytes(const uint8_t* d_rows, uint64_t rows, uint64_t d, uint64_t row_stride,
                                       uint8_t* d_packed, int32_t* d_norms, void* stream)
{
    g_last_error.clear();
    if (d == 0) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: d must be > 0");
    if (row_stride < d) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: row_stride must be >= d");
    return pack_bytes_impl(d_rows, rows, d, row_stride, d_packed, d_norms, static_cast<cudaStream_t>(stream));
}

knng_gpu_status knng_gpu_brute_force_u8(const uint8_t* rows, uint64_t n, uint64_t d, uint64_t row_stride, uint64_t k,
                                        int metric, uint32_t* ids, float* dists, knng_gpu_stats* stats)
{
    g_last_error.clear();
    KNNG_TRY(validate(n, d, k, metric));
    if (row_stride < d) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: row_stride must be >= d");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(KNNG_GPU_CUDA_ERROR, "knng::gpu::brute_force_knn: no CUDA device available");
    }
    int dev = 0;
    KNNG_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: device index out of range");
    HostCache& c = g_host_cache[dev];
    std::lock_guard<std::mutex> lock(c.mutex);
    c.device = dev;
    if (!c.stream) KNNG_CUDA(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
    cudaStream_t st = c.stream;
    // The last row needs only d bytes: a .bvecs buffer minus its final header.
    const uint64_t in_bytes = (n - 1) * row_stride + d;
    const uint64_t ws_bytes = knng_gpu_workspace_bytes(n, d, k);
    KNNG_TRY(grow(&c.x, &c.x_cap, in_bytes));
    KNNG_TRY(grow(&c.ids, &c.ids_cap, n * k * sizeof(uint32_t)));
    KNNG_TRY(grow(&c.dists, &c.dists_cap, n * k * sizeof(float)));
    KNNG_TRY(grow(&c.ws, &c.ws_cap, ws_bytes));
    uint8_t* dx = static_cast<uint8_t*>(c.x);
    uint32_t* dids = static_cast<uint32_t*>(c.ids);
    float* ddist = static_cast<float*>(c.dists);
    KNNG_TRY(copy_to_device(c.stage, dx, rows, in_bytes, st));
    KNNG_TRY(device_pipeline_u8(dx, n, d, row_stride, k, metric, dids, ddist, c.ws, c.ws_cap, st, stats));
    KNNG_TRY(copy_to_host(c.stage, ids, dids, n * k * sizeof(uint32_t), st));
    KNNG_TRY(copy_to_host(c.stage, dists, ddist, n * k * sizeof(float), st));
    KNNG_CUDA(cudaStreamSynchronize(st));
    return KNNG_GPU_OK;
}

void knng_gpu_release_cached_buffers(void)
{
    int cur = 0;
    const bool have_cur = cudaGetDevice(&cur) == cudaSuccess;
    for (int i = 0; i < kMaxDevices; ++i) {
        HostCache& c = g_host_cache[i];
        std::lock_guard<std::mutex> lock(c.mutex);
        if (!c.stream && !c.x && !c.ws && !c.stage.ring) continue;
        cudaSetDevice(c.device);
        stage_release(c.stage);
        cudaFree(c.x);
        cudaFree(c.ids);
        cudaFree(c.dists);
        cudaFree(c.ws);
        if (c.stream) cudaStreamDestroy(c.stream);
        c.x = c.ids = c.dists = c.ws = nullptr;
        c.x_cap = c.ids_cap = c.dists_cap = c.ws_cap = 0;
        c.stream = nullptr;
    }
    if (have_cur) cudaSetDevice(cur);
    cudaGetLastError();
}

knng_gpu_status knng_gpu_knn_u8_noalloc(const uint8_t* d_packed, const int32_t* d_norms, uint64_t n, uint64_t d,
                                        uint64_t q_begin, uint64_t q_count, uint64_t k, int metric, uint32_t* d_ids,
                                        float* d_dists, void* stream, knng_gpu_stats* stats)
{
    g_last_error.clear();
    KNNG_TRY(validate(n, d, k, metric));
    if (q_count > KNNG_GPU_NOALLOC_MAX_QUERIES)
        return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: knng_gpu_knn_u8_noalloc handles at most " +
                                                   std::to_string(KNNG_GPU_NOALLOC_MAX_QUERIES) +
                                                   " queries per call (got " + std::to_string(q_count) + ")");
    void* scratch = nullptr;
    KNNG_TRY(noalloc_scratch_ptr(&scratch));
    // knn_u8_impl zeroes the counters on `stream` before the kernel runs, so
    // the previous call's contents never leak into this one. The array has
    // no room for the pair kernel's partial lists, so the single-CTA kernel
    // runs; no timing events are recorded (the *_ms fields of stats stay 0).
    U8RunOptions opt;
    opt.allow_pair = false;
    opt.timing = false;
    if (stats) std::memset(stats, 0, sizeof(*stats));
    return knn_u8_impl(d_packed, d_norms, n, d, q_begin, q_count, k, metric, d_ids, d_dists, scratch,
                       kNoAllocScratchBytes, static_cast<cudaStream_t>(stream), stats, opt);
}

knng_gpu_status knng_gpu_selftest_bounded_wait(uint64_t wait_limit_cycles)
{
    g_last_error.clear();
    // A small, valid build (every row of bytes 1..n) whose pair kernel runs
    // with the given wait bound while the leader CTAs withhold the arrival
    // of their first stage: the MMA waits give up, the kernel unwinds and
    // frees its TMEM, and the call must report KNNG_GPU_TIMEOUT.
    const uint64_t n = 4096, d = 128, k = 10;
    const uint64_t pitch = knng_gpu_padded_dim(d);
    uint8_t *rows = nullptr, *packed = nullptr, *scratch = nullptr;
    int32_t* norms = nullptr;
    uint32_t* ids = nullptr;
    float* dists = nullptr;
    const uint64_t sbytes = scratch_u8_bytes(n, k);
    struct Free {
        void* p[6];
        ~Free()
        {
            for (void* q : p)
                if (q) cudaFree(q);
        }
    } guard{};
    KNNG_CUDA(cudaMalloc(&rows, n * d));
    guard.p[0] = rows;
    KNNG_CUDA(cudaMalloc(&packed, n * pitch));
    guard.p[1] = packed;
    KNNG_CUDA(cudaMalloc(&norms, n * 4));
    guard.p[2] = norms;
    KNNG_CUDA(cudaMalloc(&ids, n * k * 4));
    guard.p[3] = ids;
    KNNG_CUDA(cudaMalloc(&dists, n * k * 4));
    guard.p[4] = dists;
    KNNG_CUDA(cudaMalloc(&scratch, sbytes));
    guard.p[5] = scratch;
    KNNG_CUDA(cudaMemset(rows, 1, n * d));
    KNNG_TRY(pack_bytes_impl(rows, n, d, d, packed, norms, nullptr));
    U8RunOptions opt;
    opt.wait_limit = static_cast<long long>(std::min<uint64_t>(wait_limit_cycles, 1ull << 40));
    opt.test_mode = 1;
    opt.timing = false;
    const U8Sets z{packed, norms, n, 0, packed, norms, n, 0, 1};
    ScratchU8 sc = carve_scratch_u8(scratch, n, k, sbytes);
    if (!pair_applies(z, d, k, 0, sc, opt))
        return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: the pair kernel does not apply on this device");
    const knng_gpu_status s = knn_u8_sets_impl(z, d, k, 0, ids, dists, scratch, sbytes, nullptr, nullptr, opt);
    KNNG_CUDA(cudaDeviceSynchronize());
    return s;
}

knng_gpu_status knng_gpu_knn_u8_sets(const uint8_t* d_q_packed, const int32_t* d_q_norms, uint64_t n_q,
                                     uint64_t q_id0, const uint8_t* d_b_packed, const int32_t* d_b_norms, uint64_t n_b,
                                     uint64_t b_id0, uint64_t d, uint64_t k, int metric, int exclude_self,
                                     uint32_t* d_ids, float* d_dists, void* d_scratch, uint64_t scratch_bytes,
                                     void* stream, knng_gpu_stats* stats)
{
    g_last_error.clear();
    if (k == 0) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu::brute_force_knn: k must be > 0");
    if (k > KNNG_GPU_MAX_K)
        return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: k exceeds the GPU limit " + std::to_string(KNNG_GPU_MAX_K));
    if (metric != KNNG_METRIC_L2_SQUARED && metric != KNNG_METRIC_NEGATIVE_INNER_PRODUCT)
        return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: unknown metric id " + std::to_string(metric));
    if (d == 0 || n_b == 0) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: empty base");
    if (q_id0 + n_q > 0xFFFFFFFFull || b_id0 + n_b > 0xFFFFFFFFull)
        return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: ids exceed the 32-bit index_t range");
    const U8Sets z{d_q_packed, d_q_norms, n_q, q_id0, d_b_packed, d_b_norms, n_b, b_id0, exclude_self ? 1 : 0};
    return knn_u8_sets_impl(z, d, k, metric, d_ids, d_dists, d_scratch, scratch_bytes,
                            static_cast<cudaStream_t>(stream), stats);
}

uint64_t knng_gpu_knn_f32_sets_scratch_bytes(uint64_t n_q, uint64_t n_b, uint64_t d, uint64_t k, int exclude_self)
{
    if (n_b == 0) return 256;
    return layout_scratch_f32_sets(nullptr, n_b, n_q, d, k, exclude_self ? 1 : 0, true).total;
}

knng_gpu_status knng_gpu_knn_f32_sets(const float* d_q, uint64_t n_q, uint64_t q_id0, const float* d_b, uint64_t n_b,
                                      uint64_t b_id0, uint64_t d, uint64_t k, int metric, int exclude_self,
                                      uint32_t* d_ids, float* d_dists, void* d_scratch, uint64_t scratch_bytes,
                                      void* stream, knng_gpu_stats* stats)
{
    g_last_error.clear();
    if (k == 0) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu::brute_force_knn: k must be > 0");
    if (k > KNNG_GPU_MAX_K)
        return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: k exceeds the GPU limit " + std::to_string(KNNG_GPU_MAX_K));
    if (metric != KNNG_METRIC_L2_SQUARED && metric != KNNG_METRIC_NEGATIVE_INNER_PRODUCT)
        return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: unknown metric id " + std::to_string(metric));
    if (d == 0 || n_b == 0) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: empty base");
    if (d > (1u << 20)) return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: d must be in [1, 2^20]");
    if (q_id0 + n_q > 0xFFFFFFFFull || b_id0 + n_b > 0xFFFFFFFFull)
        return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: ids exceed the 32-bit index_t range");
    const F32Sets z{d_q, n_q, q_id0, d_b, n_b, b_id0, exclude_self ? 1 : 0, -1};
    if (stats) std::memset(stats, 0, sizeof(*stats));
    return knn_f32_sets_impl(z, d, k, metric, d_ids, d_dists, d_scratch, scratch_bytes,
                             static_cast<cudaStream_t>(stream), stats);
}

knng_gpu_status knng_gpu_recall_at_k(const uint32_t* d_approx, const uint32_t* d_truth, uint64_t n, uint64_t k,
                                     void* d_counter, void* stream, double* recall)
{
    g_last_error.clear();
    if (!recall) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::bench::recall: recall is NULL");
    if (n == 0) {
        *recall = 1.0;  // src/bench/recall.cpp: an empty graph has recall 1
        return KNNG_GPU_OK;
    }
    if (k == 0 || k > 0xFFFFFFFFull) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::bench::recall: bad k");
    if (!d_counter || (reinterpret_cast<uintptr_t>(d_counter) & 7))
        return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::bench::recall: d_counter must be 8 device bytes, 8-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto* hits = static_cast<unsigned long long*>(d_counter);
    KNNG_CUDA(cudaMemsetAsync(hits, 0, 8, st));
    const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((n + 7) / 8, 148ull * 32));
    recall_hits_kernel<<<blocks, 256, 0, st>>>(d_approx, d_truth, n, static_cast<uint32_t>(k), hits);
    KNNG_CUDA(cudaGetLastError());
    unsigned long long h = 0;
    KNNG_CUDA(cudaMemcpyAsync(&h, hits, 8, cudaMemcpyDeviceToHost, st));
    KNNG_CUDA(cudaStreamSynchronize(st));
    *recall = static_cast<double>(h) / (static_cast<double>(n) * static_cast<double>(k));
    return KNNG_GPU_OK;
}

knng_gpu_status knng_gpu_merge_topk(const uint32_t* d_a_ids, const float* d_a_dists, const uint32_t* d_b_ids,
                                    const float* d_b_dists, uint64_t rows, uint64_t k, uint32_t* d_out_ids,
                                    float* d_out_dists, void* stream)
{
    g_last_error.clear();
    if (rows == 0) return KNNG_GPU_OK;
    merge_topk_kernel<<<static_cast<uint32_t>((rows + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        d_a_ids, d_a_dists, d_b_ids, d_b_dists, rows, static_cast<uint32_t>(k), d_out_ids, d_out_dists);
    KNNG_CUDA(cudaGetLastError());
    return KNNG_GPU_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ multi-GPU builds
#include "sharded.cuh"
