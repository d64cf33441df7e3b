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

#include "knn_exact.cuh"
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
struct ScratchU8 {
    uint32_t* fallback_rows;
    uint32_t* counters;  // [0] fallback count, [1] error flag
};

// Concurrent base ranges for the last partial wave of query tiles.
constexpr int kMaxTailParts = 8;

// Fallback-row list (one entry per query) + 2 counters per launch (at most
// kMaxTailParts + 1 launches: 72 bytes of the 256).
uint64_t scratch_u8_bytes(uint64_t q_count) { return align_up(q_count * 4, 256) + 256; }

ScratchU8 carve_scratch_u8(void* p, uint64_t q_count)
{
    ScratchU8 s;
    s.fallback_rows = static_cast<uint32_t*>(p);
    s.counters = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(p) + align_up(q_count * 4, 256));
    return s;
}

struct TcMaps {
    CUtensorMap q0, q1, b0, b1;
};

template <class Elem, int MT, int NBUF, bool A_STREAM, int METRIC, class TopK, int SPLIT = 1>
knng_gpu_status launch_tc_t(const TcMaps& m, const KnnTcParams& p, cudaStream_t st)
{
    const SmemLayoutTc L = smem_layout_tc(Elem::kPlanes, MT, A_STREAM, p.kchunks, p.stages, SPLIT,
                                          SPLIT > 1 ? TopK::kRegs / 2 : 0, !Elem::kFloat && METRIC == 0);
    const uint32_t smem = L.total + 1024;
    auto kern = knn_tc_kernel<Elem, MT, NBUF, A_STREAM, METRIC, TopK, SPLIT>;
    KNNG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const uint32_t n_qtiles = (p.n_queries + MT * kTileRows - 1) / (MT * kTileRows);
    uint32_t grid = std::min<uint32_t>(n_qtiles, static_cast<uint32_t>(sm_count()));
    if (const char* gv = std::getenv("KNNG_GPU_GRID")) grid = std::min<uint32_t>(grid, std::max(1, std::atoi(gv)));  // experiments only
    kern<<<grid, 64 + 128 * MT * SPLIT, smem, st>>>(m.q0, m.q1, m.b0, m.b1, p);
    KNNG_CUDA(cudaGetLastError());
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
    if (const char* sv = std::getenv("KNNG_GPU_STAGES")) s = std::min<uint32_t>(s, std::atoi(sv));
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

// Device interval timer; ms() is 0 unless both ends were recorded (an
// elapsed-time query on an unrecorded event would leave a sticky error).
struct EventTimer {
    cudaEvent_t a = nullptr, b = nullptr;
    bool on, started = false, stopped = false;
    explicit EventTimer(bool enable) : on(enable)
    {
        if (on) {
            cudaEventCreate(&a);
            cudaEventCreate(&b);
        }
    }
    ~EventTimer()
    {
        if (a) cudaEventDestroy(a);
        if (b) cudaEventDestroy(b);
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
};

// Query tiles per CTA of the fused u8 kernel: two need k <= 32 (register
// budget of 320 threads) and at most two K chunks of resident A.
int u8_query_tiles_per_cta(uint64_t d, uint64_t k)
{
    int mt = (u8_data_bytes(d) / kChunkBytes <= 2 && k <= 32) ? 2 : 1;
    if (const char* mv = std::getenv("KNNG_GPU_MT")) mt = std::atoi(mv) == 1 ? 1 : mt;  // experiments only
    return mt;
}

// Launch the u8 search of one (query set, base set) pair on `st`: the fused
// tensor-core kernel, then the exact kernel for the rows it flags (device-side
// count), or the exact kernel alone for d > kMaxTensorDim. No host sync; the
// caller zeroes sc.counters before and reads them after. tf (optional) times
// the exact pass.
knng_gpu_status launch_u8_sets(const U8Sets& z, uint64_t d, uint64_t k, int metric, uint32_t* ids, float* dists,
                               const ScratchU8& sc, cudaStream_t st, uint32_t* launches, EventTimer* tf)
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
        if (const char* dbg = std::getenv("KNNG_GPU_DEBUG_FLAGS")) p.debug_flags = static_cast<uint32_t>(std::atoi(dbg));
        int mt = u8_query_tiles_per_cta(d, k);
        // Optional column-split epilogue (four epilogue warps per SM
        // sub-partition, each on half of a 256-column tile), KNNG_GPU_SPLIT=2.
        // Measured slower than one warp per 32 rows at n=1M d=128 k=10 on B200
        // (305 ms vs 263 ms: the 96-register budget spills), so off by default.
        int split = 1;
        if (const char* sv = std::getenv("KNNG_GPU_SPLIT")) split = (std::atoi(sv) == 2 && mt == 2 && k <= 16) ? 2 : 1;
        const bool aug = metric == 0;
        p.stages = pick_stages(1, mt, false, p.kchunks, split, split > 1 ? (k <= 10 ? 10 : 16) : 0, aug);
        if (split > 1 && p.stages < 3) {
            split = 1;
            p.stages = pick_stages(1, mt, false, p.kchunks, 1, 0, aug);
        }
        if (p.stages < 2 || (mt > 1 && p.stages < p.kchunks))
            return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: shared memory budget exceeded");
        unsigned long long* dbg_clk = nullptr;
        if (p.debug_flags & 512u) {  // profiling only
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

__global__ void merge_topk_kernel(const uint32_t* __restrict__ a_ids, const float* __restrict__ a_d,
                                  const uint32_t* __restrict__ b_ids, const float* __restrict__ b_d, uint64_t rows,
                                  uint32_t k, uint32_t* __restrict__ o_ids, float* __restrict__ o_d);

// Streams and events of one split search, released on every exit path.
struct ForkSet {
    cudaStream_t s[kMaxTailParts] = {};
    cudaEvent_t fork = nullptr, join[kMaxTailParts] = {};
    ~ForkSet()
    {
        for (int i = 0; i < kMaxTailParts; ++i) {
            if (join[i]) cudaEventDestroy(join[i]);
            if (s[i]) cudaStreamDestroy(s[i]);
        }
        if (fork) cudaEventDestroy(fork);
    }
};

// u8 search of a query set against a base set. The fused kernel is
// persistent with one CTA per SM over query tiles; when the last wave would
// hold only R < SMs/2 tiles, those tail queries are searched first by
// f = SMs / R concurrent launches, each over one 256-row-aligned range of the
// base, and the f exact partial lists are merged by (distance, id). Their
// temporary rows live in the output rows of the main range, which the main
// launch then overwrites. The result is identical to one pass.
knng_gpu_status knn_u8_sets_impl(const U8Sets& z, uint64_t d, uint64_t k, int metric, uint32_t* ids, float* dists,
                                 void* scratch, uint64_t scratch_bytes, cudaStream_t st, knng_gpu_stats* stats,
                                 bool allow_split = true)
{
    const uint64_t q_count = z.n_q;
    if (scratch_bytes < scratch_u8_bytes(q_count))
        return fail(KNNG_GPU_WORKSPACE_TOO_SMALL, "knng::gpu: scratch smaller than knng_gpu_knn_scratch_bytes");
    if (q_count == 0) return KNNG_GPU_OK;
    if (z.n_b < k + (z.exclude_self ? 1 : 0))
        return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: fewer base rows than k");
    const uint64_t pitch = knng_gpu_padded_dim(d);
    const ScratchU8 sc = carve_scratch_u8(scratch, q_count);
    // Tail plan.
    const uint64_t sms = static_cast<uint64_t>(sm_count());
    const uint64_t qt_rows = static_cast<uint64_t>(u8_query_tiles_per_cta(d, k)) * kTileRows;
    const uint64_t qtiles = (q_count + qt_rows - 1) / qt_rows;
    const uint64_t full_waves = qtiles / sms, tail_tiles = qtiles % sms;
    uint64_t parts = tail_tiles ? std::min<uint64_t>(kMaxTailParts, sms / tail_tiles) : 0;
    uint64_t part_rows = 0;
    if (parts >= 2) {
        part_rows = align_up((z.n_b + parts - 1) / parts, 256);
        parts = (z.n_b + part_rows - 1) / part_rows;
        // every part needs k (+ self) rows
        if (part_rows < k + 1 || z.n_b - (parts - 1) * part_rows < k + 1) parts = 0;
    }
    bool split = allow_split && d <= kMaxTensorDim && full_waves >= 1 && parts >= 2;
    if (const char* tv = std::getenv("KNNG_GPU_TAIL_SPLIT")) split = split && std::atoi(tv) != 0;  // experiments
    const uint64_t main_q = split ? full_waves * sms * qt_rows : q_count;
    const uint64_t tail_q = q_count - main_q;
    const uint32_t n_launch = split ? static_cast<uint32_t>(parts) + 1 : 1;
    KNNG_CUDA(cudaMemsetAsync(sc.counters, 0, 8 * n_launch, st));
    uint32_t launches = 0;
    EventTimer tk(stats != nullptr), tf(stats != nullptr && !split);
    tk.start(st);
    if (split) {
        ForkSet fs;
        KNNG_CUDA(cudaEventCreateWithFlags(&fs.fork, cudaEventDisableTiming));
        KNNG_CUDA(cudaEventRecord(fs.fork, st));
        for (uint64_t pi = 0; pi < parts; ++pi) {
            KNNG_CUDA(cudaStreamCreateWithFlags(&fs.s[pi], cudaStreamNonBlocking));
            KNNG_CUDA(cudaEventCreateWithFlags(&fs.join[pi], cudaEventDisableTiming));
            KNNG_CUDA(cudaStreamWaitEvent(fs.s[pi], fs.fork, 0));
            const uint64_t b0 = pi * part_rows;
            U8Sets zp = z;
            zp.q_packed = z.q_packed + main_q * pitch;
            zp.q_norms = z.q_norms + main_q;
            zp.n_q = tail_q;
            zp.q_id0 = z.q_id0 + main_q;
            zp.b_packed = z.b_packed + b0 * pitch;
            zp.b_norms = z.b_norms + b0;
            zp.n_b = std::min(part_rows, z.n_b - b0);
            zp.b_id0 = z.b_id0 + b0;
            const ScratchU8 scp{sc.fallback_rows + pi * tail_q, sc.counters + 2 * (1 + pi)};
            KNNG_TRY(launch_u8_sets(zp, d, k, metric, ids + pi * tail_q * k, dists + pi * tail_q * k, scp, fs.s[pi],
                                    &launches, nullptr));
            KNNG_CUDA(cudaEventRecord(fs.join[pi], fs.s[pi]));
            KNNG_CUDA(cudaStreamWaitEvent(st, fs.join[pi], 0));
        }
        // Fold the partial lists into the tail rows, alternating between the
        // tail rows and part 0's temporary rows (free after the first merge)
        // so that no merge writes the list it reads.
        uint32_t* t_ids = ids + main_q * k;
        float* t_d = dists + main_q * k;
        const uint32_t blocks = static_cast<uint32_t>((tail_q + 255) / 256);
        bool in_tail = false;  // the running result: part 0's rows at first
        for (uint64_t pi = 1; pi < parts; ++pi) {
            const uint32_t* a_ids = in_tail ? t_ids : ids;
            const float* a_d = in_tail ? t_d : dists;
            uint32_t* o_ids = in_tail ? ids : t_ids;
            float* o_d = in_tail ? dists : t_d;
            merge_topk_kernel<<<blocks, 256, 0, st>>>(a_ids, a_d, ids + pi * tail_q * k, dists + pi * tail_q * k,
                                                      tail_q, static_cast<uint32_t>(k), o_ids, o_d);
            KNNG_CUDA(cudaGetLastError());
            ++launches;
            in_tail = !in_tail;
        }
        if (!in_tail) {
            KNNG_CUDA(cudaMemcpyAsync(t_ids, ids, tail_q * k * sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));
            KNNG_CUDA(cudaMemcpyAsync(t_d, dists, tail_q * k * sizeof(float), cudaMemcpyDeviceToDevice, st));
        }
        U8Sets zm = z;
        zm.n_q = main_q;
        KNNG_TRY(launch_u8_sets(zm, d, k, metric, ids, dists, ScratchU8{sc.fallback_rows, sc.counters}, st,
                                &launches, nullptr));
        tk.stop(st);
        uint32_t host_counters[2 * (kMaxTailParts + 1)] = {};
        KNNG_CUDA(cudaMemcpyAsync(host_counters, sc.counters, 8 * n_launch, cudaMemcpyDeviceToHost, st));
        KNNG_CUDA(cudaStreamSynchronize(st));
        uint32_t fallback = 0;
        for (uint32_t i = 0; i < n_launch; ++i) {
            if (host_counters[2 * i + 1] != 0)
                return fail(KNNG_GPU_TIMEOUT, "knng::gpu: a bounded device wait gave up (code " +
                                                  std::to_string(host_counters[2 * i + 1]) + ")");
            fallback += host_counters[2 * i];
        }
        if (stats) {
            stats->path = KNNG_PATH_U8_TENSOR;
            stats->fallback_rows = fallback;
            stats->knn_ms = tk.ms();
            stats->fallback_ms = 0.f;
            stats->kernel_launches += launches;
        }
        return KNNG_GPU_OK;
    }
    KNNG_TRY(launch_u8_sets(z, d, k, metric, ids, dists, sc, st, &launches, &tf));
    tk.stop(st);
    uint32_t host_counters[2] = {0, 0};
    KNNG_TRY(read_counters(sc.counters, host_counters, st));
    if (stats) {
        stats->path = KNNG_PATH_U8_TENSOR;
        stats->fallback_rows = host_counters[0];
        stats->knn_ms = tk.ms();
        stats->fallback_ms = tf.ms();
        stats->kernel_launches += launches;
    }
    return KNNG_GPU_OK;
}

knng_gpu_status knn_u8_impl(const uint8_t* packed, const int32_t* norms, uint64_t n, uint64_t d, uint64_t q_begin,
                            uint64_t q_count, uint64_t k, int metric, uint32_t* ids, float* dists, void* scratch,
                            uint64_t scratch_bytes, cudaStream_t st, knng_gpu_stats* stats, bool allow_split = true)
{
    if (q_begin + q_count > n) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: query range exceeds the base");
    const uint64_t pitch = knng_gpu_padded_dim(d);
    const U8Sets z{packed + q_begin * pitch, norms + q_begin, q_count, q_begin, packed, norms, n, 0, 1};
    return knn_u8_sets_impl(z, d, k, metric, ids, dists, scratch, scratch_bytes, st, stats, allow_split);
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
// Candidates kept per row by the bf16x3 filter: k plus a margin, at most n - 1.
uint64_t f32_candidates(uint64_t n, uint64_t k) { return std::min<uint64_t>(n - 1, k + 32); }

uint64_t f32_pitch_elems(uint64_t d) { return align_up(d, kChunkBytes / 2); }

struct ScratchF32 {
    double* sums;
    float* mu;
    unsigned int* max_norm_bits;
    __nv_bfloat16* hi;
    __nv_bfloat16* lo;
    float* norms;
    uint32_t* cand_ids;
    int32_t* cand_keys;
    uint32_t* fallback_rows;
    uint32_t* counters;  // [0] fallback count, [1] error flag, [2] observed error ratio (fp32 bits)
    uint64_t total;
};

ScratchF32 layout_scratch_f32(void* base, uint64_t n, uint64_t d, uint64_t q_count, uint64_t k)
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
    const uint64_t c = f32_candidates(n, k);
    s.sums = reinterpret_cast<double*>(take(d * 8));
    s.mu = reinterpret_cast<float*>(take(d * 4));
    s.max_norm_bits = reinterpret_cast<unsigned int*>(take(4));
    s.hi = reinterpret_cast<__nv_bfloat16*>(take(n * pitch * 2));
    s.lo = reinterpret_cast<__nv_bfloat16*>(take(n * pitch * 2));
    s.norms = reinterpret_cast<float*>(take(n * 4));
    s.cand_ids = reinterpret_cast<uint32_t*>(take(q_count * c * 4));
    s.cand_keys = reinterpret_cast<int32_t*>(take(q_count * c * 4));
    s.fallback_rows = reinterpret_cast<uint32_t*>(take(q_count * 4));
    s.counters = reinterpret_cast<uint32_t*>(take(16));
    s.total = off;
    return s;
}

// eps coefficient of the re-rank proof (knn_rerank.cuh).
double f32_gamma(uint64_t d, int metric)
{
    const double dd = static_cast<double>(d);
    const double split = std::ldexp(1.0, -14), acc = (3.0 * dd / 16.0 + 3.0) * std::ldexp(1.0, -22);
    const double ref = (dd + 3.0) * std::ldexp(1.0, -24);
    double g = metric == 0 ? 2.0 * (split + acc) + std::ldexp(1.0, -19) + ref : split + acc + std::ldexp(1.0, -21) + ref;
    if (const char* gs = std::getenv("KNNG_GPU_GAMMA_SCALE")) g *= std::atof(gs);  // experiments only
    return g;
}

knng_gpu_status knn_f32_impl(const float* x, uint64_t n, uint64_t d, uint64_t q_begin, uint64_t q_count, uint64_t k,
                             int metric, uint32_t* ids, float* dists, void* scratch, uint64_t scratch_bytes,
                             cudaStream_t st, knng_gpu_stats* stats)
{
    if (q_begin + q_count > n) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: query range exceeds the base");
    const ScratchF32 sc = layout_scratch_f32(scratch, n, d, q_count, k);
    if (scratch_bytes < sc.total || (reinterpret_cast<uintptr_t>(scratch) & 255))
        return fail(KNNG_GPU_WORKSPACE_TOO_SMALL, "knng::gpu: fp32 scratch smaller than knng_gpu_knn_f32_scratch_bytes");
    if (q_count == 0) return KNNG_GPU_OK;
    const uint64_t pitch = f32_pitch_elems(d);
    const uint64_t c = f32_candidates(n, k);
    const uint32_t kchunks = static_cast<uint32_t>(pitch * 2 / kChunkBytes);
    EventTimer tk(stats != nullptr), tf(stats != nullptr);
    tk.start(st);
    KNNG_CUDA(cudaMemsetAsync(sc.counters, 0, 16, st));
    KNNG_CUDA(cudaMemsetAsync(sc.max_norm_bits, 0, 4, st));
    uint32_t launches = 0;
    if (metric == 0) {
        // L2 is translation invariant: centre the rows to shrink the error bound.
        KNNG_CUDA(cudaMemsetAsync(sc.sums, 0, d * 8, st));
        column_sum_kernel<<<static_cast<uint32_t>((n + 255) / 256), 256, 0, st>>>(x, n, static_cast<uint32_t>(d),
                                                                                 sc.sums);
        column_mean_kernel<<<static_cast<uint32_t>((d + 255) / 256), 256, 0, st>>>(sc.sums, n, static_cast<uint32_t>(d),
                                                                                  sc.mu);
        launches += 2;
    }
    {
        const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((n + 7) / 8, 148ull * 16));
        split_bf16_kernel<<<blocks, 256, 0, st>>>(x, n, static_cast<uint32_t>(d), static_cast<uint32_t>(pitch),
                                                  metric == 0 ? sc.mu : nullptr, sc.hi, sc.lo, sc.norms,
                                                  sc.max_norm_bits);
        KNNG_CUDA(cudaGetLastError());
        launches += 1;
    }
    // Candidate filter on the tensor cores.
    TcMaps m;
    KNNG_TRY(make_map(&m.b0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, sc.hi, n, pitch, pitch * 2));
    KNNG_TRY(make_map(&m.b1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, sc.lo, n, pitch, pitch * 2));
    m.q0 = m.b0;
    m.q1 = m.b1;
    KnnTcParams p{};
    p.base_norms = sc.norms;
    p.n_base = n;
    p.base_id0 = 0;
    p.n_queries = static_cast<uint32_t>(q_count);
    p.query_row0 = static_cast<uint32_t>(q_begin);
    p.query_id0 = static_cast<uint32_t>(q_begin);
    p.exclude_self = 1;
    p.k = static_cast<uint32_t>(c);
    p.kchunks = kchunks;
    p.out_ids = sc.cand_ids;
    p.out_keys = sc.cand_keys;
    p.error = reinterpret_cast<int*>(sc.counters + 1);
    if (const char* dbg = std::getenv("KNNG_GPU_DEBUG_FLAGS")) p.debug_flags = static_cast<uint32_t>(std::atoi(dbg));
    bool a_stream = false;
    p.stages = pick_stages(2, 1, false, kchunks);
    if (p.stages < 2) {
        a_stream = true;
        p.stages = pick_stages(2, 1, true, kchunks);
    }
    if (p.stages < 2) return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: shared memory budget exceeded");
    knng_gpu_status s;
    if (a_stream)
        s = metric == 0 ? launch_bf16_k<true, 0>(m, p, st) : launch_bf16_k<true, 1>(m, p, st);
    else
        s = metric == 0 ? launch_bf16_k<false, 0>(m, p, st) : launch_bf16_k<false, 1>(m, p, st);
    KNNG_TRY(s);
    // Exact re-rank of the candidates with the proof of exactness.
    RerankParams r{};
    r.x = x;
    r.d = d;
    r.n = n;
    r.q_begin = static_cast<uint32_t>(q_begin);
    r.n_queries = static_cast<uint32_t>(q_count);
    r.c = static_cast<uint32_t>(c);
    r.k = static_cast<uint32_t>(k);
    r.cand_ids = sc.cand_ids;
    r.cand_keys = sc.cand_keys;
    r.norms = sc.norms;
    r.max_norm_bits = sc.max_norm_bits;
    r.gamma = f32_gamma(d, metric);
    r.out_ids = ids;
    r.out_dists = dists;
    r.fallback_rows = sc.fallback_rows;
    r.fallback_count = sc.counters;
    r.err_ratio_bits = sc.counters + 2;
    {
        const uint32_t warps = 32 * kRerankWarps;
        const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((q_count + kRerankWarps - 1) / kRerankWarps,
                                                                         148ull * 8));
        const uint32_t cpl = static_cast<uint32_t>((c + 31) / 32);
        (void)warps;
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
    e.base = x;
    e.base_stride = d;
    e.n_base = n;
    e.queries = x + q_begin * d;
    e.query_stride = d;
    e.n_queries = static_cast<uint32_t>(q_count);
    e.query_id0 = static_cast<uint32_t>(q_begin);
    e.exclude_self = 1;
    e.d = static_cast<uint32_t>(d);
    e.k = static_cast<uint32_t>(k);
    e.row_list = sc.fallback_rows;
    e.row_count = sc.counters;
    e.out_ids = ids;
    e.out_dists = dists;
    KNNG_TRY(launch_exact(e, metric, static_cast<uint32_t>(q_count), st));
    tf.stop(st);
    launches += 1;
    uint32_t host_counters[2] = {0, 0};
    KNNG_TRY(read_counters(sc.counters, host_counters, st));
    uint32_t ratio_bits = 0;
    KNNG_CUDA(cudaMemcpy(&ratio_bits, sc.counters + 2, 4, cudaMemcpyDeviceToHost));
    if (stats) {
        float ratio;
        std::memcpy(&ratio, &ratio_bits, 4);
        stats->f32_err_ratio = ratio;
        stats->path = KNNG_PATH_F32_TENSOR;
        stats->fallback_rows = host_counters[0];
        stats->knn_ms = tk.ms();
        stats->fallback_ms = tf.ms();
        stats->kernel_launches += launches;
    }
    return KNNG_GPU_OK;
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
    const uint64_t u8_total = w.scratch + scratch_u8_bytes(n);
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
    EventTimer tall(stats != nullptr), tp(stats != nullptr);
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
    EventTimer tall(stats != nullptr), tp(stats != nullptr);
    tall.start(st);
    tp.start(st);
    KNNG_CUDA(cudaMemsetAsync(flag, 0, 4, st));
    KNNG_TRY(pack_impl(x, n, d, packed, norms, flag, st));
    tp.stop(st);
    int32_t nonint = 0;
    KNNG_CUDA(cudaMemcpyAsync(&nonint, flag, 4, cudaMemcpyDeviceToHost, st));
    KNNG_CUDA(cudaStreamSynchronize(st));
    if (stats) {
        std::memset(stats, 0, sizeof(*stats));
        stats->kernel_launches = 2;  // pack + augmentation
    }
    if (nonint == 0) {
        KNNG_TRY(knn_u8_impl(packed, norms, n, d, 0, n, k, metric, ids, dists, base + w.scratch, w.total - w.scratch,
                             st, stats));
    } else {
        // The packed bytes are meaningless for such data; the fp32 path
        // reuses the whole workspace.
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
// stand-in); noalloc_scratch_ptr() resolves the device address once per device.
constexpr uint64_t kNoAllocScratchBytes = (static_cast<uint64_t>(KNNG_GPU_NOALLOC_MAX_QUERIES) * 4 + 255) / 256 * 256 + 256;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxDevices] = {};

knng_gpu_status noalloc_scratch_ptr(void** out)
{
    int dev = 0;
    KNNG_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: device index out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_ptr[dev]) {
        void* ptr = nullptr;
        // The current device is `dev`, so this resolves that device's copy.
        KNNG_CUDA(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
        g_noalloc_ptr[dev] = ptr;
    }
    *out = g_noalloc_ptr[dev];
    return KNNG_GPU_OK;
}
}  // namespace

// ------------------------------------------------------------------ host-API buffer cache
// knng_gpu_brute_force keeps its device buffers and stream per device between
// calls (grown on demand, freed by knng_gpu_release_cached_buffers), so a
// build pays no cudaMalloc/cudaFree once the sizes have been seen.
namespace {
struct HostCache {
    std::mutex mutex;
    int device = 0;
    cudaStream_t stream = nullptr;
    void *x = nullptr, *ids = nullptr, *dists = nullptr, *ws = nullptr;
    uint64_t x_cap = 0, ids_cap = 0, dists_cap = 0, ws_cap = 0;
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

uint64_t knng_gpu_knn_scratch_bytes(uint64_t q_count) { return scratch_u8_bytes(q_count); }

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
    KNNG_CUDA(cudaMemcpyAsync(dx, data, n * d * sizeof(float), cudaMemcpyHostToDevice, st));
    KNNG_TRY(device_pipeline(dx, n, d, k, metric, dids, ddist, c.ws, c.ws_cap, st, stats));
    KNNG_CUDA(cudaMemcpyAsync(ids, dids, n * k * sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    KNNG_CUDA(cudaMemcpyAsync(dists, ddist, n * k * sizeof(float), cudaMemcpyDeviceToHost, st));
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
    KNNG_CUDA(cudaMemcpyAsync(dx, rows, in_bytes, cudaMemcpyHostToDevice, st));
    KNNG_TRY(device_pipeline_u8(dx, n, d, row_stride, k, metric, dids, ddist, c.ws, c.ws_cap, st, stats));
    KNNG_CUDA(cudaMemcpyAsync(ids, dids, n * k * sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
    KNNG_CUDA(cudaMemcpyAsync(dists, ddist, n * k * sizeof(float), cudaMemcpyDeviceToHost, st));
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
        if (!c.stream && !c.x && !c.ws) continue;
        cudaSetDevice(c.device);
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
    // the previous call's contents never leak into this one.
    // No tail split here: it would create streams and events.
    return knn_u8_impl(d_packed, d_norms, n, d, q_begin, q_count, k, metric, d_ids, d_dists, scratch,
                       kNoAllocScratchBytes, static_cast<cudaStream_t>(stream), stats, false);
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
