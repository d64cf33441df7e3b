// knng_gpu.cu -- C-ABI entry points (include/knng_gpu.h) and the host-side
// orchestration of the kernels: integer check + u8 pack + row norms, the
// fused tensor-core KNN, and the exact fp32 kernel.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "knn_exact.cuh"
#include "knn_u8_tc.cuh"
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
                                                      uint32_t pitch, uint8_t* __restrict__ packed,
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
        for (uint32_t c0 = lane * 4; c0 < pitch; c0 += 128) {
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

// rows x pitch u8, box 128 rows x 128 bytes, 128-byte swizzle; rows past the
// end read as zeros.
knng_gpu_status make_u8_map(CUtensorMap* map, const uint8_t* base, uint64_t rows, uint64_t pitch)
{
    EncodeTiledFn enc;
    KNNG_TRY(get_encode_fn(&enc));
    const cuuint64_t dims[2] = {pitch, rows};
    const cuuint64_t strides[1] = {pitch};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kChunkBytes), static_cast<cuuint32_t>(kTileRows)};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(KNNG_GPU_CUDA_ERROR, "knng::gpu: cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return KNNG_GPU_OK;
}

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

uint64_t scratch_u8_bytes(uint64_t q_count) { return align_up(q_count * 4, 256) + 256; }

ScratchU8 carve_scratch_u8(void* p, uint64_t q_count)
{
    ScratchU8 s;
    s.fallback_rows = static_cast<uint32_t*>(p);
    s.counters = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(p) + align_up(q_count * 4, 256));
    return s;
}

template <int MT, int BN, int NBUF, int SPLIT, int METRIC, class TopK>
knng_gpu_status launch_u8_t(const CUtensorMap& mq, const CUtensorMap& mb, const KnnU8Params& p, cudaStream_t st)
{
    const SmemLayoutU8 L = smem_layout_u8(MT, BN, p.kchunks, p.stages, SPLIT, SPLIT > 1 ? TopK::kRegs / 2 : 0);
    const uint32_t smem = L.total + 1024;
    auto kern = knn_u8_tc_kernel<MT, BN, NBUF, SPLIT, METRIC, TopK>;
    KNNG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const uint32_t n_qtiles = (p.n_queries + MT * kTileRows - 1) / (MT * kTileRows);
    const uint32_t grid = std::min<uint32_t>(n_qtiles, static_cast<uint32_t>(sm_count()));
    kern<<<grid, 64 + 128 * MT * SPLIT, smem, st>>>(mq, mb, p);
    KNNG_CUDA(cudaGetLastError());
    return KNNG_GPU_OK;
}

template <int MT, int BN, int NBUF, int METRIC>
knng_gpu_status launch_u8_k(const CUtensorMap& mq, const CUtensorMap& mb, const KnnU8Params& p, int split,
                            cudaStream_t st)
{
    (void)split;  // the column-split epilogue (SPLIT = 2) is not instantiated
    if (p.k <= 10) return launch_u8_t<MT, BN, NBUF, 1, METRIC, RegTopK<10>>(mq, mb, p, st);
    if (p.k <= 16) return launch_u8_t<MT, BN, NBUF, 1, METRIC, RegTopK<16>>(mq, mb, p, st);
    if (p.k <= 32) return launch_u8_t<MT, BN, NBUF, 1, METRIC, RegTopK<32>>(mq, mb, p, st);
    if constexpr (MT == 1) {
        if (p.k <= 64) return launch_u8_t<MT, BN, NBUF, 1, METRIC, RegTopK<64>>(mq, mb, p, st);
    }
    if (p.k <= 128) return launch_u8_t<MT, BN, NBUF, 1, METRIC, HeapTopK<128>>(mq, mb, p, st);
    return launch_u8_t<MT, BN, NBUF, 1, METRIC, HeapTopK<KNNG_GPU_MAX_K>>(mq, mb, p, st);
}

// Tile shapes of the fused kernel: (query tiles per CTA, base rows per tile,
// TMEM accumulator buffers).
struct TileShape {
    int mt, bn, nbuf, split;
};

template <int MT, int BN, int NBUF>
knng_gpu_status launch_u8_m(const CUtensorMap& mq, const CUtensorMap& mb, const KnnU8Params& p, int metric,
                            int split, cudaStream_t st)
{
    return metric == 0 ? launch_u8_k<MT, BN, NBUF, 0>(mq, mb, p, split, st)
                       : launch_u8_k<MT, BN, NBUF, 1>(mq, mb, p, split, st);
}

knng_gpu_status launch_u8(const CUtensorMap& mq, const CUtensorMap& mb, const KnnU8Params& p, TileShape ts,
                          int metric, cudaStream_t st)
{
    // Measured alternatives (BN = 256 with one TMEM buffer, MT = 1 with four
    // buffers, a two-way column split of the epilogue) were slower at d = 128.
    if (ts.mt == 2) return launch_u8_m<2, 128, 2>(mq, mb, p, metric, 1, st);
    return launch_u8_m<1, 128, 2>(mq, mb, p, metric, 1, st);
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

struct EventTimer {
    cudaEvent_t a = nullptr, b = nullptr;
    bool on;
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
        if (on) cudaEventRecord(a, s);
    }
    void stop(cudaStream_t s)
    {
        if (on) cudaEventRecord(b, s);
    }
    float ms()
    {
        float m = 0.f;
        if (on) {
            cudaEventSynchronize(b);
            cudaEventElapsedTime(&m, a, b);
        }
        return m;
    }
};

knng_gpu_status knn_u8_impl(const uint8_t* packed, const int32_t* norms, uint64_t n, uint64_t d, uint64_t q_begin,
                            uint64_t q_count, uint64_t k, int metric, uint32_t* ids, float* dists, void* scratch,
                            uint64_t scratch_bytes, cudaStream_t st, knng_gpu_stats* stats)
{
    if (q_begin + q_count > n) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: query range exceeds the base");
    if (scratch_bytes < scratch_u8_bytes(q_count))
        return fail(KNNG_GPU_WORKSPACE_TOO_SMALL, "knng::gpu: scratch smaller than knng_gpu_knn_scratch_bytes");
    if (q_count == 0) return KNNG_GPU_OK;
    const uint64_t pitch = knng_gpu_padded_dim(d);
    ScratchU8 sc = carve_scratch_u8(scratch, q_count);
    KNNG_CUDA(cudaMemsetAsync(sc.counters, 0, 8, st));
    uint32_t launches = 1;
    EventTimer tk(stats != nullptr), tf(stats != nullptr);
    tk.start(st);
    if (d <= kMaxTensorDim) {
        CUtensorMap mq, mb;
        KNNG_TRY(make_u8_map(&mq, packed, n, pitch));
        KNNG_TRY(make_u8_map(&mb, packed, n, pitch));
        KnnU8Params p{};
        p.base_norms = norms;
        p.query_norms = norms + q_begin;
        p.n_base = n;
        p.base_id0 = 0;
        p.n_queries = static_cast<uint32_t>(q_count);
        p.query_row0 = static_cast<uint32_t>(q_begin);
        p.query_id0 = static_cast<uint32_t>(q_begin);
        p.exclude_self = 1;
        p.k = static_cast<uint32_t>(k);
        p.kchunks = static_cast<uint32_t>(pitch / kChunkBytes);
        p.out_ids = ids;
        p.out_dists = dists;
        p.fallback_rows = sc.fallback_rows;
        p.fallback_count = sc.counters;
        p.error = reinterpret_cast<int*>(sc.counters + 1);
        if (const char* dbg = std::getenv("KNNG_GPU_DEBUG_FLAGS")) p.debug_flags = static_cast<uint32_t>(std::atoi(dbg));
        // Two query tiles per CTA need k <= 32 (register budget of 320 threads).
        TileShape ts = (p.kchunks <= 2 && k <= 32) ? TileShape{2, 128, 2, 1} : TileShape{1, 128, 2, 1};
        const uint32_t fixed = smem_layout_u8(ts.mt, ts.bn, p.kchunks, 0, ts.split, ts.split > 1 ? 16 : 0).total + 1024;
        const uint32_t budget = 227u * 1024u;
        const uint32_t stage_bytes = (ts.bn / kTileRows) * kBoxBytes;
        p.stages = std::min<uint32_t>(16, (budget - fixed) / stage_bytes);
        if (const char* sv = std::getenv("KNNG_GPU_STAGES")) p.stages = std::min<uint32_t>(p.stages, std::atoi(sv));
        if (p.stages < 2 || (ts.mt > 1 && p.stages < p.kchunks))
            return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: shared memory budget exceeded");
        knng_gpu_status s = launch_u8(mq, mb, p, ts, metric, st);
        KNNG_TRY(s);
        tk.stop(st);
        // Rows whose fp32 sums may round: recompute exactly (device-side
        // count; CTAs past it exit at once).
        tf.start(st);
        KnnExactParams<uint8_t> e{};
        e.base = packed;
        e.base_stride = pitch;
        e.n_base = n;
        e.queries = packed + q_begin * pitch;
        e.query_stride = pitch;
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
        launches = 2;
    } else {
        KnnExactParams<uint8_t> e{};
        e.base = packed;
        e.base_stride = pitch;
        e.n_base = n;
        e.queries = packed + q_begin * pitch;
        e.query_stride = pitch;
        e.n_queries = static_cast<uint32_t>(q_count);
        e.query_id0 = static_cast<uint32_t>(q_begin);
        e.exclude_self = 1;
        e.d = static_cast<uint32_t>(d);
        e.k = static_cast<uint32_t>(k);
        e.out_ids = ids;
        e.out_dists = dists;
        KNNG_TRY(launch_exact(e, metric, static_cast<uint32_t>(q_count), st));
        tk.stop(st);
        tf.start(st);
        tf.stop(st);
    }
    uint32_t host_counters[2] = {0, 0};
    KNNG_CUDA(cudaMemcpyAsync(host_counters, sc.counters, 8, cudaMemcpyDeviceToHost, st));
    KNNG_CUDA(cudaStreamSynchronize(st));
    if (host_counters[1] != 0)
        return fail(KNNG_GPU_TIMEOUT, "knng::gpu: a bounded device wait gave up (code " +
                                          std::to_string(host_counters[1]) + ")");
    if (stats) {
        stats->path = KNNG_PATH_U8_TENSOR;
        stats->fallback_rows = host_counters[0];
        stats->knn_ms = tk.ms();
        stats->fallback_ms = tf.ms();
        stats->kernel_launches += launches;
    }
    return KNNG_GPU_OK;
}

knng_gpu_status knn_f32_impl(const float* x, uint64_t n, uint64_t d, uint64_t q_begin, uint64_t q_count, uint64_t k,
                             int metric, uint32_t* ids, float* dists, cudaStream_t st, knng_gpu_stats* stats)
{
    if (q_begin + q_count > n) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: query range exceeds the base");
    EventTimer tk(stats != nullptr);
    tk.start(st);
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
    e.out_ids = ids;
    e.out_dists = dists;
    KNNG_TRY(launch_exact(e, metric, static_cast<uint32_t>(q_count), st));
    tk.stop(st);
    if (stats) {
        stats->path = KNNG_PATH_F32_EXACT;
        stats->knn_ms = tk.ms();
        stats->kernel_launches += 1;
    }
    return KNNG_GPU_OK;
}

struct WorkspaceLayout {
    uint64_t packed, norms, flag, scratch, total;
};

WorkspaceLayout workspace_layout(uint64_t n, uint64_t d)
{
    WorkspaceLayout w;
    const uint64_t pitch = knng_gpu_padded_dim(d);
    w.packed = 0;
    w.norms = align_up(w.packed + n * pitch, 256);
    w.flag = align_up(w.norms + n * 4, 256);
    w.scratch = w.flag + 256;
    w.total = w.scratch + scratch_u8_bytes(n);
    return w;
}

knng_gpu_status pack_impl(const float* x, uint64_t rows, uint64_t d, uint8_t* packed, int32_t* norms,
                          int32_t* nonint, cudaStream_t st)
{
    if (rows == 0) return KNNG_GPU_OK;
    const uint64_t pitch = knng_gpu_padded_dim(d);
    const uint64_t warps_needed = rows;
    const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((warps_needed + 7) / 8, 148ull * 16));
    pack_u8_kernel<<<blocks, 256, 0, st>>>(x, rows, static_cast<uint32_t>(d), static_cast<uint32_t>(pitch), packed,
                                          norms, nonint);
    KNNG_CUDA(cudaGetLastError());
    return KNNG_GPU_OK;
}

knng_gpu_status device_pipeline(const float* x, uint64_t n, uint64_t d, uint64_t k, int metric, uint32_t* ids,
                                float* dists, void* ws, uint64_t ws_bytes, cudaStream_t st, knng_gpu_stats* stats)
{
    KNNG_TRY(validate(n, d, k, metric));
    const WorkspaceLayout w = workspace_layout(n, d);
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
        stats->kernel_launches = 1;
    }
    if (nonint == 0) {
        KNNG_TRY(knn_u8_impl(packed, norms, n, d, 0, n, k, metric, ids, dists, base + w.scratch, w.total - w.scratch,
                             st, stats));
    } else {
        KNNG_TRY(knn_f32_impl(x, n, d, 0, n, k, metric, ids, dists, st, stats));
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

uint64_t knng_gpu_padded_dim(uint64_t d) { return align_up(d == 0 ? 1 : d, kChunkBytes); }

uint64_t knng_gpu_workspace_bytes(uint64_t n, uint64_t d) { return workspace_layout(n, d).total; }

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
                                 uint64_t k, int metric, uint32_t* d_ids, float* d_dists, void* stream,
                                 knng_gpu_stats* stats)
{
    g_last_error.clear();
    KNNG_TRY(validate(n, d, k, metric));
    return knn_f32_impl(d_x, n, d, q_begin, q_count, k, metric, d_ids, d_dists, static_cast<cudaStream_t>(stream),
                        stats);
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
    const uint64_t ws_bytes = knng_gpu_workspace_bytes(n, d);
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
    return knn_u8_impl(d_packed, d_norms, n, d, q_begin, q_count, k, metric, d_ids, d_dists, scratch,
                       kNoAllocScratchBytes, static_cast<cudaStream_t>(stream), stats);
}

}  // extern "C"
