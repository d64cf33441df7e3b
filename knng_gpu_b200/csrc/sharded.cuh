// sharded.cuh -- multi-GPU builds behind the C ABI (included at the end of
// knng_gpu.cu; uses its internal helpers).
//
// The reference's distributed brute force (src/dist/brute_force_mpi.cpp:36-142)
// shards query rows by compute_shard (include/knng/dist/sharded_dataset.hpp:
// 145-155: contiguous blocks, the last rank takes the remainder), passes the
// base around a ring with MPI_Sendrecv (:107-119) and gathers the Knng rows to
// rank 0 with two MPI_Gatherv (:179-200). Here one GPU is one rank of an NCCL
// communicator:
//
//   replicate mode (configs that fit one GPU's memory): every rank packs its
//     slice of rows, the integer flag is max-reduced, the packed slices are
//     all-gathered so every GPU holds the whole packed base (128 MB for
//     1M x 128), every rank searches its compute_shard query rows against it,
//     and the graph rows go to rank 0 by NCCL send/recv (NCCL has no Gatherv).
//     Non-integer data all-gathers the fp32 rows instead and takes the fp32
//     path. No host synchronisation before the search: the tensor-core
//     kernels read the reduced flag on the device and return at once for
//     fp32 data.
//   ring mode (the base never replicated): rank r's compute_shard rows are its
//     queries and its base block; in step s it searches block (r - s) mod P
//     while NCCL already sends that block to rank r + 1 and receives the next
//     from rank r - 1 on a second stream (double buffer); the block's k best
//     are merged into the running k best by (distance, id). Integer data only.
#pragma once
#include <nccl.h>

#include <thread>
#include <vector>

namespace {

#define KNNG_NCCL(call)                                                                                     \
    do {                                                                                                    \
        ncclResult_t r_ = (call);                                                                           \
        if (r_ != ncclSuccess)                                                                              \
            return fail(KNNG_GPU_CUDA_ERROR, std::string("knng::gpu: ") + #call + ": " + ncclGetErrorString(r_)); \
    } while (0)

// One rank's communicator with the stream and events its ring steps use,
// created once (knng_gpu_comm_create) and reused by every build.
struct KnngComm {
    ncclComm_t nccl = nullptr;
    int rank = 0, world = 1, device = 0;
    bool owns_nccl = true;
    cudaStream_t comm_stream = nullptr;
    cudaEvent_t ev_compute[2] = {}, ev_comm[2] = {};
    float phase_ms[6] = {};  // last build: pack, exchange, search, fp32 exchange, gather, total
    cudaEvent_t ev_phase[7] = {};
};

struct ShardRange {
    uint64_t start, count;
};

// include/knng/dist/sharded_dataset.hpp:145-155.
ShardRange compute_shard_rows(uint64_t n, int world, int rank)
{
    const uint64_t base = n / static_cast<uint64_t>(world), rem = n % static_cast<uint64_t>(world);
    return {static_cast<uint64_t>(rank) * base, base + (rank == world - 1 ? rem : 0)};
}

// Rows per rank in replicate mode: ceil(n / world) rounded up to 256, so
// every slice starts on a base tile of the pair kernel (the augmentation
// offsets are chosen per 128-row tile of one pack call).
uint64_t replicate_slice_rows(uint64_t n, int world)
{
    return align_up((n + static_cast<uint64_t>(world) - 1) / static_cast<uint64_t>(world), 256);
}

struct ShardedLayout {
    uint64_t flag, out_ids, out_dists, u;        // common part
    uint64_t packed, norms, scratch;             // u8 (relative to u)
    uint64_t qpacked, qnorms, tmp_ids, tmp_d, best_ids, best_d, bound;  // ring extras (relative to u)
    uint64_t x, f32s;                            // fp32 (relative to u)
    uint64_t total;
};

ShardedLayout sharded_layout(uint64_t n, uint64_t d, uint64_t k, int world, int mode)
{
    ShardedLayout L{};
    const uint64_t pitch = knng_gpu_padded_dim(d);
    const uint64_t ms = compute_shard_rows(n, world, world - 1).count;  // largest shard
    uint64_t off = 0;
    auto take = [&](uint64_t bytes) {
        const uint64_t r = off;
        off = align_up(off + bytes, 256);
        return r;
    };
    L.flag = take(256);
    L.out_ids = take(ms * k * 4);
    L.out_dists = take(ms * k * 4);
    L.u = off;
    off = 0;
    if (mode == 0) {
        const uint64_t s = replicate_slice_rows(n, world);
        L.packed = take(static_cast<uint64_t>(world) * s * pitch);
        L.norms = take(static_cast<uint64_t>(world) * s * 4);
        L.scratch = take(scratch_u8_bytes(ms, k));
        const uint64_t u8_end = off;
        off = 0;
        L.x = take(static_cast<uint64_t>(world) * s * d * 4);
        L.f32s = take(layout_scratch_f32(nullptr, n, d, ms, k).total);
        L.total = L.u + std::max(u8_end, off);
    } else {
        // Two ring buffers, each starting 256-byte aligned (TMA sources;
        // the key offsets are read 16 bytes at a time).
        L.packed = take(2 * align_up(ms * pitch, 256));
        L.norms = take(2 * align_up(ms * 4, 256));
        L.qpacked = take(ms * pitch);
        L.qnorms = take(ms * 4);
        L.tmp_ids = take(ms * k * 4);
        L.tmp_d = take(ms * k * 4);
        L.best_ids = take(ms * k * 4);
        L.best_d = take(ms * k * 4);
        L.bound = take(ms * 4);
        L.scratch = take(scratch_u8_bytes(ms, k));
        L.total = L.u + off;
    }
    return L;
}

struct PhaseMarks {
    KnngComm* c;
    cudaStream_t st;
    bool on;
    void mark(int i)
    {
        if (on) cudaEventRecord(c->ev_phase[i], st);
    }
    void collect()
    {
        if (!on) return;
        cudaEventSynchronize(c->ev_phase[6]);
        for (int i = 0; i < 6; ++i) {
            float m = 0.f;
            cudaEventElapsedTime(&m, c->ev_phase[i], c->ev_phase[i + 1]);
            c->phase_ms[i] = m;
        }
        float tot = 0.f;
        cudaEventElapsedTime(&tot, c->ev_phase[0], c->ev_phase[6]);
        c->phase_ms[5] = tot;
    }
};

// Graph rows of every rank to rank 0 (two MPI_Gatherv of
// src/dist/brute_force_mpi.cpp:179-200 as grouped NCCL send/recv).
knng_gpu_status gather_rows_to_root(KnngComm* c, uint64_t n, uint64_t k, const uint32_t* my_ids, const float* my_d,
                                    uint32_t* ids, float* dists, cudaStream_t st)
{
    const ShardRange sh = compute_shard_rows(n, c->world, c->rank);
    KNNG_NCCL(ncclGroupStart());
    if (c->rank == 0) {
        for (int r = 1; r < c->world; ++r) {
            const ShardRange o = compute_shard_rows(n, c->world, r);
            KNNG_NCCL(ncclRecv(ids + o.start * k, o.count * k, ncclUint32, r, c->nccl, st));
            KNNG_NCCL(ncclRecv(dists + o.start * k, o.count * k, ncclFloat32, r, c->nccl, st));
        }
    } else {
        KNNG_NCCL(ncclSend(my_ids, sh.count * k, ncclUint32, 0, c->nccl, st));
        KNNG_NCCL(ncclSend(my_d, sh.count * k, ncclFloat32, 0, c->nccl, st));
    }
    KNNG_NCCL(ncclGroupEnd());
    return KNNG_GPU_OK;
}

knng_gpu_status sharded_replicate(KnngComm* c, const float* slice, uint64_t n, uint64_t d, uint64_t k, int metric,
                                  uint32_t* ids, float* dists, uint8_t* ws, const ShardedLayout& L, cudaStream_t st,
                                  knng_gpu_stats* stats)
{
    const int P = c->world, r = c->rank;
    const uint64_t pitch = knng_gpu_padded_dim(d);
    const uint64_t s = replicate_slice_rows(n, P);
    const uint64_t lo = std::min<uint64_t>(static_cast<uint64_t>(r) * s, n);
    const uint64_t cnt = std::min<uint64_t>(s, n - lo);
    const ShardRange sh = compute_shard_rows(n, P, r);
    int32_t* flag = reinterpret_cast<int32_t*>(ws + L.flag);
    uint8_t* u = ws + L.u;
    uint8_t* packed = u + L.packed;
    int32_t* norms = reinterpret_cast<int32_t*>(u + L.norms);
    uint32_t* my_ids = r == 0 ? ids : reinterpret_cast<uint32_t*>(ws + L.out_ids);
    float* my_d = r == 0 ? dists : reinterpret_cast<float*>(ws + L.out_dists);
    PhaseMarks pm{c, st, stats != nullptr};
    pm.mark(0);
    KNNG_CUDA(cudaMemsetAsync(flag, 0, 4, st));
    KNNG_TRY(pack_impl(slice, cnt, d, packed + static_cast<uint64_t>(r) * s * pitch, norms + static_cast<uint64_t>(r) * s,
                       flag, st));
    pm.mark(1);
    KNNG_NCCL(ncclGroupStart());
    KNNG_NCCL(ncclAllReduce(flag, flag, 1, ncclInt32, ncclMax, c->nccl, st));
    KNNG_NCCL(ncclAllGather(packed + static_cast<uint64_t>(r) * s * pitch, packed, s * pitch, ncclUint8, c->nccl, st));
    KNNG_NCCL(ncclAllGather(norms + static_cast<uint64_t>(r) * s, norms, s, ncclInt32, c->nccl, st));
    KNNG_NCCL(ncclGroupEnd());
    pm.mark(2);
    if (stats) {
        std::memset(stats, 0, sizeof(*stats));
        stats->kernel_launches = 2;
    }
    const U8Sets z{packed + sh.start * pitch, norms + sh.start, sh.count, sh.start, packed, norms, n, 0, 1};
    U8RunOptions opt;
    opt.skip_flag = flag;
    // The tensor-core kernels read the reduced flag and return at once for
    // data that is not integer-valued; only the exact-only path (d > 1024)
    // needs the flag on the host first.
    const bool pair = d <= kMaxTensorDim;
    int32_t nonint = 0;
    if (!pair) {
        KNNG_CUDA(cudaMemcpyAsync(&nonint, flag, 4, cudaMemcpyDeviceToHost, st));
        KNNG_CUDA(cudaStreamSynchronize(st));
    }
    if (nonint == 0 && sh.count > 0) {
        KNNG_TRY(knn_u8_sets_impl(z, d, k, metric, my_ids, my_d, u + L.scratch, scratch_u8_bytes(sh.count, k), st,
                                  stats, opt));
    }
    if (pair || sh.count == 0) {
        KNNG_CUDA(cudaMemcpyAsync(&nonint, flag, 4, cudaMemcpyDeviceToHost, st));
        KNNG_CUDA(cudaStreamSynchronize(st));
    }
    pm.mark(3);
    if (nonint != 0) {
        // fp32 rows: every rank needs them all (the u8 region is free now).
        float* x = reinterpret_cast<float*>(u + L.x);
        if (cnt) KNNG_CUDA(cudaMemcpyAsync(x + static_cast<uint64_t>(r) * s * d, slice, cnt * d * 4,
                                           cudaMemcpyDeviceToDevice, st));
        KNNG_NCCL(ncclAllGather(x + static_cast<uint64_t>(r) * s * d, x, s * d, ncclFloat32, c->nccl, st));
        if (stats) stats->kernel_launches = 2;
        if (sh.count)
            KNNG_TRY(knn_f32_impl(x, n, d, sh.start, sh.count, k, metric, my_ids, my_d, u + L.f32s,
                                  layout_scratch_f32(nullptr, n, d, sh.count, k).total, st, stats));
    }
    pm.mark(4);
    if (P > 1) KNNG_TRY(gather_rows_to_root(c, n, k, my_ids, my_d, ids, dists, st));
    pm.mark(5);
    pm.mark(6);
    KNNG_CUDA(cudaStreamSynchronize(st));
    pm.collect();
    return KNNG_GPU_OK;
}

// Per query row of a ring build: an exact upper bound on the keys that can
// still enter its k best, from the running k-th distance D of the blocks
// searched so far (L2: D - |q|^2, inner product: D itself). D is exact when
// |D| < 2^24 (integer data: every partial sum of the reference's fp32 loop is
// an integer below it); otherwise no bound (INT_MAX).
template <int METRIC>
__global__ void ring_bound_kernel(const float* __restrict__ best_d, uint64_t rows, uint32_t k,
                                  const uint8_t* __restrict__ qpacked, const int32_t* __restrict__ qnorms,
                                  uint32_t pitch, uint32_t data_bytes, int32_t* __restrict__ bound)
{
    const uint64_t r = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const float dk = best_d[r * k + k - 1];
    int32_t b = INT_MAX;
    if (fabsf(dk) < 16777216.0f) {
        const int32_t di = static_cast<int32_t>(dk);
        if constexpr (METRIC == 0) {
            b = di - packed_sq_norm(qpacked, pitch, data_bytes, qnorms, static_cast<uint32_t>(r));
        } else {
            b = di;
        }
    }
    bound[r] = b;
}

knng_gpu_status sharded_ring(KnngComm* c, const float* shard_rows, uint64_t n, uint64_t d, uint64_t k, int metric,
                             uint32_t* ids, float* dists, uint8_t* ws, const ShardedLayout& L, cudaStream_t st,
                             knng_gpu_stats* stats)
{
    const int P = c->world, r = c->rank;
    const uint64_t pitch = knng_gpu_padded_dim(d);
    const ShardRange sh = compute_shard_rows(n, P, r);
    const uint64_t ms = compute_shard_rows(n, P, P - 1).count;
    if (compute_shard_rows(n, P, 0).count < k + 1)
        return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: ring mode needs at least k + 1 rows per rank");
    int32_t* flag = reinterpret_cast<int32_t*>(ws + L.flag);
    uint8_t* u = ws + L.u;
    const uint64_t buf_bytes = align_up(ms * pitch, 256), nbuf_bytes = align_up(ms * 4, 256);
    uint8_t* buf[2] = {u + L.packed, u + L.packed + buf_bytes};
    int32_t* nbuf[2] = {reinterpret_cast<int32_t*>(u + L.norms), reinterpret_cast<int32_t*>(u + L.norms + nbuf_bytes)};
    uint8_t* qpacked = u + L.qpacked;
    int32_t* qnorms = reinterpret_cast<int32_t*>(u + L.qnorms);
    uint32_t* tmp_ids = reinterpret_cast<uint32_t*>(u + L.tmp_ids);
    float* tmp_d = reinterpret_cast<float*>(u + L.tmp_d);
    uint32_t* best_ids[2] = {reinterpret_cast<uint32_t*>(u + L.best_ids), reinterpret_cast<uint32_t*>(ws + L.out_ids)};
    float* best_d[2] = {reinterpret_cast<float*>(u + L.best_d), reinterpret_cast<float*>(ws + L.out_dists)};
    int32_t* bound = reinterpret_cast<int32_t*>(u + L.bound);
    PhaseMarks pm{c, st, stats != nullptr};
    pm.mark(0);
    KNNG_CUDA(cudaMemsetAsync(flag, 0, 4, st));
    KNNG_TRY(pack_impl(shard_rows, sh.count, d, qpacked, qnorms, flag, st));
    KNNG_NCCL(ncclAllReduce(flag, flag, 1, ncclInt32, ncclMax, c->nccl, st));
    int32_t nonint = 0;
    KNNG_CUDA(cudaMemcpyAsync(&nonint, flag, 4, cudaMemcpyDeviceToHost, st));
    KNNG_CUDA(cudaStreamSynchronize(st));
    if (nonint) return fail(KNNG_GPU_NOT_SUPPORTED, "knng::gpu: ring mode needs integer-valued data in [0, 255]");
    KNNG_CUDA(cudaMemcpyAsync(buf[0], qpacked, sh.count * pitch, cudaMemcpyDeviceToDevice, st));
    KNNG_CUDA(cudaMemcpyAsync(nbuf[0], qnorms, sh.count * 4, cudaMemcpyDeviceToDevice, st));
    pm.mark(1);
    pm.mark(2);  // no separate base exchange: the ring passes blocks during the search
    if (stats) {
        std::memset(stats, 0, sizeof(*stats));
        stats->kernel_launches = 2;
    }
    const int right = (r + 1) % P, left = (r + P - 1) % P;
    int cur_best = -1;
    float tc_ms = 0.f, knn_ms = 0.f;
    uint64_t fallback = 0;
    for (int step = 0; step < P; ++step) {
        const int cur = step & 1;
        const int blk = (r - step + P) % P;
        const ShardRange bsh = compute_shard_rows(n, P, blk);
        if (step + 1 < P) {
            // The buffer received into was last read by the previous step.
            KNNG_CUDA(cudaEventRecord(c->ev_compute[cur], st));
            KNNG_CUDA(cudaStreamWaitEvent(c->comm_stream, c->ev_compute[cur], 0));
            KNNG_NCCL(ncclGroupStart());
            KNNG_NCCL(ncclSend(buf[cur], ms * pitch, ncclUint8, right, c->nccl, c->comm_stream));
            KNNG_NCCL(ncclRecv(buf[1 - cur], ms * pitch, ncclUint8, left, c->nccl, c->comm_stream));
            KNNG_NCCL(ncclSend(nbuf[cur], ms, ncclInt32, right, c->nccl, c->comm_stream));
            KNNG_NCCL(ncclRecv(nbuf[1 - cur], ms, ncclInt32, left, c->nccl, c->comm_stream));
            KNNG_NCCL(ncclGroupEnd());
            KNNG_CUDA(cudaEventRecord(c->ev_comm[cur], c->comm_stream));
        }
        // Global ids; the own block excludes self by id (brute_force_mpi.cpp:80-82).
        U8Sets z{qpacked, qnorms, sh.count, sh.start, buf[cur], nbuf[cur], bsh.count, bsh.start, blk == r ? 1 : 0};
        if (step > 0) {
            // From the second block on, only keys at or below the running
            // k-th key can change a row's list.
            const uint32_t db = static_cast<uint32_t>(u8_data_bytes(d));
            const uint32_t grid = static_cast<uint32_t>((sh.count + 255) / 256);
            if (metric == 0)
                ring_bound_kernel<0><<<grid, 256, 0, st>>>(best_d[cur_best], sh.count, static_cast<uint32_t>(k),
                                                           qpacked, qnorms, static_cast<uint32_t>(pitch), db, bound);
            else
                ring_bound_kernel<1><<<grid, 256, 0, st>>>(best_d[cur_best], sh.count, static_cast<uint32_t>(k),
                                                           qpacked, qnorms, static_cast<uint32_t>(pitch), db, bound);
            KNNG_CUDA(cudaGetLastError());
            if (stats) ++stats->kernel_launches;
            z.seed = bound;
        }
        uint32_t* out_i = step == 0 ? best_ids[0] : tmp_ids;
        float* out_d = step == 0 ? best_d[0] : tmp_d;
        knng_gpu_stats bs{};
        KNNG_TRY(knn_u8_sets_impl(z, d, k, metric, out_i, out_d, u + L.scratch, scratch_u8_bytes(ms, k), st,
                                  stats ? &bs : nullptr));
        tc_ms += bs.tc_ms;
        knn_ms += bs.knn_ms;
        fallback += bs.fallback_rows;
        if (stats) stats->kernel_launches += bs.kernel_launches;
        if (step == 0) {
            cur_best = 0;
        } else {
            const int nb = 1 - cur_best;
            merge_topk_kernel<<<static_cast<uint32_t>((sh.count + 255) / 256), 256, 0, st>>>(
                best_ids[cur_best], best_d[cur_best], tmp_ids, tmp_d, sh.count, static_cast<uint32_t>(k),
                best_ids[nb], best_d[nb]);
            KNNG_CUDA(cudaGetLastError());
            if (stats) ++stats->kernel_launches;
            cur_best = nb;
        }
        if (step + 1 < P) KNNG_CUDA(cudaStreamWaitEvent(st, c->ev_comm[cur], 0));
    }
    pm.mark(3);  // search, overlapped with the ring exchange
    pm.mark(4);
    uint32_t* my_ids = best_ids[cur_best];
    float* my_d = best_d[cur_best];
    if (r == 0) {
        KNNG_CUDA(cudaMemcpyAsync(ids, my_ids, sh.count * k * 4, cudaMemcpyDeviceToDevice, st));
        KNNG_CUDA(cudaMemcpyAsync(dists, my_d, sh.count * k * 4, cudaMemcpyDeviceToDevice, st));
    }
    if (P > 1) KNNG_TRY(gather_rows_to_root(c, n, k, my_ids, my_d, ids, dists, st));
    pm.mark(5);
    pm.mark(6);
    KNNG_CUDA(cudaStreamSynchronize(st));
    pm.collect();
    if (stats) {
        stats->path = KNNG_PATH_U8_TENSOR;
        stats->tc_ms = tc_ms;
        stats->knn_ms = knn_ms;
        stats->fallback_rows = fallback;
    }
    return KNNG_GPU_OK;
}

knng_gpu_status comm_resources(KnngComm* c)
{
    KNNG_CUDA(cudaStreamCreateWithFlags(&c->comm_stream, cudaStreamNonBlocking));
    for (int i = 0; i < 2; ++i) {
        KNNG_CUDA(cudaEventCreateWithFlags(&c->ev_compute[i], cudaEventDisableTiming));
        KNNG_CUDA(cudaEventCreateWithFlags(&c->ev_comm[i], cudaEventDisableTiming));
    }
    for (int i = 0; i < 7; ++i) KNNG_CUDA(cudaEventCreate(&c->ev_phase[i]));
    return KNNG_GPU_OK;
}

void comm_release(KnngComm* c)
{
    if (!c) return;
    int cur = 0;
    const bool have = cudaGetDevice(&cur) == cudaSuccess;
    cudaSetDevice(c->device);
    if (c->comm_stream) cudaStreamDestroy(c->comm_stream);
    for (int i = 0; i < 2; ++i) {
        if (c->ev_compute[i]) cudaEventDestroy(c->ev_compute[i]);
        if (c->ev_comm[i]) cudaEventDestroy(c->ev_comm[i]);
    }
    for (int i = 0; i < 7; ++i)
        if (c->ev_phase[i]) cudaEventDestroy(c->ev_phase[i]);
    if (c->nccl && c->owns_nccl) ncclCommDestroy(c->nccl);
    if (have) cudaSetDevice(cur);
    delete c;
}

// ---- one process, several GPUs (knng_gpu_brute_force_multi)
struct MultiDevice {
    KnngComm* comm = nullptr;
    cudaStream_t stream = nullptr;
    void *ws = nullptr, *slice = nullptr, *ids = nullptr, *dists = nullptr;
    uint64_t ws_cap = 0, slice_cap = 0, ids_cap = 0, dists_cap = 0;
    HostStage stage;  // pinned chunks for host buffers the caller did not pin
};
struct MultiCache {
    std::mutex mutex;
    int gpus = 0;
    std::vector<MultiDevice> dev;
};
MultiCache g_multi;

void multi_release_locked()
{
    for (size_t g = 0; g < g_multi.dev.size(); ++g) {
        MultiDevice& m = g_multi.dev[g];
        cudaSetDevice(static_cast<int>(g));
        stage_release(m.stage);
        cudaFree(m.ws);
        cudaFree(m.slice);
        cudaFree(m.ids);
        cudaFree(m.dists);
        if (m.stream) cudaStreamDestroy(m.stream);
        comm_release(m.comm);
    }
    g_multi.dev.clear();
    g_multi.gpus = 0;
    cudaGetLastError();
}

}  // namespace

extern "C" {

uint64_t knng_gpu_nccl_id_bytes(void) { return sizeof(ncclUniqueId); }

knng_gpu_status knng_gpu_nccl_unique_id(void* id_out)
{
    g_last_error.clear();
    if (!id_out) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: id_out is NULL");
    ncclUniqueId id;
    KNNG_NCCL(ncclGetUniqueId(&id));
    std::memcpy(id_out, &id, sizeof(id));
    return KNNG_GPU_OK;
}

knng_gpu_status knng_gpu_comm_create(const void* id, int world, int rank, void** comm_out)
{
    g_last_error.clear();
    if (!id || !comm_out || world < 1 || rank < 0 || rank >= world)
        return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: bad communicator arguments");
    KnngComm* c = new KnngComm();
    c->rank = rank;
    c->world = world;
    cudaGetDevice(&c->device);
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    const ncclResult_t r = ncclCommInitRank(&c->nccl, world, uid, rank);
    if (r != ncclSuccess) {
        delete c;
        return fail(KNNG_GPU_CUDA_ERROR, std::string("knng::gpu: ncclCommInitRank: ") + ncclGetErrorString(r));
    }
    const knng_gpu_status s = comm_resources(c);
    if (s != KNNG_GPU_OK) {
        comm_release(c);
        return s;
    }
    *comm_out = c;
    return KNNG_GPU_OK;
}

void knng_gpu_comm_destroy(void* comm) { comm_release(static_cast<KnngComm*>(comm)); }

void knng_gpu_shard_rows(uint64_t n, int world, int rank, int mode, uint64_t* begin, uint64_t* count)
{
    if (world < 1 || rank < 0 || rank >= world) {
        *begin = *count = 0;
        return;
    }
    if (mode == 0) {
        const uint64_t s = replicate_slice_rows(n, world);
        const uint64_t lo = std::min<uint64_t>(static_cast<uint64_t>(rank) * s, n);
        *begin = lo;
        *count = std::min<uint64_t>(s, n - lo);
    } else {
        const ShardRange sh = compute_shard_rows(n, world, rank);
        *begin = sh.start;
        *count = sh.count;
    }
}

uint64_t knng_gpu_sharded_workspace_bytes(uint64_t n, uint64_t d, uint64_t k, int world, int mode)
{
    if (world < 1) return 0;
    return sharded_layout(n, d, k, world, mode).total;
}

knng_gpu_status knng_gpu_brute_force_sharded(const float* d_rows, uint64_t n, uint64_t d, uint64_t k, int metric,
                                             int mode, void* comm, uint32_t* d_ids, float* d_dists,
                                             void* d_workspace, uint64_t workspace_bytes, void* stream,
                                             knng_gpu_stats* stats)
{
    g_last_error.clear();
    KNNG_TRY(validate(n, d, k, metric));
    KnngComm* c = static_cast<KnngComm*>(comm);
    if (!c) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: communicator is NULL");
    if (mode != 0 && mode != 1) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: mode must be 0 or 1");
    if (c->rank == 0 && (!d_ids || !d_dists))
        return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: rank 0 needs the n x k output arrays");
    const ShardedLayout L = sharded_layout(n, d, k, c->world, mode);
    if (workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(d_workspace) & 255))
        return fail(KNNG_GPU_WORKSPACE_TOO_SMALL, "knng::gpu: workspace smaller than knng_gpu_sharded_workspace_bytes or "
                                                  "not 256-byte aligned");
    uint8_t* ws = static_cast<uint8_t*>(d_workspace);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return mode == 0 ? sharded_replicate(c, d_rows, n, d, k, metric, d_ids, d_dists, ws, L, st, stats)
                     : sharded_ring(c, d_rows, n, d, k, metric, d_ids, d_dists, ws, L, st, stats);
}

knng_gpu_status knng_gpu_comm_phase_ms(void* comm, float* out6)
{
    KnngComm* c = static_cast<KnngComm*>(comm);
    if (!c || !out6) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: NULL argument");
    std::memcpy(out6, c->phase_ms, sizeof(c->phase_ms));
    return KNNG_GPU_OK;
}

knng_gpu_status knng_gpu_brute_force_multi(const float* data, uint64_t n, uint64_t d, uint64_t k, int metric,
                                           int num_gpus, int mode, uint32_t* ids, float* dists,
                                           knng_gpu_stats* stats)
{
    g_last_error.clear();
    KNNG_TRY(validate(n, d, k, metric));
    if (mode != 0 && mode != 1) return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: mode must be 0 or 1");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(KNNG_GPU_CUDA_ERROR, "knng::gpu::brute_force_knn: no CUDA device available");
    }
    if (num_gpus < 1 || num_gpus > ndev)
        return fail(KNNG_GPU_INVALID_ARGUMENT, "knng::gpu: num_gpus must be in [1, " + std::to_string(ndev) + "]");
    std::lock_guard<std::mutex> lock(g_multi.mutex);
    int cur = 0;
    cudaGetDevice(&cur);
    if (g_multi.gpus != num_gpus) {
        multi_release_locked();
        std::vector<ncclComm_t> comms(num_gpus);
        std::vector<int> devs(num_gpus);
        for (int g = 0; g < num_gpus; ++g) devs[g] = g;
        KNNG_NCCL(ncclCommInitAll(comms.data(), num_gpus, devs.data()));
        g_multi.dev.resize(num_gpus);
        g_multi.gpus = num_gpus;
        for (int g = 0; g < num_gpus; ++g) {
            KNNG_CUDA(cudaSetDevice(g));
            KnngComm* c = new KnngComm();
            c->nccl = comms[g];
            c->rank = g;
            c->world = num_gpus;
            c->device = g;
            g_multi.dev[g].comm = c;
            KNNG_TRY(comm_resources(c));
            KNNG_CUDA(cudaStreamCreateWithFlags(&g_multi.dev[g].stream, cudaStreamNonBlocking));
        }
    }
    std::vector<knng_gpu_status> status(num_gpus, KNNG_GPU_OK);
    std::vector<std::string> errors(num_gpus);
    std::vector<knng_gpu_stats> st(num_gpus);
    auto run = [&](int g) {
        MultiDevice& m = g_multi.dev[g];
        auto body = [&]() -> knng_gpu_status {
            KNNG_CUDA(cudaSetDevice(g));
            uint64_t lo = 0, cnt = 0;
            knng_gpu_shard_rows(n, num_gpus, g, mode, &lo, &cnt);
            KNNG_TRY(grow(&m.ws, &m.ws_cap, knng_gpu_sharded_workspace_bytes(n, d, k, num_gpus, mode)));
            KNNG_TRY(grow(&m.slice, &m.slice_cap, std::max<uint64_t>(cnt, 1) * d * 4));
            if (g == 0) {
                KNNG_TRY(grow(&m.ids, &m.ids_cap, n * k * 4));
                KNNG_TRY(grow(&m.dists, &m.dists_cap, n * k * 4));
            }
            KNNG_TRY(copy_to_device(m.stage, m.slice, data + lo * d, cnt * d * 4, m.stream));
            KNNG_TRY(knng_gpu_brute_force_sharded(static_cast<const float*>(m.slice), n, d, k, metric, mode, m.comm,
                                                  static_cast<uint32_t*>(m.ids), static_cast<float*>(m.dists), m.ws,
                                                  m.ws_cap, m.stream, stats ? &st[g] : nullptr));
            if (g == 0) {
                KNNG_TRY(copy_to_host(m.stage, ids, m.ids, n * k * 4, m.stream));
                KNNG_TRY(copy_to_host(m.stage, dists, m.dists, n * k * 4, m.stream));
            }
            KNNG_CUDA(cudaStreamSynchronize(m.stream));
            return KNNG_GPU_OK;
        };
        status[g] = body();
        if (status[g] != KNNG_GPU_OK) errors[g] = g_last_error;
    };
    std::vector<std::thread> threads;
    for (int g = 1; g < num_gpus; ++g) threads.emplace_back(run, g);
    run(0);
    for (auto& t : threads) t.join();
    cudaSetDevice(cur);
    for (int g = 0; g < num_gpus; ++g)
        if (status[g] != KNNG_GPU_OK) return fail(status[g], errors[g]);
    if (stats) *stats = st[0];
    return KNNG_GPU_OK;
}

void knng_gpu_release_multi(void)
{
    std::lock_guard<std::mutex> lock(g_multi.mutex);
    int cur = 0;
    const bool have = cudaGetDevice(&cur) == cudaSuccess;
    multi_release_locked();
    if (have) cudaSetDevice(cur);
}

}  // extern "C"
