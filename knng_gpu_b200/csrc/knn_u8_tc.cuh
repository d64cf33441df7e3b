// knn_u8_tc.cuh -- fused exact KNN for integer-valued data on the 5th-gen
// tensor cores: u8 x u8 -> s32 UMMA (tcgen05.mma kind::i8) into TMEM, with
// the top-k selection in the epilogue so the n x n distance matrix never
// leaves the SM.
//
// Restates, for data whose every coordinate is an integer in [0, 255],
//   knng::cpu::brute_force_knn<L2Squared | NegativeInnerProduct>
//   (include/knng/cpu/brute_force.hpp:336-376)
// with the norm identity of brute_force_knn_l2_with_norms
// (src/cpu/brute_force.cpp:261-323): for a fixed query q the ranking key of a
// base row r is  s(q, r) = |r|^2 - 2 q.r  (L2; dist = |q|^2 + s) or -q.r
// (negative inner product). All of it is exact int32 arithmetic, so ranks,
// ties and the emitted fp32 distances equal the reference's sequential fp32
// sums bit for bit whenever those sums stay below 2^24 (always for L2 at
// d <= 258); rows where they may not are routed to the exact fp32 kernel.
//
// CTA layout (persistent, one CTA per SM):
//   warp 0       TMA producer: A = MT query tiles of 128 rows (resident for a
//                query tile), B = ring of STAGES base tiles (BN rows x 128 B)
//   warp 1       TMEM allocator and UMMA issuer (one elected lane)
//   warps 2..    4*MT epilogue warps; thread <-> one query row (TMEM lane),
//                all BN columns of every base tile
// TMEM: NBUF accumulator buffers x MT x BN columns (s32). With NBUF = 2 the
// epilogue of base tile j overlaps the MMAs of tile j+1; with NBUF = 1 and
// MT = 2 the two query tiles alternate (epilogue of one, MMAs of the other).
#pragma once
#include <climits>
#include <cstdint>

#include "ptx.cuh"
#include "topk.cuh"

namespace knng_b200 {

constexpr int kTileRows = 128;      // M per UMMA; rows per TMA box
constexpr int kChunkBytes = 128;    // K bytes per TMA box / swizzle atom
constexpr int kBoxBytes = kTileRows * kChunkBytes;  // 16 KiB
constexpr int kSlowPitch = 36;      // ints per thread in the slow-path spill area

struct KnnU8Params {
    const int32_t* base_norms;   // L2: |r|^2 per base row
    const int32_t* query_norms;  // L2: |q|^2 per query row of this launch
    uint64_t n_base;             // valid base rows
    uint32_t base_id0;           // global id of base row 0
    uint32_t n_queries;          // query rows in this launch
    uint32_t query_row0;         // first query row inside the A tensor map
    uint32_t query_id0;          // global id of query row 0 (self exclusion)
    uint32_t exclude_self;
    uint32_t k;
    uint32_t kchunks;            // padded d / 128
    uint32_t stages;
    uint32_t* out_ids;           // n_queries x k
    float* out_dists;            // n_queries x k
    uint32_t* fallback_rows;     // rows whose fp32 sums may be inexact
    uint32_t* fallback_count;
    int* error;                  // non-zero: a bounded wait gave up
    uint32_t debug_flags;        // profiling only: 1 skip filtering, 2 skip insertion, 4 skip TMEM loads
};

struct SmemLayoutU8 {
    uint32_t a_off, b_off, nb_off, slow_off, merge_off, bar_off, total;
};

// split: epilogue warps per (M tile, TMEM lane quarter); each covers 1/split
// of the columns, and the partial lists are merged through `merge`.
__host__ __device__ inline SmemLayoutU8 smem_layout_u8(int mt, int bn, uint32_t kchunks, uint32_t stages,
                                                       int split = 1, int kcap = 0)
{
    SmemLayoutU8 L;
    const int epi_threads = mt * kTileRows * split;
    L.a_off = 0;
    L.b_off = L.a_off + mt * kchunks * kBoxBytes;
    L.nb_off = L.b_off + stages * (bn / kTileRows) * kBoxBytes;
    L.slow_off = L.nb_off + (epi_threads / 32) * 2 * bn * 4;  // per epilogue warp, double-buffered
    L.merge_off = L.slow_off + epi_threads * kSlowPitch * 4;
    L.bar_off = L.merge_off + (split > 1 ? mt * kTileRows * 2 * kcap * 4 : 0);
    L.total = L.bar_off + 512;  // barriers + tmem slot + abort flag
    return L;
}

// Balanced three-way minimum tree over N registers (compile-time shape, so
// the operands stay in registers).
template <int N>
__device__ __forceinline__ int32_t tree_min(const int32_t* v)
{
    if constexpr (N == 1) {
        return v[0];
    } else if constexpr (N == 2) {
        return min(v[0], v[1]);
    } else if constexpr (N == 3) {
        return __vimin3_s32(v[0], v[1], v[2]);
    } else {
        constexpr int a = N / 3, b = (N - a) / 2, c = N - a - b;
        return __vimin3_s32(tree_min<a>(v), tree_min<b>(v + a), tree_min<c>(v + a + b));
    }
}

template <int MT, int BN, int NBUF, int SPLIT, int METRIC, class TopK>
__global__ void __launch_bounds__(64 + 128 * MT * SPLIT, 1)
    knn_u8_tc_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_b,
                     const KnnU8Params p)
{
    static_assert(NBUF <= 4 && MT * NBUF <= 4, "barrier slots");
    static_assert(MT * NBUF * BN <= 512, "TMEM holds 512 columns");
    static_assert(BN % 128 == 0 && BN <= 256, "BN is 128 or 256");
    constexpr int kBoxesPerStage = BN / kTileRows;
    constexpr uint32_t kStageBytes = kBoxesPerStage * kBoxBytes;
    constexpr uint32_t kTmemCols = MT * NBUF * BN <= 256 ? 256 : 512;
    // Every tcgen05.commit costs the MMA pipe several hundred cycles, so with
    // two TMEM buffers all M tiles of a base tile share one handoff barrier;
    // with one buffer each M tile gets its own so the two tiles alternate.
    constexpr bool kPerMtBars = NBUF == 1 && MT > 1;
    static_assert(SPLIT == 1 || (SPLIT == 2 && TopK::kRegs <= 32), "split epilogue needs register lists");
    constexpr int kCap = TopK::kRegs / 2;

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const SmemLayoutU8 L = smem_layout_u8(MT, BN, p.kchunks, p.stages, SPLIT, SPLIT > 1 ? kCap : 0);
    uint8_t* sA = smem + L.a_off;
    uint8_t* sB = smem + L.b_off;
    int32_t* sNB = reinterpret_cast<int32_t*>(smem + L.nb_off);
    int32_t* sSlow = reinterpret_cast<int32_t*>(smem + L.slow_off);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    const uint32_t S = p.stages;
    uint64_t* full = bars;             // [S], S <= 16
    uint64_t* empty = bars + 16;       // [S]
    uint64_t* a_full = bars + 32;
    uint64_t* a_empty = bars + 33;
    uint64_t* tfull = bars + 34;       // [NBUF * MT]
    uint64_t* tempty = bars + 38;      // [NBUF * MT]
    uint64_t* merge_full = bars + 42;  // [MT]
    uint64_t* merge_empty = bars + 44; // [MT]
    int32_t* sMerge = reinterpret_cast<int32_t*>(smem + L.merge_off);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 46);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 47);
    // Base tiles whose MMAs are known complete (published by one epilogue
    // thread after its handoff wait). The producer reuses a B stage once the
    // tile that read it is counted here, so the MMA warp issues one
    // tcgen05.commit per tile (the TMEM handoff) instead of two.
    volatile uint32_t* tiles_done = reinterpret_cast<volatile uint32_t*>(bars + 48);
    // With fewer stages than two tiles' worth of K chunks a tile cannot wait
    // for a whole earlier tile, so stages are released per chunk instead.
    const bool stage_commits = p.stages < 2 * p.kchunks;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t n_qtiles = (p.n_queries + MT * kTileRows - 1) / (MT * kTileRows);
    const uint32_t n_btiles = static_cast<uint32_t>((p.n_base + BN - 1) / BN);

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(a_full, 1);
        mbar_init(a_empty, 1);
        for (int b = 0; b < NBUF * MT; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kPerMtBars ? 4 * SPLIT : 4 * MT * SPLIT);
        }
        for (int m = 0; m < MT; ++m) {
            mbar_init(&merge_full[m], 4);
            mbar_init(&merge_empty[m], 4);
        }
        *abort_flag = 0;
        *tiles_done = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmap_q);
        prefetch_tensormap(&tmap_b);
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, a_par = 0, load_idx = 0;
            bool ok = true;
            for (uint32_t t = blockIdx.x; t < n_qtiles && ok; t += gridDim.x) {
                ok = mbar_wait(a_empty, a_par ^ 1, abort_flag);
                if (!ok) break;
                a_par ^= 1;
                mbar_arrive_expect_tx(a_full, MT * p.kchunks * kBoxBytes);
                for (int mt = 0; mt < MT; ++mt)
                    for (uint32_t kc = 0; kc < p.kchunks; ++kc)
                        tma_load_2d(sA + (mt * p.kchunks + kc) * kBoxBytes, &tmap_q, kc * kChunkBytes,
                                    p.query_row0 + (t * MT + mt) * kTileRows, a_full);
                for (uint32_t j = 0; j < n_btiles && ok; ++j) {
                    for (uint32_t kc = 0; kc < p.kchunks; ++kc) {
                        if (stage_commits) {
                            ok = mbar_wait(&empty[stage], phase ^ 1, abort_flag);
                            if (!ok) break;
                        } else if (load_idx >= S) {
                            // The stage last held load (load_idx - S), part of
                            // tile (load_idx - S) / kchunks.
                            ok = spin_until_geq(tiles_done, (load_idx - S) / p.kchunks + 1, abort_flag);
                            if (!ok) break;
                        }
                        ++load_idx;
                        mbar_arrive_expect_tx(&full[stage], kStageBytes);
#pragma unroll
                        for (int bx = 0; bx < kBoxesPerStage; ++bx)
                            tma_load_2d(sB + stage * kStageBytes + bx * kBoxBytes, &tmap_b, kc * kChunkBytes,
                                        j * BN + bx * kTileRows, &full[stage]);
                        if (++stage == S) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            if (!ok) {
                atomicOr(p.error, 1);
                *abort_flag = 1;
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ UMMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_u8_s32(kTileRows, BN);
            uint32_t stage0 = 0, phase0 = 0, a_par = 0, acc_i = 0;
            bool ok = true;
            const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
            for (uint32_t t = blockIdx.x; t < n_qtiles && ok; t += gridDim.x) {
                ok = mbar_wait(a_full, a_par, abort_flag);
                if (!ok) break;
                a_par ^= 1;
                tc_fence_after();
                for (uint32_t j = 0; j < n_btiles && ok; ++j, ++acc_i) {
                    const uint32_t buf = acc_i % NBUF;
                    const uint32_t tpar = (acc_i / NBUF) & 1;
                    if (kPerMtBars) {
                        // One buffer per M tile: M tile mt waits for its own
                        // epilogue; a B stage is released after the last M tile.
                        for (int mt = 0; mt < MT && ok; ++mt) {
                            ok = mbar_wait(&tempty[mt], tpar ^ 1, abort_flag);
                            if (!ok) break;
                            tc_fence_after();
                            const uint32_t d_tmem = tmem_base + mt * BN;
                            for (uint32_t kc = 0; kc < p.kchunks; ++kc) {
                                const uint32_t idx = stage0 + kc;
                                const uint32_t s = idx % S;
                                if (mt == 0) {
                                    ok = mbar_wait(&full[s], phase0 ^ ((idx / S) & 1), abort_flag);
                                    if (!ok) break;
                                    tc_fence_after();
                                }
                                const uint32_t bs = b_base + s * kStageBytes;
                                const uint32_t as = a_base + (mt * p.kchunks + kc) * kBoxBytes;
#pragma unroll
                                for (int ks = 0; ks < kChunkBytes / 32; ++ks)
                                    umma_u8(d_tmem, umma_desc_sw128(as + ks * 32), umma_desc_sw128(bs + ks * 32),
                                            idesc, (kc | ks) != 0);
                                if (stage_commits && mt == MT - 1) umma_commit(&empty[s]);
                            }
                            if (ok) umma_commit(&tfull[mt]);
                        }
                    } else {
                        ok = mbar_wait(&tempty[buf], tpar ^ 1, abort_flag);
                        if (!ok) break;
                        tc_fence_after();
                        for (uint32_t kc = 0; kc < p.kchunks && ok; ++kc) {
                            const uint32_t idx = stage0 + kc;
                            const uint32_t s = idx % S;
                            ok = mbar_wait(&full[s], phase0 ^ ((idx / S) & 1), abort_flag);
                            if (!ok) break;
                            tc_fence_after();
                            const uint32_t bs = b_base + s * kStageBytes;
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt) {
                                const uint32_t as = a_base + (mt * p.kchunks + kc) * kBoxBytes;
                                const uint32_t d_tmem = tmem_base + (buf * MT + mt) * BN;
#pragma unroll
                                for (int ks = 0; ks < kChunkBytes / 32; ++ks)
                                    umma_u8(d_tmem, umma_desc_sw128(as + ks * 32), umma_desc_sw128(bs + ks * 32),
                                            idesc, (kc | ks) != 0);
                            }
                            if (stage_commits) umma_commit(&empty[s]);
                        }
                        if (ok) umma_commit(&tfull[buf]);
                    }
                    const uint32_t next = stage0 + p.kchunks;
                    phase0 ^= (next / S) & 1;
                    stage0 = next % S;
                }
                if (ok) umma_commit(a_empty);
            }
            if (!ok) {
                atomicOr(p.error, 2);
                *abort_flag = 1;
            }
        }
    } else {
        // ------------------------------------------------ epilogue
        const int ew = warp - 2;
        const int grp = ew >> 2;
        const int mt = grp % MT;
        const int half = grp / MT;  // which 1/SPLIT of the columns
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        int32_t* nbuf = sNB + ew * 2 * BN;  // this warp's copy of the base-tile norms
        int32_t* slow = sSlow + (ew * 32 + lane) * kSlowPitch;
        int32_t* merge_slot = sMerge + (mt * kTileRows + row) * 2 * kCap;
        uint32_t qt_iter = 0;
        // Column keys are  nb - scale * dot  with nb = |r|^2 (L2) or 0 (IP)
        // for real rows and INT_MAX for padding rows (dot == 0 there), so
        // padding never enters the list. Lane l fetches columns 4l..4l+3 of
        // every 128-column block.
        auto load_norms = [&](uint32_t j, int blk) -> int4 {
            const uint64_t b0 = static_cast<uint64_t>(j) * BN + blk * kTileRows + lane * 4;
            if (b0 + 3 < p.n_base)
                return METRIC == 0 ? __ldg(reinterpret_cast<const int4*>(p.base_norms + b0)) : make_int4(0, 0, 0, 0);
            int4 nn;
            nn.x = b0 + 0 < p.n_base ? (METRIC == 0 ? p.base_norms[b0 + 0] : 0) : INT_MAX;
            nn.y = b0 + 1 < p.n_base ? (METRIC == 0 ? p.base_norms[b0 + 1] : 0) : INT_MAX;
            nn.z = b0 + 2 < p.n_base ? (METRIC == 0 ? p.base_norms[b0 + 2] : 0) : INT_MAX;
            nn.w = b0 + 3 < p.n_base ? (METRIC == 0 ? p.base_norms[b0 + 3] : 0) : INT_MAX;
            return nn;
        };
        uint32_t acc_i = 0;
        bool ok = true;
        for (uint32_t t = blockIdx.x; t < n_qtiles && ok; t += gridDim.x, ++qt_iter) {
            const uint32_t qlocal = (t * MT + mt) * kTileRows + row;
            const bool qvalid = qlocal < p.n_queries;
            const uint32_t self_id = p.exclude_self ? p.query_id0 + qlocal : UINT32_MAX;
            const int32_t qnorm = (METRIC == 0 && qvalid) ? p.query_norms[qlocal] : 0;
            TopK tk;
            tk.init(p.k);
            int32_t thr = tk.thr();
            int4 nn_next[kBoxesPerStage];
#pragma unroll
            for (int b = 0; b < kBoxesPerStage; ++b) nn_next[b] = load_norms(0, b);
            for (uint32_t j = 0; j < n_btiles; ++j, ++acc_i) {
                // Publish this tile's norms (fetched one tile earlier) and
                // start fetching the next tile's, so the global latency hides
                // behind a whole tile of work.
#pragma unroll
                for (int b = 0; b < kBoxesPerStage; ++b) {
                    reinterpret_cast<int4*>(nbuf + (j & 1) * BN + b * kTileRows)[lane] = nn_next[b];
                    if (j + 1 < n_btiles) nn_next[b] = load_norms(j + 1, b);
                }
                __syncwarp();
                const uint32_t buf = acc_i % NBUF;
                const uint32_t hb = kPerMtBars ? mt : buf;  // handoff barrier
                ok = mbar_wait(&tfull[hb], (acc_i / NBUF) & 1, abort_flag);
                if (!ok) break;
                tc_fence_after();
                if (ew == (kPerMtBars ? 4 * (MT - 1) : 0) && lane == 0) *tiles_done = acc_i + 1;
                const uint32_t tb =
                    tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + (buf * MT + mt) * BN;
                const int4* nb4 = reinterpret_cast<const int4*>(nbuf + (j & 1) * BN);
                // 32-column chunks, software-pipelined: the TMEM load of chunk
                // c+1 is in flight while chunk c is filtered.
                // Steps of kW columns: one TMEM wait per step, all keys of the
                // step computed before one threshold test (ILP over kW keys).
                constexpr int kCols = BN / SPLIT;
                constexpr int kW = (SPLIT == 1 && TopK::kRegs <= 64) ? 64 : 32;
                const uint32_t tbh = tb + half * kCols;
                const int4* nb4h = nb4 + half * kCols / 4;
#pragma unroll
                for (int st = 0; st < kCols / kW; ++st) {
                    int32_t v[kW];
                    __syncwarp();
                    if (!(p.debug_flags & 4u)) {
#pragma unroll
                        for (int c = 0; c < kW / 32; ++c) tmem_ld_32cols(tbh + st * kW + c * 32, v + c * 32);
                        tmem_ld_wait_n<kW>(v);
                    }
                    if (st + 1 == kCols / kW) {
                        // Every column of this buffer is in registers: hand it
                        // back to the MMA warp before the last filtering step.
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[hb]);
                    }
                    if (p.debug_flags & 1u) continue;
#pragma unroll
                    for (int i4 = 0; i4 < kW / 4; ++i4) {
                        const int4 nn = nb4h[st * kW / 4 + i4];
                        if (METRIC == 0) {
                            v[4 * i4 + 0] = nn.x - 2 * v[4 * i4 + 0];
                            v[4 * i4 + 1] = nn.y - 2 * v[4 * i4 + 1];
                            v[4 * i4 + 2] = nn.z - 2 * v[4 * i4 + 2];
                            v[4 * i4 + 3] = nn.w - 2 * v[4 * i4 + 3];
                        } else {
                            v[4 * i4 + 0] = nn.x - v[4 * i4 + 0];
                            v[4 * i4 + 1] = nn.y - v[4 * i4 + 1];
                            v[4 * i4 + 2] = nn.z - v[4 * i4 + 2];
                            v[4 * i4 + 3] = nn.w - v[4 * i4 + 3];
                        }
                    }
                    const int32_t step_min = tree_min<kW>(v);  // depth log3(kW)
                    if (step_min < thr && !(p.debug_flags & 2u)) {
                        // Rare path, per 32 columns: spill the keys and insert
                        // those under the running threshold, in id order.
#pragma unroll
                        for (int c = 0; c < kW / 32; ++c) {
                            const int32_t* vc = v + c * 32;
                            uint32_t mask = 0;
#pragma unroll
                            for (int i = 0; i < 32; ++i) mask |= (vc[i] < thr ? 1u : 0u) << i;
                            if (!mask) continue;
#pragma unroll
                            for (int i4 = 0; i4 < 8; ++i4)
                                *reinterpret_cast<int4*>(slow + 4 * i4) =
                                    make_int4(vc[4 * i4], vc[4 * i4 + 1], vc[4 * i4 + 2], vc[4 * i4 + 3]);
                            const uint32_t col0 = p.base_id0 + j * BN + half * kCols + st * kW + c * 32;
                            while (mask) {
                                const int i = __ffs(mask) - 1;
                                mask &= mask - 1;
                                const int32_t key = slow[i];
                                const uint32_t id = col0 + i;
                                if (key < thr && id != self_id) {
                                    tk.insert_increasing(key, id);
                                    thr = tk.thr();
                                }
                            }
                        }
                    }
                }
            }
            if (!ok) break;
            if constexpr (SPLIT > 1) {
                // Merge the column halves: half 1 publishes its sorted list,
                // half 0 inserts it into its own (same (key, id) order).
                const uint32_t mpar = qt_iter & 1;
                if (half == 1) {
                    ok = mbar_wait(&merge_empty[mt], mpar ^ 1, abort_flag);
                    if (!ok) break;
                    tk.for_each(p.k, [&](int jj, int32_t key, uint32_t id) {
                        merge_slot[jj] = key;
                        merge_slot[kCap + jj] = static_cast<int32_t>(id);
                    });
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&merge_full[mt]);
                    continue;
                }
                ok = mbar_wait(&merge_full[mt], mpar, abort_flag);
                if (!ok) break;
                for (uint32_t jj = 0; jj < p.k; ++jj) {
                    const int32_t key = merge_slot[jj];
                    const uint32_t id = static_cast<uint32_t>(merge_slot[kCap + jj]);
                    if (key_gt(tk.thr(), tk.thr_id(), key, id)) tk.insert(key, id);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&merge_empty[mt]);
            }
            if (qvalid) {
                uint32_t* oid = p.out_ids + static_cast<uint64_t>(qlocal) * p.k;
                float* odist = p.out_dists + static_cast<uint64_t>(qlocal) * p.k;
                bool inexact = false;
                if (METRIC == 0) {
                    // Partial sums of squares are monotone: every retained sum
                    // is exact in fp32 iff the k-th is below 2^24.
                    inexact = static_cast<int64_t>(qnorm) + tk.thr() >= (1 << 24);
                    tk.for_each(p.k, [&](int jj, int32_t key, uint32_t id) {
                        oid[jj] = id;
                        odist[jj] = __int2float_rn(qnorm + key);
                    });
                } else {
                    // Largest dot first: exact iff it is below 2^24.
                    inexact = -static_cast<int64_t>(tk.best(p.k)) >= (1 << 24);
                    tk.for_each(p.k, [&](int jj, int32_t key, uint32_t id) {
                        oid[jj] = id;
                        odist[jj] = -__int2float_rn(-key);
                    });
                }
                if (inexact && p.debug_flags == 0) {
                    const uint32_t slot = atomicAdd(p.fallback_count, 1u);
                    p.fallback_rows[slot] = qlocal;
                }
            }
        }
        if (!ok) {
            atomicOr(p.error, 4);
            *abort_flag = 1;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

}  // namespace knng_b200
