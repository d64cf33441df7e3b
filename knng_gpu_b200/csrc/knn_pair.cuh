// knn_pair.cuh -- exact u8 brute-force KNN on a CTA pair (cta_group::2).
//
// Same arithmetic and output as the u8 path of knn_tc.cuh (exact int32 keys
// |r|^2 - 2 q.r or -q.r from u8 x u8 -> s32 UMMAs, norms folded into K by the
// augmentation bytes, top-k in the epilogue; knng::cpu::brute_force_knn,
// include/knng/cpu/brute_force.hpp:336-376), with a tile shape that keeps the
// tensor pipe fed:
//
//  * Two CTAs on two SMs form a cluster. The leader issues
//    tcgen05.mma.cta_group::2 with M = 256 (128 query rows resident in each
//    CTA) and N = 256 base rows per tile, each CTA holding 128 of those base
//    rows in its own shared memory (plain TMA, no multicast). Per SM and per
//    MMA the tensor core then reads 4 KiB of A and 4 KiB of B for 128 x 256 x
//    32 MACs: half the shared-memory traffic per MAC of a single-CTA
//    128 x 128 tile, and one commit/hand-off per 256 base columns.
//  * TMEM: two 256-column accumulator buffers per CTA, so the epilogue of
//    base tile j overlaps the MMAs of tile j + 1.
//  * Work is split stream-K style: the (query tile, base tile) space is cut
//    into one contiguous range per CTA pair, so every pair does the same
//    number of tiles and there is no partial last wave. A query tile cut
//    between pairs leaves partial (key, id) lists that merge_pair_partials
//    combines by (key, id) afterwards -- exact, since the keys are exact.
//
// CTA roles (each CTA of the pair):
//   warp 0    TMA producer: this CTA's 128 query rows (kchunks boxes, resident
//             per query tile) and its 128-row half of every base tile; the
//             byte counts land on the leader's barriers. L2 also fetches the
//             256 key offsets of each base tile into a local slot.
//   warp 1    TMEM allocation (both CTAs); UMMA issue (leader, one lane)
//   warps 2-5 epilogue: thread <-> one query row (TMEM lane), all 256
//             columns of every tile, one sorted register list per row
#pragma once
#include <climits>
#include <cstdint>

#include "knn_tc.cuh"
#include "schedule.cuh"

namespace knng_b200 {

constexpr int kPairTile = 256;    // base rows per tile, query rows per pair
// Threads of a pair CTA with EPI epilogue warps (4: one per TMEM lane
// quarter, each over all 256 columns of a tile; 8 or 16: two or four per
// quarter, each over a 128- or 64-column slice).
constexpr int pair_threads(int epi) { return 64 + 32 * epi; }
constexpr int kPairNormSlots = 8;  // key-offset slots (one base tile each)

struct PairParams {
    const int32_t* query_norms;  // key offset per query row (L2)
    const uint8_t* query_packed; // packed query rows (augmentation bytes give |q|^2)
    uint32_t pitch;
    uint32_t data_bytes;
    uint64_t n_base;
    uint32_t base_id0;
    uint32_t n_queries;
    uint32_t query_id0;
    uint32_t exclude_self;
    uint32_t k;
    uint32_t kchunks;
    uint32_t stages;
    TileSchedule sched;  // units = CTA pairs; 256-row query tiles, 256-row base tiles
    uint32_t* out_ids;
    float* out_dists;
    int32_t* part_keys;  // [2 * n_pairs][256][k] partial lists of cut query tiles
    uint32_t* part_ids;
    uint32_t* fallback_rows;
    uint32_t* fallback_count;
    int* error;
    const int* skip_flag;  // optional: non-zero -> the data is not integer-valued, do nothing
    const int32_t* seed_in;  // optional: per query row, an upper bound on the keys its list admits
    int32_t* seed_out;       // seeding pass: write each query row's k-th key instead of its list
    long long wait_limit;  // clock cycles before a wait gives up
    uint32_t test_mode;    // 1: the leader's producer withholds one arrival (timeout test)
    uint32_t debug_flags;  // profiling builds only: 1 no filtering, 2 no TMEM loads, 4 no MMAs, 512 clocks
    unsigned long long* debug_clocks;  // profiling builds only (flag 512): per-role cycle counters
};

#ifdef KNNG_GPU_EXPERIMENTS
constexpr bool kPairProfile = true;
#else
constexpr bool kPairProfile = false;
#endif

struct SmemLayoutPair {
    uint32_t a_off, aug_off, b_off, norm_off, merge_off, bar_off, total, stage_bytes;
};

// merge_kcap > 0: two slots of 128 rows x merge_kcap (key, id) pairs where
// the column slices' lists of a row meet at the end of a segment.
__host__ __device__ inline SmemLayoutPair smem_layout_pair(uint32_t kchunks, uint32_t stages, bool l2,
                                                           uint32_t merge_kcap = 0)
{
    SmemLayoutPair L;
    L.stage_bytes = kBoxBytes + (l2 ? kAugBox : 0);
    L.a_off = 0;
    L.aug_off = kchunks * kBoxBytes;
    L.b_off = L.aug_off + (l2 ? kAugBox : 0);
    L.norm_off = L.b_off + stages * L.stage_bytes;
    L.merge_off = L.norm_off + (l2 ? kPairNormSlots * kPairTile * 4 : 0);
    L.bar_off = L.merge_off + 2 * kTileRows * merge_kcap * 8;
    L.total = L.bar_off + 512;
    return L;
}

// UMMA instruction descriptor of the pair tile (M = 256 over two CTAs).
__host__ __device__ constexpr uint32_t idesc_pair_u8() { return idesc_u8_s32(2 * kTileRows, kPairTile); }

template <int METRIC, class TopK, int EPI>
__global__ void __launch_bounds__(pair_threads(EPI), 1) knn_pair_kernel(const __grid_constant__ CUtensorMap tmap_q,
                                                                   const __grid_constant__ CUtensorMap tmap_b,
                                                                   const __grid_constant__ CUtensorMap tmap_baug,
                                                                   const __grid_constant__ CUtensorMap tmap_norm,
                                                                   const PairParams p)
{
    constexpr bool kL2 = METRIC == 0;
    static_assert(EPI == 4 || EPI == 8 || EPI == 16, "epilogue warps");
    constexpr int kSlices = EPI / 4;             // column slices per tile
    constexpr int kSliceCols = kPairTile / kSlices;
    constexpr int kSteps = kSliceCols / 32;      // 32-column steps per tile and warp
    constexpr int kMergeCap = kSlices > 1 ? TopK::kRegs / 2 : 0;
    // With four epilogue warps the load of the next 32 columns overlaps the
    // filter of the current ones (when the register list is small).
    constexpr bool kPipe = EPI == 4 && TopK::kRegs <= 32;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const SmemLayoutPair L = smem_layout_pair(p.kchunks, p.stages, kL2, kMergeCap);
    uint8_t* sA = smem + L.a_off;
    uint8_t* sAaug = smem + L.aug_off;
    uint8_t* sB = smem + L.b_off;
    int32_t* sNorm = reinterpret_cast<int32_t*>(smem + L.norm_off);
    int32_t* sMerge = reinterpret_cast<int32_t*>(smem + L.merge_off);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    const uint32_t S = p.stages;
    uint64_t* full = bars;         // [S] leader: stage loaded (both CTAs' bytes)
    uint64_t* empty = bars + 16;   // [S] both: stage consumed (per-chunk release mode)
    uint64_t* a_full = bars + 32;  // leader: query rows loaded
    uint64_t* a_empty = bars + 33; // both: MMAs of a query tile done
    uint64_t* tfull = bars + 34;   // [2] both: accumulator buffer ready
    uint64_t* tempty = bars + 36;  // [2] leader: buffer drained by the epilogue warps of both CTAs
    uint64_t* nfull = bars + 38;   // [8] local: key offsets of a tile landed
    uint64_t* nempty = bars + 46;  // [8] local: key offsets read by the epilogue warps
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 54);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 55);
    // Base tiles whose MMAs are complete (published by one epilogue thread
    // after its hand-off wait): a B stage is reused once its tile is counted.
    volatile uint32_t* tiles_done = reinterpret_cast<volatile uint32_t*>(bars + 56);
    // Per lane quarter: arrivals of its slice warps at the segment-end merge
    // (a bounded counter barrier, so an aborting warp cannot strand the others).
    uint32_t* merge_cnt = reinterpret_cast<uint32_t*>(bars + 57);
    const bool stage_commits = S < 2 * p.kchunks;
    const uint32_t stage_bytes = L.stage_bytes;
    const long long lim_cycles = p.wait_limit;

    // Both CTAs of a pair read the same flag, so they leave together.
    if (p.skip_flag && *p.skip_flag) return;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t crank = cluster_ctarank();
    const uint32_t cta = crank & 1u;
    const bool leader = cta == 0;
    const uint32_t leader_rank = crank & ~1u;
    const uint32_t pair = blockIdx.x >> 1;
    const uint32_t nbt = p.sched.n_btiles;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(a_full, 1);
        mbar_init(a_empty, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * EPI);
        }
        for (int s = 0; s < kPairNormSlots; ++s) {
            mbar_init(&nfull[s], 1);
            mbar_init(&nempty[s], EPI);
        }
        *abort_flag = 0;
        *tiles_done = 0;
        for (int q = 0; q < 4; ++q) merge_cnt[q] = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmap_q);
        prefetch_tensormap(&tmap_b);
        if (kL2) {
            prefetch_tensormap(&tmap_baug);
            prefetch_tensormap(&tmap_norm);
        }
    }
    if constexpr (kL2) {
        for (uint32_t i = threadIdx.x; i < kAugBox / 16; i += blockDim.x)
            reinterpret_cast<uint4*>(sAaug)[i] = make_uint4(~0u, ~0u, ~0u, ~0u);
        fence_proxy_async_smem();
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, 512);
    tc_fence_before();
    // Barriers of both CTAs initialised before any remote arrive / TMA.
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Raise the abort flag in both CTAs of the pair.
    auto abort_pair = [&](int code) {
        atomicOr(p.error, code);
        *abort_flag = 1;
        st_cluster_u32(mapa_shared(smem_u32(const_cast<int*>(abort_flag)), crank ^ 1u), 1u);
    };

    if (warp == 0) {
        // ------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            const uint32_t full0 = mapa_shared(smem_u32(full), leader_rank);
            const uint32_t a_full_l = mapa_shared(smem_u32(a_full), leader_rank);
            uint32_t stage = 0, phase = 0, a_par = 0, rel_tile = 0, rel_kc = 0;
            uint32_t last_use[16];
            for (int i = 0; i < 16; ++i) last_use[i] = 0;
            uint64_t load_idx = 0;
            bool ok = true, withheld = false;
            uint32_t acc_i = 0;
            uint32_t qt, b0, b1, pslot;
            for (uint32_t sg = 0; ok && schedule_segment(p.sched, pair, sg, qt, b0, b1, pslot); ++sg) {
                ok = mbar_wait(a_empty, a_par ^ 1, abort_flag, lim_cycles);
                if (!ok) break;
                a_par ^= 1;
                if (leader) mbar_arrive_expect_tx(a_full, 2 * p.kchunks * kBoxBytes);
                for (uint32_t kc = 0; kc < p.kchunks; ++kc)
                    tma_load_2d_pair(sA + kc * kBoxBytes, &tmap_q, kc * kChunkBytes, qt * kPairTile + cta * kTileRows,
                                     a_full_l);
                for (uint32_t bt = b0; bt < b1 && ok; ++bt, ++acc_i) {
                    if constexpr (kL2) {
                        const uint32_t slot = acc_i % kPairNormSlots;
                        if (acc_i >= kPairNormSlots) {
                            ok = mbar_wait(&nempty[slot], (acc_i / kPairNormSlots - 1) & 1, abort_flag, lim_cycles);
                            if (!ok) break;
                        }
                        mbar_arrive_expect_tx(&nfull[slot], kPairTile * 4);
                        tma_load_1d(sNorm + slot * kPairTile, &tmap_norm, bt * kPairTile, &nfull[slot]);
                    }
                    for (uint32_t kc = 0; kc < p.kchunks; ++kc) {
                        if (stage_commits) {
                            ok = mbar_wait(&empty[stage], phase ^ 1, abort_flag, lim_cycles);
                            if (!ok) break;
                        } else if (load_idx >= S) {
                            ok = spin_until_geq(tiles_done, rel_tile + 1, abort_flag, 128, lim_cycles);
                            if (!ok) break;
                            if (++rel_kc == p.kchunks) {
                                rel_kc = 0;
                                ++rel_tile;
                            }
                        }
                        ++load_idx;
                        const bool aug_here = kL2 && kc + 1 == p.kchunks;
                        const uint32_t bytes = 2 * (kBoxBytes + (aug_here ? kAugBox : 0));
                        // Timeout test: the leader withholds the arrival of one
                        // stage, so its phase never completes.
                        const bool skip = p.test_mode == 1 && leader && !withheld;
                        if (skip) withheld = true;
                        if (leader && !skip) mbar_arrive_expect_tx(&full[stage], bytes);
                        uint8_t* dst = sB + stage * stage_bytes;
                        const uint32_t bar = full0 + stage * 8;
                        tma_load_2d_pair(dst, &tmap_b, kc * kChunkBytes, bt * kPairTile + cta * kTileRows, bar);
                        if (aug_here)
                            tma_load_2d_pair(dst + kBoxBytes, &tmap_baug, 0, bt * kPairTile + cta * kTileRows, bar);
                        last_use[stage] = phase + 1;  // completes phase `phase`
                        if (++stage == S) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            if (!ok) abort_pair(1);
            // Drain: the leader waits (bounded) until every stage load it
            // counted has landed, in both CTAs; a timed-out phase is skipped.
            if (!ok && leader) {
                for (uint32_t s = 0; s < S; ++s)
                    if (last_use[s]) (void)mbar_wait_drain(&full[s], (last_use[s] - 1) & 1, lim_cycles / 8);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ UMMA issuer (leader)
        if (leader && lane == 0) {
            const uint32_t idesc = idesc_pair_u8();
            const uint64_t a_desc0 = umma_desc_sw128(smem_u32(sA));
            const uint64_t b_desc0 = umma_desc_sw128(smem_u32(sB));
            const uint64_t a_aug_desc = umma_desc_sw32(smem_u32(sAaug));
            const uint64_t b_aug_desc0 = umma_desc_sw32(smem_u32(sB + kBoxBytes));
            constexpr uint64_t kBoxStep = kBoxBytes >> 4;
            const uint64_t stage_step = stage_bytes >> 4;
            uint32_t s = 0, ph = 0, a_par = 0, acc_i = 0;
            bool ok = true;
            const bool prof = kPairProfile && (p.debug_flags & 512u) && p.debug_clocks;
            long long c_te = 0, c_fu = 0, c_t0 = clock64();
            uint32_t qt, b0, b1, pslot;
            for (uint32_t sg = 0; ok && schedule_segment(p.sched, pair, sg, qt, b0, b1, pslot); ++sg) {
                ok = mbar_wait_sleep(a_full, a_par, abort_flag, lim_cycles);
                if (!ok) break;
                a_par ^= 1;
                tc_fence_after();
                for (uint32_t bt = b0; bt < b1; ++bt, ++acc_i) {
                    const uint32_t buf = acc_i & 1u;
                    const long long w_te = prof ? clock64() : 0;
                    // profiling flag 8: plain try_wait polling instead of the suspend hint
                    ok = (kPairProfile && (p.debug_flags & 8u))
                             ? mbar_wait(&tempty[buf], ((acc_i >> 1) & 1u) ^ 1u, abort_flag, lim_cycles)
                             : mbar_wait_sleep(&tempty[buf], ((acc_i >> 1) & 1u) ^ 1u, abort_flag, lim_cycles);
                    if (prof) c_te += clock64() - w_te;
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + buf * kPairTile;
                    for (uint32_t kc = 0; kc < p.kchunks; ++kc) {
                        const long long w_fu = prof ? clock64() : 0;
                        ok = (kPairProfile && (p.debug_flags & 8u)) ? mbar_wait(&full[s], ph, abort_flag, lim_cycles)
                                                                    : mbar_wait_sleep(&full[s], ph, abort_flag, lim_cycles);
                        if (prof) c_fu += clock64() - w_fu;
                        if (!ok) break;
                        tc_fence_after();
                        const uint64_t ad = a_desc0 + kc * kBoxStep;
                        const uint64_t bd = b_desc0 + s * stage_step;
                        if (!(p.debug_flags & 4u)) {
#pragma unroll
                            for (int ks = 0; ks < kChunkBytes / 32; ++ks)
                                umma_u8_pair(d_tmem, ad + 2 * ks, bd + 2 * ks, idesc, (kc > 0 || ks > 0) ? 1u : 0u);
                            if constexpr (kL2) {
                                if (kc + 1 == p.kchunks && !(kPairProfile && (p.debug_flags & 1024u)))
                                    umma_u8_pair(d_tmem, a_aug_desc, b_aug_desc0 + s * stage_step, idesc, 1u);
                            }
                        }
                        if (stage_commits) umma_commit_pair(&empty[s]);
                        if (++s == S) {
                            s = 0;
                            ph ^= 1;
                        }
                    }
                    if (!ok) break;
                    umma_commit_pair(&tfull[buf]);
                }
                // The query tile's MMAs are issued: its A buffer frees when they complete.
                if (ok) umma_commit_pair(a_empty);
            }
            if (prof) {
                atomicAdd(p.debug_clocks + 4, static_cast<unsigned long long>(c_te));
                atomicAdd(p.debug_clocks + 5, static_cast<unsigned long long>(c_fu));
                atomicAdd(p.debug_clocks + 6, static_cast<unsigned long long>(clock64() - c_t0));
            }
            if (!ok) abort_pair(2);
        }
    } else {
        // ------------------------------------------------ epilogue (EPI warps per CTA)
        // Warp -> TMEM lane quarter (hardware rule: warp w reads lanes
        // 32 (w % 4) ..) and column slice; thread <-> one query row.
        const int quarter = warp & 3;
        const int slice = (warp - 2) >> 2;
        const uint32_t row = quarter * 32 + lane;
        const int cbase = slice * kSliceCols;  // first column of this warp's slice
        const uint32_t tempty_l = mapa_shared(smem_u32(tempty), leader_rank);
        uint32_t acc_i = 0;
        bool ok = true;
        const bool prof = kPairProfile && (p.debug_flags & 512u) && p.debug_clocks && lane == 0;
        long long c_tf = 0, c_slow = 0, c_t0 = clock64();
        unsigned long long n_slow = 0, n_slow_calls = 0;
        uint32_t merge_round = 0;  // target of this warp's next merge barrier
        uint32_t qt, b0, b1, pslot;
        for (uint32_t sg = 0; ok && schedule_segment(p.sched, pair, sg, qt, b0, b1, pslot); ++sg) {
            const bool complete = b0 == 0 && b1 == nbt;
            const uint32_t qlocal = qt * kPairTile + cta * kTileRows + row;
            const bool qvalid = qlocal < p.n_queries;
            const uint32_t self_id = p.exclude_self ? p.query_id0 + qlocal : UINT32_MAX;
            TopK tk;
            tk.init(p.k);
            // A seeded upper bound on the row's k-th key (from a pass over a
            // sample of the base) admits only keys <= seed from the start.
            int32_t seed_thr = INT_MAX;
            if (p.seed_in && qvalid) {
                const int32_t sd = p.seed_in[qlocal];
                seed_thr = sd < INT_MAX ? sd + 1 : INT_MAX;
            }
            int32_t thr = min(tk.thr(), seed_thr);
            for (uint32_t bt = b0; bt < b1; ++bt, ++acc_i) {
                const uint32_t buf = acc_i & 1u;
                const long long w_tf = prof ? clock64() : 0;
                ok = mbar_wait(&tfull[buf], (acc_i >> 1) & 1u, abort_flag, lim_cycles);
                if (prof) c_tf += clock64() - w_tf;
                if (!ok) break;
                tc_fence_after();
                if (warp == 2 && lane == 0) *tiles_done = acc_i + 1;
                const uint32_t slot = acc_i % kPairNormSlots;
                const int32_t* nb = sNorm + slot * kPairTile;
                const uint64_t tile0 = static_cast<uint64_t>(bt) * kPairTile;
                const uint32_t nvalid =
                    p.n_base - tile0 < kPairTile ? static_cast<uint32_t>(p.n_base - tile0) : kPairTile;
                const uint32_t col0 = p.base_id0 + static_cast<uint32_t>(tile0);
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * kPairTile;
                // A column can hold a key < thr only if its accumulator
                // exceeds lim: L2 keys are keyoff - 2 acc >= hmin - 2 acc,
                // with hmin the smallest key offset of the column's 128-row
                // half of the tile (the augmentation bytes are chosen per
                // 128-row pack tile, so offsets are near-uniform within a
                // half but not across halves); inner-product keys are -acc.
                int32_t hmin_lo = 0, hmin_hi = 0;
                if constexpr (kL2) {
                    ok = mbar_wait(&nfull[slot], (acc_i / kPairNormSlots) & 1u, abort_flag, lim_cycles);
                    if (!ok) break;
                    const int4 h0 = reinterpret_cast<const int4*>(nb)[2 * lane];
                    const int4 h1 = reinterpret_cast<const int4*>(nb)[2 * lane + 1];
                    const int32_t hv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                    int32_t hm = INT_MAX;
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (8u * lane + e < nvalid) hm = min(hm, hv[e]);
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) hm = min(hm, __shfl_xor_sync(0xffffffffu, hm, o));
                    hmin_lo = __shfl_sync(0xffffffffu, hm, 0);
                    hmin_hi = __shfl_sync(0xffffffffu, hm, 16);
                }
                auto lim_of = [](int32_t h, int32_t t) -> int32_t {
                    if constexpr (kL2) {
                        return static_cast<int32_t>((static_cast<long long>(h) - t) >> 1);  // floor
                    } else {
                        return -t;
                    }
                };
                int32_t lim_lo = lim_of(hmin_lo, thr), lim_hi = lim_of(hmin_hi, thr);
                // 32 columns from c0 hold an accumulator above lim: scan the
                // 8-column sub-groups in registers; for those that pass,
                // compute exact keys and insert in id order.
                auto slow_path = [&](const int32_t* vc, int c0) {
                    const long long w_sl = prof ? clock64() : 0;
                    if (prof) ++n_slow_calls;
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        const int cg = c0 + 8 * g;
                        const int32_t* a = vc + 8 * g;
                        const int32_t lim = cg < 128 ? lim_lo : lim_hi;
                        const int32_t m = max(__vimax3_s32(a[0], a[1], a[2]), __vimax3_s32(a[3], a[4], a[5]));
                        if (max(m, max(a[6], a[7])) <= lim) continue;
                        int32_t kv[8];
                        if constexpr (kL2) {
                            const int4 n0 = reinterpret_cast<const int4*>(nb + cg)[0];
                            const int4 n1 = reinterpret_cast<const int4*>(nb + cg)[1];
                            const int32_t nv[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll
                            for (int j = 0; j < 8; ++j) kv[j] = nv[j] - 2 * a[j];
                        } else {
#pragma unroll
                            for (int j = 0; j < 8; ++j) kv[j] = -a[j];
                        }
                        uint32_t mask = 0;
#pragma unroll
                        for (int j = 0; j < 8; ++j) mask |= (kv[j] < thr ? 1u : 0u) << j;
                        if (cg + 8 > static_cast<int>(nvalid))
                            mask &= cg >= static_cast<int>(nvalid) ? 0u : (0xffu >> (8 - (nvalid - cg)));
                        if (prof && mask) ++n_slow;
                        while (mask) {
                            const int j = __ffs(mask) - 1;
                            mask &= mask - 1;
                            int32_t key = kv[7];
#pragma unroll
                            for (int jj = 6; jj >= 0; --jj) key = j == jj ? kv[jj] : key;
                            const uint32_t id = col0 + cg + j;
                            if (key < thr && id != self_id) {
                                tk.insert_increasing(key, id);
                                thr = min(tk.thr(), seed_thr);
                            }
                        }
                        lim_lo = lim_of(hmin_lo, thr);
                        lim_hi = lim_of(hmin_hi, thr);
                    }
                    if (prof) c_slow += clock64() - w_sl;
                };
                // 32 columns from c0: one maximum against lim.
                auto filter32 = [&](const int32_t* v, int c0) {
                    if (tree_max<32>(v) > (c0 < 128 ? lim_lo : lim_hi)) slow_path(v, c0);
                };
                auto release = [&]() {
                    tc_fence_before();
                    __syncwarp();
                    // Default semantics (release at CTA scope): the tcgen05
                    // fence above orders the TMEM reads; a cluster-scope
                    // release here would cost a membar per hand-off.
                    if (lane == 0) mbar_arrive_remote(tempty_l + buf * 8);
                };
                const uint32_t tslice = taddr + cbase;
                if (p.debug_flags & 3u) {
                    // profiling: hand-off (with or without the loads), no filtering
                    if (!(p.debug_flags & 2u)) {
                        int32_t v[32];
#pragma unroll 1
                        for (int st = 0; st < kSteps; ++st) {
                            __syncwarp();
                            tmem_ld_32cols(tslice + st * 32, v);
                            tmem_ld_wait_n<32>(v);
                            if (v[0] == INT_MIN && v[31] == INT_MIN) thr = 0;  // keep the loads
                        }
                    }
                    release();
                } else if constexpr (kPipe) {
                    // The load of the next 32 columns is in flight while the
                    // current ones are filtered; the buffer goes back as soon
                    // as the last columns are in registers.
                    int32_t va[32], vb[32];
                    __syncwarp();
                    tmem_ld_32cols(tslice, va);
                    tmem_ld_wait_n<32>(va);
#pragma unroll 1
                    for (int st = 0; st < kSteps; st += 2) {
                        __syncwarp();
                        tmem_ld_32cols(tslice + (st + 1) * 32, vb);
                        filter32(va, cbase + st * 32);
                        __syncwarp();
                        tmem_ld_wait_n<32>(vb);
                        if (st + 2 < kSteps) {
                            tmem_ld_32cols(tslice + (st + 2) * 32, va);
                        } else {
                            release();
                        }
                        filter32(vb, cbase + (st + 1) * 32);
                        if (st + 2 < kSteps) {
                            __syncwarp();
                            tmem_ld_wait_n<32>(va);
                        }
                    }
                } else {
#pragma unroll 1
                    for (int st = 0; st < kSteps; ++st) {
                        int32_t v[32];
                        __syncwarp();
                        tmem_ld_32cols(tslice + st * 32, v);
                        tmem_ld_wait_n<32>(v);
                        if (st == kSteps - 1) release();
                        filter32(v, cbase + st * 32);
                    }
                }
                if constexpr (kL2) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&nempty[slot]);
                }
            }
            if (!ok) break;
            if constexpr (kSlices > 1) {
                // The four slices' lists of each row meet in slice 0 (named
                // barrier per lane quarter: its four warps): slices 1 and 3
                // hand their lists to slices 0 and 2, then slice 2 to 0.
                int32_t* m0 = sMerge + (0 * kTileRows + row) * 2 * kMergeCap;
                int32_t* m1 = sMerge + (1 * kTileRows + row) * 2 * kMergeCap;
                auto put = [&](int32_t* m) {
                    tk.for_each(p.k, [&](int jj, int32_t key, uint32_t id) {
                        m[jj] = key;
                        m[kMergeCap + jj] = static_cast<int32_t>(id);
                    });
                };
                auto take = [&](const int32_t* m) {
                    for (uint32_t jj = 0; jj < p.k; ++jj) {
                        const int32_t key = m[jj];
                        const uint32_t id = static_cast<uint32_t>(m[kMergeCap + jj]);
                        if (key_gt(tk.thr(), tk.thr_id(), key, id)) tk.insert(key, id);
                    }
                };
                auto group_sync = [&]() -> bool {
                    merge_round += kSlices;
                    __syncwarp();
                    if (lane == 0) {
                        __threadfence_block();
                        atomicAdd(&merge_cnt[quarter], 1u);
                    }
                    const bool r = spin_until_geq(reinterpret_cast<volatile uint32_t*>(&merge_cnt[quarter]),
                                                  merge_round, abort_flag, 32, lim_cycles);
                    __threadfence_block();
                    return __all_sync(0xffffffffu, r);
                };
                if constexpr (kSlices == 4) {
                    if (slice == 1) put(m0);
                    if (slice == 3) put(m1);
                    ok = group_sync();
                    if (ok && slice == 0) take(m0);
                    if (ok && slice == 2) take(m1);
                    ok = ok && group_sync();
                    if (ok && slice == 2) put(m0);
                    ok = ok && group_sync();
                    if (ok && slice == 0) take(m0);
                    ok = ok && group_sync();
                } else {
                    (void)m1;
                    if (slice == 1) put(m0);
                    ok = group_sync();
                    if (ok && slice == 0) take(m0);
                    ok = ok && group_sync();
                }
                if (!ok) break;
            }
            // Segment done (slice 0): final graph rows, or a partial list of a
            // query tile cut between pairs; in the seeding pass only the k-th key.
            if (qvalid && slice == 0) {
                const int32_t bound = seed_thr == INT_MAX ? INT_MAX : seed_thr - 1;
                if (complete && p.seed_out) {
                    p.seed_out[qlocal] = min(tk.thr(), bound);
                } else if (complete) {
                    const int32_t qnorm =
                        kL2 ? packed_sq_norm(p.query_packed, p.pitch, p.data_bytes, p.query_norms, qlocal) : 0;
                    emit_graph_row<METRIC>(tk, p.k, qlocal, qnorm, p.out_ids, p.out_dists, p.fallback_rows,
                                           p.fallback_count, bound);
                } else {
                    const uint64_t o = (static_cast<uint64_t>(pslot) * kPairTile + cta * kTileRows + row) * p.k;
                    tk.for_each(p.k, [&](int jj, int32_t key, uint32_t id) {
                        p.part_keys[o + jj] = key;
                        p.part_ids[o + jj] = id;
                    });
                }
            }
        }
        if (prof) {
            atomicAdd(p.debug_clocks + 0, static_cast<unsigned long long>(c_tf));
            atomicAdd(p.debug_clocks + 1, static_cast<unsigned long long>(c_slow));
            atomicAdd(p.debug_clocks + 2, n_slow);
            atomicAdd(p.debug_clocks + 3, static_cast<unsigned long long>(clock64() - c_t0));
            atomicAdd(p.debug_clocks + 7, n_slow_calls);
        }
        if (!ok) abort_pair(4);
    }

    __syncwarp();
    tc_fence_before();
    // No CTA of the pair leaves while its peer may still arrive on its
    // barriers or read its shared memory through the pair UMMAs.
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, 512);
    }
}

}  // namespace knng_b200
