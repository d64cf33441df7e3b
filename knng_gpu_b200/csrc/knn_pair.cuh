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

namespace knng_b200 {

constexpr int kPairTile = 256;    // base rows per tile, query rows per pair
constexpr int kPairThreads = 64 + 128;
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
    uint32_t n_qtiles;   // ceil(n_queries / 256)
    uint32_t n_btiles;   // ceil(n_base / 256)
    uint32_t n_pairs;    // CTA pairs in the grid
    uint64_t total;      // n_qtiles * n_btiles
    uint32_t* out_ids;
    float* out_dists;
    int32_t* part_keys;  // [2 * n_pairs][256][k] partial lists of cut query tiles
    uint32_t* part_ids;
    uint32_t* fallback_rows;
    uint32_t* fallback_count;
    int* error;
    const int* skip_flag;  // optional: non-zero -> the data is not integer-valued, do nothing
    long long wait_limit;  // clock cycles before a wait gives up
    uint32_t test_mode;    // 1: the leader's producer withholds one arrival (timeout test)
    uint32_t debug_flags;  // profiling builds only: 1 no filtering, 2 no TMEM loads, 4 no MMAs
};

// First work item of pair p (stream-K split of [0, total)).
__host__ __device__ inline uint64_t pair_work_begin(uint64_t total, uint32_t n_pairs, uint32_t p)
{
    return total * p / n_pairs;
}

struct SmemLayoutPair {
    uint32_t a_off, aug_off, b_off, norm_off, slow_off, bar_off, total, stage_bytes;
};

__host__ __device__ inline SmemLayoutPair smem_layout_pair(uint32_t kchunks, uint32_t stages, bool l2)
{
    SmemLayoutPair L;
    L.stage_bytes = kBoxBytes + (l2 ? kAugBox : 0);
    L.a_off = 0;
    L.aug_off = kchunks * kBoxBytes;
    L.b_off = L.aug_off + (l2 ? kAugBox : 0);
    L.norm_off = L.b_off + stages * L.stage_bytes;
    L.slow_off = L.norm_off + (l2 ? kPairNormSlots * kPairTile * 4 : 0);
    L.bar_off = L.slow_off + 128 * kSlowPitch * 4;
    L.total = L.bar_off + 512;
    return L;
}

// UMMA instruction descriptor of the pair tile (M = 256 over two CTAs).
__host__ __device__ constexpr uint32_t idesc_pair_u8() { return idesc_u8_s32(2 * kTileRows, kPairTile); }

template <int METRIC, class TopK>
__global__ void __launch_bounds__(kPairThreads, 1) knn_pair_kernel(const __grid_constant__ CUtensorMap tmap_q,
                                                                   const __grid_constant__ CUtensorMap tmap_b,
                                                                   const __grid_constant__ CUtensorMap tmap_baug,
                                                                   const __grid_constant__ CUtensorMap tmap_norm,
                                                                   const PairParams p)
{
    constexpr bool kL2 = METRIC == 0;
    // Loads of the next 64 columns overlap the filter of the current ones
    // when the register list is small.
    constexpr bool kPipe = TopK::kRegs <= 32;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const SmemLayoutPair L = smem_layout_pair(p.kchunks, p.stages, kL2);
    uint8_t* sA = smem + L.a_off;
    uint8_t* sAaug = smem + L.aug_off;
    uint8_t* sB = smem + L.b_off;
    int32_t* sNorm = reinterpret_cast<int32_t*>(smem + L.norm_off);
    int32_t* sSlow = reinterpret_cast<int32_t*>(smem + L.slow_off);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    const uint32_t S = p.stages;
    uint64_t* full = bars;         // [S] leader: stage loaded (both CTAs' bytes)
    uint64_t* empty = bars + 16;   // [S] both: stage consumed (per-chunk release mode)
    uint64_t* a_full = bars + 32;  // leader: query rows loaded
    uint64_t* a_empty = bars + 33; // both: MMAs of a query tile done
    uint64_t* tfull = bars + 34;   // [2] both: accumulator buffer ready
    uint64_t* tempty = bars + 36;  // [2] leader: buffer drained by all 8 epilogue warps
    uint64_t* nfull = bars + 38;   // [8] local: key offsets of a tile landed
    uint64_t* nempty = bars + 46;  // [8] local: key offsets read by the 4 epilogue warps
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 54);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 55);
    // Base tiles whose MMAs are complete (published by one epilogue thread
    // after its hand-off wait): a B stage is reused once its tile is counted.
    volatile uint32_t* tiles_done = reinterpret_cast<volatile uint32_t*>(bars + 56);
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
    const uint64_t w0 = pair_work_begin(p.total, p.n_pairs, pair);
    const uint64_t w1 = pair_work_begin(p.total, p.n_pairs, pair + 1);
    const uint32_t nbt = p.n_btiles;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(a_full, 1);
        mbar_init(a_empty, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 8);
        }
        for (int s = 0; s < kPairNormSlots; ++s) {
            mbar_init(&nfull[s], 1);
            mbar_init(&nempty[s], 4);
        }
        *abort_flag = 0;
        *tiles_done = 0;
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
            uint32_t qt = static_cast<uint32_t>(w0 / nbt), bt = static_cast<uint32_t>(w0 % nbt);
            uint32_t acc_i = 0;
            for (uint64_t w = w0; w < w1 && ok; ++w, ++acc_i) {
                if (w == w0 || bt == 0) {
                    ok = mbar_wait(a_empty, a_par ^ 1, abort_flag, lim_cycles);
                    if (!ok) break;
                    a_par ^= 1;
                    if (leader) mbar_arrive_expect_tx(a_full, 2 * p.kchunks * kBoxBytes);
                    for (uint32_t kc = 0; kc < p.kchunks; ++kc)
                        tma_load_2d_pair(sA + kc * kBoxBytes, &tmap_q, kc * kChunkBytes,
                                         qt * kPairTile + cta * kTileRows, a_full_l);
                }
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
                    if (aug_here) tma_load_2d_pair(dst + kBoxBytes, &tmap_baug, 0, bt * kPairTile + cta * kTileRows, bar);
                    last_use[stage] = phase + 1;  // completes phase `phase`
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                if (++bt == nbt) {
                    bt = 0;
                    ++qt;
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
            uint32_t bt = static_cast<uint32_t>(w0 % nbt);
            for (uint64_t w = w0; w < w1 && ok; ++w, ++acc_i) {
                if (w == w0 || bt == 0) {
                    ok = mbar_wait_sleep(a_full, a_par, abort_flag, lim_cycles);
                    if (!ok) break;
                    a_par ^= 1;
                    tc_fence_after();
                }
                const uint32_t buf = acc_i & 1u;
                ok = mbar_wait_sleep(&tempty[buf], ((acc_i >> 1) & 1u) ^ 1u, abort_flag, lim_cycles);
                if (!ok) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + buf * kPairTile;
                for (uint32_t kc = 0; kc < p.kchunks; ++kc) {
                    ok = mbar_wait_sleep(&full[s], ph, abort_flag, lim_cycles);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t ad = a_desc0 + kc * kBoxStep;
                    const uint64_t bd = b_desc0 + s * stage_step;
                    if (!(p.debug_flags & 4u)) {
#pragma unroll
                        for (int ks = 0; ks < kChunkBytes / 32; ++ks)
                            umma_u8_pair(d_tmem, ad + 2 * ks, bd + 2 * ks, idesc, (kc > 0 || ks > 0) ? 1u : 0u);
                        if constexpr (kL2) {
                            if (kc + 1 == p.kchunks)
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
                const bool qtile_ends = bt + 1 == nbt || w + 1 == w1;
                if (qtile_ends) umma_commit_pair(a_empty);
                if (++bt == nbt) bt = 0;
            }
            if (!ok) abort_pair(2);
        }
    } else {
        // ------------------------------------------------ epilogue (4 warps per CTA)
        const int quarter = warp & 3;
        const uint32_t row = quarter * 32 + lane;
        int32_t* slow = sSlow + row * kSlowPitch;
        const uint32_t tempty_l = mapa_shared(smem_u32(tempty), leader_rank);
        uint32_t qt = static_cast<uint32_t>(w0 / nbt), bt = static_cast<uint32_t>(w0 % nbt);
        uint32_t acc_i = 0;
        bool ok = true;
        uint64_t w = w0;
        while (w < w1 && ok) {
            const uint64_t seg_lo = w;
            const uint64_t q_end = static_cast<uint64_t>(qt + 1) * nbt;
            const uint64_t seg_hi = q_end < w1 ? q_end : w1;
            const bool complete = bt == 0 && seg_hi == q_end;
            const uint32_t qlocal = qt * kPairTile + cta * kTileRows + row;
            const bool qvalid = qlocal < p.n_queries;
            const uint32_t self_id = p.exclude_self ? p.query_id0 + qlocal : UINT32_MAX;
            int32_t qnorm = 0;
            if constexpr (kL2) {
                if (qvalid && complete) {
                    const uint4* a4 = reinterpret_cast<const uint4*>(p.query_packed + static_cast<uint64_t>(qlocal) * p.pitch +
                                                                     p.data_bytes);
                    const uint4 x0 = a4[0], x1 = a4[1];
                    uint32_t sb = 0;
                    sb = __dp4a(x0.x, 0x01010101u, sb);
                    sb = __dp4a(x0.y, 0x01010101u, sb);
                    sb = __dp4a(x0.z, 0x01010101u, sb);
                    sb = __dp4a(x0.w, 0x01010101u, sb);
                    sb = __dp4a(x1.x, 0x01010101u, sb);
                    sb = __dp4a(x1.y, 0x01010101u, sb);
                    sb = __dp4a(x1.z, 0x01010101u, sb);
                    sb = __dp4a(x1.w, 0x01010101u, sb);
                    qnorm = p.query_norms[qlocal] - 510 * static_cast<int32_t>(sb);
                }
            }
            TopK tk;
            tk.init(p.k);
            int32_t thr = tk.thr();
            for (; w < seg_hi; ++w, ++acc_i, ++bt) {
                const uint32_t buf = acc_i & 1u;
                ok = mbar_wait(&tfull[buf], (acc_i >> 1) & 1u, abort_flag, lim_cycles);
                if (!ok) break;
                tc_fence_after();
                if (warp == 2 && lane == 0) *tiles_done = acc_i + 1;
                const uint32_t slot = acc_i % kPairNormSlots;
                const int32_t* nb = sNorm + slot * kPairTile;
                if constexpr (kL2) {
                    ok = mbar_wait(&nfull[slot], (acc_i / kPairNormSlots) & 1u, abort_flag, lim_cycles);
                    if (!ok) break;
                    // Smallest key offset of each 128-column half of the
                    // tile (valid rows only; padding rows read as 0 from TMA
                    // and are masked in the slow path). The augmentation
                    // bytes are chosen per 128-row tile of the pack call, so
                    // key offsets are near-uniform within a half but not
                    // across the two halves: one bound per half keeps the
                    // filter sharp. Lanes 0-15 hold columns 0-127.
                    const uint64_t tile0 = static_cast<uint64_t>(bt) * kPairTile;
                    const int4 h0 = reinterpret_cast<const int4*>(nb)[2 * lane];
                    const int4 h1 = reinterpret_cast<const int4*>(nb)[2 * lane + 1];
                    const int32_t hv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                    int32_t hm = INT_MAX;
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (tile0 + 8 * lane + e < p.n_base) hm = min(hm, hv[e]);
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) hm = min(hm, __shfl_xor_sync(0xffffffffu, hm, o));
                    const int32_t hmin_lo = __shfl_sync(0xffffffffu, hm, 0);
                    const int32_t hmin_hi = __shfl_sync(0xffffffffu, hm, 16);
                    auto lim_of = [](int32_t h, int32_t t) -> int32_t {
                        return static_cast<int32_t>((static_cast<long long>(h) - t) >> 1);  // floor
                    };
                    int32_t lim_lo = lim_of(hmin_lo, thr), lim_hi = lim_of(hmin_hi, thr);
                    const uint32_t nvalid = p.n_base - tile0 < kPairTile ? static_cast<uint32_t>(p.n_base - tile0) : kPairTile;
                    const uint32_t col0 = p.base_id0 + static_cast<uint32_t>(tile0);
                    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * kPairTile;
                    // 32 columns starting at c0 hold a candidate: exact keys,
                    // then insertion in id order.
                    auto slow_path = [&](int32_t* vc, int c0) {
#pragma unroll
                        for (int i4 = 0; i4 < 8; ++i4) {
                            const int4 nn = reinterpret_cast<const int4*>(nb + c0)[i4];
                            vc[4 * i4 + 0] = nn.x - 2 * vc[4 * i4 + 0];
                            vc[4 * i4 + 1] = nn.y - 2 * vc[4 * i4 + 1];
                            vc[4 * i4 + 2] = nn.z - 2 * vc[4 * i4 + 2];
                            vc[4 * i4 + 3] = nn.w - 2 * vc[4 * i4 + 3];
                        }
                        uint32_t mask = 0;
#pragma unroll
                        for (int i = 0; i < 32; ++i) mask |= (vc[i] < thr ? 1u : 0u) << i;
                        if (c0 + 32 > static_cast<int>(nvalid))
                            mask &= c0 >= static_cast<int>(nvalid) ? 0u : (0xffffffffu >> (32 - (nvalid - c0)));
                        if (!mask) return;
#pragma unroll
                        for (int i4 = 0; i4 < 8; ++i4)
                            *reinterpret_cast<int4*>(slow + 4 * i4) =
                                make_int4(vc[4 * i4], vc[4 * i4 + 1], vc[4 * i4 + 2], vc[4 * i4 + 3]);
                        while (mask) {
                            const int i = __ffs(mask) - 1;
                            mask &= mask - 1;
                            const int32_t key = slow[i];
                            const uint32_t id = col0 + c0 + i;
                            if (key < thr && id != self_id) {
                                tk.insert_increasing(key, id);
                                thr = tk.thr();
                            }
                        }
                        lim_lo = lim_of(hmin_lo, thr);
                        lim_hi = lim_of(hmin_hi, thr);
                    };
                    auto filter64 = [&](int32_t* v, int c0) {
                        const int32_t lim = c0 < 128 ? lim_lo : lim_hi;
                        if (tree_max<64>(v) > lim) {
                            if (tree_max<32>(v) > lim) slow_path(v, c0);
                            const int32_t lim2 = c0 < 128 ? lim_lo : lim_hi;
                            if (tree_max<32>(v + 32) > lim2) slow_path(v + 32, c0 + 32);
                        }
                    };
                    auto release = [&]() {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive_cluster(tempty_l + buf * 8);
                    };
                    if (p.debug_flags & 3u) {
                        // profiling: hand-off (with or without the loads), no filtering
                        if (!(p.debug_flags & 2u)) {
                            int32_t v[64];
#pragma unroll
                            for (int st = 0; st < 4; ++st) {
                                __syncwarp();
                                tmem_ld_32cols(taddr + st * 64, v);
                                tmem_ld_32cols(taddr + st * 64 + 32, v + 32);
                                tmem_ld_wait_n<64>(v);
                                if (v[0] == INT_MIN && v[63] == INT_MIN) thr = 0;  // keep the loads
                            }
                        }
                        release();
                    } else if constexpr (kPipe) {
                        int32_t va[64], vb[64];
                        __syncwarp();
                        tmem_ld_32cols(taddr, va);
                        tmem_ld_32cols(taddr + 32, va + 32);
                        tmem_ld_wait_n<64>(va);
                        // st 0
                        tmem_ld_32cols(taddr + 64, vb);
                        tmem_ld_32cols(taddr + 96, vb + 32);
                        filter64(va, 0);
                        __syncwarp();
                        tmem_ld_wait_n<64>(vb);
                        // st 1
                        tmem_ld_32cols(taddr + 128, va);
                        tmem_ld_32cols(taddr + 160, va + 32);
                        filter64(vb, 64);
                        __syncwarp();
                        tmem_ld_wait_n<64>(va);
                        // st 2
                        tmem_ld_32cols(taddr + 192, vb);
                        tmem_ld_32cols(taddr + 224, vb + 32);
                        filter64(va, 128);
                        __syncwarp();
                        tmem_ld_wait_n<64>(vb);
                        // st 3: every column is in registers
                        release();
                        filter64(vb, 192);
                    } else {
#pragma unroll
                        for (int st = 0; st < 4; ++st) {
                            int32_t v[64];
                            __syncwarp();
                            tmem_ld_32cols(taddr + st * 64, v);
                            tmem_ld_32cols(taddr + st * 64 + 32, v + 32);
                            tmem_ld_wait_n<64>(v);
                            if (st == 3) release();
                            filter64(v, st * 64);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&nempty[slot]);
                } else {
                    // Inner product: key = -acc, no offsets.
                    int32_t lim = -thr;
                    const uint64_t tile0 = static_cast<uint64_t>(bt) * kPairTile;
                    const uint32_t nvalid = p.n_base - tile0 < kPairTile ? static_cast<uint32_t>(p.n_base - tile0) : kPairTile;
                    const uint32_t col0 = p.base_id0 + static_cast<uint32_t>(tile0);
                    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * kPairTile;
                    auto slow_path = [&](int32_t* vc, int c0) {
                        uint32_t mask = 0;
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            vc[i] = -vc[i];
                            mask |= (vc[i] < thr ? 1u : 0u) << i;
                        }
                        if (c0 + 32 > static_cast<int>(nvalid))
                            mask &= c0 >= static_cast<int>(nvalid) ? 0u : (0xffffffffu >> (32 - (nvalid - c0)));
                        if (!mask) return;
#pragma unroll
                        for (int i4 = 0; i4 < 8; ++i4)
                            *reinterpret_cast<int4*>(slow + 4 * i4) =
                                make_int4(vc[4 * i4], vc[4 * i4 + 1], vc[4 * i4 + 2], vc[4 * i4 + 3]);
                        while (mask) {
                            const int i = __ffs(mask) - 1;
                            mask &= mask - 1;
                            const int32_t key = slow[i];
                            const uint32_t id = col0 + c0 + i;
                            if (key < thr && id != self_id) {
                                tk.insert_increasing(key, id);
                                thr = tk.thr();
                            }
                        }
                        lim = -thr;
                    };
                    auto filter64 = [&](int32_t* v, int c0) {
                        if (tree_max<64>(v) > lim) {
                            if (tree_max<32>(v) > lim) slow_path(v, c0);
                            if (tree_max<32>(v + 32) > lim) slow_path(v + 32, c0 + 32);
                        }
                    };
                    auto release = [&]() {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive_cluster(tempty_l + buf * 8);
                    };
#pragma unroll
                    for (int st = 0; st < 4; ++st) {
                        int32_t v[64];
                        __syncwarp();
                        tmem_ld_32cols(taddr + st * 64, v);
                        tmem_ld_32cols(taddr + st * 64 + 32, v + 32);
                        tmem_ld_wait_n<64>(v);
                        if (st == 3) release();
                        filter64(v, st * 64);
                    }
                }
            }
            if (!ok) break;
            // Segment done: final graph rows, or a partial list of a query
            // tile cut between pairs.
            if (qvalid) {
                if (complete) {
                    uint32_t* oid = p.out_ids + static_cast<uint64_t>(qlocal) * p.k;
                    float* odist = p.out_dists + static_cast<uint64_t>(qlocal) * p.k;
                    bool inexact;
                    if constexpr (kL2) {
                        inexact = static_cast<int64_t>(qnorm) + tk.thr() >= (1 << 24);
                        tk.for_each(p.k, [&](int jj, int32_t key, uint32_t id) {
                            oid[jj] = id;
                            odist[jj] = __int2float_rn(qnorm + key);
                        });
                    } else {
                        inexact = -static_cast<int64_t>(tk.best(p.k)) >= (1 << 24);
                        tk.for_each(p.k, [&](int jj, int32_t key, uint32_t id) {
                            oid[jj] = id;
                            odist[jj] = -__int2float_rn(-key);
                        });
                    }
                    if (inexact) {
                        const uint32_t fs = atomicAdd(p.fallback_count, 1u);
                        p.fallback_rows[fs] = qlocal;
                    }
                } else {
                    const uint32_t pslot = 2 * pair + (seg_lo == w0 ? 0u : 1u);
                    const uint64_t o = (static_cast<uint64_t>(pslot) * kPairTile + cta * kTileRows + row) * p.k;
                    tk.for_each(p.k, [&](int jj, int32_t key, uint32_t id) {
                        p.part_keys[o + jj] = key;
                        p.part_ids[o + jj] = id;
                    });
                }
            }
            if (bt == nbt) {
                bt = 0;
                ++qt;
            }
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

// The pair holding work item w (largest p with pair_work_begin(p) <= w).
__device__ inline uint32_t pair_of_work(uint64_t total, uint32_t n_pairs, uint64_t w)
{
    uint32_t p = static_cast<uint32_t>(w * n_pairs / total);
    while (p + 1 < n_pairs && pair_work_begin(total, n_pairs, p + 1) <= w) ++p;
    while (p > 0 && pair_work_begin(total, n_pairs, p) > w) --p;
    return p;
}

// Merge the partial lists of query tiles cut between pairs. Block b looks at
// the boundary between pairs b and b + 1; it handles the query tile that
// boundary falls inside (if it does not fall on a tile start), unless the
// previous boundary cut the same tile. One thread per query row.
template <int METRIC, int KCAP>
__global__ void __launch_bounds__(kPairTile) merge_pair_partials(const PairParams p)
{
    const uint32_t pb = blockIdx.x + 1;  // boundary: start of pair pb
    if (pb >= p.n_pairs || (p.skip_flag && *p.skip_flag)) return;
    const uint32_t nbt = p.n_btiles;
    const uint64_t wb = pair_work_begin(p.total, p.n_pairs, pb);
    if (wb % nbt == 0) return;
    const uint32_t q = static_cast<uint32_t>(wb / nbt);
    if (pb > 1) {
        const uint64_t wprev = pair_work_begin(p.total, p.n_pairs, pb - 1);
        if (wprev / nbt == q && wprev % nbt != 0) return;
    }
    const uint64_t qlo = static_cast<uint64_t>(q) * nbt, qhi = qlo + nbt;
    const uint32_t p_first = pair_of_work(p.total, p.n_pairs, qlo);
    const uint32_t p_last = pair_of_work(p.total, p.n_pairs, qhi - 1);
    const uint32_t r = threadIdx.x;
    const uint32_t qlocal = q * kPairTile + r;
    if (qlocal >= p.n_queries) return;
    RegTopK<KCAP> tk;
    tk.init(p.k);
    for (uint32_t pp = p_first; pp <= p_last; ++pp) {
        const uint32_t slot = (pp == p_first && pair_work_begin(p.total, p.n_pairs, pp) != qlo) ? 1u : 0u;
        const uint64_t o = (static_cast<uint64_t>(2 * pp + slot) * kPairTile + r) * p.k;
        for (uint32_t j = 0; j < p.k; ++j) {
            const int32_t key = p.part_keys[o + j];
            const uint32_t id = p.part_ids[o + j];
            if (key_gt(tk.thr(), tk.thr_id(), key, id)) tk.insert(key, id);
        }
    }
    uint32_t* oid = p.out_ids + static_cast<uint64_t>(qlocal) * p.k;
    float* odist = p.out_dists + static_cast<uint64_t>(qlocal) * p.k;
    bool inexact;
    if constexpr (METRIC == 0) {
        const uint4* a4 = reinterpret_cast<const uint4*>(p.query_packed + static_cast<uint64_t>(qlocal) * p.pitch +
                                                         p.data_bytes);
        const uint4 x0 = a4[0], x1 = a4[1];
        uint32_t sb = 0;
        sb = __dp4a(x0.x, 0x01010101u, sb);
        sb = __dp4a(x0.y, 0x01010101u, sb);
        sb = __dp4a(x0.z, 0x01010101u, sb);
        sb = __dp4a(x0.w, 0x01010101u, sb);
        sb = __dp4a(x1.x, 0x01010101u, sb);
        sb = __dp4a(x1.y, 0x01010101u, sb);
        sb = __dp4a(x1.z, 0x01010101u, sb);
        sb = __dp4a(x1.w, 0x01010101u, sb);
        const int32_t qnorm = p.query_norms[qlocal] - 510 * static_cast<int32_t>(sb);
        inexact = static_cast<int64_t>(qnorm) + tk.thr() >= (1 << 24);
        tk.for_each(p.k, [&](int jj, int32_t key, uint32_t id) {
            oid[jj] = id;
            odist[jj] = __int2float_rn(qnorm + key);
        });
    } else {
        inexact = -static_cast<int64_t>(tk.best(p.k)) >= (1 << 24);
        tk.for_each(p.k, [&](int jj, int32_t key, uint32_t id) {
            oid[jj] = id;
            odist[jj] = -__int2float_rn(-key);
        });
    }
    if (inexact) {
        const uint32_t fs = atomicAdd(p.fallback_count, 1u);
        p.fallback_rows[fs] = qlocal;
    }
}

}  // namespace knng_b200
