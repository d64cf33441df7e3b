// knn_tc.cuh -- fused brute-force KNN on the 5th-gen tensor cores: UMMA
// (tcgen05.mma) into TMEM, top-k selection in the epilogue, so the n x n
// distance matrix never leaves the SM. Two element kinds share the pipeline:
//
//  ElemU8     exact path for data whose every coordinate is an integer in
//             [0, 255]: u8 x u8 -> s32 (kind::i8). For a fixed query q the key
//             of base row r is |r|^2 - 2 q.r (L2; dist = |q|^2 + key) or -q.r
//             (negative inner product), exact int32; the kernel writes the
//             final graph rows. This restates knng::cpu::brute_force_knn
//             (include/knng/cpu/brute_force.hpp:336-376) with the norm
//             identity of src/cpu/brute_force.cpp:261-323; the emitted fp32
//             distances equal the reference's sequential sums bit for bit
//             whenever those stay below 2^24, and rows where they may not are
//             flagged for the exact fp32 kernel.
//  ElemBf16x3 candidate filter for arbitrary fp32 data: every (centred) row
//             is split into bf16 hi + lo planes and q.r ~ hi.hi + hi.lo + lo.hi
//             is accumulated in fp32 (kind::f16, three UMMAs per K step). The
//             kernel keeps the C best approximate keys per query; the re-rank
//             kernel (knn_rerank.cuh) recomputes them exactly and proves the
//             result with an error bound.
//
// CTA layout (persistent, one CTA per SM):
//   warp 0    TMA producer: A = MT query tiles of 128 rows, resident for a
//             query tile (or streamed per K chunk when A_STREAM); B = ring of
//             `stages` base tiles of 128 rows x 128 B per plane
//   warp 1    TMEM allocator and UMMA issuer (one lane)
//   warps 2.. 4*MT epilogue warps; thread <-> one query row (TMEM lane)
// TMEM: NBUF buffers x MT tiles x 128 columns (s32 or f32).
#pragma once
#include <climits>
#include <cstdint>
#include <type_traits>

#include "ptx.cuh"
#include "schedule.cuh"
#include "topk.cuh"

namespace knng_b200 {

constexpr int kTileRows = 128;      // M per UMMA, N per base tile, rows per TMA box
constexpr int kChunkBytes = 128;    // K bytes per TMA box / swizzle atom
constexpr int kBoxBytes = kTileRows * kChunkBytes;  // 16 KiB
constexpr int kAugBytes = 32;       // augmentation K bytes per packed u8 row (after the data)
constexpr int kAugBox = kTileRows * kAugBytes;  // 4 KiB: one tile of augmentation bytes
constexpr int kSlowPitch = 36;      // ints per thread in the slow-path spill area
constexpr int kNormRing = 4;        // base-tile norm slots per epilogue warp (prefetch depth + 1)
// Software-pipelined TMEM loads in the epilogue (measured slower at d = 128).
constexpr bool kPipelineTmemLoads = false;
// Small lists: load a whole tile before handing the TMEM buffer back.
constexpr bool kLoadWholeTile = false;
// u8, two buffers x two M tiles: a handoff barrier pair per (buffer, M tile).
constexpr bool kSplitHandoffOpt = true;

struct ElemU8 {
    static constexpr int kPlanes = 1;
    static constexpr bool kFloat = false;
    __device__ static uint32_t idesc() { return idesc_u8_s32(kTileRows, kTileRows); }
    // One K step = 32 bytes of each operand; a/b are smem descriptors.
    __device__ static void mma_step(uint32_t d, const uint64_t* a, const uint64_t* b, uint32_t idesc,
                                    uint32_t accumulate)
    {
        umma_u8(d, a[0], b[0], idesc, accumulate);
    }
};

struct ElemBf16x3 {
    static constexpr int kPlanes = 2;  // hi, lo
    static constexpr bool kFloat = true;
    __device__ static uint32_t idesc() { return idesc_bf16_f32(kTileRows, kTileRows); }
    __device__ static void mma_step(uint32_t d, const uint64_t* a, const uint64_t* b, uint32_t idesc,
                                    uint32_t accumulate)
    {
        umma_f16(d, a[0], b[0], idesc, accumulate);  // hi.hi
        umma_f16(d, a[0], b[1], idesc, 1u);          // hi.lo
        umma_f16(d, a[1], b[0], idesc, 1u);          // lo.hi
    }
};

struct KnnTcParams {
    const void* base_norms;      // per base row: int32 key offset (u8 L2) or fp32 |r'|^2 (bf16x3 L2)
    const int32_t* query_norms;  // u8: key offset per query row of this launch (see below)
    // u8: packed query rows (augmentation bytes at data_bytes within each
    // pitch-byte row); L2 recovers |q|^2 = keyoff - 510 * sum(aug bytes).
    const uint8_t* query_packed;
    uint32_t pitch;
    uint32_t data_bytes;
    uint64_t n_base;             // valid base rows
    uint32_t base_id0;           // global id of base row 0
    uint32_t n_queries;          // query rows in this launch
    uint32_t query_row0;         // first query row inside the A tensor maps
    uint32_t query_id0;          // global id of query row 0 (self exclusion)
    uint32_t exclude_self;
    uint32_t k;                  // neighbours (u8) or candidates kept (bf16x3)
    uint32_t kchunks;            // 128-byte K chunks per row
    uint32_t stages;
    uint32_t* out_ids;           // u8: n_queries x k graph rows; bf16x3: candidates
    float* out_dists;            // u8: distances
    int32_t* out_keys;           // bf16x3: ordered approximate keys of the candidates
    uint32_t* fallback_rows;     // u8: rows whose fp32 sums may be inexact
    uint32_t* fallback_count;
    int* error;                  // non-zero: a bounded wait gave up
    TileSchedule sched;          // units = CTAs; MT*128-row query tiles, 128-row base tiles
    int32_t* part_keys;          // u8: [2 * n_units][MT*128][k] partial lists of cut query tiles
    uint32_t* part_ids;
    uint32_t part_units;         // units whose partial lists fit (0: whole query tiles only)
    const int* skip_flag;        // u8: non-zero -> the data is not integer-valued, do nothing
    uint32_t debug_flags;        // profiling only: 1 skip filtering, 2 skip insertion, 4 skip TMEM loads
    unsigned long long* debug_clocks;  // profiling only: per-role wait cycles (flag 512)
};

struct SmemLayoutTc {
    uint32_t a_off, aug_off, b_off, nb_off, slow_off, merge_off, bar_off, total, stage_bytes, a_bytes;
};

// split: epilogue warps per (M tile, TMEM lane quarter), each covering
// 1/split of the columns; their lists meet in `merge` (2 * kcap ints per row).
// aug: u8 L2 -- a constant 4 KiB block of query-side augmentation bytes
// after A, and 4 KiB of base-side augmentation bytes in every stage.
__host__ __device__ inline SmemLayoutTc smem_layout_tc(int planes, int mt, bool a_stream, uint32_t kchunks,
                                                       uint32_t stages, int split = 1, int kcap = 0, bool aug = false)
{
    SmemLayoutTc L;
    // A resident: all K chunks of MT tiles. A streamed: a stage carries the
    // A chunk(s) next to the B chunk.
    L.a_bytes = a_stream ? 0 : mt * kchunks * planes * kBoxBytes;
    L.stage_bytes = (a_stream ? mt + 1 : 1) * planes * kBoxBytes + (aug ? kAugBox : 0);
    const int epi_threads = mt * kTileRows * split;
    L.a_off = 0;
    L.aug_off = L.a_off + L.a_bytes;
    L.b_off = L.aug_off + (aug ? kAugBox : 0);
    L.nb_off = L.b_off + stages * L.stage_bytes;
    L.slow_off = L.nb_off + (epi_threads / 32) * kNormRing * kTileRows * 4;  // per epilogue warp ring
    L.merge_off = L.slow_off + epi_threads * kSlowPitch * 4;
    L.bar_off = L.merge_off + (split > 1 ? mt * kTileRows * 2 * kcap * 4 : 0);
    L.total = L.bar_off + 512;  // barriers + tmem slot + abort flag + stage counter
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

template <int N>
__device__ __forceinline__ int32_t tree_max(const int32_t* v)
{
    if constexpr (N == 1) {
        return v[0];
    } else if constexpr (N == 2) {
        return max(v[0], v[1]);
    } else if constexpr (N == 3) {
        return __vimax3_s32(v[0], v[1], v[2]);
    } else {
        constexpr int a = N / 3, b = (N - a) / 2, c = N - a - b;
        return __vimax3_s32(tree_max<a>(v), tree_max<b>(v + a), tree_max<c>(v + a + b));
    }
}

// Order-preserving int image of an fp32 key, branch-free (finite or +inf).
__device__ __forceinline__ int32_t ordered_bits(int32_t b) { return b ^ ((b >> 31) & 0x7FFFFFFF); }

template <class Elem, int MT, int NBUF, bool A_STREAM, int METRIC, class TopK, int SPLIT>
__global__ void __launch_bounds__(64 + 128 * MT * SPLIT, 1)
    knn_tc_kernel(const __grid_constant__ CUtensorMap tmap_q0, const __grid_constant__ CUtensorMap tmap_q1,
                  const __grid_constant__ CUtensorMap tmap_b0, const __grid_constant__ CUtensorMap tmap_b1,
                  const KnnTcParams p)
{
    constexpr int P = Elem::kPlanes;
    constexpr int BN = kTileRows;
    static_assert(NBUF <= 4 && MT * NBUF <= 4, "barrier slots");
    static_assert(MT * NBUF * BN <= 512, "TMEM holds 512 columns");
    constexpr uint32_t kTmemCols = MT * NBUF * BN <= 256 ? 256 : 512;
    // Every tcgen05.commit costs the MMA pipe several hundred cycles, so with
    // two TMEM buffers all M tiles of a base tile share one handoff barrier;
    // with one buffer each M tile gets its own so the two tiles alternate.
    constexpr bool kPerMtBars = NBUF == 1 && MT > 1;
    // Two TMEM buffers and two M tiles (u8): one handoff barrier pair per
    // (buffer, M tile), so each M tile's epilogue starts when its own MMAs
    // finish and releases independently of the other M tile.
    constexpr bool kSplitHandoff = kSplitHandoffOpt && !Elem::kFloat && NBUF == 2 && MT == 2 && SPLIT == 1 && !A_STREAM;
    // SPLIT == 2: two epilogue warps per TMEM lane quarter (four per SM
    // sub-partition instead of two), each filtering half of every tile's
    // columns into its own list; the halves merge at the end of a query tile.
    static_assert(SPLIT == 1 || (SPLIT == 2 && TopK::kRegs <= 32 && !kPerMtBars), "split epilogue");
    constexpr int kCap = TopK::kRegs / 2;

    if (p.skip_flag && *p.skip_flag) return;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // u8 L2: the K dimension is extended by 32 bytes so that the accumulator
    // already holds q.r + 255 * S(r); the key is keyoff(r) - 2 * acc with
    // keyoff(r) = |r|^2 + 510 * S(r), and the filter needs only a maximum.
    constexpr bool kAug = !Elem::kFloat && METRIC == 0;
    const SmemLayoutTc L = smem_layout_tc(P, MT, A_STREAM, p.kchunks, p.stages, SPLIT, SPLIT > 1 ? kCap : 0, kAug);
    uint8_t* sA = smem + L.a_off;
    uint8_t* sAaug = smem + L.aug_off;
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
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 46);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 47);
    // Base tiles whose MMAs are known complete (published by one epilogue
    // thread after its handoff wait). The producer reuses a B stage once the
    // tile that read it is counted here, so the MMA warp issues one
    // tcgen05.commit per tile (the TMEM handoff) instead of two.
    volatile uint32_t* tiles_done = reinterpret_cast<volatile uint32_t*>(bars + 48);
    uint64_t* merge_full = bars + 50;   // [MT]
    uint64_t* merge_empty = bars + 52;  // [MT]
    int32_t* sMerge = reinterpret_cast<int32_t*>(smem + L.merge_off);
    // With fewer stages than two tiles' worth of K chunks a tile cannot wait
    // for a whole earlier tile, so stages are released per chunk instead.
    const bool stage_commits = p.stages < 2 * p.kchunks;
    const uint32_t stage_bytes = L.stage_bytes;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t unit = blockIdx.x;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(a_full, 1);
        mbar_init(a_empty, 1);
        for (int b = 0; b < NBUF * MT; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], (kPerMtBars || kSplitHandoff) ? 4 : 4 * MT * SPLIT);
        }
        *abort_flag = 0;
        *tiles_done = 0;
        mbar_init(&bars[60], 1);
        for (int m = 0; m < MT; ++m) {
            mbar_init(&merge_full[m], 4);
            mbar_init(&merge_empty[m], 4);
        }
        fence_barrier_init();
        prefetch_tensormap(&tmap_q0);
        prefetch_tensormap(&tmap_b0);
        if (P > 1) {
            prefetch_tensormap(&tmap_q1);
            prefetch_tensormap(&tmap_b1);
        }
    }
    if constexpr (kAug) {
        // Query-side augmentation bytes: 255 in every position (so the
        // swizzle of the 32-byte rows is immaterial).
        for (uint32_t i = threadIdx.x; i < kAugBox / 16; i += blockDim.x)
            reinterpret_cast<uint4*>(sAaug)[i] = make_uint4(~0u, ~0u, ~0u, ~0u);
        fence_proxy_async_smem();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            const CUtensorMap* qmap[2] = {&tmap_q0, &tmap_q1};
            const CUtensorMap* bmap[2] = {&tmap_b0, &tmap_b1};
            uint32_t stage = 0, phase = 0, a_par = 0, load_idx = 0, rel_tile = 0, rel_kc = 0;
            bool ok = true;
            const bool dbg = (p.debug_flags & 512u) && p.debug_clocks;
            const bool no_tma = (p.debug_flags & 2048u) != 0;  // profiling only
            long long c_wait = 0, c_start = clock64();
            uint32_t t, b0, b1, pslot;
            for (uint32_t sg = 0; ok && schedule_segment(p.sched, unit, sg, t, b0, b1, pslot); ++sg) {
                if (!A_STREAM) {
                    ok = mbar_wait(a_empty, a_par ^ 1, abort_flag);
                    if (!ok) break;
                    a_par ^= 1;
                    mbar_arrive_expect_tx(a_full, MT * p.kchunks * P * kBoxBytes);
                    for (int mt = 0; mt < MT; ++mt)
                        for (uint32_t kc = 0; kc < p.kchunks; ++kc)
                            for (int pl = 0; pl < P; ++pl)
                                tma_load_2d(sA + ((mt * p.kchunks + kc) * P + pl) * kBoxBytes, qmap[pl],
                                            kc * kChunkBytes / (Elem::kFloat ? 2 : 1),
                                            p.query_row0 + (t * MT + mt) * kTileRows, a_full);
                }
                for (uint32_t j = b0; j < b1 && ok; ++j) {
                    for (uint32_t kc = 0; kc < p.kchunks; ++kc) {
                        if (stage_commits) {
                            ok = mbar_wait(&empty[stage], phase ^ 1, abort_flag);
                            if (!ok) break;
                        } else if (load_idx >= S) {
                            // The stage last held load (load_idx - S), chunk
                            // rel_kc of tile rel_tile (counted incrementally:
                            // no division in this single-thread loop).
                            if (dbg) {
                                const long long w0 = clock64();
                                ok = spin_until_geq(tiles_done, rel_tile + 1, abort_flag, 256);
                                c_wait += clock64() - w0;
                            } else {
                                ok = spin_until_geq(tiles_done, rel_tile + 1, abort_flag, 256);
                            }
                            if (!ok) break;
                            if (++rel_kc == p.kchunks) {
                                rel_kc = 0;
                                ++rel_tile;
                            }
                        }
                        ++load_idx;
                        // The augmentation tile rides with the last K chunk.
                        const bool aug_here = kAug && kc + 1 == p.kchunks;
                        if (no_tma) {  // profiling: stage handoff without data
                            mbar_arrive(&full[stage]);
                        } else {
                            mbar_arrive_expect_tx(&full[stage], stage_bytes - ((kAug && !aug_here) ? kAugBox : 0));
                        }
                        const int32_t x = kc * kChunkBytes / (Elem::kFloat ? 2 : 1);
                        uint8_t* dst = sB + stage * stage_bytes;
                        if (!no_tma) {
                            for (int pl = 0; pl < P; ++pl)
                                tma_load_2d(dst + pl * kBoxBytes, bmap[pl], x, j * BN, &full[stage]);
                            if (aug_here) tma_load_2d(dst + kBoxBytes, &tmap_b1, 0, j * BN, &full[stage]);
                        }
                        if (A_STREAM && !no_tma) {
                            for (int mt = 0; mt < MT; ++mt)
                                for (int pl = 0; pl < P; ++pl)
                                    tma_load_2d(dst + ((1 + mt) * P + pl) * kBoxBytes, qmap[pl], x,
                                                p.query_row0 + (t * MT + mt) * kTileRows, &full[stage]);
                        }
                        if (++stage == S) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            if (dbg) {
                atomicAdd(p.debug_clocks + 5, static_cast<unsigned long long>(c_wait));
                atomicAdd(p.debug_clocks + 6, static_cast<unsigned long long>(clock64() - c_start));
            }
            if (!ok) {
                atomicOr(p.error, 1);
                *abort_flag = 1;
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ UMMA issuer
        // One thread issues every MMA of the CTA, so its loop is kept lean:
        // descriptors are precomputed and advanced by adding (byte offset
        // >> 4) to the start-address field, stage/phase counters advance
        // incrementally, and nothing is divided.
        if (lane == 0) {
            const uint32_t idesc = Elem::idesc();
            const uint64_t a_desc0 = umma_desc_sw128(smem_u32(sA));
            const uint64_t b_desc0 = umma_desc_sw128(smem_u32(sB));
            // u8 L2: augmentation operands (32-byte swizzled rows)
            const uint64_t a_aug_desc = umma_desc_sw32(smem_u32(sAaug));
            const uint64_t b_aug_desc0 = umma_desc_sw32(smem_u32(sB + kBoxBytes));
            constexpr uint64_t kBoxStep = kBoxBytes >> 4;  // descriptor units per 16 KiB box
            const uint64_t stage_step = stage_bytes >> 4;
            uint32_t s = 0, ph = 0, a_par = 0, acc_i = 0;
            bool ok = true;
            const bool dbg = (p.debug_flags & 512u) && p.debug_clocks;
            const bool no_mma = (p.debug_flags & 128u) != 0;  // profiling: epilogue without MMAs
            // profiling only: 64 = do not wait for the TMEM handoff (idle
            // epilogue), 32 = one extra commit per tile
            const bool skip_tempty = (p.debug_flags & 64u) != 0, extra_commit = (p.debug_flags & 32u) != 0;
            const bool lean = !Elem::kFloat && !A_STREAM && NBUF == 2 && !kPerMtBars && p.kchunks == 1 &&
                              !stage_commits && (p.debug_flags & (64u | 32u | 128u | 512u | 4096u)) == 0;
            long long c_tempty = 0, c_full = 0, c_start = clock64();
            // Issue the K steps of one 128-byte K chunk for M tile mt.
            auto issue_chunk = [&](uint32_t d_tmem, int mt, uint32_t kc, uint32_t stage, bool first) {
                uint64_t a[2], b[2];
#pragma unroll
                for (int pl = 0; pl < P; ++pl) {
                    a[pl] = A_STREAM ? b_desc0 + stage * stage_step + ((1 + mt) * P + pl) * kBoxStep
                                     : a_desc0 + ((mt * p.kchunks + kc) * P + pl) * kBoxStep;
                    b[pl] = b_desc0 + stage * stage_step + pl * kBoxStep;
                }
                // Straight-line MMAs: no branch between them (control flow
                // around each tcgen05.mma costs the issuing thread dearly).
#pragma unroll
                for (int ks = 0; ks < kChunkBytes / 32; ++ks) {
                    Elem::mma_step(d_tmem, a, b, idesc, (first && ks == 0) ? 0u : 1u);
#pragma unroll
                    for (int pl = 0; pl < P; ++pl) {
                        a[pl] += 2;  // 32 bytes
                        b[pl] += 2;
                    }
                }
                if constexpr (kAug) {
                    if (kc + 1 == p.kchunks) umma_u8(d_tmem, a_aug_desc, b_aug_desc0 + stage * stage_step, idesc, 1u);
                }
            };
            uint32_t t, b0, b1, pslot;
            for (uint32_t sg = 0; ok && schedule_segment(p.sched, unit, sg, t, b0, b1, pslot); ++sg) {
                (void)t;
                (void)pslot;
                if (!A_STREAM) {
                    ok = mbar_wait(a_full, a_par, abort_flag);
                    if (!ok) break;
                    a_par ^= 1;
                    tc_fence_after();
                }
                if constexpr (!Elem::kFloat && !A_STREAM && NBUF == 2 && !kPerMtBars) if (lean) {
                    // Hot configuration (one K chunk, resident A, two TMEM
                    // buffers, stages released by counter): per tile two waits,
                    // one fence, the MMAs as straight-line code, one commit.
                    for (uint32_t j = b0; j < b1; ++j, ++acc_i) {
                        const uint32_t buf = acc_i & 1u;
                        const uint32_t tpar = ((acc_i >> 1) & 1u) ^ 1u;
                        if (!mbar_wait_sleep(&full[s], ph, abort_flag) ||
                            (!kSplitHandoff && !mbar_wait_sleep(&tempty[buf], tpar, abort_flag))) {
                            ok = false;
                            break;
                        }
                        if (!kSplitHandoff) tc_fence_after();
                        const uint64_t bd = b_desc0 + s * stage_step;
                        const uint32_t d0 = tmem_base + buf * (MT * BN);
                        const uint64_t bd_aug = b_aug_desc0 + s * stage_step;
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            if constexpr (kSplitHandoff) {
                                if (!mbar_wait_sleep(&tempty[buf * MT + mt], tpar, abort_flag)) {
                                    ok = false;
                                    break;
                                }
                                tc_fence_after();
                            }
#pragma unroll
                            for (int ks = 0; ks < kChunkBytes / 32; ++ks)
                                umma_u8(d0 + mt * BN, a_desc0 + mt * kBoxStep + 2 * ks, bd + 2 * ks, idesc,
                                        ks > 0 ? 1u : 0u);
                            if constexpr (kAug) umma_u8(d0 + mt * BN, a_aug_desc, bd_aug, idesc, 1u);
                            if constexpr (kSplitHandoff) umma_commit(&tfull[buf * MT + mt]);
                        }
                        if (!ok) break;
                        if (++s == S) {
                            s = 0;
                            ph ^= 1;
                        }
                        if constexpr (!kSplitHandoff) umma_commit(&tfull[buf]);
                    }
                }
                for (uint32_t j = b0; !lean && j < b1 && ok; ++j, ++acc_i) {
                    const uint32_t buf = NBUF == 1 ? 0u : acc_i & (NBUF - 1);
                    const uint32_t tpar = (acc_i / NBUF) & 1;
                    if (kPerMtBars) {
                        // One buffer per M tile: M tile mt waits for its own
                        // epilogue; a B stage is released after the last M tile
                        // (the host keeps kchunks <= 2 here).
                        uint32_t st_k[2] = {s, s}, ph_k[2] = {ph, ph};
                        {
                            uint32_t s2 = s, ph2 = ph;
                            for (uint32_t kc = 0; kc < p.kchunks && kc < 2; ++kc) {
                                st_k[kc] = s2;
                                ph_k[kc] = ph2;
                                if (++s2 == S) {
                                    s2 = 0;
                                    ph2 ^= 1;
                                }
                            }
                            s = s2;
                            ph = ph2;
                        }
                        for (int mt = 0; mt < MT && ok; ++mt) {
                            const long long w0 = clock64();
                            ok = mbar_wait(&tempty[mt], tpar ^ 1, abort_flag);
                            c_tempty += clock64() - w0;
                            if (!ok) break;
                            tc_fence_after();
                            for (uint32_t kc = 0; kc < p.kchunks && kc < 2; ++kc) {
                                if (mt == 0) {
                                    const long long w1 = clock64();
                                    ok = mbar_wait(&full[st_k[kc]], ph_k[kc], abort_flag);
                                    c_full += clock64() - w1;
                                    if (!ok) break;
                                    tc_fence_after();
                                }
                                if (!no_mma) issue_chunk(tmem_base + mt * BN, mt, kc, st_k[kc], kc == 0);
                                if (stage_commits && mt == MT - 1) umma_commit(&empty[st_k[kc]]);
                            }
                            if (ok) umma_commit(&tfull[mt]);
                        }
                    } else {
                        // Both waits first, then one fence for the MMAs that
                        // follow. Clock reads only when profiling: every extra
                        // instruction in this thread delays the next MMAs.
                        if (!skip_tempty) {
                            // (split handoff: both M tiles' barriers of this buffer)
                            for (int hm = 0; hm < (kSplitHandoff ? MT : 1) && ok; ++hm) {
                                uint64_t* te = kSplitHandoff ? &tempty[buf * MT + hm] : &tempty[buf];
                                if (dbg) {
                                    const long long w0 = clock64();
                                    ok = mbar_wait(te, tpar ^ 1, abort_flag);
                                    c_tempty += clock64() - w0;
                                } else {
                                    ok = mbar_wait(te, tpar ^ 1, abort_flag);
                                }
                            }
                            if (!ok) break;
                        }
                        for (uint32_t kc = 0; kc < p.kchunks && ok; ++kc) {
                            if (dbg) {
                                const long long w1 = clock64();
                                ok = mbar_wait(&full[s], ph, abort_flag);
                                c_full += clock64() - w1;
                            } else {
                                ok = mbar_wait(&full[s], ph, abort_flag);
                            }
                            if (!ok) break;
                            tc_fence_after();
                            if (!no_mma) {
#pragma unroll
                                for (int mt = 0; mt < MT; ++mt)
                                    issue_chunk(tmem_base + (buf * MT + mt) * BN, mt, kc, s, kc == 0);
                            }
                            if (stage_commits) umma_commit(&empty[s]);
                            if (++s == S) {
                                s = 0;
                                ph ^= 1;
                            }
                        }
                        if (ok) {
                            if constexpr (kSplitHandoff) {
                                for (int hm = 0; hm < MT; ++hm) umma_commit(&tfull[buf * MT + hm]);
                            } else {
                                umma_commit(&tfull[buf]);
                            }
                        }
                        if (extra_commit) umma_commit(&bars[60]);  // profiling: one extra commit per tile
                    }
                }
                if (ok && !A_STREAM) umma_commit(a_empty);
            }
            if (dbg) {
                atomicAdd(p.debug_clocks + 0, static_cast<unsigned long long>(c_tempty));
                atomicAdd(p.debug_clocks + 1, static_cast<unsigned long long>(c_full));
                atomicAdd(p.debug_clocks + 2, static_cast<unsigned long long>(clock64() - c_start));
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
        int32_t* nbuf = sNB + ew * kNormRing * BN;  // this warp's ring of base-tile norms
        int32_t* slow = sSlow + (ew * 32 + lane) * kSlowPitch;
        // Per-column addend of the key: u8 L2 |r|^2, bf16x3 L2 |r'|^2 (fp32
        // bits), 0 for inner product; padding rows (dot == 0 there) get
        // INT_MAX (u8) or +inf (bf16x3), so they never beat a real row.
        const int32_t kPad = Elem::kFloat ? 0x7F800000 : INT_MAX;
        // Norms of base tile j reach slot j % kNormRing by cp.async issued
        // kNormRing - 1 tiles ahead (no register dependency, so the global
        // latency never stalls the epilogue); lane l covers columns 4l..4l+3.
        auto fetch_norms = [&](uint32_t j) {
            int32_t* dst = nbuf + (j % kNormRing) * BN + lane * 4;
            const uint64_t b0 = static_cast<uint64_t>(j) * BN + lane * 4;
            if (METRIC == 0) {
                const uint64_t valid = b0 < p.n_base ? (p.n_base - b0 < 4 ? p.n_base - b0 : 4) : 0;
                const int32_t* src = static_cast<const int32_t*>(p.base_norms) + (valid ? b0 : 0);
                cp_async_16_zfill(dst, src, static_cast<uint32_t>(valid * 4));
            }
        };
        // Columns past the base (last tile only) and inner-product tiles are
        // written directly once the copies of tile j have landed.
        auto finish_norms = [&](uint32_t j) {
            int32_t* dst = nbuf + (j % kNormRing) * BN + lane * 4;
            const uint64_t b0 = static_cast<uint64_t>(j) * BN + lane * 4;
            if (METRIC != 0 || b0 + 3 >= p.n_base) {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (METRIC != 0 || b0 + e >= p.n_base) dst[e] = b0 + e < p.n_base ? 0 : kPad;
            }
        };
        // The key of one column from its accumulator and norm addend.
        auto key_of = [](int32_t acc, int32_t nb) -> int32_t {
            if constexpr (Elem::kFloat) {
                const float f = fmaf(METRIC == 0 ? -2.0f : -1.0f, __int_as_float(acc), __int_as_float(nb));
                return ordered_bits(__float_as_int(f));
            } else {
                return METRIC == 0 ? nb - 2 * acc : nb - acc;
            }
        };
        int32_t* merge_slot = sMerge + (mt * kTileRows + row) * 2 * kCap;
        uint32_t qt_iter = 0;
        uint32_t acc_i = 0;
        bool ok = true;
        const bool dbg = (p.debug_flags & 512u) && p.debug_clocks && ew == 0 && lane == 0;
        long long c_tfull = 0, c_start = clock64();
        uint32_t t, b0, b1, pslot;
        for (uint32_t sg = 0; ok && schedule_segment(p.sched, unit, sg, t, b0, b1, pslot); ++sg, ++qt_iter) {
            const bool complete = b0 == 0 && b1 == p.sched.n_btiles;
            const uint32_t qlocal = (t * MT + mt) * kTileRows + row;
            const bool qvalid = qlocal < p.n_queries;
            const uint32_t self_id = p.exclude_self ? p.query_id0 + qlocal : UINT32_MAX;
            int32_t qnorm = 0;
            if constexpr (kAug) {
                if (qvalid) {
                    // |q|^2 = keyoff(q) - 510 * (sum of q's augmentation bytes)
                    const uint4* a4 = reinterpret_cast<const uint4*>(p.query_packed + static_cast<uint64_t>(qlocal) * p.pitch +
                                                                     p.data_bytes);
                    const uint4 w0 = a4[0], w1 = a4[1];
                    uint32_t sb = 0;
                    sb = __dp4a(w0.x, 0x01010101u, sb);
                    sb = __dp4a(w0.y, 0x01010101u, sb);
                    sb = __dp4a(w0.z, 0x01010101u, sb);
                    sb = __dp4a(w0.w, 0x01010101u, sb);
                    sb = __dp4a(w1.x, 0x01010101u, sb);
                    sb = __dp4a(w1.y, 0x01010101u, sb);
                    sb = __dp4a(w1.z, 0x01010101u, sb);
                    sb = __dp4a(w1.w, 0x01010101u, sb);
                    qnorm = p.query_norms[qlocal] - 510 * static_cast<int32_t>(sb);
                }
            }
            TopK tk;
            tk.init(p.k);
            int32_t thr = tk.thr();
            // u8: a column can enter the list only if its accumulator exceeds
            // lim (keys are keyoff - 2 acc >= keyoff_min(tile) - 2 acc for L2,
            // -acc for IP); recomputed per tile and after every insertion.
            int32_t hmin = 0, lim = 0;
            auto lim_of = [&](int32_t t) -> int32_t {
                if constexpr (METRIC == 0) {
                    return static_cast<int32_t>((static_cast<long long>(hmin) - t) >> 1);  // floor
                } else {
                    return -t;
                }
            };
            __syncwarp();
            for (uint32_t jj = b0; jj + 1 < b0 + kNormRing; ++jj) {
                if (jj < b1) fetch_norms(jj);
                cp_async_commit();
            }
            for (uint32_t j = b0; j < b1; ++j, ++acc_i) {
                // Every lane is done with tile j-1, whose slot now receives
                // tile j + kNormRing - 1; then wait for tile j's copies.
                __syncwarp();
                if (j + kNormRing - 1 < b1) fetch_norms(j + kNormRing - 1);
                cp_async_commit();
                cp_async_wait_group<kNormRing - 1>();
                finish_norms(j);
                __syncwarp();
                const uint32_t buf = acc_i % NBUF;
                const uint32_t hb = kPerMtBars ? mt : (kSplitHandoff ? buf * MT + mt : buf);  // handoff barrier
                const long long w0 = clock64();
                ok = (p.debug_flags & 256u) ? mbar_wait_spin(&tfull[hb], (acc_i / NBUF) & 1, abort_flag)
                                                : mbar_wait(&tfull[hb], (acc_i / NBUF) & 1, abort_flag);
                c_tfull += clock64() - w0;
                if (!ok) break;
                tc_fence_after();
                if (ew == ((kPerMtBars || kSplitHandoff) ? 4 * (MT - 1) : 0) && lane == 0) *tiles_done = acc_i + 1;
                const uint32_t tb = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + (buf * MT + mt) * BN +
                                    half * (BN / SPLIT);
                constexpr int kCols = BN / SPLIT;  // columns of each tile this thread filters
                const int4* nb4 = reinterpret_cast<const int4*>(nbuf + (j % kNormRing) * BN + half * kCols);
                if constexpr (!Elem::kFloat) {
                    if constexpr (METRIC == 0) {
                        // Smallest key offset of the tile (padding columns
                        // hold INT_MAX): one 16-byte read per lane + a reduce.
                        const int4 h4 = reinterpret_cast<const int4*>(nbuf + (j % kNormRing) * BN)[lane];
                        hmin = __reduce_min_sync(0xffffffffu, min(min(h4.x, h4.y), min(h4.z, h4.w)));
                    }
                    lim = lim_of(thr);
                }
                // Insertion path for W columns starting at column c0 of the
                // tile, whose keys are in v: spill them and insert those under
                // the running threshold, in id order.
                auto insert_keys = [&](const int32_t* v, auto w_tag, int c0) {
                    constexpr int W = decltype(w_tag)::value;
#pragma unroll
                    for (int c = 0; c < W / 32; ++c) {
                        const int32_t* vc = v + c * 32;
                        uint32_t mask = 0;
#pragma unroll
                        for (int i = 0; i < 32; ++i) mask |= (vc[i] < thr ? 1u : 0u) << i;
                        if (!mask) continue;
#pragma unroll
                        for (int i4 = 0; i4 < 8; ++i4)
                            *reinterpret_cast<int4*>(slow + 4 * i4) =
                                make_int4(vc[4 * i4], vc[4 * i4 + 1], vc[4 * i4 + 2], vc[4 * i4 + 3]);
                        const uint32_t col0 = p.base_id0 + j * BN + half * kCols + c0 + c * 32;
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
                };
                // One threshold test per W columns (starting at column c0 of
                // the tile). u8: on the raw accumulators (maximum against lim);
                // bf16x3: on the keys (minimum against the threshold).
                auto filter = [&](int32_t* v, auto w_tag, int c0) {
                    constexpr int W = decltype(w_tag)::value;
                    if constexpr (!Elem::kFloat) {
                        if (tree_max<W>(v) > lim && !(p.debug_flags & 2u)) {
                            // Only the 32-column groups that hold a candidate.
#pragma unroll
                            for (int c = 0; c < W / 32; ++c) {
                                int32_t* vc = v + c * 32;
                                if (W > 32 && tree_max<32>(vc) <= lim) continue;
#pragma unroll
                                for (int i4 = 0; i4 < 8; ++i4) {
                                    const int4 nn = nb4[(c0 + c * 32) / 4 + i4];
                                    vc[4 * i4 + 0] = key_of(vc[4 * i4 + 0], nn.x);
                                    vc[4 * i4 + 1] = key_of(vc[4 * i4 + 1], nn.y);
                                    vc[4 * i4 + 2] = key_of(vc[4 * i4 + 2], nn.z);
                                    vc[4 * i4 + 3] = key_of(vc[4 * i4 + 3], nn.w);
                                }
                                insert_keys(vc, std::integral_constant<int, 32>{}, c0 + c * 32);
                                lim = lim_of(thr);
                            }
                        }
                    } else {
#pragma unroll
                        for (int i4 = 0; i4 < W / 4; ++i4) {
                            const int4 nn = nb4[c0 / 4 + i4];
                            v[4 * i4 + 0] = key_of(v[4 * i4 + 0], nn.x);
                            v[4 * i4 + 1] = key_of(v[4 * i4 + 1], nn.y);
                            v[4 * i4 + 2] = key_of(v[4 * i4 + 2], nn.z);
                            v[4 * i4 + 3] = key_of(v[4 * i4 + 3], nn.w);
                        }
                        const int32_t step_min = tree_min<W>(v);  // depth log3(W)
                        if (step_min < thr && !(p.debug_flags & 2u)) insert_keys(v, w_tag, c0);
                    }
                };
                auto release = [&]() {
                    // Every column of this buffer is in registers: hand it back
                    // to the MMA warp before the last filtering step.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[hb]);
                };
                const bool loads = !(p.debug_flags & 4u), filtering = !(p.debug_flags & 1u);
                if constexpr (TopK::kRegs <= 32 && kPipelineTmemLoads) {
                    // Small lists: 32-column chunks, software-pipelined -- the
                    // TMEM load of chunk c+1 is in flight while chunk c is
                    // filtered (two epilogue warps per sub-partition cannot
                    // hide the load latency otherwise).
                    int32_t va[32], vb[32];
                    __syncwarp();
                    if (loads) {
                        tmem_ld_32cols(tb, va);
                        tmem_ld_wait_n<32>(va);
                    }
#pragma unroll
                    for (int c = 0; c < kCols / 32; ++c) {
                        int32_t* vc = (c & 1) ? vb : va;
                        int32_t* vn = (c & 1) ? va : vb;
                        if (c + 1 < kCols / 32) {
                            __syncwarp();
                            if (loads) tmem_ld_32cols(tb + (c + 1) * 32, vn);
                        } else {
                            release();
                        }
                        if (filtering) filter(vc, std::integral_constant<int, 32>{}, c * 32);
                        if (c + 1 < kCols / 32) {
                            __syncwarp();
                            if (loads) tmem_ld_wait_n<32>(vn);
                        }
                    }
                } else if constexpr (kLoadWholeTile && SPLIT == 1 && TopK::kRegs <= 32) {
                    // Small lists: the whole 128-column tile into registers,
                    // the buffer handed back at once (the TMEM round trip is
                    // the throughput limit), then filtered in two halves.
                    int32_t v[kCols];
                    __syncwarp();
                    if (loads) {
#pragma unroll
                        for (int c = 0; c < kCols / 32; ++c) tmem_ld_32cols(tb + c * 32, v + c * 32);
                        tmem_ld_wait_n<kCols>(v);
                    }
                    release();
                    if (filtering) {
                        filter(v, std::integral_constant<int, kCols / 2>{}, 0);
                        filter(v + kCols / 2, std::integral_constant<int, kCols / 2>{}, kCols / 2);
                    }
                } else {
                    // Larger lists: steps of kW columns, one TMEM wait per step.
                    constexpr int kW = (SPLIT == 1 && TopK::kRegs <= 64) ? 64 : 32;
#pragma unroll
                    for (int st = 0; st < kCols / kW; ++st) {
                        int32_t v[kW];
                        __syncwarp();
                        if (loads) {
#pragma unroll
                            for (int c = 0; c < kW / 32; ++c) tmem_ld_32cols(tb + st * kW + c * 32, v + c * 32);
                            tmem_ld_wait_n<kW>(v);
                        }
                        if (st + 1 == kCols / kW) release();
                        if (filtering) filter(v, std::integral_constant<int, kW>{}, st * kW);
                    }
                }
            }
            if (!ok) break;
            if constexpr (SPLIT > 1) {
                // Merge the column halves: half 1 publishes its list, half 0
                // inserts it (ids interleave, so the full (key, id) order).
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
            if (!qvalid) continue;
            uint32_t* oid = p.out_ids + static_cast<uint64_t>(qlocal) * p.k;
            if constexpr (Elem::kFloat) {
                // Candidates and their approximate (ordered) keys, ascending.
                int32_t* okey = p.out_keys + static_cast<uint64_t>(qlocal) * p.k;
                tk.for_each(p.k, [&](int jj, int32_t key, uint32_t id) {
                    oid[jj] = id;
                    okey[jj] = key;
                });
            } else if (!complete) {
                // A piece of a tail query tile cut between CTAs: its partial
                // list, merged with the other pieces' afterwards.
                const uint64_t o = (static_cast<uint64_t>(pslot) * (MT * kTileRows) + mt * kTileRows + row) * p.k;
                tk.for_each(p.k, [&](int jj, int32_t key, uint32_t id) {
                    p.part_keys[o + jj] = key;
                    p.part_ids[o + jj] = id;
                });
            } else {
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
        if (dbg) {
            atomicAdd(p.debug_clocks + 3, static_cast<unsigned long long>(c_tfull));
            atomicAdd(p.debug_clocks + 4, static_cast<unsigned long long>(clock64() - c_start));
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
