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

#include "ptx.cuh"
#include "topk.cuh"

namespace knng_b200 {

constexpr int kTileRows = 128;      // M per UMMA, N per base tile, rows per TMA box
constexpr int kChunkBytes = 128;    // K bytes per TMA box / swizzle atom
constexpr int kBoxBytes = kTileRows * kChunkBytes;  // 16 KiB
constexpr int kSlowPitch = 36;      // ints per thread in the slow-path spill area

struct ElemU8 {
    static constexpr int kPlanes = 1;
    static constexpr bool kFloat = false;
    __device__ static uint32_t idesc() { return idesc_u8_s32(kTileRows, kTileRows); }
    // One K step = 32 bytes of each operand.
    __device__ static void mma_step(uint32_t d, const uint32_t* a, const uint32_t* b, uint32_t off, uint32_t idesc,
                                    bool accumulate)
    {
        umma_u8(d, umma_desc_sw128(a[0] + off), umma_desc_sw128(b[0] + off), idesc, accumulate);
    }
};

struct ElemBf16x3 {
    static constexpr int kPlanes = 2;  // hi, lo
    static constexpr bool kFloat = true;
    __device__ static uint32_t idesc() { return idesc_bf16_f32(kTileRows, kTileRows); }
    __device__ static void mma_step(uint32_t d, const uint32_t* a, const uint32_t* b, uint32_t off, uint32_t idesc,
                                    bool accumulate)
    {
        umma_f16(d, umma_desc_sw128(a[0] + off), umma_desc_sw128(b[0] + off), idesc, accumulate);  // hi.hi
        umma_f16(d, umma_desc_sw128(a[0] + off), umma_desc_sw128(b[1] + off), idesc, true);        // hi.lo
        umma_f16(d, umma_desc_sw128(a[1] + off), umma_desc_sw128(b[0] + off), idesc, true);        // lo.hi
    }
};

struct KnnTcParams {
    const void* base_norms;      // per base row: int32 |r|^2 (u8 L2) or fp32 |r'|^2 (bf16x3 L2)
    const int32_t* query_norms;  // u8 L2: |q|^2 per query row of this launch
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
    uint32_t debug_flags;        // profiling only: 1 skip filtering, 2 skip insertion, 4 skip TMEM loads
};

struct SmemLayoutTc {
    uint32_t a_off, b_off, nb_off, slow_off, bar_off, total, stage_bytes, a_bytes;
};

__host__ __device__ inline SmemLayoutTc smem_layout_tc(int planes, int mt, bool a_stream, uint32_t kchunks,
                                                       uint32_t stages)
{
    SmemLayoutTc L;
    // A resident: all K chunks of MT tiles. A streamed: a stage carries the
    // A chunk(s) next to the B chunk.
    L.a_bytes = a_stream ? 0 : mt * kchunks * planes * kBoxBytes;
    L.stage_bytes = (a_stream ? mt + 1 : 1) * planes * kBoxBytes;
    const int epi_threads = mt * kTileRows;
    L.a_off = 0;
    L.b_off = L.a_off + L.a_bytes;
    L.nb_off = L.b_off + stages * L.stage_bytes;
    L.slow_off = L.nb_off + (epi_threads / 32) * 2 * kTileRows * 4;  // per epilogue warp, double-buffered
    L.bar_off = L.slow_off + epi_threads * kSlowPitch * 4;
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

// Order-preserving int image of an fp32 key, branch-free (finite or +inf).
__device__ __forceinline__ int32_t ordered_bits(int32_t b) { return b ^ ((b >> 31) & 0x7FFFFFFF); }

template <class Elem, int MT, int NBUF, bool A_STREAM, int METRIC, class TopK>
__global__ void __launch_bounds__(64 + 128 * MT, 1)
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

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const SmemLayoutTc L = smem_layout_tc(P, MT, A_STREAM, p.kchunks, p.stages);
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
    const uint32_t stage_bytes = L.stage_bytes;

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
            mbar_init(&tempty[b], kPerMtBars ? 4 : 4 * MT);
        }
        *abort_flag = 0;
        *tiles_done = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmap_q0);
        prefetch_tensormap(&tmap_b0);
        if (P > 1) {
            prefetch_tensormap(&tmap_q1);
            prefetch_tensormap(&tmap_b1);
        }
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
            uint32_t stage = 0, phase = 0, a_par = 0, load_idx = 0;
            bool ok = true;
            for (uint32_t t = blockIdx.x; t < n_qtiles && ok; t += gridDim.x) {
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
                        mbar_arrive_expect_tx(&full[stage], stage_bytes);
                        const int32_t x = kc * kChunkBytes / (Elem::kFloat ? 2 : 1);
                        uint8_t* dst = sB + stage * stage_bytes;
                        for (int pl = 0; pl < P; ++pl) tma_load_2d(dst + pl * kBoxBytes, bmap[pl], x, j * BN, &full[stage]);
                        if (A_STREAM) {
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
            if (!ok) {
                atomicOr(p.error, 1);
                *abort_flag = 1;
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ UMMA issuer
        if (lane == 0) {
            const uint32_t idesc = Elem::idesc();
            uint32_t stage0 = 0, phase0 = 0, a_par = 0, acc_i = 0;
            bool ok = true;
            const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
            // Operand plane addresses of M tile mt / the B tile in stage s.
            auto a_planes = [&](int mt, uint32_t kc, uint32_t s, uint32_t* a) {
                for (int pl = 0; pl < P; ++pl)
                    a[pl] = A_STREAM ? b_base + s * stage_bytes + ((1 + mt) * P + pl) * kBoxBytes
                                     : a_base + ((mt * p.kchunks + kc) * P + pl) * kBoxBytes;
            };
            for (uint32_t t = blockIdx.x; t < n_qtiles && ok; t += gridDim.x) {
                if (!A_STREAM) {
                    ok = mbar_wait(a_full, a_par, abort_flag);
                    if (!ok) break;
                    a_par ^= 1;
                    tc_fence_after();
                }
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
                                uint32_t a[2], b[2];
                                a_planes(mt, kc, s, a);
                                for (int pl = 0; pl < P; ++pl) b[pl] = b_base + s * stage_bytes + pl * kBoxBytes;
#pragma unroll
                                for (int ks = 0; ks < kChunkBytes / 32; ++ks)
                                    Elem::mma_step(d_tmem, a, b, ks * 32, idesc, (kc | ks) != 0);
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
                            uint32_t b[2];
                            for (int pl = 0; pl < P; ++pl) b[pl] = b_base + s * stage_bytes + pl * kBoxBytes;
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt) {
                                uint32_t a[2];
                                a_planes(mt, kc, s, a);
                                const uint32_t d_tmem = tmem_base + (buf * MT + mt) * BN;
#pragma unroll
                                for (int ks = 0; ks < kChunkBytes / 32; ++ks)
                                    Elem::mma_step(d_tmem, a, b, ks * 32, idesc, (kc | ks) != 0);
                            }
                            if (stage_commits) umma_commit(&empty[s]);
                        }
                        if (ok) umma_commit(&tfull[buf]);
                    }
                    const uint32_t next = stage0 + p.kchunks;
                    phase0 ^= (next / S) & 1;
                    stage0 = next % S;
                }
                if (ok && !A_STREAM) umma_commit(a_empty);
            }
            if (!ok) {
                atomicOr(p.error, 2);
                *abort_flag = 1;
            }
        }
    } else {
        // ------------------------------------------------ epilogue
        const int ew = warp - 2;
        const int mt = ew >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        int32_t* nbuf = sNB + ew * 2 * BN;  // this warp's copy of the base-tile norms
        int32_t* slow = sSlow + (ew * 32 + lane) * kSlowPitch;
        // Per-column addend of the key: u8 L2 |r|^2, bf16x3 L2 |r'|^2 (fp32
        // bits), 0 for inner product; padding rows (dot == 0 there) get
        // INT_MAX (u8) or +inf (bf16x3), so they never beat a real row.
        const int32_t kPad = Elem::kFloat ? 0x7F800000 : INT_MAX;
        auto load_norms = [&](uint32_t j) -> int4 {
            const uint64_t b0 = static_cast<uint64_t>(j) * BN + lane * 4;
            const int32_t* nb = static_cast<const int32_t*>(p.base_norms);
            if (b0 + 3 < p.n_base)
                return METRIC == 0 ? __ldg(reinterpret_cast<const int4*>(nb + b0)) : make_int4(0, 0, 0, 0);
            int4 nn;
            nn.x = b0 + 0 < p.n_base ? (METRIC == 0 ? nb[b0 + 0] : 0) : kPad;
            nn.y = b0 + 1 < p.n_base ? (METRIC == 0 ? nb[b0 + 1] : 0) : kPad;
            nn.z = b0 + 2 < p.n_base ? (METRIC == 0 ? nb[b0 + 2] : 0) : kPad;
            nn.w = b0 + 3 < p.n_base ? (METRIC == 0 ? nb[b0 + 3] : 0) : kPad;
            return nn;
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
        uint32_t acc_i = 0;
        bool ok = true;
        for (uint32_t t = blockIdx.x; t < n_qtiles && ok; t += gridDim.x) {
            const uint32_t qlocal = (t * MT + mt) * kTileRows + row;
            const bool qvalid = qlocal < p.n_queries;
            const uint32_t self_id = p.exclude_self ? p.query_id0 + qlocal : UINT32_MAX;
            const int32_t qnorm = (!Elem::kFloat && METRIC == 0 && qvalid) ? p.query_norms[qlocal] : 0;
            TopK tk;
            tk.init(p.k);
            int32_t thr = tk.thr();
            int4 nn_next = load_norms(0);
            for (uint32_t j = 0; j < n_btiles; ++j, ++acc_i) {
                // Publish this tile's norms (fetched one tile earlier) and
                // start fetching the next tile's, so the global latency hides
                // behind a whole tile of work.
                reinterpret_cast<int4*>(nbuf + (j & 1) * BN)[lane] = nn_next;
                if (j + 1 < n_btiles) nn_next = load_norms(j + 1);
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
                // Steps of kW columns: one TMEM wait per step, all keys of the
                // step computed before one threshold test (ILP over kW keys).
                constexpr int kW = TopK::kRegs <= 64 ? 64 : 32;
#pragma unroll
                for (int st = 0; st < BN / kW; ++st) {
                    int32_t v[kW];
                    __syncwarp();
                    if (!(p.debug_flags & 4u)) {
#pragma unroll
                        for (int c = 0; c < kW / 32; ++c) tmem_ld_32cols(tb + st * kW + c * 32, v + c * 32);
                        tmem_ld_wait_n<kW>(v);
                    }
                    if (st + 1 == BN / kW) {
                        // Every column of this buffer is in registers: hand it
                        // back to the MMA warp before the last filtering step.
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[hb]);
                    }
                    if (p.debug_flags & 1u) continue;
#pragma unroll
                    for (int i4 = 0; i4 < kW / 4; ++i4) {
                        const int4 nn = nb4[st * kW / 4 + i4];
                        v[4 * i4 + 0] = key_of(v[4 * i4 + 0], nn.x);
                        v[4 * i4 + 1] = key_of(v[4 * i4 + 1], nn.y);
                        v[4 * i4 + 2] = key_of(v[4 * i4 + 2], nn.z);
                        v[4 * i4 + 3] = key_of(v[4 * i4 + 3], nn.w);
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
                            const uint32_t col0 = p.base_id0 + j * BN + st * kW + c * 32;
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
            if (!qvalid) continue;
            uint32_t* oid = p.out_ids + static_cast<uint64_t>(qlocal) * p.k;
            if constexpr (Elem::kFloat) {
                // Candidates and their approximate (ordered) keys, ascending.
                int32_t* okey = p.out_keys + static_cast<uint64_t>(qlocal) * p.k;
                tk.for_each(p.k, [&](int jj, int32_t key, uint32_t id) {
                    oid[jj] = id;
                    okey[jj] = key;
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
