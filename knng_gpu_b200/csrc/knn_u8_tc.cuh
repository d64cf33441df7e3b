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
//                query tile), B = ring of STAGES base tiles (128 rows x 128 B)
//   warp 1       TMEM allocator and UMMA issuer (one elected lane)
//   warps 2..    4*MT epilogue warps; thread <-> one query row (TMEM lane)
// TMEM: 2 accumulator buffers x MT x 128 columns (s32), so the epilogue of
// base tile j overlaps the MMAs of tile j+1.
#pragma once
#include <climits>
#include <cstdint>

#include "ptx.cuh"
#include "topk.cuh"

namespace knng_b200 {

constexpr int kTileRows = 128;      // M per UMMA and N per base tile
constexpr int kChunkBytes = 128;    // K bytes per TMA box / swizzle atom
constexpr int kTileBytes = kTileRows * kChunkBytes;  // 16 KiB
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
};

struct SmemLayoutU8 {
    uint32_t a_off, b_off, nb_off, slow_off, bar_off, total;
};

__host__ __device__ inline SmemLayoutU8 smem_layout_u8(int mt, uint32_t kchunks, uint32_t stages)
{
    SmemLayoutU8 L;
    L.a_off = 0;
    L.b_off = L.a_off + mt * kchunks * kTileBytes;
    L.nb_off = L.b_off + stages * kTileBytes;
    L.slow_off = L.nb_off + mt * 4 * 2 * kTileRows * 4;  // per epilogue warp, double-buffered
    L.bar_off = L.slow_off + mt * kTileRows * kSlowPitch * 4;
    L.total = L.bar_off + 256;  // barriers + tmem slot + abort flag
    return L;
}

template <int MT, int METRIC, class TopK>
__global__ void __launch_bounds__(64 + 128 * MT, 1)
    knn_u8_tc_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_b,
                     const KnnU8Params p)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const SmemLayoutU8 L = smem_layout_u8(MT, p.kchunks, p.stages);
    uint8_t* sA = smem + L.a_off;
    uint8_t* sB = smem + L.b_off;
    int32_t* sNB = reinterpret_cast<int32_t*>(smem + L.nb_off);
    int32_t* sSlow = reinterpret_cast<int32_t*>(smem + L.slow_off);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    const uint32_t S = p.stages;
    uint64_t* full = bars;             // [S]
    uint64_t* empty = bars + 8;        // [S], S <= 8
    uint64_t* a_full = bars + 16;
    uint64_t* a_empty = bars + 17;
    uint64_t* tfull = bars + 18;       // [2]
    uint64_t* tempty = bars + 20;      // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 23);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t n_qtiles = (p.n_queries + MT * kTileRows - 1) / (MT * kTileRows);
    const uint32_t n_btiles = static_cast<uint32_t>((p.n_base + kTileRows - 1) / kTileRows);
    constexpr uint32_t kTmemCols = MT == 2 ? 512 : 256;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(a_full, 1);
        mbar_init(a_empty, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4 * MT);
        }
        *abort_flag = 0;
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
            uint32_t stage = 0, phase = 0, a_par = 0;
            bool ok = true;
            for (uint32_t t = blockIdx.x; t < n_qtiles && ok; t += gridDim.x) {
                ok = mbar_wait(a_empty, a_par ^ 1, abort_flag);
                if (!ok) break;
                a_par ^= 1;
                mbar_arrive_expect_tx(a_full, MT * p.kchunks * kTileBytes);
                for (int mt = 0; mt < MT; ++mt)
                    for (uint32_t kc = 0; kc < p.kchunks; ++kc)
                        tma_load_2d(sA + (mt * p.kchunks + kc) * kTileBytes, &tmap_q, kc * kChunkBytes,
                                    p.query_row0 + (t * MT + mt) * kTileRows, a_full);
                for (uint32_t j = 0; j < n_btiles && ok; ++j) {
                    for (uint32_t kc = 0; kc < p.kchunks; ++kc) {
                        ok = mbar_wait(&empty[stage], phase ^ 1, abort_flag);
                        if (!ok) break;
                        mbar_arrive_expect_tx(&full[stage], kTileBytes);
                        tma_load_2d(sB + stage * kTileBytes, &tmap_b, kc * kChunkBytes, j * kTileRows, &full[stage]);
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
            constexpr uint32_t idesc = idesc_u8_s32(kTileRows, kTileRows);
            uint32_t stage = 0, phase = 0, a_par = 0, acc_i = 0;
            bool ok = true;
            const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
            for (uint32_t t = blockIdx.x; t < n_qtiles && ok; t += gridDim.x) {
                ok = mbar_wait(a_full, a_par, abort_flag);
                if (!ok) break;
                a_par ^= 1;
                tc_fence_after();
                for (uint32_t j = 0; j < n_btiles && ok; ++j, ++acc_i) {
                    const uint32_t buf = acc_i & 1;
                    ok = mbar_wait(&tempty[buf], ((acc_i >> 1) & 1) ^ 1, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + buf * (MT * kTileRows);
                    for (uint32_t kc = 0; kc < p.kchunks; ++kc) {
                        ok = mbar_wait(&full[stage], phase, abort_flag);
                        if (!ok) break;
                        tc_fence_after();
                        const uint32_t bs = b_base + stage * kTileBytes;
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            const uint32_t as = a_base + (mt * p.kchunks + kc) * kTileBytes;
#pragma unroll
                            for (int ks = 0; ks < kChunkBytes / 32; ++ks) {
                                umma_u8(d_tmem + mt * kTileRows, umma_desc_sw128(as + ks * 32),
                                        umma_desc_sw128(bs + ks * 32), idesc, (kc | ks) != 0);
                            }
                        }
                        umma_commit(&empty[stage]);
                        if (++stage == S) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                    if (ok) umma_commit(&tfull[buf]);
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
        const int mt = ew >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        int32_t* nbuf = sNB + ew * 2 * kTileRows;  // this warp's copy of the base-tile norms
        int32_t* slow = sSlow + (mt * kTileRows + row) * kSlowPitch;
        uint32_t acc_i = 0;
        bool ok = true;
        for (uint32_t t = blockIdx.x; t < n_qtiles && ok; t += gridDim.x) {
            const uint32_t qlocal = (t * MT + mt) * kTileRows + row;
            const bool qvalid = qlocal < p.n_queries;
            const uint32_t self_id = p.exclude_self ? p.query_id0 + qlocal : UINT32_MAX;
            const int32_t qnorm = (METRIC == 0 && qvalid) ? p.query_norms[qlocal] : 0;
            TopK tk;
            tk.init(p.k);
            int32_t thr = tk.thr();
            for (uint32_t j = 0; j < n_btiles; ++j, ++acc_i) {
                // Column keys are  nb - scale * dot  with nb = |r|^2 (L2) or 0
                // (IP) for real rows and INT_MAX for padding rows (dot == 0
                // there), so padding never enters the list.
                {
                    const uint64_t b0 = static_cast<uint64_t>(j) * kTileRows + lane * 4;
                    int4 nn;
                    if (b0 + 3 < p.n_base) {
                        nn = METRIC == 0 ? __ldg(reinterpret_cast<const int4*>(p.base_norms + b0)) : make_int4(0, 0, 0, 0);
                    } else {
                        nn.x = b0 + 0 < p.n_base ? (METRIC == 0 ? p.base_norms[b0 + 0] : 0) : INT_MAX;
                        nn.y = b0 + 1 < p.n_base ? (METRIC == 0 ? p.base_norms[b0 + 1] : 0) : INT_MAX;
                        nn.z = b0 + 2 < p.n_base ? (METRIC == 0 ? p.base_norms[b0 + 2] : 0) : INT_MAX;
                        nn.w = b0 + 3 < p.n_base ? (METRIC == 0 ? p.base_norms[b0 + 3] : 0) : INT_MAX;
                    }
                    reinterpret_cast<int4*>(nbuf + (j & 1) * kTileRows)[lane] = nn;
                    __syncwarp();
                }
                const uint32_t buf = acc_i & 1;
                ok = mbar_wait(&tfull[buf], (acc_i >> 1) & 1, abort_flag);
                if (!ok) break;
                tc_fence_after();
                const uint32_t tb = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * (MT * kTileRows) +
                                    mt * kTileRows;
                const int4* nb4 = reinterpret_cast<const int4*>(nbuf + (j & 1) * kTileRows);
#pragma unroll
                for (int c = 0; c < kTileRows / 32; ++c) {
                    int32_t v[32];
                    __syncwarp();
                    tmem_ld_32cols(tb + c * 32, v);
                    tmem_ld_wait(v);
                    if (c == kTileRows / 32 - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[buf]);
                    }
                    int32_t m = INT_MAX;
#pragma unroll
                    for (int i4 = 0; i4 < 8; ++i4) {
                        const int4 nn = nb4[c * 8 + i4];
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
                        m = min(m, min(min(v[4 * i4 + 0], v[4 * i4 + 1]), min(v[4 * i4 + 2], v[4 * i4 + 3])));
                    }
                    if (m < thr) {
                        // Rare path: spill this chunk's keys and insert the
                        // ones under the running threshold, in id order.
                        uint32_t mask = 0;
#pragma unroll
                        for (int i = 0; i < 32; ++i) mask |= (v[i] < thr ? 1u : 0u) << i;
#pragma unroll
                        for (int i4 = 0; i4 < 8; ++i4)
                            *reinterpret_cast<int4*>(slow + 4 * i4) =
                                make_int4(v[4 * i4], v[4 * i4 + 1], v[4 * i4 + 2], v[4 * i4 + 3]);
                        const uint32_t col0 = p.base_id0 + j * kTileRows + c * 32;
                        while (mask) {
                            const int i = __ffs(mask) - 1;
                            mask &= mask - 1;
                            const int32_t key = slow[i];
                            const uint32_t id = col0 + i;
                            if (key < thr && id != self_id) {
                                tk.insert(key, id);
                                thr = tk.thr();
                            }
                        }
                    }
                }
            }
            if (!ok) break;
            if (qvalid) {
                uint32_t* oid = p.out_ids + static_cast<uint64_t>(qlocal) * p.k;
                float* odist = p.out_dists + static_cast<uint64_t>(qlocal) * p.k;
                bool inexact = false;
                if (METRIC == 0) {
                    // Partial sums of squares are monotone: every retained sum
                    // is exact in fp32 iff the k-th is below 2^24.
                    inexact = static_cast<int64_t>(qnorm) + tk.thr() >= (1 << 24);
                    tk.for_each(p.k, [&](int j, int32_t key, uint32_t id) {
                        oid[j] = id;
                        odist[j] = __int2float_rn(qnorm + key);
                    });
                } else {
                    // Largest dot first: exact iff it is below 2^24.
                    inexact = -static_cast<int64_t>(tk.best(p.k)) >= (1 << 24);
                    tk.for_each(p.k, [&](int j, int32_t key, uint32_t id) {
                        oid[j] = id;
                        odist[j] = -__int2float_rn(-key);
                    });
                }
                if (inexact) {
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
