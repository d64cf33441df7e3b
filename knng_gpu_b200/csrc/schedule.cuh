// schedule.cuh -- how the persistent u8 KNN kernels split the (query tile,
// base tile) work space over their units (CTAs, or CTA pairs), and the merge
// of query tiles that end up split between units.
//
// Query tiles [0, full_waves * n_units) go round-robin to the units, each
// searched against the whole base: all units then sweep the base in the same
// order and share it in L2. The last, partial wave -- tail_total = its query
// tiles x n_btiles work items -- is cut into equal contiguous ranges, one per
// unit, so every unit finishes at about the same time instead of most of
// them idling through the last wave. A query tile cut between units leaves
// one partial (key, id) list per piece; merge_partials combines them by
// (key, id) -- exact, since the keys are exact integers.
#pragma once
#include <climits>
#include <cstdint>

#include "topk.cuh"

namespace knng_b200 {

struct TileSchedule {
    uint32_t n_units;
    uint32_t full_waves;
    uint32_t n_qtiles;
    uint32_t n_btiles;
    uint64_t tail_total;
};

// full_waves = n_qtiles / n_units and the remainder as the tail; with
// no_tail every query tile is whole (round-robin over ceil(n_qtiles / n_units)
// waves).
__host__ __device__ inline TileSchedule make_schedule(uint32_t n_units, uint32_t n_qtiles, uint32_t n_btiles,
                                                      bool no_tail)
{
    TileSchedule s;
    s.n_units = n_units;
    s.n_qtiles = n_qtiles;
    s.n_btiles = n_btiles;
    if (no_tail) {
        s.full_waves = (n_qtiles + n_units - 1) / n_units;
        s.tail_total = 0;
    } else {
        s.full_waves = n_qtiles / n_units;
        s.tail_total = static_cast<uint64_t>(n_qtiles % n_units) * n_btiles;
    }
    return s;
}

// First tail work item of unit u (equal contiguous ranges of [0, total)).
__host__ __device__ inline uint64_t range_begin(uint64_t total, uint32_t n_units, uint32_t u)
{
    return total * u / n_units;
}

// Segment idx of unit u: query tile qt, base tiles [b0, b1). Segments
// 0 .. full_waves-1 are whole query tiles; then at most two pieces of the
// unit's tail range (a range shorter than n_btiles spans at most two query
// tiles). pslot: the slot of the piece's partial lists (2 per unit: the
// range's first and last piece).
__device__ inline bool schedule_segment(const TileSchedule& s, uint32_t u, uint32_t idx, uint32_t& qt, uint32_t& b0,
                                        uint32_t& b1, uint32_t& pslot)
{
    const uint32_t nbt = s.n_btiles;
    if (idx < s.full_waves) {
        qt = u + idx * s.n_units;
        b0 = 0;
        b1 = nbt;
        pslot = 2 * u;
        return qt < s.n_qtiles;
    }
    idx -= s.full_waves;
    if (idx > 1 || s.tail_total == 0) return false;
    const uint64_t tw0 = range_begin(s.tail_total, s.n_units, u);
    const uint64_t tw1 = range_begin(s.tail_total, s.n_units, u + 1);
    uint64_t s0 = tw0;
    if (idx == 1) s0 = (tw0 / nbt + 1) * nbt;
    if (s0 >= tw1) return false;
    const uint64_t qe = (s0 / nbt + 1) * nbt;
    const uint64_t s1 = qe < tw1 ? qe : tw1;
    qt = s.full_waves * s.n_units + static_cast<uint32_t>(s0 / nbt);
    b0 = static_cast<uint32_t>(s0 % nbt);
    b1 = b0 + static_cast<uint32_t>(s1 - s0);
    pslot = 2 * u + idx;
    return true;
}

// The unit holding tail work item w (largest u with range_begin(u) <= w).
__device__ inline uint32_t unit_of_work(uint64_t total, uint32_t n_units, uint64_t w)
{
    uint32_t u = static_cast<uint32_t>(w * n_units / total);
    while (u + 1 < n_units && range_begin(total, n_units, u + 1) <= w) ++u;
    while (u > 0 && range_begin(total, n_units, u) > w) --u;
    return u;
}

struct MergeParams {
    TileSchedule s;
    uint32_t qtile_rows;         // query rows per query tile
    uint32_t k;
    uint32_t n_queries;
    const int32_t* part_keys;    // [2 * n_units][qtile_rows][k]
    const uint32_t* part_ids;
    uint32_t* out_ids;           // n_queries x k graph rows
    float* out_dists;
    int32_t* seed_out;           // seeding pass: the k-th key per query instead
    const int32_t* seed_in;      // optional: per query an upper bound on the keys its list admits
    const int32_t* query_norms;  // key offset per query row (L2)
    const uint8_t* query_packed; // packed query rows (augmentation bytes give |q|^2)
    uint32_t pitch;
    uint32_t data_bytes;
    uint32_t* fallback_rows;
    uint32_t* fallback_count;
    const int* skip_flag;
};

// |q|^2 of a packed query row: its key offset minus 510 x the sum of its
// augmentation bytes.
__device__ __forceinline__ int32_t packed_sq_norm(const uint8_t* packed, uint32_t pitch, uint32_t data_bytes,
                                                  const int32_t* keyoff, uint32_t qlocal)
{
    const uint4* a4 = reinterpret_cast<const uint4*>(packed + static_cast<uint64_t>(qlocal) * pitch + data_bytes);
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
    return keyoff[qlocal] - 510 * static_cast<int32_t>(sb);
}

// Graph row of query qlocal from its sorted (key, id) list: distances
// |q|^2 + key (L2) or key (inner product) as fp32; rows whose fp32 sums may
// round (L2: k-th distance >= 2^24; inner product: largest dot >= 2^24) are
// appended to the fallback list for the exact kernel. `bound` is the largest
// key the list could admit (INT_MAX: none). A list searched under an outside
// bound (the running k-th key of a ring build) may hold fewer than k
// entries; its empty slots are emitted as (id 0xFFFFFFFF, +inf), which sort
// after every real entry when the lists are merged, and its exactness test
// uses the bound in place of the missing k-th key.
template <int METRIC, class TopK>
__device__ inline void emit_graph_row(TopK& tk, uint32_t k, uint32_t qlocal, int32_t qnorm, uint32_t* out_ids,
                                      float* out_dists, uint32_t* fallback_rows, uint32_t* fallback_count,
                                      int32_t bound = INT_MAX)
{
    uint32_t* oid = out_ids + static_cast<uint64_t>(qlocal) * k;
    float* odist = out_dists + static_cast<uint64_t>(qlocal) * k;
    bool inexact;
    if constexpr (METRIC == 0) {
        inexact = static_cast<int64_t>(qnorm) + min(tk.thr(), bound) >= (1 << 24);
        tk.for_each(k, [&](int jj, int32_t key, uint32_t id) {
            oid[jj] = id;
            odist[jj] = key == INT_MAX ? __int_as_float(0x7F800000) : __int2float_rn(qnorm + key);
        });
    } else {
        inexact = -static_cast<int64_t>(tk.best(k)) >= (1 << 24);
        tk.for_each(k, [&](int jj, int32_t key, uint32_t id) {
            oid[jj] = id;
            odist[jj] = key == INT_MAX ? __int_as_float(0x7F800000) : -__int2float_rn(-key);
        });
    }
    if (inexact) {
        const uint32_t fs = atomicAdd(fallback_count, 1u);
        fallback_rows[fs] = qlocal;
    }
}

// Merge the partial lists of the tail's query tiles that are cut between
// units. Block b looks at the boundary between units b and b + 1 in the tail
// range; it handles the query tile that boundary falls inside (if it does not
// fall on a tile start), unless the previous boundary cut the same tile.
// One thread per query row of the tile.
template <int METRIC, int KCAP>
__global__ void merge_partials(const MergeParams p)
{
    const uint32_t ub = blockIdx.x + 1;  // boundary: start of unit ub's tail range
    const TileSchedule& s = p.s;
    if (ub >= s.n_units || s.tail_total == 0 || (p.skip_flag && *p.skip_flag)) return;
    const uint32_t nbt = s.n_btiles;
    const uint64_t total = s.tail_total;
    const uint64_t wb = range_begin(total, s.n_units, ub);
    if (wb % nbt == 0 || wb >= total) return;
    const uint32_t qt_tail = static_cast<uint32_t>(wb / nbt);
    if (ub > 1) {
        const uint64_t wprev = range_begin(total, s.n_units, ub - 1);
        if (wprev / nbt == qt_tail && wprev % nbt != 0) return;
    }
    const uint64_t qlo = static_cast<uint64_t>(qt_tail) * nbt, qhi = qlo + nbt;
    const uint32_t u_first = unit_of_work(total, s.n_units, qlo);
    const uint32_t u_last = unit_of_work(total, s.n_units, qhi - 1);
    const uint32_t q = s.full_waves * s.n_units + qt_tail;
    const uint32_t r = threadIdx.x;
    const uint32_t qlocal = q * p.qtile_rows + r;
    if (r >= p.qtile_rows || qlocal >= p.n_queries) return;
    RegTopK<KCAP> tk;
    tk.init(p.k);
    for (uint32_t uu = u_first; uu <= u_last; ++uu) {
        // Units with an empty range (fewer tail items than units) wrote nothing.
        if (range_begin(total, s.n_units, uu) == range_begin(total, s.n_units, uu + 1)) continue;
        // The piece of unit uu in this tile is its range's first piece
        // (slot 0) unless the range began in the previous tile (slot 1).
        const uint32_t slot = range_begin(total, s.n_units, uu) < qlo ? 1u : 0u;
        const uint64_t o = (static_cast<uint64_t>(2 * uu + slot) * p.qtile_rows + r) * p.k;
        for (uint32_t j = 0; j < p.k; ++j) {
            const int32_t key = p.part_keys[o + j];
            const uint32_t id = p.part_ids[o + j];
            if (key_gt(tk.thr(), tk.thr_id(), key, id)) tk.insert(key, id);
        }
    }
    const int32_t bound = p.seed_in ? p.seed_in[qlocal] : INT_MAX;
    if (p.seed_out) {
        p.seed_out[qlocal] = min(tk.thr(), bound);
        return;
    }
    const int32_t qnorm =
        METRIC == 0 ? packed_sq_norm(p.query_packed, p.pitch, p.data_bytes, p.query_norms, qlocal) : 0;
    emit_graph_row<METRIC>(tk, p.k, qlocal, qnorm, p.out_ids, p.out_dists, p.fallback_rows, p.fallback_count,
                           bound);
}

}  // namespace knng_b200
