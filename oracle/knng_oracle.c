/*
 * knng_oracle.c -- CPU restatement of the reference's exact brute-force
 * KNN-graph path. TEST INFRASTRUCTURE ONLY: this file is the checker that
 * the CUDA path is compared against. Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg load it; the product library never links
 * or calls it.
 *
 * Pinned by: tests/test_oracle.py, which checks it against
 *   - the reference's own known-answer tests (tests/brute_force_test.cpp:36-150,
 *     tests/top_k_test.cpp:82-97, tests/core_test.cpp:38-100), restated as data;
 *   - golden vectors produced by the reference itself, compiled from its own
 *     sources (oracle/Makefile -> oracle/_ref/libknng_ref.so), committed under
 *     tests/golden/ together with the script that made them.
 *
 * Each function cites the reference file:line whose behaviour it restates.
 * Build: gcc -std=c11 -O2 -fopenmp -shared -fPIC (see oracle/Makefile).
 * The arithmetic is deliberately plain: no FMA contraction
 * (-ffp-contract=off), sequential left-to-right fp32 sums, exactly like the
 * reference built in ISO C++20 mode without -ffast-math or -march.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---- XorShift64 (include/knng/random.hpp:48-144) ---------------------- */

/* One step of the (13, 7, 17) xorshift, random.hpp:79-87. */
uint64_t oracle_xorshift64_next(uint64_t *state)
{
    uint64_t x = *state;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *state = x;
    return x;
}

/* Top 24 bits scaled by 2^-24, random.hpp:115-123. */
float oracle_next_float01(uint64_t *state)
{
    const uint64_t bits = (oracle_xorshift64_next(state) >> 40) & ((1ull << 24) - 1);
    return (float)bits * (1.0f / (float)(1u << 24));
}

/* Lemire multiply-high, random.hpp:131-140. */
uint64_t oracle_next_below(uint64_t *state, uint64_t bound)
{
    if (bound <= 1) return 0;
    const unsigned __int128 p = (unsigned __int128)oracle_xorshift64_next(state) * bound;
    return (uint64_t)(p >> 64);
}

/* Fill `out` with `count` raw 64-bit outputs (golden-vector hook). */
void oracle_xorshift64_stream(uint64_t seed, uint64_t count, uint64_t *out)
{
    uint64_t s = seed;
    for (uint64_t i = 0; i < count; ++i) out[i] = oracle_xorshift64_next(&s);
}

/* ---- distances (include/knng/core/distance.hpp:52-116) ---------------- */

/* squared_l2: acc += (a-b)^2, sequential fp32, distance.hpp:52-62. */
float oracle_squared_l2(const float *a, const float *b, uint64_t dim)
{
    float acc = 0.0f;
    for (uint64_t i = 0; i < dim; ++i) {
        const float delta = a[i] - b[i];
        const float sq = delta * delta;
        acc = acc + sq;
    }
    return acc;
}

/* NegativeInnerProduct: -(sum a*b), sequential fp32, distance.hpp:105-116. */
float oracle_negative_inner_product(const float *a, const float *b, uint64_t dim)
{
    float acc = 0.0f;
    for (uint64_t i = 0; i < dim; ++i) {
        const float p = a[i] * b[i];
        acc = acc + p;
    }
    return -acc;
}

/* compute_norms_squared: sequential fp32 sum of squares, src/cpu/distance.cpp:17-38. */
void oracle_norms_squared(const float *x, uint64_t n, uint64_t d, float *out)
{
    for (uint64_t i = 0; i < n; ++i) {
        const float *row = x + i * d;
        float acc = 0.0f;
        for (uint64_t j = 0; j < d; ++j) {
            const float sq = row[j] * row[j];
            acc = acc + sq;
        }
        out[i] = acc;
    }
}

/* ---- TopK (include/knng/top_k.hpp:43-127) ----------------------------- */
/*
 * Bounded max-heap keyed on (dist, id) lexicographically; the root is the
 * worst retained entry. Admission rule top_k.hpp:56-72: admit when not full,
 * or dist < worst.dist, or (dist == worst.dist && id < worst.id).
 */
typedef struct {
    float dist;
    uint32_t id;
} oracle_entry;

static int entry_worse(oracle_entry a, oracle_entry b) /* a > b in (dist, id) */
{
    if (a.dist != b.dist) return a.dist > b.dist;
    return a.id > b.id;
}

typedef struct {
    oracle_entry *h;
    uint64_t size, cap;
} oracle_topk;

static void topk_push(oracle_topk *t, uint32_t id, float dist)
{
    if (t->cap == 0) return;
    oracle_entry e = {dist, id};
    if (t->size < t->cap) {
        uint64_t i = t->size++;
        while (i > 0) {
            uint64_t p = (i - 1) / 2;
            if (!entry_worse(e, t->h[p])) break;
            t->h[i] = t->h[p];
            i = p;
        }
        t->h[i] = e;
        return;
    }
    const oracle_entry w = t->h[0];
    if (!(dist < w.dist || (dist == w.dist && id < w.id))) return;
    /* replace root, sift down */
    uint64_t i = 0;
    for (;;) {
        uint64_t l = 2 * i + 1, r = l + 1, m = i;
        oracle_entry best = e;
        if (l < t->size && entry_worse(t->h[l], best)) { m = l; best = t->h[l]; }
        if (r < t->size && entry_worse(t->h[r], best)) { m = r; best = t->h[r]; }
        if (m == i) break;
        t->h[i] = t->h[m];
        i = m;
    }
    t->h[i] = e;
}

/* extract_sorted: ascending (dist, id), top_k.hpp:78-91. */
static uint64_t topk_extract_sorted(oracle_topk *t, uint32_t *ids, float *dists)
{
    const uint64_t m = t->size;
    for (uint64_t out = m; out-- > 0;) {
        ids[out] = t->h[0].id;
        dists[out] = t->h[0].dist;
        oracle_entry last = t->h[--t->size];
        uint64_t i = 0;
        for (;;) {
            uint64_t l = 2 * i + 1, r = l + 1, mm = i;
            oracle_entry best = last;
            if (l < t->size && entry_worse(t->h[l], best)) { mm = l; best = t->h[l]; }
            if (r < t->size && entry_worse(t->h[r], best)) { mm = r; best = t->h[r]; }
            if (mm == i) break;
            t->h[i] = t->h[mm];
            i = mm;
        }
        if (t->size) t->h[i] = last;
    }
    return m;
}

/* Public TopK hook for golden tests: push (ids[i], dists[i]) in order into a
 * TopK(k) and extract. Returns the number of extracted entries. */
uint64_t oracle_topk_run(uint64_t k, uint64_t count, const uint32_t *ids, const float *dists,
                         uint32_t *out_ids, float *out_dists)
{
    oracle_topk t = {NULL, 0, k};
    t.h = (oracle_entry *)malloc(sizeof(oracle_entry) * (k ? k : 1));
    for (uint64_t i = 0; i < count; ++i) topk_push(&t, ids[i], dists[i]);
    const uint64_t m = topk_extract_sorted(&t, out_ids, out_dists);
    free(t.h);
    return m;
}

/* ---- brute force (include/knng/cpu/brute_force.hpp:336-376) ----------- */

enum { ORACLE_OK = 0, ORACLE_EMPTY = 1, ORACLE_K_ZERO = 2, ORACLE_K_TOO_LARGE = 3 };

/*
 * For each query row q in `queries` (indices into x), score every base row
 * r != q with the metric (0 = L2Squared, 1 = NegativeInnerProduct), keep the
 * k smallest in a TopK and write the sorted row. Argument checks follow
 * brute_force.hpp:339-352. The canonical path is `queries == NULL`
 * (all rows, in order); a non-NULL list is the subset harness: the same loop
 * body (brute_force.hpp:355-374) for a chosen list of query rows. Rows are
 * independent, so the OpenMP split over queries leaves every row bit-identical.
 */
int oracle_brute_force_knn(const float *x, uint64_t n, uint64_t d, uint64_t k, int metric,
                           const uint64_t *queries, uint64_t n_queries,
                           uint32_t *out_ids, float *out_dists)
{
    if (n == 0) return ORACLE_EMPTY;
    if (k == 0) return ORACLE_K_ZERO;
    if (k > n - 1) return ORACLE_K_TOO_LARGE;
    const uint64_t nq = queries ? n_queries : n;
#pragma omp parallel
    {
        oracle_topk t = {NULL, 0, k};
        t.h = (oracle_entry *)malloc(sizeof(oracle_entry) * k);
#pragma omp for schedule(dynamic, 16)
        for (int64_t qi = 0; qi < (int64_t)nq; ++qi) {
            const uint64_t q = queries ? queries[qi] : (uint64_t)qi;
            const float *qr = x + q * d;
            t.size = 0;
            for (uint64_t r = 0; r < n; ++r) {
                if (r == q) continue;
                const float dist = metric == 0 ? oracle_squared_l2(qr, x + r * d, d)
                                               : oracle_negative_inner_product(qr, x + r * d, d);
                topk_push(&t, (uint32_t)r, dist);
            }
            topk_extract_sorted(&t, out_ids + (uint64_t)qi * k, out_dists + (uint64_t)qi * k);
        }
        free(t.h);
    }
    return ORACLE_OK;
}

/*
 * Cross-set variant of the same loop body (brute_force.hpp:355-374): every
 * query row of `q` (id q_id0 + i) against every base row of `b` (id
 * b_id0 + r), skipping equal ids when exclude_self is set -- the reference's
 * distributed builder scores its local queries against a remote block this
 * way, excluding self by global index (src/dist/brute_force_mpi.cpp:76-82).
 */
int oracle_knn_sets(const float *q, uint64_t n_q, uint64_t q_id0, const float *b, uint64_t n_b, uint64_t b_id0,
                    uint64_t d, uint64_t k, int metric, int exclude_self, uint32_t *out_ids, float *out_dists)
{
    if (n_b == 0) return ORACLE_EMPTY;
    if (k == 0) return ORACLE_K_ZERO;
    if (k > n_b - (exclude_self ? 1 : 0)) return ORACLE_K_TOO_LARGE;
#pragma omp parallel
    {
        oracle_topk t = {NULL, 0, k};
        t.h = (oracle_entry *)malloc(sizeof(oracle_entry) * k);
#pragma omp for schedule(dynamic, 16)
        for (int64_t qi = 0; qi < (int64_t)n_q; ++qi) {
            const float *qr = q + (uint64_t)qi * d;
            const uint64_t qid = q_id0 + (uint64_t)qi;
            t.size = 0;
            for (uint64_t r = 0; r < n_b; ++r) {
                if (exclude_self && b_id0 + r == qid) continue;
                const float dist = metric == 0 ? oracle_squared_l2(qr, b + r * d, d)
                                               : oracle_negative_inner_product(qr, b + r * d, d);
                topk_push(&t, (uint32_t)(b_id0 + r), dist);
            }
            topk_extract_sorted(&t, out_ids + (uint64_t)qi * k, out_dists + (uint64_t)qi * k);
        }
        free(t.h);
    }
    return ORACLE_OK;
}

/* ---- dataset hash (src/bench/ground_truth.cpp:45-56, 90-101) ---------- */

static uint64_t fnv_update(uint64_t s, const void *bytes, uint64_t n)
{
    const uint8_t *p = (const uint8_t *)bytes;
    for (uint64_t i = 0; i < n; ++i) {
        s ^= (uint64_t)p[i];
        s *= 1099511628211ull;
    }
    return s;
}

/* FNV-1a 64 over (u64 n, u64 d, fp32 payload), ground_truth.cpp:90-101. */
uint64_t oracle_dataset_hash(const float *x, uint64_t n, uint64_t d)
{
    uint64_t s = 14695981039346656037ull;
    s = fnv_update(s, &n, sizeof n);
    s = fnv_update(s, &d, sizeof d);
    if (n * d) s = fnv_update(s, x, n * d * sizeof(float));
    return s;
}

/* ---- recall (src/bench/recall.cpp:52-96) ------------------------------ */

/* Mean over rows of |unique(approx_row) ∩ truth_row| / k. */
double oracle_recall_at_k(const uint32_t *approx, const uint32_t *truth, uint64_t n, uint64_t k)
{
    if (n == 0) return 1.0;
    uint64_t hits = 0;
    for (uint64_t q = 0; q < n; ++q) {
        const uint32_t *a = approx + q * k, *t = truth + q * k;
        for (uint64_t i = 0; i < k; ++i) {
            int dup = 0;
            for (uint64_t j = 0; j < i; ++j) if (a[j] == a[i]) { dup = 1; break; }
            if (dup) continue;
            for (uint64_t j = 0; j < k; ++j) if (t[j] == a[i]) { ++hits; break; }
        }
    }
    return (double)hits / ((double)n * (double)k);
}
