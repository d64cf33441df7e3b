// topk.cuh -- per-thread bounded top-k candidate lists.
//
// Both structures keep the k smallest (key, id) pairs under the total order
// "key ascending, then id ascending": the order of knng::TopK
// (include/knng/top_k.hpp:56-72, comparator :113-121). Keys are int32: exact
// integer distance keys on the u8 path, order-preserving images of fp32
// distances on the fp32 path (ordered_key below).
#pragma once
#include <climits>
#include <cstdint>

namespace knng_b200 {

// (a, ia) > (b, ib) lexicographically.
__device__ __forceinline__ bool key_gt(int32_t a, uint32_t ia, int32_t b, uint32_t ib)
{
    return a > b || (a == b && ia > ib);
}

// Map an fp32 distance to an int32 whose signed order equals the float
// order. -0.0 and +0.0 map to the same key (they compare equal in C++).
__device__ __forceinline__ int32_t ordered_key(float f)
{
    const int32_t b = __float_as_int(f + 0.0f);
    return b >= 0 ? b : (b ^ 0x7FFFFFFF);
}

__device__ __forceinline__ float key_to_float(int32_t key)
{
    return __int_as_float(key >= 0 ? key : (key ^ 0x7FFFFFFF));
}

// Sorted list held in registers, capacity KCAP >= k. Slots [0, KCAP-k) hold
// INT_MIN sentinels that never move, so the worst retained entry is always
// slot KCAP-1 and the threshold read is a static register.
template <int KCAP>
struct RegTopK {
    static constexpr int kRegs = 2 * KCAP;
    static constexpr int kCap = KCAP;  // register lists: the capacity (merge kernels take it)
    int32_t key[KCAP];
    uint32_t id[KCAP];

    __device__ __forceinline__ void init(uint32_t k)
    {
#pragma unroll
        for (int i = 0; i < KCAP; ++i) {
            const bool sentinel = i < KCAP - static_cast<int>(k);
            key[i] = sentinel ? INT_MIN : INT_MAX;
            id[i] = sentinel ? 0u : UINT32_MAX;
        }
    }
    __device__ __forceinline__ int32_t thr() const { return key[KCAP - 1]; }
    __device__ __forceinline__ uint32_t thr_id() const { return id[KCAP - 1]; }

    // Precondition: (v, vid) < (key[KCAP-1], id[KCAP-1]).
    __device__ __forceinline__ void insert(int32_t v, uint32_t vid)
    {
#pragma unroll
        for (int i = KCAP - 1; i > 0; --i) {
            const bool shift = key_gt(key[i - 1], id[i - 1], v, vid);
            const bool here = key_gt(key[i], id[i], v, vid);
            const int32_t nk = shift ? key[i - 1] : (here ? v : key[i]);
            const uint32_t ni = shift ? id[i - 1] : (here ? vid : id[i]);
            key[i] = nk;
            id[i] = ni;
        }
        if (key_gt(key[0], id[0], v, vid)) {
            key[0] = v;
            id[0] = vid;
        }
    }

    // Insert when ids arrive in increasing order (one thread scanning base
    // rows in order): an equal key never displaces an earlier id, so only
    // keys need comparing. Precondition: v < key[KCAP-1].
    __device__ __forceinline__ void insert_increasing(int32_t v, uint32_t vid)
    {
#pragma unroll
        for (int i = KCAP - 1; i > 0; --i) {
            const bool shift = key[i - 1] > v;
            const bool here = key[i] > v;
            const int32_t nk = shift ? key[i - 1] : (here ? v : key[i]);
            const uint32_t ni = shift ? id[i - 1] : (here ? vid : id[i]);
            key[i] = nk;
            id[i] = ni;
        }
        if (key[0] > v) {
            key[0] = v;
            id[0] = vid;
        }
    }

    // Entry j (0-based, ascending) of the k retained.
    template <class F>
    __device__ __forceinline__ void for_each(uint32_t k, F&& f) const
    {
#pragma unroll
        for (int i = 0; i < KCAP; ++i) {
            const int j = i - (KCAP - static_cast<int>(k));
            if (j >= 0) f(j, key[i], id[i]);
        }
    }
    __device__ __forceinline__ int32_t best(uint32_t k) const
    {
        int32_t b = INT_MAX;
#pragma unroll
        for (int i = 0; i < KCAP; ++i)
            if (i == KCAP - static_cast<int>(k)) b = key[i];
        return b;
    }
};

// Binary max-heap in thread-local memory for large k (up to KMAX); the root
// is the worst retained entry. Used where k does not fit in registers.
template <int KMAX>
struct HeapTopK {
    static constexpr int kRegs = 4;
    static constexpr int kCap = 0;  // not a register list
    int32_t hk[KMAX];
    uint32_t hi[KMAX];
    uint32_t size;
    uint32_t cap;

    __device__ __forceinline__ void init(uint32_t k)
    {
        size = 0;
        cap = k;
    }
    __device__ __forceinline__ int32_t thr() const { return size < cap ? INT_MAX : hk[0]; }
    __device__ __forceinline__ uint32_t thr_id() const { return size < cap ? UINT32_MAX : hi[0]; }

    __device__ void insert(int32_t v, uint32_t vid)
    {
        if (size < cap) {
            uint32_t i = size++;
            while (i > 0) {
                const uint32_t p = (i - 1) >> 1;
                if (!key_gt(v, vid, hk[p], hi[p])) break;
                hk[i] = hk[p];
                hi[i] = hi[p];
                i = p;
            }
            hk[i] = v;
            hi[i] = vid;
            return;
        }
        sift_down_from_root(v, vid, size);
    }

    __device__ __forceinline__ void insert_increasing(int32_t v, uint32_t vid) { insert(v, vid); }

    __device__ void sift_down_from_root(int32_t v, uint32_t vid, uint32_t sz)
    {
        uint32_t i = 0;
        for (;;) {
            const uint32_t l = 2 * i + 1, r = l + 1;
            uint32_t m = i;
            int32_t bk = v;
            uint32_t bi = vid;
            if (l < sz && key_gt(hk[l], hi[l], bk, bi)) {
                m = l;
                bk = hk[l];
                bi = hi[l];
            }
            if (r < sz && key_gt(hk[r], hi[r], bk, bi)) {
                m = r;
                bk = hk[r];
                bi = hi[r];
            }
            if (m == i) break;
            hk[i] = hk[m];
            hi[i] = hi[m];
            i = m;
        }
        hk[i] = v;
        hi[i] = vid;
    }

    // Heap-sort in place: afterwards hk/hi[0..size) ascend.
    __device__ void sort()
    {
        for (uint32_t end = size; end > 1; --end) {
            const int32_t tk = hk[0];
            const uint32_t ti = hi[0];
            const int32_t lk = hk[end - 1];
            const uint32_t li = hi[end - 1];
            sift_down_from_root(lk, li, end - 1);
            hk[end - 1] = tk;
            hi[end - 1] = ti;
        }
    }

    template <class F>
    __device__ void for_each(uint32_t k, F&& f)
    {
        sort();
        for (uint32_t j = 0; j < size && j < k; ++j) f(static_cast<int>(j), hk[j], hi[j]);
    }
    __device__ int32_t best(uint32_t) const
    {
        int32_t b = INT_MAX;
        for (uint32_t i = 0; i < size; ++i) b = hk[i] < b ? hk[i] : b;
        return b;
    }
};

}  // namespace knng_b200
