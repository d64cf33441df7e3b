/*
 * knng_gpu.h -- C ABI of the B200 brute-force KNN-graph builder
 * (libknng_gpu.so). Plain pointers and sizes only; no C++ or torch types.
 *
 * The reference has no FFI: its boundary is the C++ template
 *   template <Distance D>
 *   Knng knng::cpu::brute_force_knn(const Dataset& ds, std::size_t k, D d = D{});
 * (include/knng/cpu/brute_force.hpp:336-337, instantiated for L2Squared and
 * NegativeInnerProduct at src/cpu/brute_force.cpp:39-43). These entry points
 * are what a binding of that template to a GPU library needs; the header-only
 * C++ drop-in include/knng/gpu/brute_force.hpp wraps them back into the
 * reference's signature.
 *
 * Output layout (every entry point): row q of the graph is
 *   ids[q*k .. q*k+k), dists[q*k .. q*k+k)
 * sorted ascending by (distance, id), self excluded by index: the layout of
 * knng::Knng (include/knng/core/graph.hpp:35-84).
 *
 * Errors: every entry point returns a knng_gpu_status and never aborts; the
 * message of the last failure on the calling thread is knng_gpu_last_error().
 * Argument errors use the reference's wording (brute_force.hpp:339-352).
 */
#ifndef KNNG_GPU_H
#define KNNG_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    KNNG_GPU_OK = 0,
    KNNG_GPU_INVALID_ARGUMENT = 1, /* maps to std::invalid_argument */
    KNNG_GPU_CUDA_ERROR = 2,       /* a CUDA runtime/driver call failed */
    KNNG_GPU_TIMEOUT = 3,          /* a bounded device-side wait gave up */
    KNNG_GPU_NOT_SUPPORTED = 4,    /* e.g. k above KNNG_GPU_MAX_K */
    KNNG_GPU_OUT_OF_MEMORY = 5,
    KNNG_GPU_WORKSPACE_TOO_SMALL = 6
} knng_gpu_status;

/* Metric ids equal the .knng file header's metric_id
 * (tools/build_knng.cpp:183-188): 0 = L2Squared, 1 = NegativeInnerProduct. */
typedef enum { KNNG_METRIC_L2_SQUARED = 0, KNNG_METRIC_NEGATIVE_INNER_PRODUCT = 1 } knng_metric;

/* Which kernel family produced the result: exact u8 UMMA (integer data in
 * [0,255]) or bf16x3 UMMA candidate filter + exact fp32 re-rank (other data). */
typedef enum { KNNG_PATH_U8_TENSOR = 0, KNNG_PATH_F32_TENSOR = 1 } knng_path;

#define KNNG_GPU_MAX_K 1024u

typedef struct {
    int path;                 /* knng_path */
    uint64_t fallback_rows;   /* rows recomputed by the exact fp32 kernel */
    float pack_ms;            /* integer check + u8 pack + row norms */
    float knn_ms;             /* fused KNN kernel (device time, CUDA events) */
    float fallback_ms;        /* exact kernel on fallback rows */
    float total_ms;           /* whole call, device time */
    uint32_t kernel_launches; /* kernels this call launched */
    float f32_err_ratio;      /* fp32 path: max |approximate - exact| / proof margin seen (< 1) */
    float tc_ms;              /* the tensor-core kernel alone (device time; the roofline's denominator) */
} knng_gpu_stats;

/* Message of the last failure on this thread ("" if none). */
const char* knng_gpu_last_error(void);

/* Number of CUDA devices visible (0 if none / no driver). */
int knng_gpu_device_count(void);

/* ---- one-shot host API (the drop-in) ------------------------------------
 * Replaces knng::cpu::brute_force_knn<L2Squared|NegativeInnerProduct>
 * (include/knng/cpu/brute_force.hpp:336-376). `data` is the row-major
 * n x d fp32 payload of a knng::Dataset (dataset.hpp:76-152, data_ptr()),
 * `ids`/`dists` are caller-allocated n*k arrays (Knng::neighbors/distances).
 * Runs on the current CUDA device. Device buffers are cached per device and
 * reused by later calls (see knng_gpu_release_cached_buffers); calls on one
 * device are serialised. `stats` may be NULL. Host buffers may be pageable or
 * pinned: pinned ones (cudaMallocHost / cudaHostRegister) are copied
 * directly; pageable ones of 4 MiB or more go through a ring of four 32 MiB
 * pinned chunks that the library allocates on first use and keeps per
 * device, with the host-side copies spread over up to 8 threads. */
knng_gpu_status knng_gpu_brute_force(const float* data, uint64_t n, uint64_t d, uint64_t k, int metric,
                                     uint32_t* ids, float* dists, knng_gpu_stats* stats);

/* Same build from rows that are already bytes (.bvecs records: the u8 path
 * without the fp32 round trip, src/io/fvecs.cpp:189-206 reads them into
 * floats). Row r's d values start at rows + r * row_stride (row_stride >= d;
 * d + 4 passes a .bvecs payload with its per-row dimension headers after
 * skipping the first header). Output identical to knng_gpu_brute_force on the
 * same values as floats. */
knng_gpu_status knng_gpu_brute_force_u8(const uint8_t* rows, uint64_t n, uint64_t d, uint64_t row_stride, uint64_t k,
                                        int metric, uint32_t* ids, float* dists, knng_gpu_stats* stats);

/* Free the device buffers, pinned staging chunks and stream that
 * knng_gpu_brute_force keeps per device between calls (they are grown on
 * demand and otherwise held until process exit). No counterpart in the
 * reference. */
void knng_gpu_release_cached_buffers(void);

/* ---- device-resident API (inputs already in HBM) ------------------------
 * All pointers are device pointers; `stream` is a cudaStream_t (NULL = the
 * legacy default stream). Nothing is allocated: the caller passes a
 * workspace of at least knng_gpu_workspace_bytes(n, d, k) bytes, 256-byte
 * aligned. Same semantics and output layout as knng_gpu_brute_force; the
 * call synchronises `stream` once (to read which path applies). */
uint64_t knng_gpu_workspace_bytes(uint64_t n, uint64_t d, uint64_t k);
knng_gpu_status knng_gpu_brute_force_device(const float* d_data, uint64_t n, uint64_t d, uint64_t k, int metric,
                                            uint32_t* d_ids, float* d_dists, void* d_workspace,
                                            uint64_t workspace_bytes, void* stream, knng_gpu_stats* stats);

/* ---- building blocks for sharded (multi-GPU) builds ---------------------
 * The distributed driver (one process per GPU) packs its slice of rows,
 * exchanges packed rows with NCCL, and runs the fused kernel on its query
 * shard against the full base, mirroring the reference's query sharding
 * (include/knng/dist/sharded_dataset.hpp:145-155, src/dist/brute_force_mpi.cpp:36-142).
 *
 * knng_gpu_padded_dim: row pitch in bytes of the packed u8 layout: the row's
 *   d bytes rounded up to 128, then 32 bytes of augmentation.
 * knng_gpu_pack_u8: rows x d fp32 -> rows x pitch u8 + one int32 per row;
 *   atomically ORs 1 into *d_nonint if any value is not an integer in [0,255]
 *   (then the packed output is meaningless and the fp32 path must be used).
 *   The int32 is the row's key offset keyoff = |x|^2 + 510 * S, where S is
 *   the sum of the row's augmentation bytes: the packed set computes
 *   squared L2 as keyoff(r) - 2 (q.r + 255 S(r)) on the tensor cores. S is
 *   chosen per 128-row tile of the pack call (the tile's largest
 *   ceil(|x|^2/2) minus the row's, over 255, at most 8160), so packs whose
 *   first row sits on a multiple of 128 of the searched base filter most
 *   sharply; any split stays exact. Pass these arrays as the d_norms /
 *   d_q_norms / d_b_norms arguments below.
 * knng_gpu_knn_u8: queries are packed rows [q_begin, q_begin+q_count) of the
 *   base; results for query row i go to row i of d_ids/d_dists (q_count x k).
 *   d_scratch: >= knng_gpu_knn_scratch_bytes(q_count, k) bytes, 256-byte aligned.
 * knng_gpu_knn_f32: any fp32 data: bf16x3 tensor-core candidate filter over
 *   all n rows, exact re-rank with the reference's arithmetic and a proven
 *   error bound, exact kernel for rows the bound cannot certify.
 *   d_scratch: >= knng_gpu_knn_f32_scratch_bytes(n, d, q_count, k) bytes,
 *   256-byte aligned. */
uint64_t knng_gpu_padded_dim(uint64_t d);
knng_gpu_status knng_gpu_pack_u8(const float* d_x, uint64_t rows, uint64_t d, uint8_t* d_packed,
                                 int32_t* d_norms, int32_t* d_nonint, void* stream);
/* knng_gpu_pack_u8_bytes: as knng_gpu_pack_u8 for device rows that are
 *   already bytes (row r at d_rows + r * row_stride, row_stride >= d). */
knng_gpu_status knng_gpu_pack_u8_bytes(const uint8_t* d_rows, uint64_t rows, uint64_t d, uint64_t row_stride,
                                       uint8_t* d_packed, int32_t* d_norms, void* stream);
uint64_t knng_gpu_knn_scratch_bytes(uint64_t q_count, uint64_t k);
knng_gpu_status knng_gpu_knn_u8(const uint8_t* d_packed, const int32_t* d_norms, uint64_t n, uint64_t d,
                                uint64_t q_begin, uint64_t q_count, uint64_t k, int metric, uint32_t* d_ids,
                                float* d_dists, void* d_scratch, uint64_t scratch_bytes, void* stream,
                                knng_gpu_stats* stats);
/* knng_gpu_knn_u8_sets: query rows and base rows as separate packed sets
 *   (cross-set KNN and the base blocks of a ring pass). Ids are global: base
 *   row r is b_id0 + r, query row i is q_id0 + i; with exclude_self a query
 *   never returns its own id (src/dist/brute_force_mpi.cpp:80-82 excludes by
 *   global index the same way). Needs n_b >= k (+1 with exclude_self).
 *   d_q_packed, d_b_packed and d_b_norms must be 16-byte aligned (tensor-map
 *   sources; the key offsets are copied 16 bytes at a time), else
 *   KNNG_GPU_INVALID_ARGUMENT.
 *   d_scratch: >= knng_gpu_knn_scratch_bytes(n_q, k) bytes, 256-byte aligned.
 * knng_gpu_merge_topk: row-wise merge of two sorted k-lists into the k best
 *   by (distance, id), the TopK order (include/knng/top_k.hpp:56-72); merges
 *   the per-block results of a ring pass. */
knng_gpu_status knng_gpu_knn_u8_sets(const uint8_t* d_q_packed, const int32_t* d_q_norms, uint64_t n_q,
                                     uint64_t q_id0, const uint8_t* d_b_packed, const int32_t* d_b_norms, uint64_t n_b,
                                     uint64_t b_id0, uint64_t d, uint64_t k, int metric, int exclude_self,
                                     uint32_t* d_ids, float* d_dists, void* d_scratch, uint64_t scratch_bytes,
                                     void* stream, knng_gpu_stats* stats);
knng_gpu_status knng_gpu_merge_topk(const uint32_t* d_a_ids, const float* d_a_dists, const uint32_t* d_b_ids,
                                    const float* d_b_dists, uint64_t rows, uint64_t k, uint32_t* d_out_ids,
                                    float* d_out_dists, void* stream);
uint64_t knng_gpu_knn_f32_scratch_bytes(uint64_t n, uint64_t d, uint64_t q_count, uint64_t k);
/* knng_gpu_knn_f32_sets: fp32 query rows against separate fp32 base rows
 *   (cross-set KNN: the batched query != base search the reference's recall
 *   harness needs, src/bench/recall.cpp and src/bench/ground_truth.cpp).
 *   Same exactness as knng_gpu_knn_f32 (bf16x3 tensor-core filter, exact
 *   re-rank with the reference's arithmetic, exact kernel for rows the bound
 *   cannot certify); ids are global as in knng_gpu_knn_u8_sets. Needs
 *   n_b >= k (+1 with exclude_self). d_scratch: >=
 *   knng_gpu_knn_f32_sets_scratch_bytes(n_q, n_b, d, k, exclude_self) bytes,
 *   256-byte aligned. */
uint64_t knng_gpu_knn_f32_sets_scratch_bytes(uint64_t n_q, uint64_t n_b, uint64_t d, uint64_t k, int exclude_self);
knng_gpu_status knng_gpu_knn_f32_sets(const float* d_q, uint64_t n_q, uint64_t q_id0, const float* d_b, uint64_t n_b,
                                      uint64_t b_id0, uint64_t d, uint64_t k, int metric, int exclude_self,
                                      uint32_t* d_ids, float* d_dists, void* d_scratch, uint64_t scratch_bytes,
                                      void* stream, knng_gpu_stats* stats);
/* knng_gpu_recall_at_k: recall@k of an approximate graph against the true
 *   graph, both n x k device id arrays -- knng::bench::recall_at_k
 *   (src/bench/recall.cpp:79-96): the fraction of true neighbours found,
 *   where a repeated approximate id counts once (:52-77); 1.0 for n == 0.
 *   d_counter: 8 device bytes of scratch. Synchronises `stream`. */
knng_gpu_status knng_gpu_recall_at_k(const uint32_t* d_approx, const uint32_t* d_truth, uint64_t n, uint64_t k,
                                     void* d_counter, void* stream, double* recall);
knng_gpu_status knng_gpu_knn_f32(const float* d_x, uint64_t n, uint64_t d, uint64_t q_begin, uint64_t q_count,
                                 uint64_t k, int metric, uint32_t* d_ids, float* d_dists, void* d_scratch,
                                 uint64_t scratch_bytes, void* stream, knng_gpu_stats* stats);

/* ---- allocation-free variant of knng_gpu_knn_u8 -------------------------
 * No counterpart in the reference (it has no GPU code). For callers that may
 * not allocate device memory at all -- code running under a custom or
 * pre-reserved memory pool, inside a host that forbids cudaMalloc after
 * start-up, or a plugin that only receives device pointers from its host --
 * and therefore cannot provide the `d_scratch` buffer knng_gpu_knn_u8 needs.
 * Same arguments, semantics and output as knng_gpu_knn_u8 minus the scratch:
 * the fallback-row list and counters live in a fixed device array built into
 * the library (4 MiB + 256 B, held on every GPU that loads the library until
 * the process exits). Limits and caveats:
 *   - q_count must be <= KNNG_GPU_NOALLOC_MAX_QUERIES, else
 *     KNNG_GPU_INVALID_ARGUMENT;
 *   - every call looks up the array's address in the CUDA context current
 *     on the calling thread (cudaGetSymbolAddress): a host may use its own,
 *     non-primary context, or reset the device, between calls;
 *   - all calls share the one array: calls that overlap on the GPU (other
 *     streams, other host threads) race and must be serialised by the caller.
 * The call allocates nothing: no cudaMalloc/cudaFree and no allocating
 * library routine; it runs the single-CTA kernel (the array has no room for
 * the partial lists of the CTA-pair kernel) and records no timing events, so
 * the *_ms fields of `stats` are 0. Like every entry point here it ends by
 * synchronising `stream` once, to read the fallback count and the error
 * word of the bounded device waits. */
#define KNNG_GPU_NOALLOC_MAX_QUERIES (1u << 20)
knng_gpu_status knng_gpu_knn_u8_noalloc(const uint8_t* d_packed, const int32_t* d_norms, uint64_t n, uint64_t d,
                                        uint64_t q_begin, uint64_t q_count, uint64_t k, int metric, uint32_t* d_ids,
                                        float* d_dists, void* stream, knng_gpu_stats* stats);

/* ---- multi-GPU builds (NCCL) ---------------------------------------------
 * The reference's distributed build (src/dist/brute_force_mpi.cpp:36-203 over
 * MPI, sharded by include/knng/dist/sharded_dataset.hpp:145-155) as NCCL
 * ranks, one GPU each. Two ways to drive it:
 *
 * (1) one process per GPU (e.g. torchrun): rank 0 calls
 *     knng_gpu_nccl_unique_id, hands the knng_gpu_nccl_id_bytes() bytes to
 *     every rank by any channel, and every rank calls knng_gpu_comm_create
 *     with its device current, then knng_gpu_brute_force_sharded for each
 *     build. d_rows holds the rank's rows [begin, begin + count) given by
 *     knng_gpu_shard_rows. Rank 0 receives the whole n x k graph in
 *     d_ids/d_dists (device pointers; other ranks may pass NULL).
 * (2) one process driving num_gpus GPUs (devices 0..num_gpus-1):
 *     knng_gpu_brute_force_multi with host buffers, like
 *     knng_gpu_brute_force; communicators, streams and device buffers are
 *     kept between calls until knng_gpu_release_multi.
 *
 * mode 0 (replicate): the packed base is all-gathered to every GPU and each
 *   rank searches its compute_shard query rows against it; any data.
 * mode 1 (ring): the base stays sharded; blocks are passed around the ring
 *   (the reference's MPI_Sendrecv ring, brute_force_mpi.cpp:71-124) while the
 *   kernel searches the current block, and the per-query lists are merged by
 *   (distance, id). Integer-valued data in [0, 255] only, and at least k + 1
 *   rows per rank.
 * Every rank must make the same calls with the same arguments. Output is
 * identical to knng_gpu_brute_force for every rank count and mode. */
uint64_t knng_gpu_nccl_id_bytes(void);
knng_gpu_status knng_gpu_nccl_unique_id(void* id_out);
knng_gpu_status knng_gpu_comm_create(const void* id, int world, int rank, void** comm_out);
void knng_gpu_comm_destroy(void* comm);
void knng_gpu_shard_rows(uint64_t n, int world, int rank, int mode, uint64_t* begin, uint64_t* count);
uint64_t knng_gpu_sharded_workspace_bytes(uint64_t n, uint64_t d, uint64_t k, int world, int mode);
knng_gpu_status knng_gpu_brute_force_sharded(const float* d_rows, uint64_t n, uint64_t d, uint64_t k, int metric,
                                             int mode, void* comm, uint32_t* d_ids, float* d_dists,
                                             void* d_workspace, uint64_t workspace_bytes, void* stream,
                                             knng_gpu_stats* stats);
/* Device time of the phases of the last sharded build on this rank (filled
 * when that build had non-NULL stats): pack, base exchange, search, fp32
 * exchange + search, gather to rank 0, total. */
knng_gpu_status knng_gpu_comm_phase_ms(void* comm, float* out6);
knng_gpu_status knng_gpu_brute_force_multi(const float* data, uint64_t n, uint64_t d, uint64_t k, int metric,
                                           int num_gpus, int mode, uint32_t* ids, float* dists,
                                           knng_gpu_stats* stats);
void knng_gpu_release_multi(void);

/* ---- test hook -----------------------------------------------------------
 * Runs one small build whose device-side waits give up after
 * `wait_limit_cycles` clock cycles while the kernel's producer withholds one
 * arrival on purpose. Returns KNNG_GPU_TIMEOUT when the bounded waits work
 * (the kernel unwinds, frees its TMEM and the CUDA context stays usable).
 * Allocates and frees its own small buffers. No counterpart in the
 * reference, whose code has no device waits. */
knng_gpu_status knng_gpu_selftest_bounded_wait(uint64_t wait_limit_cycles);

#ifdef __cplusplus
}
#endif

#endif /* KNNG_GPU_H */
