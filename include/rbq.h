/*
 * rbq.h -- C ABI of the B200-native IVF-RaBitQ retrieval library (librbq.so).
 *
 * Drop-in boundary for Neurosamble's retrieval hot path.  The reference path is the vendored
 * cuVS fork's C++ API (third-party/cuvs_rabitq/cpp/include/cuvs/neighbors/ivf_rabitq.hpp),
 * driven by the rabitq_search CLI (src/rabitq_gpu/rabitq_search.cu) and consumed by
 * src/neurosamble/overlap/map_full.py.  Every entry point below names the reference
 * interface it replaces.
 *
 * Conventions
 *   - Every function returns an int status (RBQ_OK == 0).  Nothing throws across the ABI,
 *     nothing calls exit() or traps; rbq_last_error() returns the calling thread's message.
 *   - Pointers named *_dev are device pointers on the index's device, owned by the caller.
 *     The library owns the index memory.  `stream` is a cudaStream_t (0 = legacy default);
 *     work is enqueued asynchronously on it unless the function says it synchronises.
 *   - One handle per stream/thread at a time; distinct handles are independent.
 *   - Distances are squared L2 (ascending); missing results have id -1 and distance +inf.
 */
#ifndef RBQ_H_
#define RBQ_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RBQ_OK 0
#define RBQ_ERR_INVALID 1 /* bad argument (size, nprobe > nlist, null pointer, ...) */
#define RBQ_ERR_CUDA 2    /* a CUDA runtime call failed */
#define RBQ_ERR_OOM 3     /* device allocation failed */
#define RBQ_ERR_IO 4      /* file open/read/write failed */
#define RBQ_ERR_STATE 5   /* wrong call order (search before add, add before train, ...) */
#define RBQ_ERR_FORMAT 6  /* index file malformed or truncated */

typedef struct rbq_index rbq_index_t;

/* Build-time parameters.  Replaces cuvs::neighbors::ivf_rabitq::index_params
 * (ivf_rabitq.hpp:50-103). */
typedef struct {
  int32_t dim;                          /* D; padded internally to Dp = ceil(D/32)*32       */
  int32_t n_lists;                      /* K (n_lists)                                        */
  uint64_t seed;                        /* rotation / t4 seed (reference: RAFT seed 7)        */
  int32_t kmeans_n_iters;               /* reference default 20                               */
  int32_t max_train_points_per_cluster; /* reference default 256                              */
  int32_t device;                       /* CUDA device ordinal holding the index              */
  int32_t shard_rank;                   /* this handle stores the lists owned by this rank    */
  int32_t shard_count;                  /* 1 = unsharded                                      */
  int32_t shard_policy;                 /* list -> rank map: RBQ_SHARD_ROUND_ROBIN (l % count) */
                                        /* or RBQ_SHARD_BALANCED (fixed at the first add)     */
  int32_t kmeans_kind;                  /* RBQ_KMEANS_BALANCED (reference) or RBQ_KMEANS_LLOYD */
  int32_t raw_store;                    /* where the raw fp32 rows of the exact rerank live:  */
                                        /* RBQ_RAW_DEVICE (HBM, default) or RBQ_RAW_HOST      */
                                        /* (pinned host memory the GPU reads over PCIe: an   */
                                        /* index whose N*D*4 raw bytes exceed the GPU's      */
                                        /* memory keeps only codes, factors and ids in HBM;  */
                                        /* the rerank then reads R rows per query over the   */
                                        /* bus).  Loaded and imported indexes use the device. */
  int32_t bits_per_dim;                 /* code bits per dimension, 1..9 (index_params.      */
                                        /* bits_per_dim, ivf_rabitq.cu:388-393).  1: 1-bit   */
                                        /* RaBitQ codes.  b > 1 adds ExRaBitQ's b - 1 extra  */
                                        /* bits per dimension (quantizer_gpu.cu:347-468) and  */
                                        /* two factors per vector: the scan admits by the     */
                                        /* 1-bit estimate's error bound as before and ranks   */
                                        /* the admitted vectors by the extra-bit distance     */
                                        /* (searcher_gpu_quantize_query.cu:405-473).  Default 1. */
} rbq_index_params_t;

/* Raw-row stores (rbq_index_params_t.raw_store).  The reference builds from a host dataset in
 * batches (construct_on_gpu_streaming, gpu_index/ivf_gpu.cu:814-1066) and keeps no raw rows. */
#define RBQ_RAW_DEVICE 0
#define RBQ_RAW_HOST 1

/* Coarse quantiser trainers.  BALANCED: hierarchical balanced k-means, the algorithm of
 * cuvs::cluster::kmeans::fit(balanced_params) that build calls (ivf_rabitq.cu:141-147,
 * src/cluster/detail/kmeans_balanced.cuh:443-1134): ~sqrt(K) mesoclusters, fine clusters
 * per mesocluster in proportion to its size, then a fine-tuning pass; every EM pass moves
 * the centres of clusters below a size threshold towards rows of large clusters.  Made
 * deterministic (fixed rebalancing order, double-accumulated means).  LLOYD: plain Lloyd
 * iterations from evenly strided initial rows. */
#define RBQ_KMEANS_BALANCED 0
#define RBQ_KMEANS_LLOYD 1

/* List ownership across shards.  ROUND_ROBIN: list l on rank l % shard_count (the layout
 * BASELINE's sharded configuration names).  BALANCED: the lists, taken by decreasing size^2
 * (ties: smaller list id first), each go to the rank with the smallest sum of size^2 so far
 * (ties: smaller rank), sizes counted over the first rbq_add batch, which every rank passes
 * whole; a list's expected scan work grows with its size times how often it is probed, and
 * both grow with its size. */
#define RBQ_SHARD_ROUND_ROBIN 0
#define RBQ_SHARD_BALANCED 1

/* Search-time parameters.  Replaces cuvs::neighbors::ivf_rabitq::search_params
 * (ivf_rabitq.hpp:178-228) in QUANT4 mode. */
typedef struct {
  int32_t n_probes;      /* P (n_probes)                                                      */
  int32_t k;             /* neighbours returned per query                                      */
  int32_t rerank;        /* R: exact fp32 rerank depth; 0 = return the estimator's top-k       */
  int32_t prune;         /* 1 = RaBitQ error-bound prune (reference behaviour), 0 = off        */
  int32_t probe_split;   /* probe slices per query (0 = auto from nq and P)                    */
  int32_t cand_cap;      /* candidate buffer entries per slice (0 = default 1024)              */
  int32_t coarse_margin; /* extra lists kept by the approximate coarse pass (0 = default)      */
  int32_t seeded;        /* every slice starts from the nearest probed list's bound seed      */
                         /* (rbq_bound_seed); -1 = auto (on when the probes are split into      */
                         /* slices), 0 = off (each slice seeds itself), 1 = on                  */
  int32_t query_bits;    /* search mode (search_mode, ivf_rabitq.hpp:111-120; ivf_rabitq.cu:      */
                         /* 294-345): 4 = QUANT4 (default; 0 means 4), 8 = QUANT8 (popcount     */
                         /* estimator over 4- / 8-bit query codes), 16 = LUT16, 32 = LUT32      */
                         /* (the estimate from fp16 / fp32 tables of the float query, one entry */
                         /* per 4-dim code nibble; it is the candidate's distance, so there is  */
                         /* no exact pass, no error-bound prune and no bound seed)             */
  int32_t graph;         /* 1: the first search of a batch size (and these parameters) is       */
                         /* captured as a CUDA graph and later ones replay it: copy in, one     */
                         /* graph launch, copy out (small batches are launch-bound).  Up to 8   */
                         /* graphs per index; adding, training or setting centroids drops them. */
                         /* A graph reads and writes buffers of its own: replays of one graph   */
                         /* issued on different streams are serialised (each replay's copy-in   */
                         /* waits for the previous replay's copy-out).  Like every call on one  */
                         /* index, they must come from one host thread at a time.               */
                         /* 0 (default): launch the kernels one by one.                         */
  int32_t scan_kind;     /* the list scan's schedule.  1: the tile scan (each query walks its   */
                         /* probed lists in tiles of rbq_scan_tile() vectors, the threshold     */
                         /* tightening between tiles).  2: the list scan: the nearest probe is  */
                         /* tile-scanned from its bound seed; every query's threshold for its   */
                         /* other probes is then fixed at min(seed, the nearest list's R-th     */
                         /* distance), and each of those lists is scored against all         */
                         /* the batch's queries that probe it in one int8 GEMM on the tensor    */
                         /* cores (4- or 8-bit query codes x code bits, exactly the popcount    */
                         /* estimator's integers, as the reference scans one (list, query) pair */
                         /* per block, searcher_gpu_quantize_query.cu:172-300); the admitted    */
                         /* vectors' exact distances then rank per query.  Needs QUANT4 /       */
                         /* QUANT8, the prune on and a padded dim <= 768.  0 (default, auto):   */
                         /* the list scan when nq * n_probes >= 64 * n_lists (the lists are     */
                         /* shared by many queries) and the index holds >= R vectors per list   */
                         /* on average (R = max(rerank, k)), else the tile scan.                */
} rbq_search_params_t;

typedef struct {
  int32_t dim, padded_dim, n_lists, shard_rank, shard_count, trained;
  int64_t n_total; /* vectors added (global id space)   */
  int64_t n_local; /* vectors stored by this shard      */
  float query_scale;
  uint64_t seed;
  int64_t device_bytes; /* index memory held on the device */
  int32_t shard_policy; /* RBQ_SHARD_*                      */
  int32_t owners_fixed; /* 1 once the list -> rank map is final (ROUND_ROBIN: always) */
  int32_t kmeans_kind;  /* RBQ_KMEANS_*                     */
  int32_t bits_per_dim; /* 1 + extra bits per dimension     */
  float ex_scale;       /* data scale of the extra-bit codes (0 at 1 bit) */
} rbq_index_info_t;

/* ---- errors / defaults ------------------------------------------------------------------ */
const char* rbq_last_error(void);
int rbq_version(void);
/* Kernels this library has launched in this process (all devices).  No reference
 * counterpart: lets a benchmark count the library's launches inside a timed region. */
uint64_t rbq_kernel_launches(void);
/* Vectors per scan tile: the prune threshold tightens between tiles, and every candidate buffer
 * holds at least R + tile keys (cap = max(pow2(cand_cap or 1024), pow2(R + tile))).  Callers that
 * plan scans themselves (a sharded search) read it here.  No reference counterpart. */
int rbq_scan_tile(void);
void rbq_index_params_default(rbq_index_params_t* p);
void rbq_search_params_default(rbq_search_params_t* p);

/* ---- host-only index constants (no GPU needed) ------------------------------------------ */
/* Seeded orthogonal rotation P [Dp, Dp] row-major (X_rot = X * P).  Replaces
 * RotatorGPU::init_matmul (gpu_index/rotator_gpu.cu:52-59). */
int rbq_make_rotation(int32_t padded_dim, uint64_t seed, float* P_host);
/* Query scaling constant t4 for 4-bit queries (ex_bits = 3).  Replaces
 * DataQuantizerGPU::get_const_scaling_factors (gpu_index/quantizer_gpu.cu:947-980). */
int rbq_query_scale(int32_t padded_dim, uint64_t seed, int32_t ex_bits, float* t_out);

/* ---- index lifecycle -------------------------------------------------------------------- */
/* Create an empty index: generates the seeded rotation and the query scale t4.
 * Replaces index(handle, n_rows, dim, n_lists, bits_per_dim) (ivf_rabitq.hpp:265-272) and the
 * IVFGPU / RotatorGPU constructors (gpu_index/ivf_gpu.cu:37-53, rotator_gpu.cu:52-59). */
int rbq_index_create(const rbq_index_params_t* params, rbq_index_t** out);
int rbq_index_free(rbq_index_t* index);
int rbq_index_info(rbq_index_t* index, rbq_index_info_t* out);

/* Train the coarse quantiser (k-means of kind params.kmeans_kind on an evenly strided sample
 * of at most max_train_points_per_cluster * K rows) on device rows.
 * Replaces the k-means part of build (src/neighbors/ivf_rabitq.cu:117-152).  Synchronises. */
int rbq_train(rbq_index_t* index, const float* X_dev, int64_t n, void* stream);

/* One-call build, ivf_rabitq::build (ivf_rabitq.cu:32-194): with C_host (caller-given centroids
 * [K, D], host memory) the centroids are installed, else k-means trains on X_dev; then the n
 * rows are added (labels_dev: caller-given lists, only together with C_host).  d must equal the
 * index's dim.  Synchronises. */
int rbq_build(rbq_index_t* index, const float* X_dev, int64_t n, int32_t d, const float* C_host,
              const uint32_t* labels_dev, void* stream);

/* Install caller-given centroids [K, D] (host memory) instead of training.  Synchronises. */
int rbq_set_centroids(rbq_index_t* index, const float* C_host, int32_t n_lists);

/* Add rows [n, D] (device) with global ids n_total .. n_total+n-1: assign lists (or take
 * labels_dev), rotate, 1-bit quantise, compute factors, lay out per list.  Replaces
 * build's construct_on_gpu (gpu_index/ivf_gpu.cu:623-812) + serialise/deserialise reorg
 * (rabitq_search.cu:152-158).  Synchronises. */
int rbq_add(rbq_index_t* index, const float* X_dev, int64_t n, const uint32_t* labels_dev, void* stream);

/* Search: queries [nq, D] (device) -> dist [nq, k] f32, ids [nq, k] i64 (device).
 * Replaces ivf_rabitq::search (ivf_rabitq.hpp:361-366; src/neighbors/ivf_rabitq.cu:197-354)
 * and the id cast (:349-353).  Asynchronous on `stream`. */
int rbq_search(rbq_index_t* index, const rbq_search_params_t* params, const float* Q_dev, int64_t nq,
               float* dist_dev, int64_t* ids_dev, void* stream);

/* Same as rbq_search with host buffers: copies queries in and results out on `stream`
 * (pinned buffers are fastest) and synchronises before returning.  Replaces the CLI's
 * H2D -> search -> D2H batch loop (rabitq_search.cu:188-204). */
int rbq_search_host(rbq_index_t* index, const rbq_search_params_t* params, const float* Q_host, int64_t nq,
                    float* dist_host, int64_t* ids_host, void* stream);

/* Persist / restore.  Replaces serialize / deserialize (ivf_rabitq.hpp:395-423;
 * gpu_index/ivf_gpu.cu:100-289, 367-461).  This library's own format ("RBQB200"). */
int rbq_save(rbq_index_t* index, const char* path);
int rbq_load(const char* path, int32_t device, int32_t shard_rank, int32_t shard_count, rbq_index_t** out);

/* The reference's index file (IVFGPU::save / load_transposed, gpu_index/ivf_gpu.cu:367-461,
 * 100-289, as written by ivf_rabitq::serialize, ivf_rabitq.cu:357-368): import a
 * matmul-rotator file with 0..8 extra bits (its rotation, query constants, rotated centroids,
 * codes, long codes, factors and ids are used as stored; lists are split over shards by
 * shard_policy), optionally with the raw
 * vectors X_host [n_x = num_vectors, D] (row = id) for the exact rerank — without them the
 * index searches with rerank = 0 only.  Export writes an unsharded index in that format. */
int rbq_import_reference(const char* path, int32_t device, const float* X_host, int64_t n_x, int32_t shard_rank,
                         int32_t shard_count, int32_t shard_policy, rbq_index_t** out);
int rbq_export_reference(rbq_index_t* index, const char* path);

/* ---- introspection (parity tests) ------------------------------------------------------- */
/* Host copies.  rotation: [Dp*Dp]; centroids: [K*D]; rotated centroids: [K*Dp]. */
int rbq_get_rotation(rbq_index_t* index, float* P_host);
int rbq_get_centroids(rbq_index_t* index, float* C_host, float* C_rot_host);
/* Host copies of the list layout: list_off [K+1], ids [n_local], codes [n_local*W],
 * f_add / f_rescale / f_err [n_local].  Any output may be NULL. */
int rbq_export_lists(rbq_index_t* index, int64_t* list_off, uint32_t* ids, uint32_t* codes, float* fadd,
                     float* frescale, float* ferr);
/* The extra bits of an index with bits_per_dim > 1, in the same slot order: ex_codes
 * [n_local, ex, W] (plane p word w, dim 32w+j -> bit 31-j = bit p of the dim's extra-bit code,
 * ex = bits_per_dim - 1), f_ex_add / f_ex_rescale [n_local].  Any output may be NULL. */
int rbq_export_ex_lists(rbq_index_t* index, uint32_t* ex_codes, float* fexadd, float* fexr);
/* owners [K]: the rank holding each list (-1 while a BALANCED map awaits the first add). */
int rbq_get_list_owners(rbq_index_t* index, int32_t* owners);

/* ---- stage entry points (device pointers; parity tests and the sharded driver) ----------- */
/* Y [n, Dp] = pad(X [n, D]) * P.  Replaces RotatorGPU::rotate (rotator_gpu.cu:162-176). */
int rbq_rotate(rbq_index_t* index, const float* X_dev, int64_t n, float* Y_dev, void* stream);
/* B-bit query quantisation, B = query_bits (4 = QUANT4 with t4, 8 = QUANT8 with t8; 0 means
 * 4): planes [nq, B, W], delta [nq], k1 [nq] (= -0.5 sum q).  Replaces exrabitq_quantize_query
 * (searcher_gpu_quantize_query.cu:655-793) and computeQueryFactorsWarpKernel
 * (gpu_index/ivf_gpu.cu:1451-1490).  The scan entry points below take the same query_bits
 * as the planes they are given.  query_bits 16 / 32 (LUT16 / LUT32) prepare 4-bit planes: those
 * modes read only k1, and their scan builds its tables from the rotated query itself. */
int rbq_query_prep(rbq_index_t* index, const float* Qr_dev, int64_t nq, uint32_t* planes_dev,
                   float* delta_dev, float* k1_dev, int32_t query_bits, void* stream);
/* Approximate coarse scores S [nq, K] = |c_rot|^2 - 2 <q_rot, c_rot> (the shortlist ranking).
 * tensor_cores = 1: tcgen05 kind::tf32 MMA (the search path); 0: fp32 CUDA-core reference.
 * Replaces the -2 Q C^T GEMM + add_norms of PrepareClusterSearchInputs
 * (gpu_index/ivf_gpu.cu:1531-1596). */
int rbq_coarse_scores(rbq_index_t* index, const float* Qr_dev, int64_t nq, float* S_dev, int32_t tensor_cores,
                      void* stream);
/* Synchronises the index's device and reports device-side failures recorded since the last
 * call (a tensor-core pipeline wait that timed out): RBQ_ERR_CUDA with a message, else RBQ_OK.
 * No reference counterpart (the reference has no bounded device waits). */
int rbq_check_errors(rbq_index_t* index);
/* Coarse quantiser: top-nprobe lists per rotated query, ascending exact distance g.
 * Replaces PrepareClusterSearchInputs steps 1-4 (gpu_index/ivf_gpu.cu:1513-1628). */
int rbq_coarse(rbq_index_t* index, const float* Qr_dev, int64_t nq, int32_t nprobe, int32_t margin,
               int32_t* probes_dev, float* g_dev, void* stream);
/* List scan: top-R candidates (estimated distance, id) per query over its probed lists.
 * Replaces SearchClusterQueryPairsQuantizeQuery (searcher_gpu_quantize_query.cu:1006-1596).
 * Optional seeds of a two-phase search (the query's nearest list scanned first):
 *   tau0_dev (f32[nq]): the threshold every slice of query q starts from (default +inf), e.g.
 *     the smallest R-th distance any shard found in its first phase;
 *   init_ids_dev / init_dist_dev ([nq, R], id -1 = none): candidates of that earlier scan,
 *     merged into the result (slice 0 starts from them, and from their R-th distance when
 *     all R are present).
 * Query q's probes are probes_dev[q * probe_stride + p], p < nprobe (g alike; probe_stride
 * 0 = nprobe), so the two phases can read columns 0 and 1.. of one [nq, P] array.
 * stats_dev (optional, u64[2]) accumulates vectors scanned / admitted by the prune.
 * query_bits 16 / 32 (LUT16 / LUT32, computeInnerProductsWithLUT16Opt,
 * searcher_gpu_shared_mem_opt.cu:36-200): the candidates are the top R by the table estimate
 * (prune has no effect; "admitted" counts the estimates kept below the running threshold). */
int rbq_scan(rbq_index_t* index, const float* Qr_dev, const uint32_t* planes_dev, const float* delta_dev,
             const float* k1_dev, int64_t nq, const int32_t* probes_dev, const float* g_dev, int32_t nprobe,
             int32_t probe_stride, const float* tau0_dev, const int64_t* init_ids_dev, const float* init_dist_dev, int32_t R,
             int32_t prune, int32_t slices, int32_t cand_cap, int64_t* cand_ids_dev, float* cand_dist_dev,
             uint64_t* stats_dev, int32_t query_bits, void* stream);
/* The list scan with fixed thresholds (rbq_search_params_t.scan_kind = 2) as a stage: every query
 * admits a vector of its probed lists (this shard's) while the vector's lower bound is below
 * tau0_dev[q] (no tightening), keeps the admitted vectors whose distance is <= tau0_dev[q], and
 * returns its R smallest (distance, id) candidates, ascending (id -1 / +inf past the last).
 * Each probed list is scored against all the queries that probe it by an int8 GEMM on the
 * tensor cores (tcgen05 kind::i8: query codes x code bits = the popcount estimator's integers);
 * the prune is always on.  query_bits 4 or 8 (the planes' width); padded dim <= 768.  stats_dev
 * (optional): += (vectors scanned, vectors admitted).  Replaces the reference's pair-per-block
 * scan (computeInnerProductsWithBitwiseBlockSort, searcher_gpu_quantize_query.cu:172-626). */
int rbq_scan_lists(rbq_index_t* index, const float* Qr_dev, const uint32_t* planes_dev, const float* delta_dev,
                   const float* k1_dev, int64_t nq, const int32_t* probes_dev, const float* g_dev, int32_t nprobe,
                   int32_t probe_stride, const float* tau0_dev, int32_t R, int64_t* cand_ids_dev, float* cand_dist_dev,
                   uint64_t* stats_dev, int32_t query_bits, void* stream);
/* Bound seed per query: the R-th smallest RaBitQ upper bound est + f_err * sqrt(g) over the
 * query's leading owned probed lists that hold >= R vectors (+inf if they hold fewer), the
 * threshold a pruning scan starts from.  With nprobe = 1 it is the nearest list's seed that
 * a sharded search all-reduces (min) and hands to rbq_scan as tau0.  tau_dev: f32[nq].
 * No reference counterpart (the reference seeds with 1.45 x a centroid distance,
 * searcher_gpu_common.cuh:178-193). */
int rbq_bound_seed(rbq_index_t* index, const float* Qr_dev, const uint32_t* planes_dev, const float* delta_dev,
                   const float* k1_dev, int64_t nq, const int32_t* probes_dev, const float* g_dev, int32_t nprobe,
                   int32_t probe_stride, int32_t R, int32_t cand_cap, float* tau_dev, int32_t query_bits,
                   void* stream);
/* rbq_bound_seed for the queries whose nearest probe (column 0 of probes_dev) this shard owns;
 * +inf for the others.  A sharded search all-reduces (min) it: each query's seed is then its
 * nearest list's owner's, over that shard's leading owned lists, at 1/N of the work per shard. */
int rbq_bound_seed_owned(rbq_index_t* index, const float* Qr_dev, const uint32_t* planes_dev, const float* delta_dev,
                         const float* k1_dev, int64_t nq, const int32_t* probes_dev, const float* g_dev, int32_t nprobe,
                         int32_t probe_stride, int32_t R, int32_t cand_cap, float* tau_dev, int32_t query_bits,
                         void* stream);
/* rbq_scan without any device allocation, for callers that cannot allocate GPU memory at
 * search time: a host program whose device memory is handed out up front by its own pool
 * (so a library cudaMalloc would fail or break its budget), or a latency-critical search
 * thread that must not pay for an allocation (cudaMalloc can synchronise the whole device).
 * The scan's only scratch, the per-slice candidate keys, lives in a fixed array of
 * RBQ_NOALLOC_SCRATCH_BYTES compiled into librbq.so; every GPU that loads the library holds
 * that much memory until the process exits.  Inputs, outputs and their meaning are exactly
 * those of rbq_scan without its initial candidates (tau0_dev is accepted).  Limits and rules:
 *   - needs nq*slices*R*8 bytes, plus nq*R*8 when slices > 1 (each part rounded up to 256);
 *     anything larger is rejected with RBQ_ERR_INVALID before any work is queued;
 *   - the first call on a device looks up the array's device address (cudaGetSymbolAddress)
 *     with that device current; make that first call before any stream capture.  The address
 *     is kept with the id of the context it belongs to and looked up again (by the next call,
 *     which then counts as a first call) when the device's context has been re-created, as
 *     after cudaDeviceReset;
 *   - all calls share the one array and it keeps the last call's contents (nothing in it has
 *     to start at zero: every key read is written earlier in the same call); calls that can
 *     overlap on the GPU (other streams, other host threads, same device) race on it and must
 *     be serialised by the caller.
 * It calls no cudaMalloc / cudaFree / cudaMallocAsync.  No counterpart in the reference. */
#define RBQ_NOALLOC_SCRATCH_BYTES (32u << 20)
int rbq_scan_noalloc(rbq_index_t* index, const float* Qr_dev, const uint32_t* planes_dev, const float* delta_dev,
                     const float* k1_dev, int64_t nq, const int32_t* probes_dev, const float* g_dev, int32_t nprobe,
                     int32_t probe_stride, const float* tau0_dev, int32_t R, int32_t prune, int32_t slices, int32_t cand_cap,
                     int64_t* cand_ids_dev, float* cand_dist_dev, uint64_t* stats_dev, int32_t query_bits,
                     void* stream);
/* Phase-1 estimator of one query against every vector of list `list`: integer popcount
 * inner product acc, estimate est and lower bound low (slot order of the list).  Replaces the
 * phase-1 loop of computeInnerProductsWithBitwiseBlockSort (searcher_gpu_quantize_query.cu:
 * 233-281) for inspection; planes_dev is one query's [query_bits, W] planes. */
int rbq_list_estimates(rbq_index_t* index, const uint32_t* planes_dev, float delta, float k1, float g,
                       int32_t list, int32_t* acc_dev, float* est_dev, float* low_dev, int32_t query_bits,
                       void* stream);
/* Exact fp32 rerank of candidates [nq, R] (id -1 = empty) in the original space -> top-k.
 * Semantics of cuvs::neighbors::refine (src/neighbors/refine/refine_device.cuh:31-150). */
int rbq_rerank(rbq_index_t* index, const float* Q_dev, int64_t nq, const int64_t* cand_ids_dev, int32_t R,
               int32_t k, float* dist_dev, int64_t* ids_dev, void* stream);
/* k-way merge of per-shard results [parts, nq, k] -> [nq, k] by (dist, id).  The on-device
 * merge after the NCCL all-gather of a list-sharded search. */
int rbq_merge_results(const float* dist_dev, const int64_t* ids_dev, int32_t parts, int64_t nq, int32_t k,
                      float* out_dist_dev, int64_t* out_ids_dev, void* stream);
/* Results (dist f32, id i64; id < 0 = empty) -> 8-byte keys: (order-preserving bits of dist) << 32 |
 * id, all ones when empty.  A sharded search all-gathers these instead of the 12-byte pairs and
 * merges them with rbq_merge_result_keys ([parts, nq, k] keys, same output as rbq_merge_results).
 * No reference counterpart (the reference has no multi-GPU search, rabitq_search.cu:11). */
int rbq_pack_results(const float* dist_dev, const int64_t* ids_dev, int64_t n, uint64_t* keys_dev, void* stream);
int rbq_merge_result_keys(const uint64_t* keys_dev, int32_t parts, int64_t nq, int32_t k, float* out_dist_dev,
                          int64_t* out_ids_dev, void* stream);

/* ---- fault injection (tests) --------------------------------------------------------------- */
/* Host-side: the (after+1)-th device allocation the library makes from now on fails with
 * RBQ_ERR_OOM exactly as a failed cudaMalloc would (one shot; after < 0 turns it off).  Used to
 * test out-of-memory handling without exhausting a shared GPU; the GPU is not touched. */
int rbq_debug_fail_alloc(int64_t after);

/* ---- synthetic data (benchmarks and tests) ---------------------------------------------- */
/* X [n, D]: row i = centre[h(i) % n_centres] + sigma * N(0,1) per dim, centres ~ N(0,1)
 * (per-dim scale sqrt(1/(1+d/64)) when aniso), L2-normalised when normalize. */
int rbq_gen_mixture(float* X_dev, int64_t n, int32_t D, int32_t n_centres, float sigma, int32_t aniso,
                    int32_t normalize, uint64_t seed, void* stream);
/* Q [nq, D]: row = X[src] + sigma * N(0,1), renormalised when normalize; src_rows_dev
 * (optional) receives the source rows. */
int rbq_gen_queries(const float* X_dev, int64_t n, int32_t D, float* Q_dev, int64_t nq, float sigma,
                    int32_t normalize, uint64_t seed, int64_t* src_rows_dev, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RBQ_H_ */
