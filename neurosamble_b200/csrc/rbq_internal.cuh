// Internal declarations of the B200 IVF-RaBitQ library (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/rbq.h"

namespace rbq {

// ---------------------------------------------------------------------------------------
// Error plumbing: every C-ABI entry point returns an int status and never throws or exits.
// ---------------------------------------------------------------------------------------
void set_error(const std::string& msg);
struct Error {
  int code;
  std::string msg;
};

#define RBQ_CUDA(call)                                                                     \
  do {                                                                                     \
    cudaError_t e_ = (call);                                                               \
    if (e_ != cudaSuccess)                                                                 \
      throw ::rbq::Error{RBQ_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)}; \
  } while (0)

#define RBQ_CHECK(cond, code, msg)                        \
  do {                                                    \
    if (!(cond)) throw ::rbq::Error{(code), (msg)};       \
  } while (0)

// Process-wide count of kernels launched by this library (rbq_kernel_launches()).
void count_launch();
// Follows every kernel launch: counts it and surfaces launch-configuration errors.
#define RBQ_LAUNCHED()                  \
  do {                                  \
    ::rbq::count_launch();              \
    RBQ_CUDA(cudaGetLastError());       \
  } while (0)

// ---------------------------------------------------------------------------------------
// Keys: (order-preserving float bits << 32) | id.  Ascending keys = ascending distance,
// ties broken by the smaller id.  All-ones = empty slot.
// ---------------------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint32_t ordered_bits(float f)
{
  uint32_t u;
#ifdef __CUDA_ARCH__
  u = __float_as_uint(f);
#else
  __builtin_memcpy(&u, &f, 4);
#endif
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__host__ __device__ __forceinline__ float from_ordered_bits(uint32_t o)
{
  uint32_t u = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
  float f;
#ifdef __CUDA_ARCH__
  f = __uint_as_float(u);
#else
  __builtin_memcpy(&f, &u, 4);
#endif
  return f;
}
__host__ __device__ __forceinline__ unsigned long long make_key(float d, uint32_t id)
{
  return ((unsigned long long)ordered_bits(d) << 32) | id;
}
constexpr unsigned long long kEmptyKey = ~0ull;

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int next_pow2(int v)
{
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

// ---------------------------------------------------------------------------------------
// Device-resident index.  All per-vector arrays are in list-slot order: list l owns slots
// [list_off[l], list_off[l+1]), members in ascending global id.
// ---------------------------------------------------------------------------------------
struct Index {
  int device = 0;
  int D = 0, Dp = 0, W = 0, K = 0;
  uint64_t seed = 0;
  int kmeans_iters = 20;
  int kmeans_kind = RBQ_KMEANS_BALANCED;
  int max_train_per_list = 256;
  int shard_rank = 0, shard_count = 1;
  int shard_policy = RBQ_SHARD_ROUND_ROBIN;
  bool has_raw = true;              // X_r holds the raw rows (false for an index imported without them)
  bool raw_on_host = false;         // X_r is pinned, mapped host memory (RBQ_RAW_HOST), else HBM
  int64_t min_list = 0;             // vectors in this shard's smallest list (set by relayout)
  float t8 = 0.0f / 0.0f;           // 8-bit query constant of an imported reference file (NaN: derive)
  bool owners_fixed = false;
  std::vector<int32_t> owner_host;  // [K] rank holding list l
  float t4 = 0.0f;
  bool trained = false;
  // ExRaBitQ (bits_per_dim = ex_bits + 1): ex_bits extra bits per dimension beyond the 1-bit
  // code, quantised with data scale tex (0 extra bits: 1-bit codes only).
  int ex_bits = 0;
  float tex = 0.0f;

  std::vector<float> P_host;       // [Dp*Dp] rotation (row-major)
  std::vector<float> C_host;       // [K*D] centroids, original space
  std::vector<int64_t> off_host;   // [K+1]
  int64_t n_total = 0;             // vectors added across all shards (global id space)
  int64_t n_rows = 0;              // vectors stored on this shard

  float* P = nullptr;          // [Dp*Dp]
  float* C = nullptr;          // [K*D]
  float* C_rot = nullptr;      // [K*Dp]
  float* C_rot_n2 = nullptr;   // [K] |c_rot|^2 (float, for the approximate coarse pass)
  float* C_rot_n2_max = nullptr;  // device scalar: max of C_rot_n2 (error bound of the coarse shortlist)
  float* C_n2 = nullptr;       // [K] |c|^2 (original space, for assignment)

  // Row order: append-only storage of this shard's vectors, in the order they were added.
  int64_t cap_rows = 0;
  float* X_r = nullptr;          // [n_rows*D] raw vectors (rerank store)
  uint32_t* codes_r = nullptr;   // [n_rows*W]
  float* fadd_r = nullptr;       // [n_rows]
  float* frescale_r = nullptr;   // [n_rows]
  float* ferr_r = nullptr;       // [n_rows]
  uint32_t* ex_codes_r = nullptr;  // [n_rows*ex_bits*W] extra-bit planes (ex_bits > 0)
  float* fexadd_r = nullptr;       // [n_rows]
  float* fexr_r = nullptr;         // [n_rows]
  uint32_t* labels_r = nullptr;  // [n_rows]
  uint32_t* ids_r = nullptr;     // [n_rows] global ids
  int64_t cap_ids = 0;
  uint32_t* id2row = nullptr;    // [n_total] row of a global id, 0xFFFFFFFF if not on this shard
  int* dev_err = nullptr;        // [1] device-side error code (tensor-core waits that timed out)
  int32_t* owner = nullptr;      // [K] device copy of owner_host
  cudaStream_t copy_stream = nullptr;  // host-buffer searches: uploads / downloads beside compute

  // Searches captured as CUDA graphs (rbq_search_params_t.graph): one per batch size and search
  // parameters, reading and writing their own device buffers; dropped whenever the index's
  // arrays change (add, train, set_centroids, free).
  struct SearchGraph {
    int64_t nq = 0;
    rbq_search_params_t p{};
    cudaGraphExec_t exec = nullptr;
    float* q = nullptr;
    float* d = nullptr;
    int64_t* i = nullptr;
    // Recorded after a replay's results are copied out; the next replay's copy into q waits on
    // it, so replays issued on different streams cannot overwrite each other's buffers.
    cudaEvent_t done = nullptr;
  };
  std::vector<SearchGraph> graphs;

  // Slot order (rebuilt after every add): list l owns slots [list_off[l], list_off[l+1]).
  int64_t* list_off = nullptr;   // [K+1]
  uint32_t* ids = nullptr;       // [n_rows] global ids
  uint32_t* codes = nullptr;     // [n_rows*W] vector-major 1-bit codes
  float* fadd = nullptr;         // [n_rows]
  float* frescale = nullptr;     // [n_rows]
  float* ferr = nullptr;         // [n_rows]
  // Extra bits (ex_bits > 0): one vector = ex_bits planes of W words (plane p word w, dim 32w+j
  // -> bit 31-j = bit p of the dim's extra-bit code), then the two extra-bit factors.
  uint32_t* ex_codes = nullptr;  // [n_rows*ex_bits*W]
  float* fexadd = nullptr;       // [n_rows]
  float* fexr = nullptr;         // [n_rows]
};

void free_index_memory(Index& ix);
// Destroys the index's captured search graphs (their pointers into the index go stale).
void drop_graphs(Index& ix);
// The list -> rank map of a policy for list sizes `sizes` (ROUND_ROBIN ignores them).
std::vector<int32_t> list_owners(int policy, const std::vector<int64_t>& sizes, int count);
// Uploads the map (allocating the device copy on first use); fixed = final for later adds.
void install_owners(Index& ix, const std::vector<int32_t>& owners, bool fixed);

// ---------------------------------------------------------------------------------------
// Host math (rbq_host_math.cpp): rotation and query scaling constant.
// ---------------------------------------------------------------------------------------
void make_rotation(int Dp, uint64_t seed, float* P_out);
float query_scale(int Dp, uint64_t seed, int ex_bits);

// ---------------------------------------------------------------------------------------
// Kernel launchers.
// ---------------------------------------------------------------------------------------
// Y[n, Dp] = pad(X[n, D]) * P  (double accumulation in k order).
void launch_rotate(const float* X, int64_t n, int D, int Dp, const float* P, float* Y, cudaStream_t s);
// 1-bit codes + factors of rotated rows Y against rotated centroids of their labels.
void launch_quantize(const float* Y, int64_t n, int Dp, const float* C_rot, const uint32_t* labels,
                     uint32_t* codes, float* fadd, float* frescale, float* ferr, cudaStream_t s);
// ExRaBitQ extra-bit planes [n, ex, W] and factors f_ex_add / f_ex_rescale of rotated rows Y
// (data scale t), against the rotated centroids of their labels.
void launch_quantize_ex(const float* Y, int64_t n, int Dp, const float* C_rot, const uint32_t* labels, int ex,
                        float t, uint32_t* planes, float* fexadd, float* fexr, cudaStream_t s);
// Row squared norms (float, any order) of A[n, d].
void launch_row_norms(const float* A, int64_t n, int d, float* out, cudaStream_t s);
// Approximate scores S[q, c] = |c|^2 - 2 <a_q, c> for ranking (fp32).
// Same scores on the tensor cores (tcgen05 kind::tf32); err[0] is set if a wait timed out.
bool coarse_tc_supported(int dp);
// Fused tensor-core scores + m-best shortlist for large K: cand [nq, m] (any order) and bounds
// [nq] as launch_topm_rows gives them, without writing the [nq, K] scores.  rowbuf: scratch of
// ceil(nq / 128) * 128 * coarse_topm_row_cap(m) keys.
int coarse_topm_row_cap(int m);
int coarse_topm_max_shortlist();  // the largest m the fused kernel takes
void launch_coarse_topm_tc(const float* A, int64_t nq, const float* C, const float* cn2, int K, int dp, int m, int p,
                           unsigned long long* rowbuf, int32_t* cand, float2* bounds, int* err, cudaStream_t s);
void launch_coarse_scores_tc(const float* A, int64_t nq, const float* C, const float* cn2, int K, int dp, float* S,
                             int* err, cudaStream_t s);
void launch_coarse_scores(const float* A, int64_t nq, const float* C, const float* c_n2, int K, int d,
                          float* S, cudaStream_t s);
// Per row of S [nq, K]: the m smallest (score, id) keys -> cand [nq, m] (any order).  With
// bounds, also the row's m-th smallest score in bounds[q].y (+inf when all K are kept).
void launch_topm_rows(const float* S, int64_t nq, int K, int m, int32_t* cand, cudaStream_t s, int p = 0,
                      float2* bounds = nullptr);
// Exact refine: g = sum_j double(a_j - c_j)^2 for the m candidates, then top-p by (g, id).  With
// bounds (from launch_topm_rows), cmax2 (max |c|^2, device scalar) and unsafe ([1 + nq] ints,
// unsafe[0] = 0 on entry), queries whose shortlist may miss a true top-p list are appended to
// unsafe: a list outside the shortlist has exact distance >= |q|^2 + (m-th tf32 score) - E (E the
// tf32 score error bound), which must exceed the p-th exact distance found.
void launch_refine_topp(const float* A, int64_t nq, const float* C, int d, const int32_t* cand, int m,
                        int p, int32_t* probes, float* g, cudaStream_t s, const float2* bounds = nullptr,
                        const float* cmax2 = nullptr, int* unsafe = nullptr);
// Exact top-p over all K lists for the queries queued in unsafe; overwrites their probes / g.
void launch_refine_all(const float* A, int64_t nq, const float* C, int d, int K, int p, const int* unsafe,
                       int32_t* probes, float* g, cudaStream_t s);
// *out = max of v[0..n).
void launch_max_reduce(const float* v, int n, float* out, cudaStream_t s);
// B-bit query planes (B = qbits: 4 for QUANT4, 8 for QUANT8; planes [nq, B, W]), delta and k1;
// t is the index's scale constant for that width (t4 or t8).
void launch_query_prep(const float* Qr, int64_t nq, int Dp, float t, int qbits, uint32_t* planes, float* delta,
                       float* k1, cudaStream_t s);

struct ScanArgs {
  const int64_t* list_off;
  const uint32_t* ids;
  const uint32_t* codes;
  const float* fadd;
  const float* frescale;
  const float* ferr;
  // ExRaBitQ: an admitted vector's distance is the extra-bit one (ex_bits > 0; null otherwise)
  const uint32_t* ex_codes = nullptr;  // [n_slots, ex_bits, W]
  const float* fexadd = nullptr;
  const float* fexr = nullptr;
  int ex_bits = 0;
  int64_t n_slots;  // vectors on the shard (the scan indexes slots with 32-bit ints)
  int Dp, W;
  const float* Qr;
  const uint32_t* planes;  // [nq, qbits, W]
  int qbits = 4;           // query code width: 4 (QUANT4) or 8 (QUANT8)
  const float* delta;
  const float* k1;
  int64_t nq;
  const int32_t* probes;  // query q's probes: probes[q * pstride + p], p < nprobe (g alike)
  const float* g;
  int nprobe;
  int pstride = 0;  // 0: nprobe
  int R;
  int cap;
  int prune;
  int slices;
  const int32_t* owner;  // [K] rank holding list l; this shard scans lists with owner[l] == shard_rank
  int shard_rank;
  // Optional seeds.  tau0 [nq]: every slice of query q starts from threshold tau0[q] (default
  // +inf).  init_keys [nq, R] (kEmptyKey = none, any order): candidates of an earlier scan of
  // the same query, loaded into slice 0's buffer; when all R are present the slice starts from
  // min(tau0, their largest distance).
  const float* tau0 = nullptr;
  const unsigned long long* init_keys = nullptr;
  // Seed-only launch (slices 1, prune on): write the slice's starting threshold to tau_out[q]
  // (the bound seed, or +inf when its lists hold fewer than R vectors) and scan nothing.
  float* tau_out = nullptr;
  // With tau_out: only queries whose nearest probe (column 0) this shard owns compute the seed;
  // the others get +inf (a sharded search takes the minimum over the shards).
  int seed_nearest_owned = 0;
  // Optional [nq]: slice 0 writes the threshold it starts its scan from (tau0, the bound seed it
  // computed, or +inf) and then scans as usual.
  float* seed_out = nullptr;
  unsigned long long* out_keys;  // [nq, slices, R]
  unsigned long long* stats;     // optional [2]: scanned, admitted
  // Optional [nq] visiting order: block i scans query qorder[i / slices] (a permutation of
  // 0..nq-1).  Only the order in which queries run changes; every query's result is its own.
  const int32_t* qorder = nullptr;
  // Optional (device): scan only the first *unit_count queries of qorder, their units spread by
  // a grid-stride loop over grid_blocks blocks (a list whose length only the device knows).
  const int32_t* unit_count = nullptr;
  int grid_blocks = 0;
  // Fixed-threshold scan (the list scan's semantics): the prune admits a vector while
  // low < tau0[q] (+inf when tau0 is null), however far the kept candidates have tightened the
  // threshold; only the keep test and the buffer cuts use the running threshold.
  int fixed_tau = 0;
  // Optional: only queries whose admitted count over_cnt[q] exceeds over_cap run (the list
  // scan's candidate rows that overflowed); the other blocks return at once.
  const int32_t* over_cnt = nullptr;
  int over_cap = 0;
  // Output rows: query q's slice s goes to out_keys + (q * out_slices + out_slice + s) * R
  // (out_slices 0: slices), so that two scans can fill the halves of one [nq, 2, R] buffer.
  int out_slices = 0;
  int out_slice = 0;
};
// ---------------------------------------------------------------------------------------
// List scan on the tensor cores (fixed per-query threshold).  For every (list, query) pair of
// the batch: acc = <query code, vector bits> as an int8 GEMM on tcgen05 (kind::i8; exactly the
// popcount estimator's integer), est = (f_add + g) + f_rescale * (acc * delta + k1),
// low = est - f_err * sqrt(g); a vector with low < tau0[q] is appended to its query's candidate
// row: cand[q * cap + i] = (float bits of g) << 32 | slot.  cand_cnt[q] counts every admitted
// vector, also past cap (an overflowed row).
// ---------------------------------------------------------------------------------------
struct ListScanArgs {
  const int64_t* list_off;
  const uint32_t* codes;
  const float* fadd;
  const float* frescale;
  const float* ferr;
  int W, Dp;
  const int8_t* qcodes;  // [nq, Dp] query codes
  const float* delta;
  const float* k1;
  const float* tau0;          // [nq] fixed thresholds
  const int32_t* pair_q;      // (list, query) pairs in list order: the query
  const float* pair_g;        //   and its coarse distance to the list
  const int32_t* list_start;  // [K + 1] first pair of list l
  const int32_t* item_start;  // [K + 1] first work item of list l (128 pairs per item)
  int K;
  unsigned long long* cand;  // [nq, cap]
  int32_t* cand_cnt;         // [nq]
  int cap;
  unsigned long long* stats;  // optional [2]: scanned, admitted
  int* err;
};
bool list_scan_tc_supported(int dp);
// SMs of the current device (grid sizes of the persistent and grid-stride kernels).
int device_sm_count();
constexpr int kListScanRows = 128;  // (list, query) pairs per work item
void launch_list_scan_tc(const ListScanArgs& a, int64_t max_items, cudaStream_t s);
// The work plan of a list scan: codes of the queries ([nq, Dp] int8, from planes [nq, QB, W]),
// the (list, query) pairs of this shard's probed lists bucketed by list, and the work items.
// The queries q < nq with cnt[q] > cap into list[0..*n) (n zeroed first), in no fixed order.
void launch_over_list(const int32_t* cnt, int64_t nq, int cap, int32_t* list, int32_t* n, cudaStream_t s);
void launch_planes_to_codes(const uint32_t* planes, int64_t nq, int W, int QB, int8_t* codes, cudaStream_t s);
void launch_list_pairs(const int32_t* probes, const float* g, int64_t nq, int nprobe, int pstride,
                       const int32_t* owner, int rank, int K, int32_t* list_start, int32_t* item_start,
                       int32_t* cursor, int32_t* pair_q, float* pair_g, cudaStream_t s);
// Exact pass of the list scan: per query the candidates of its row (1-bit exact distance, or
// the extra-bit distance), kept while dist <= tau0[q], cut to the R smallest keys -> out_keys
// [nq, R].  Rows that overflowed (cand_cnt > cap) are left to the fixed-threshold tile scan.
struct ExactArgs {
  const uint32_t* codes;
  const float* fadd;
  const float* frescale;
  const uint32_t* ids;
  const uint32_t* ex_codes = nullptr;
  const float* fexadd = nullptr;
  const float* fexr = nullptr;
  int ex_bits = 0;
  int W;
  const float* Qr;  // [nq, Dp]
  const float* k1;
  const float* tau0;
  const unsigned long long* cand;
  const int32_t* cand_cnt;
  int cap;
  int R;
  int64_t nq;
  unsigned long long* out_keys;  // query q's R keys at out_keys + (q * out_slices + out_slice) * R
  int out_slices = 1;
  int out_slice = 0;
};
void launch_exact_topr(const ExactArgs& a, cudaStream_t s);
// tau[q] = min(tau[q], the R-th key's distance of keys[q * stride .. + R)) when that key is present.
// The R smallest keys of `parts` ascending key rows per query ([nq, parts, R]) into row
// out + (q * out_rows + out_row) * R; with over_cnt only the queries with over_cnt[q] > over_cap.
void launch_merge_sorted_keys(const unsigned long long* in, int64_t nq, int parts, int R, unsigned long long* out,
                              int out_rows, int out_row, const int32_t* over_cnt, int over_cap, cudaStream_t s);
void launch_tighten_tau(const unsigned long long* keys, int64_t nq, int stride, int R, float* tau, cudaStream_t s);

// qorder[0..nq) = the queries sorted by their nearest probe probes[q * pstride] (ascending list id;
// queries without probes last), so that queries searching the same region of the index run at
// the same time and share its lists in L2.  counts: scratch of K + 2 ints.  The order inside
// one list's bucket is unspecified.
void launch_query_order(const int32_t* probes, int64_t nq, int pstride, int K, int32_t* counts, int32_t* qorder,
                        cudaStream_t s);
// The scan sorts queries (launch_query_order) for batches of at least this many.
#ifndef RBQ_QUERY_ORDER_MIN_BATCH
#define RBQ_QUERY_ORDER_MIN_BATCH 2048
#endif
constexpr int64_t kQueryOrderMinBatch = RBQ_QUERY_ORDER_MIN_BATCH;
#ifndef RBQ_SCAN_TILE
#define RBQ_SCAN_TILE 1024
#endif
constexpr int kScanTile = RBQ_SCAN_TILE;  // vectors per scan tile (256 threads x tile / 256)
void launch_scan(const ScanArgs& a, cudaStream_t s);
// Phase-1 dump for one query and one list.
void launch_list_estimates(const Index& ix, const uint32_t* planes, int qbits, float delta, float k1, float g,
                           int list, int32_t* acc, float* est, float* low, cudaStream_t s);
// Merge [nq, parts, R] keys -> [nq, R] keys (ascending).
void launch_merge_keys(const unsigned long long* in, int64_t nq, int parts, int R, unsigned long long* out,
                       cudaStream_t s);
// Keys [nq, R] -> dist f32 [nq, k], ids i64 [nq, k] (first k of each row).
void launch_keys_to_result(const unsigned long long* keys, int64_t nq, int R, int k, float* dist,
                           int64_t* ids, cudaStream_t s);
// Exact rerank: candidate keys [nq, R] -> top-k exact L2^2 in the original space.
void launch_rerank(const float* Xslots, const uint32_t* id2slot, int D, const float* Q, int64_t nq,
                   const unsigned long long* cand, int R, int k, float* dist, int64_t* ids, cudaStream_t s);

// k-means helpers.
void launch_centroid_update(const float* X, int64_t n, int D, const uint32_t* labels, const int64_t* off,
                            const uint32_t* order, int K, float* C, bool zero_empty, cudaStream_t s);
// Balanced k-means: C[l] = (wc * C[li] + X[i]) / (wc + 1) for adj = {l, li, i, wc} x n_adj.
void launch_adjust_centers(float* C, int D, const float* X, const int64_t* adj, int n_adj, cudaStream_t s);
void launch_gather_rows_f32(const float* src, int64_t rows, int cols, const int64_t* src_row, float* dst,
                            cudaStream_t s);
// dst[r*cols + j] = src[src_row[r]*cols + j] for 32-bit words.
void launch_gather_rows_u32(const uint32_t* src, int64_t rows, int cols, const int64_t* src_row, uint32_t* dst,
                            cudaStream_t s);
// id2row[ids[r]] = r for r < n.
void launch_scatter_id2row(const uint32_t* ids, int64_t n, uint32_t* id2row, cudaStream_t s);
// keys[i] = ids[i] < 0 ? empty : (0 << 32 | ids[i]).
void launch_ids_to_keys(const int64_t* ids, int64_t n, unsigned long long* keys, cudaStream_t s);
// (id, distance) pairs -> keys (id < 0 -> kEmptyKey).
void launch_cands_to_keys(const int64_t* ids, const float* dist, int64_t n, unsigned long long* keys, cudaStream_t s);
void launch_keys_to_ids(const unsigned long long* keys, int64_t n, int64_t* ids, float* dist, cudaStream_t s);
// k-way merge of [parts, nq, k] results.
// keys (optional): the results already packed as keys [parts, nq, k]; dist and ids unused.
void launch_merge_results(const float* dist, const int64_t* ids, int parts, int64_t nq, int k, float* out_dist,
                          int64_t* out_ids, cudaStream_t s, const unsigned long long* keys = nullptr);

// Synthetic data (benchmarks): Gaussian mixture rows, optionally normalised.
void launch_gen_mixture(float* X, int64_t n, int D, int n_centres, float sigma, int aniso, int normalize,
                        uint64_t seed, uint32_t stream, float* centres_scratch, cudaStream_t s);
void launch_gen_queries(const float* X, int64_t n, int D, float* Q, int64_t nq, float sigma, int normalize,
                        uint64_t seed, uint32_t stream, int64_t* src_rows, cudaStream_t s);

}  // namespace rbq
