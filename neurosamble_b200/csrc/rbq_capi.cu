// C ABI of librbq.so: index lifecycle, k-means training, add (quantise + list layout),
// the search pipeline, persistence, stage entry points and synthetic data.
//
// Every entry point catches everything, stores a message for rbq_last_error() and returns
// a status code; nothing throws across the ABI and nothing exits or traps.
#include <cuda.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <utility>
#include <vector>

#include "rbq_internal.cuh"

struct rbq_index {
  rbq::Index ix;
};

namespace rbq {
namespace {

thread_local std::string g_last_error;

// NVTX range for the scope (entry points and search / training stages; free without a tool).
struct Range {
  explicit Range(const char* name) { nvtxRangePushA(name); }
  ~Range() { nvtxRangePop(); }
};

// Host-side fault injection for tests (rbq_debug_fail_alloc): the device allocation that takes
// the counter from 0 fails as a failed cudaMalloc would; -1 = off.
std::atomic<int64_t> g_fail_alloc_after{-1};

void maybe_inject_alloc_failure(size_t bytes)
{
  int64_t v = g_fail_alloc_after.load();
  while (v >= 0) {
    if (g_fail_alloc_after.compare_exchange_weak(v, v - 1)) {
      if (v == 0)
        throw Error{RBQ_ERR_OOM, "device allocation of " + std::to_string(bytes) +
                                     " bytes failed (injected by rbq_debug_fail_alloc)"};
      return;
    }
  }
}

// Switches to `dev` for the scope and restores the caller's device.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev)
  {
    RBQ_CUDA(cudaGetDevice(&prev));
    if (prev != dev) RBQ_CUDA(cudaSetDevice(dev));
  }
  ~DeviceGuard()
  {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

template <typename F>
int guarded(F&& f)
{
  try {
    f();
    return RBQ_OK;
  } catch (const Error& e) {
    g_last_error = e.msg;
    return e.code;
  } catch (const std::bad_alloc&) {
    g_last_error = "host allocation failed";
    return RBQ_ERR_OOM;
  } catch (...) {
    g_last_error = "unknown error";
    return RBQ_ERR_INVALID;
  }
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

template <typename T>
T* dev_alloc(size_t count)
{
  if (count == 0) count = 1;
  maybe_inject_alloc_failure(count * sizeof(T));
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, count * sizeof(T));
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw Error{RBQ_ERR_OOM, std::string("cudaMalloc of ") + std::to_string(count * sizeof(T)) +
                                 " bytes failed: " + cudaGetErrorString(e)};
  }
  return static_cast<T*>(p);
}

template <typename T>
void dev_free(T*& p)
{
  if (p) cudaFree(p);
  p = nullptr;
}

// Stream-ordered scratch from the device's default memory pool (kept cached between calls).
struct Scratch {
  cudaStream_t s;
  std::vector<void*> bufs;
  explicit Scratch(cudaStream_t st) : s(st) {}
  template <typename T>
  T* get(size_t count)
  {
    if (count == 0) count = 1;
    maybe_inject_alloc_failure(count * sizeof(T));
    void* p = nullptr;
    cudaError_t e = cudaMallocAsync(&p, count * sizeof(T), s);
    if (e != cudaSuccess) {
      cudaGetLastError();
      throw Error{RBQ_ERR_OOM, std::string("cudaMallocAsync of ") + std::to_string(count * sizeof(T)) +
                                   " bytes failed: " + cudaGetErrorString(e)};
    }
    bufs.push_back(p);
    return static_cast<T*>(p);
  }
  ~Scratch()
  {
    for (void* p : bufs) cudaFreeAsync(p, s);
  }
};

void keep_pool_cached(int device)
{
  static bool done[64] = {false};
  if (device < 0 || device >= 64 || done[device]) return;
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
    uint64_t thr = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
  }
  done[device] = true;
}

// Grow a device array to `count` elements, keeping the first `keep` elements.
template <typename T>
void dev_grow(T*& p, size_t keep, size_t count)
{
  T* np = dev_alloc<T>(count);
  if (p && keep) RBQ_CUDA(cudaMemcpy(np, p, keep * sizeof(T), cudaMemcpyDeviceToDevice));
  dev_free(p);
  p = np;
}

void install_centroids(Index& ix, cudaStream_t s)
{
  drop_graphs(ix);
  dev_free(ix.C);
  dev_free(ix.C_rot);
  dev_free(ix.C_rot_n2);
  dev_free(ix.C_rot_n2_max);
  dev_free(ix.C_n2);
  ix.C = dev_alloc<float>((size_t)ix.K * ix.D);
  ix.C_rot = dev_alloc<float>((size_t)ix.K * ix.Dp);
  ix.C_rot_n2 = dev_alloc<float>(ix.K);
  ix.C_rot_n2_max = dev_alloc<float>(1);
  ix.C_n2 = dev_alloc<float>(ix.K);
  RBQ_CUDA(cudaMemcpyAsync(ix.C, ix.C_host.data(), ix.C_host.size() * 4, cudaMemcpyHostToDevice, s));
  launch_rotate(ix.C, ix.K, ix.D, ix.Dp, ix.P, ix.C_rot, s);
  launch_row_norms(ix.C_rot, ix.K, ix.Dp, ix.C_rot_n2, s);
  launch_max_reduce(ix.C_rot_n2, ix.K, ix.C_rot_n2_max, s);
  launch_row_norms(ix.C, ix.K, ix.D, ix.C_n2, s);
  RBQ_CUDA(cudaStreamSynchronize(s));
  ix.trained = true;
}

// Exact nearest centroid (ties -> lower id) of rows A [n, d] among C [K, d]: approximate
// shortlist (tcgen05 tf32 scores when d is a multiple of 32 and the rows are 16-byte aligned,
// else fp32 SIMT), then the double-accumulated distance over the shortlist decides.
}  // namespace

// Exact top-p probes of rows A [n, d] among C [K, d] (double distances, ties to the lower id):
// approximate scores (tcgen05 tf32 when d is a multiple of 32 and the operands are 16-byte
// aligned, else fp32 SIMT) shortlist the m best per row, the exact distance over the shortlist
// decides, and rows whose shortlist the score error bound cannot vouch for (the m-th shortlisted
// score is not clear of the p-th by twice the bound) are recomputed over all K lists.  For
// K >= kFusedCoarseMinK on tensor cores the scores and the shortlist come from one fused kernel
// (rowbuf: its per-row candidate buffers) and S is not used; otherwise S [n, K] holds the scores.
// cand [n, m], bounds [n], unsafe [1 + n]; cmax2 = max_l |c_l|^2 (device scalar).  At K = 1024
// the fused kernel measured slower (a 10,000-query search step 3.30 vs 2.90 ms): its 128 queries
// per CTA leave most SMs idle where the two kernels spread over the whole GPU.
constexpr int kFusedCoarseMinK = 2048;

bool coarse_uses_tc(const float* A, const float* C, int d)
{
  return coarse_tc_supported(d) && d % 32 == 0 && (reinterpret_cast<uintptr_t>(A) & 15u) == 0 &&
         (reinterpret_cast<uintptr_t>(C) & 15u) == 0;
}

// Scratch of coarse_probes for up to n rows: fused (rowbuf keys) or two-kernel (S floats).
struct CoarseScratch {
  float* S = nullptr;
  unsigned long long* rowbuf = nullptr;
  int32_t* cand = nullptr;
  float2* bounds = nullptr;
  int* unsafe = nullptr;
};

bool coarse_fused(int K, int d, int m)
{
  return K >= kFusedCoarseMinK && coarse_tc_supported(d) && d % 32 == 0 && m < K && m <= coarse_topm_max_shortlist();
}

// Rows per coarse_probes call: the [rows, K] scores (two-kernel) or the per-row candidate
// buffers (fused) stay within 512 MiB.
int64_t coarse_rows_per_call(const float* A, const float* C, int K, int d, int m, int64_t n)
{
  const bool fused = coarse_fused(K, d, m) && coarse_uses_tc(A, C, d);
  const int64_t per_row = fused ? (int64_t)coarse_topm_row_cap(m) * 8 : (int64_t)K * 4;
  return std::min<int64_t>(n, std::max<int64_t>(128, (512ll << 20) / per_row));
}

// A, C: the rows' and centroids' base pointers (the fused kernel reads both by TMA; d % 32 == 0
// keeps every row block of A as aligned as its base).
CoarseScratch coarse_scratch(Scratch& sc, const float* A, const float* C, int K, int d, int m, int64_t rows)
{
  CoarseScratch cs;
  if (coarse_fused(K, d, m) && coarse_uses_tc(A, C, d))
    cs.rowbuf = sc.get<unsigned long long>((size_t)ceil_div(rows, 128) * 128 * coarse_topm_row_cap(m));
  else
    cs.S = sc.get<float>((size_t)rows * K);
  cs.cand = sc.get<int32_t>((size_t)rows * m);
  cs.bounds = sc.get<float2>((size_t)rows);
  cs.unsafe = sc.get<int>((size_t)rows + 1);
  return cs;
}

void coarse_probes(const Index& ix, const float* A, int64_t n, const float* C, const float* cn2, const float* cmax2,
                   int K, int d, int m, int p, const CoarseScratch& cs, int32_t* probes, float* g, cudaStream_t s)
{
  if (n <= 0) return;
  RBQ_CUDA(cudaMemsetAsync(cs.unsafe, 0, sizeof(int), s));
  int32_t* cand = cs.cand;
  float2* bounds = cs.bounds;
  int* unsafe = cs.unsafe;
  if (coarse_uses_tc(A, C, d) && cs.rowbuf && m < K) {
    launch_coarse_topm_tc(A, n, C, cn2, K, d, m, p, cs.rowbuf, cand, bounds, ix.dev_err, s);
  } else {
    RBQ_CHECK(cs.S != nullptr, RBQ_ERR_INVALID, "coarse: no score buffer");
    if (coarse_uses_tc(A, C, d))
      launch_coarse_scores_tc(A, n, C, cn2, K, d, cs.S, ix.dev_err, s);
    else
      launch_coarse_scores(A, n, C, cn2, K, d, cs.S, s);
    launch_topm_rows(cs.S, n, K, m, cand, s, p, bounds);
  }
  launch_refine_topp(A, n, C, d, cand, m, p, probes, g, s, bounds, cmax2, unsafe);
  launch_refine_all(A, n, C, d, K, p, unsafe, probes, g, s);
}

namespace {

// Exact nearest centroid (ties -> lower id) of rows A [n, d] among C [K, d] (coarse_probes with
// p = 1 over a shortlist of 32).
void assign_labels(const Index& ix, const float* A, int64_t n, const float* C, const float* cn2, int K, int d,
                   uint32_t* labels_out, cudaStream_t s)
{
  const int m = std::min(K, 32);
  const int64_t chunk = std::min<int64_t>(65535 * 64, coarse_rows_per_call(A, C, K, d, m, n));
  Scratch sc(s);
  const CoarseScratch cs = coarse_scratch(sc, A, C, K, d, m, std::min(n, chunk));
  float* cmax2 = sc.get<float>(1);
  launch_max_reduce(cn2, K, cmax2, s);
  for (int64_t a = 0; a < n; a += chunk) {
    const int64_t cn = std::min(chunk, n - a);
    coarse_probes(ix, A + a * d, cn, C, cn2, cmax2, K, d, m, 1, cs, reinterpret_cast<int32_t*>(labels_out + a),
                  nullptr, s);
  }
}

// Stable counting sort of labels: off [K+1], order (row indices grouped by label, ascending).
void counting_sort(const std::vector<uint32_t>& lab, int K, std::vector<int64_t>& off, std::vector<int64_t>& order)
{
  off.assign(K + 1, 0);
  for (uint32_t l : lab) off[l + 1]++;
  for (int k = 0; k < K; ++k) off[k + 1] += off[k];
  std::vector<int64_t> pos(off.begin(), off.end() - 1);
  order.resize(lab.size());
  for (size_t i = 0; i < lab.size(); ++i) order[pos[lab[i]]++] = (int64_t)i;
}

// Rebuild slot-order arrays from the row-order storage.
void relayout(Index& ix, cudaStream_t s)
{
  drop_graphs(ix);
  std::vector<uint32_t> lab(ix.n_rows);
  if (ix.n_rows)
    RBQ_CUDA(cudaMemcpyAsync(lab.data(), ix.labels_r, ix.n_rows * 4, cudaMemcpyDeviceToHost, s));
  RBQ_CUDA(cudaStreamSynchronize(s));
  std::vector<int64_t> off, order;
  counting_sort(lab, ix.K, off, order);
  ix.off_host = off;
  ix.min_list = -1;
  for (int l = 0; l < ix.K; ++l)
    if (ix.owner_host[l] == ix.shard_rank && (ix.min_list < 0 || off[l + 1] - off[l] < ix.min_list))
      ix.min_list = off[l + 1] - off[l];
  if (ix.min_list < 0) ix.min_list = 0;
  dev_free(ix.list_off);
  dev_free(ix.ids);
  dev_free(ix.codes);
  dev_free(ix.fadd);
  dev_free(ix.frescale);
  dev_free(ix.ferr);
  dev_free(ix.ex_codes);
  dev_free(ix.fexadd);
  dev_free(ix.fexr);
  const size_t n = (size_t)ix.n_rows;
  ix.list_off = dev_alloc<int64_t>(ix.K + 1);
  ix.ids = dev_alloc<uint32_t>(n);
  ix.codes = dev_alloc<uint32_t>(n * ix.W);
  ix.fadd = dev_alloc<float>(n);
  ix.frescale = dev_alloc<float>(n);
  ix.ferr = dev_alloc<float>(n);
  if (ix.ex_bits > 0) {
    ix.ex_codes = dev_alloc<uint32_t>(n * ix.ex_bits * ix.W);
    ix.fexadd = dev_alloc<float>(n);
    ix.fexr = dev_alloc<float>(n);
  }
  RBQ_CUDA(cudaMemcpyAsync(ix.list_off, off.data(), (ix.K + 1) * 8, cudaMemcpyHostToDevice, s));
  if (n) {
    Scratch sc(s);
    int64_t* ord = sc.get<int64_t>(n);
    RBQ_CUDA(cudaMemcpyAsync(ord, order.data(), n * 8, cudaMemcpyHostToDevice, s));
    launch_gather_rows_u32(ix.ids_r, ix.n_rows, 1, ord, ix.ids, s);
    launch_gather_rows_u32(ix.codes_r, ix.n_rows, ix.W, ord, ix.codes, s);
    launch_gather_rows_u32(reinterpret_cast<const uint32_t*>(ix.fadd_r), ix.n_rows, 1, ord,
                           reinterpret_cast<uint32_t*>(ix.fadd), s);
    launch_gather_rows_u32(reinterpret_cast<const uint32_t*>(ix.frescale_r), ix.n_rows, 1, ord,
                           reinterpret_cast<uint32_t*>(ix.frescale), s);
    launch_gather_rows_u32(reinterpret_cast<const uint32_t*>(ix.ferr_r), ix.n_rows, 1, ord,
                           reinterpret_cast<uint32_t*>(ix.ferr), s);
    if (ix.ex_bits > 0) {
      launch_gather_rows_u32(ix.ex_codes_r, ix.n_rows, ix.ex_bits * ix.W, ord, ix.ex_codes, s);
      launch_gather_rows_u32(reinterpret_cast<const uint32_t*>(ix.fexadd_r), ix.n_rows, 1, ord,
                             reinterpret_cast<uint32_t*>(ix.fexadd), s);
      launch_gather_rows_u32(reinterpret_cast<const uint32_t*>(ix.fexr_r), ix.n_rows, 1, ord,
                             reinterpret_cast<uint32_t*>(ix.fexr), s);
    }
  }
  RBQ_CUDA(cudaStreamSynchronize(s));
}

// The raw-row store: HBM, or pinned host memory mapped into the device's address space (the
// GPU reads and writes it through the same pointer).
float* raw_alloc(const Index& ix, size_t count)
{
  if (!ix.raw_on_host) return dev_alloc<float>(count);
  if (count == 0) count = 1;
  maybe_inject_alloc_failure(count * sizeof(float));
  void* p = nullptr;
  const cudaError_t e = cudaHostAlloc(&p, count * sizeof(float), cudaHostAllocMapped | cudaHostAllocPortable);
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw Error{RBQ_ERR_OOM, std::string("cudaHostAlloc of ") + std::to_string(count * sizeof(float)) +
                                 " bytes failed: " + cudaGetErrorString(e)};
  }
  void* dp = nullptr;
  RBQ_CUDA(cudaHostGetDevicePointer(&dp, p, 0));
  RBQ_CHECK(dp == p, RBQ_ERR_CUDA, "mapped host memory has a different device address (no unified addressing)");
  return static_cast<float*>(p);
}

void raw_free(const Index& ix, float*& p)
{
  if (!p) return;
  if (ix.raw_on_host)
    cudaFreeHost(p);
  else
    cudaFree(p);
  p = nullptr;
}

void ensure_row_capacity(Index& ix, int64_t need)
{
  if (need <= ix.cap_rows) return;
  int64_t cap = std::max<int64_t>(need, ix.cap_rows + ix.cap_rows / 2);
  const size_t keep = (size_t)ix.n_rows;
  {
    float* np = raw_alloc(ix, (size_t)cap * ix.D);
    if (ix.X_r && keep) RBQ_CUDA(cudaMemcpy(np, ix.X_r, keep * ix.D * 4, cudaMemcpyDefault));
    raw_free(ix, ix.X_r);
    ix.X_r = np;
  }
  dev_grow(ix.codes_r, keep * ix.W, (size_t)cap * ix.W);
  dev_grow(ix.fadd_r, keep, cap);
  dev_grow(ix.frescale_r, keep, cap);
  dev_grow(ix.ferr_r, keep, cap);
  if (ix.ex_bits > 0) {
    dev_grow(ix.ex_codes_r, keep * ix.ex_bits * ix.W, (size_t)cap * ix.ex_bits * ix.W);
    dev_grow(ix.fexadd_r, keep, cap);
    dev_grow(ix.fexr_r, keep, cap);
  }
  dev_grow(ix.labels_r, keep, cap);
  dev_grow(ix.ids_r, keep, cap);
  ix.cap_rows = cap;
}

void ensure_id_capacity(Index& ix, int64_t need)
{
  if (need <= ix.cap_ids) return;
  int64_t cap = std::max<int64_t>(need, ix.cap_ids + ix.cap_ids / 2);
  RBQ_CHECK(cap <= 0xFFFFFFFFll, RBQ_ERR_INVALID, "index supports at most 2^32-1 vectors");
  uint32_t* np = dev_alloc<uint32_t>(cap);
  RBQ_CUDA(cudaMemset(np, 0xFF, cap * 4));
  if (ix.id2row && ix.n_total) RBQ_CUDA(cudaMemcpy(np, ix.id2row, ix.n_total * 4, cudaMemcpyDeviceToDevice));
  dev_free(ix.id2row);
  ix.id2row = np;
  ix.cap_ids = cap;
}

// Append already-quantised or raw rows: X_dev [n, D] with labels (device) -> this shard's rows.
void add_rows(Index& ix, const float* X, int64_t n, const uint32_t* labels_dev, cudaStream_t s)
{
  RBQ_CHECK(ix.trained, RBQ_ERR_STATE, "add called before train / set_centroids");
  RBQ_CHECK(n >= 0, RBQ_ERR_INVALID, "add: negative row count");
  if (n == 0) return;
  RBQ_CHECK(ix.n_total + n <= 0xFFFFFFFFll, RBQ_ERR_INVALID, "index supports at most 2^32-1 vectors");
  Scratch sc(s);
  uint32_t* lab = sc.get<uint32_t>(n);
  if (labels_dev) {
    RBQ_CUDA(cudaMemcpyAsync(lab, labels_dev, n * 4, cudaMemcpyDeviceToDevice, s));
  } else {
    assign_labels(ix, X, n, ix.C, ix.C_n2, ix.K, ix.D, lab, s);
  }
  std::vector<uint32_t> hl(n);
  RBQ_CUDA(cudaMemcpyAsync(hl.data(), lab, n * 4, cudaMemcpyDeviceToHost, s));
  RBQ_CUDA(cudaStreamSynchronize(s));
  for (int64_t i = 0; i < n; ++i) RBQ_CHECK(hl[i] < (uint32_t)ix.K, RBQ_ERR_INVALID, "add: label out of range");
  if (!ix.owners_fixed) {  // BALANCED: the map follows the list sizes of the first batch
    std::vector<int64_t> sizes(ix.K, 0);
    for (int64_t i = 0; i < n; ++i) ++sizes[hl[i]];
    install_owners(ix, list_owners(ix.shard_policy, sizes, ix.shard_count), true);
  }
  std::vector<int64_t> own;
  std::vector<uint32_t> own_lab, own_ids;
  own.reserve(n);
  for (int64_t i = 0; i < n; ++i) {
    if (ix.owner_host[hl[i]] == ix.shard_rank) {
      own.push_back(i);
      own_lab.push_back(hl[i]);
      own_ids.push_back((uint32_t)(ix.n_total + i));
    }
  }
  const int64_t m = (int64_t)own.size();
  ensure_id_capacity(ix, ix.n_total + n);
  if (m > 0) {
    ensure_row_capacity(ix, ix.n_rows + m);
    const int64_t r0 = ix.n_rows;
    int64_t* src = sc.get<int64_t>(m);
    RBQ_CUDA(cudaMemcpyAsync(src, own.data(), m * 8, cudaMemcpyHostToDevice, s));
    if (!ix.raw_on_host) launch_gather_rows_f32(X, m, ix.D, src, ix.X_r + (size_t)r0 * ix.D, s);
    RBQ_CUDA(cudaMemcpyAsync(ix.labels_r + r0, own_lab.data(), m * 4, cudaMemcpyHostToDevice, s));
    RBQ_CUDA(cudaMemcpyAsync(ix.ids_r + r0, own_ids.data(), m * 4, cudaMemcpyHostToDevice, s));
    // Rotate + quantise in chunks to bound the rotated-row scratch.  A host store receives each
    // chunk's raw rows from a device copy the chunk is quantised from (one trip over the bus).
    const int64_t chunk = std::max<int64_t>(1, (512ll << 20) / ((int64_t)ix.Dp * 4));
    float* Y = sc.get<float>((size_t)std::min(chunk, m) * ix.Dp);
    float* Xs = ix.raw_on_host ? sc.get<float>((size_t)std::min(chunk, m) * ix.D) : nullptr;
    for (int64_t a = 0; a < m; a += chunk) {
      const int64_t cn = std::min(chunk, m - a);
      const int64_t r = r0 + a;
      const float* rows = ix.X_r + (size_t)r * ix.D;
      if (ix.raw_on_host) {
        launch_gather_rows_f32(X, cn, ix.D, src + a, Xs, s);
        RBQ_CUDA(cudaMemcpyAsync(ix.X_r + (size_t)r * ix.D, Xs, (size_t)cn * ix.D * 4, cudaMemcpyDeviceToHost, s));
        rows = Xs;
      }
      launch_rotate(rows, cn, ix.D, ix.Dp, ix.P, Y, s);
      launch_quantize(Y, cn, ix.Dp, ix.C_rot, ix.labels_r + r, ix.codes_r + (size_t)r * ix.W, ix.fadd_r + r,
                      ix.frescale_r + r, ix.ferr_r + r, s);
      launch_quantize_ex(Y, cn, ix.Dp, ix.C_rot, ix.labels_r + r, ix.ex_bits, ix.tex,
                         ix.ex_codes_r + (size_t)r * ix.ex_bits * ix.W, ix.fexadd_r + r, ix.fexr_r + r, s);
    }
    // id2row for this call's id range [n_total, n_total + n): ids are contiguous per call.
    std::vector<uint32_t> id2row_new(n, 0xFFFFFFFFu);
    for (int64_t i = 0; i < m; ++i) id2row_new[own[i]] = (uint32_t)(r0 + i);
    RBQ_CUDA(cudaMemcpyAsync(ix.id2row + ix.n_total, id2row_new.data(), n * 4, cudaMemcpyHostToDevice, s));
    RBQ_CUDA(cudaStreamSynchronize(s));
    ix.n_rows += m;
  }
  ix.n_total += n;
  relayout(ix, s);
}

// ---------------------------------------------------------------------------------------
// k-means.  One EM problem: rows X [n, D] (device), k centres C [k, D] (device), labels on
// device and host, cluster sizes on the host.
// ---------------------------------------------------------------------------------------
struct KmProblem {
  const float* X = nullptr;
  int64_t n = 0;
  int k = 0;
  float* C = nullptr;
  uint32_t* lab_d = nullptr;
  float* cn2 = nullptr;
  std::vector<uint32_t> lab;
  std::vector<int64_t> size;
};

// E step: exact nearest centre of every row (ties -> lower id), labels copied to the host.
void km_predict(const Index& ix, KmProblem& p, cudaStream_t s)
{
  launch_row_norms(p.C, p.k, ix.D, p.cn2, s);
  assign_labels(ix, p.X, p.n, p.C, p.cn2, p.k, ix.D, p.lab_d, s);
  p.lab.resize(p.n);
  RBQ_CUDA(cudaMemcpyAsync(p.lab.data(), p.lab_d, p.n * 4, cudaMemcpyDeviceToHost, s));
  RBQ_CUDA(cudaStreamSynchronize(s));
}

// M step: centres = means of their rows (members summed in ascending row order, in double),
// sizes from the same labels.
void km_update(const Index& ix, KmProblem& p, bool zero_empty, cudaStream_t s)
{
  std::vector<int64_t> off, order;
  counting_sort(p.lab, p.k, off, order);
  std::vector<uint32_t> ho(p.n);
  for (int64_t i = 0; i < p.n; ++i) ho[i] = (uint32_t)order[i];
  p.size.resize(p.k);
  for (int c = 0; c < p.k; ++c) p.size[c] = off[c + 1] - off[c];
  Scratch sc(s);
  int64_t* off_d = sc.get<int64_t>(p.k + 1);
  uint32_t* order_d = sc.get<uint32_t>(p.n);
  RBQ_CUDA(cudaMemcpyAsync(off_d, off.data(), (p.k + 1) * 8, cudaMemcpyHostToDevice, s));
  RBQ_CUDA(cudaMemcpyAsync(order_d, ho.data(), p.n * 4, cudaMemcpyHostToDevice, s));
  launch_centroid_update(p.X, p.n, ix.D, p.lab_d, off_d, order_d, p.k, p.C, zero_empty, s);
  RBQ_CUDA(cudaStreamSynchronize(s));  // the host vectors above are the copies' sources
}

// Stride of the rebalancing walk over the rows (the reference draws it from a cycle of 40
// primes, kmeans_balanced.cuh:569-582): the next entry of a fixed cycle of 40 primes (the
// smallest prime >= 61 + 64 t, t = 0..39) that does not divide n, so the walk i = stride *
// j mod n reaches every row.  The cursor runs on across all EM passes of one training run.
int64_t km_walk_stride(int& cursor, int64_t n)
{
  auto next_prime = [](int64_t x) {
    for (;; ++x) {
      bool prime = x > 1;
      for (int64_t d = 2; d * d <= x && prime; ++d) prime = x % d != 0;
      if (prime) return x;
    }
  };
  for (;;) {
    cursor = (cursor + 1) % 40;
    const int64_t p = next_prime(61 + 64 * (int64_t)cursor);
    if (n % p != 0) return p;
  }
}

// Rebalancing (kmeans_balanced.cuh:498-591): every cluster of size <= (float)(n / k) * threshold,
// taken in ascending id, moves its centre towards the next row of the walk whose cluster holds
// >= n / k rows (one walk counter shared by all clusters).  Returns whether any centre moved.
bool km_adjust(const Index& ix, KmProblem& p, float threshold, int& cursor, cudaStream_t s)
{
  const int64_t average = p.n / p.k;
  const int64_t limit = (int64_t)((float)average * threshold);
  const int64_t stride = km_walk_stride(cursor, p.n);
  std::vector<int64_t> adj;
  int64_t count = 0;
  for (int l = 0; l < p.k; ++l) {
    if (p.size[l] > limit) continue;
    int64_t i;
    do {
      const int64_t old = count++;
      i = (int64_t)(((__int128)stride * (old + 1)) % p.n);
    } while (p.size[p.lab[i]] < average);
    adj.insert(adj.end(), {(int64_t)l, (int64_t)p.lab[i], i, std::min<int64_t>(p.size[l], 7)});
  }
  if (adj.empty()) return false;
  Scratch sc(s);
  int64_t* adj_d = sc.get<int64_t>(adj.size());
  RBQ_CUDA(cudaMemcpyAsync(adj_d, adj.data(), adj.size() * 8, cudaMemcpyHostToDevice, s));
  launch_adjust_centers(p.C, ix.D, p.X, adj_d, (int)(adj.size() / 4), s);
  RBQ_CUDA(cudaStreamSynchronize(s));
  return true;
}

// EM with rebalancing (kmeans_balanced.cuh:593-704): n_iters passes of adjust (not on the
// first pass) -> predict -> update; the first and then every pullback-th pass that moved a
// centre adds one pass.
void km_em(const Index& ix, KmProblem& p, int n_iters, int pullback, float threshold, int& cursor, cudaStream_t s)
{
  int counter = pullback;
  for (int iter = 0; iter < n_iters; ++iter) {
    if (iter > 0 && km_adjust(ix, p, threshold, cursor, s)) {
      if (counter++ >= pullback) {
        counter -= pullback;
        ++n_iters;
      }
    }
    km_predict(ix, p, s);
    km_update(ix, p, true, s);
  }
}

// Clusters from scratch (kmeans_balanced.cuh:706-757): labels i mod k, their means, then EM
// (pullback 2, threshold 0.25).
void km_build_clusters(const Index& ix, KmProblem& p, int n_iters, int& cursor, cudaStream_t s)
{
  p.lab.resize(p.n);
  for (int64_t i = 0; i < p.n; ++i) p.lab[i] = (uint32_t)(i % p.k);
  RBQ_CUDA(cudaMemcpyAsync(p.lab_d, p.lab.data(), p.n * 4, cudaMemcpyHostToDevice, s));
  km_update(ix, p, true, s);
  km_em(ix, p, n_iters, 2, 0.25f, cursor, s);
}

// Hierarchical balanced k-means (kmeans_balanced.cuh:759-1132) of the rows X [n, D] into K
// centres C_out [K, D] (device).
void train_balanced(const Index& ix, const float* X, int64_t n, int K, float* C_out, cudaStream_t s)
{
  const int D = ix.D, iters = ix.kmeans_iters;
  int cursor = 0;
  Scratch sc(s);
  Range r("rbq balanced k-means");
  const int n_meso = std::min<int>(K, (int)(std::sqrt((double)K) + 0.5));
  uint32_t* lab_d = sc.get<uint32_t>(n);
  float* cn2 = sc.get<float>(K);
  KmProblem meso;
  meso.X = X;
  meso.n = n;
  meso.k = n_meso;
  meso.C = sc.get<float>((size_t)n_meso * D);
  meso.lab_d = lab_d;
  meso.cn2 = cn2;
  km_build_clusters(ix, meso, iters, cursor, s);

  // Fine clusters per mesocluster, in proportion to its rows (kmeans_balanced.cuh:759-826).
  std::vector<int64_t> nums(n_meso), csum(n_meso + 1, 0);
  int64_t lists_rem = K, rows_rem = n, nonempty_rem = 0, size_max = 0, nums_max = 0;
  for (int i = 0; i < n_meso; ++i) nonempty_rem += meso.size[i] > 0;
  for (int i = 0; i < n_meso; ++i) {
    if (i < n_meso - 1) {
      if (meso.size[i] == 0) {
        nums[i] = 0;
      } else {
        --nonempty_rem;
        int64_t f = (int64_t)((double)(lists_rem * meso.size[i]) / (double)rows_rem + 0.5);
        f = std::min<int64_t>(f, lists_rem - nonempty_rem);
        nums[i] = std::max<int64_t>(f, 1);
      }
    } else {
      nums[i] = lists_rem;
    }
    lists_rem -= nums[i];
    rows_rem -= meso.size[i];
    size_max = std::max(size_max, meso.size[i]);
    nums_max = std::max(nums_max, nums[i]);
    csum[i + 1] = csum[i] + nums[i];
  }
  RBQ_CHECK(csum[n_meso] == K, RBQ_ERR_INVALID, "balanced k-means: fine cluster counts do not add up");
  // At most 2n / n_meso rows of one mesocluster train its fine clusters (kmeans_balanced.cuh:1068-1083).
  size_max = std::min<int64_t>(size_max, (2 * n + n_meso - 1) / std::max(n_meso, 1));

  // Fine clusters of each mesocluster (kmeans_balanced.cuh:828-946).
  {
    Scratch fs(s);
    float* Xm = fs.get<float>((size_t)size_max * D);
    int64_t* rows_d = fs.get<int64_t>(size_max);
    float* Cm = fs.get<float>((size_t)std::max<int64_t>(nums_max, 1) * D);
    std::vector<int64_t> moff, morder;  // rows of each mesocluster, ascending
    counting_sort(meso.lab, n_meso, moff, morder);
    std::vector<int64_t> rows;
    for (int i = 0; i < n_meso; ++i) {
      rows.assign(morder.begin() + moff[i], morder.begin() + std::min(moff[i + 1], moff[i] + size_max));
      if (rows.empty()) {
        RBQ_CHECK(nums[i] == 0, RBQ_ERR_INVALID, "balanced k-means: an empty mesocluster was given fine clusters");
        continue;
      }
      RBQ_CUDA(cudaMemcpyAsync(rows_d, rows.data(), rows.size() * 8, cudaMemcpyHostToDevice, s));
      launch_gather_rows_f32(X, (int64_t)rows.size(), D, rows_d, Xm, s);
      KmProblem fine;
      fine.X = Xm;
      fine.n = (int64_t)rows.size();
      fine.k = (int)nums[i];
      fine.C = Cm;
      fine.lab_d = lab_d;
      fine.cn2 = cn2;
      km_build_clusters(ix, fine, iters, cursor, s);
      RBQ_CUDA(cudaMemcpyAsync(C_out + (size_t)csum[i] * D, Cm, (size_t)nums[i] * D * 4, cudaMemcpyDeviceToDevice, s));
      RBQ_CUDA(cudaStreamSynchronize(s));  // `rows` is the next upload's source
    }
  }

  // Fine-tuning over all rows (kmeans_balanced.cuh:1096-1117): max(iters / 10, 2) passes,
  // pullback 5, threshold 0.2.
  KmProblem all;
  all.X = X;
  all.n = n;
  all.k = K;
  all.C = C_out;
  all.lab_d = lab_d;
  all.cn2 = cn2;
  km_em(ix, all, std::max(iters / 10, 2), 5, 0.2f, cursor, s);
}

// Plain Lloyd iterations from the evenly strided rows i * n / K; empty lists keep their centre.
void train_lloyd(const Index& ix, const float* X, int64_t n, int K, float* C, cudaStream_t s)
{
  Scratch sc(s);
  std::vector<int64_t> ipick(K);
  for (int k = 0; k < K; ++k) ipick[k] = (int64_t)(((__int128)k * n) / K);
  int64_t* ipick_d = sc.get<int64_t>(K);
  RBQ_CUDA(cudaMemcpyAsync(ipick_d, ipick.data(), K * 8, cudaMemcpyHostToDevice, s));
  launch_gather_rows_f32(X, K, ix.D, ipick_d, C, s);
  KmProblem p;
  p.X = X;
  p.n = n;
  p.k = K;
  p.C = C;
  p.lab_d = sc.get<uint32_t>(n);
  p.cn2 = sc.get<float>(K);
  for (int it = 0; it < ix.kmeans_iters; ++it) {
    km_predict(ix, p, s);
    km_update(ix, p, false, s);
  }
}

void train_kmeans(Index& ix, const float* X, int64_t n, cudaStream_t s)
{
  const int K = ix.K, D = ix.D;
  RBQ_CHECK(n >= K, RBQ_ERR_INVALID, "train: need at least n_lists rows");
  const int64_t n_train = std::min<int64_t>(n, (int64_t)ix.max_train_per_list * K);
  Scratch sc(s);
  std::vector<int64_t> pick(n_train);
  for (int64_t i = 0; i < n_train; ++i) pick[i] = (int64_t)(((__int128)i * n) / n_train);
  int64_t* pick_d = sc.get<int64_t>(n_train);
  RBQ_CUDA(cudaMemcpyAsync(pick_d, pick.data(), n_train * 8, cudaMemcpyHostToDevice, s));
  float* Xs = sc.get<float>((size_t)n_train * D);
  launch_gather_rows_f32(X, n_train, D, pick_d, Xs, s);
  float* C = sc.get<float>((size_t)K * D);
  if (ix.kmeans_kind == RBQ_KMEANS_LLOYD)
    train_lloyd(ix, Xs, n_train, K, C, s);
  else
    train_balanced(ix, Xs, n_train, K, C, s);
  ix.C_host.resize((size_t)K * D);
  RBQ_CUDA(cudaMemcpyAsync(ix.C_host.data(), C, (size_t)K * D * 4, cudaMemcpyDeviceToHost, s));
  RBQ_CUDA(cudaStreamSynchronize(s));
  install_centroids(ix, s);
}

struct SearchPlan {
  int P, k, R, cap, slices, m;
  int prune;
  int qbits;    // search mode: 4 (QUANT4), 8 (QUANT8), 16 (LUT16) or 32 (LUT32)
  bool seeded;  // two-phase scan (search_scan)
  bool lists;   // list scan on the tensor cores with a fixed per-query threshold
  int lcap;     // its candidate row per query
};

// The list scan serves batches whose probed lists are shared by at least this many queries on
// average (at the benchmark shapes, 98 to 390 per list, it beats the tile scan by 1.3x at D = 128
// and 256 and 3x at D = 768; at 32 per list it loses, 1.5 against 0.8 ms), on indexes whose lists
// hold R vectors on average (the nearest list then gives a tight fixed threshold; with lists of
// 98 vectors and R = 800 the threshold admits 93 % of the probed vectors); others take the tile
// scan.
constexpr int64_t kListScanMinPairsPerList = 64;

// Whether a search takes the list scan: scan_kind 2 asks for it, 1 for the tile scan; 0 (auto)
// takes the list scan for popcount modes with the prune on when nq * P >= 64 K and the index
// holds n_total >= R K vectors.
bool use_list_scan(int scan_kind, int qbits, int prune, int dp, int64_t nq, int P, int K, int64_t n_total, int R)
{
  RBQ_CHECK(scan_kind >= 0 && scan_kind <= 2, RBQ_ERR_INVALID,
            "scan_kind must be 0 (auto), 1 (tile scan) or 2 (list scan)");
  const bool able = (qbits == 4 || qbits == 8) && prune && list_scan_tc_supported(dp);
  RBQ_CHECK(scan_kind != 2 || able, RBQ_ERR_INVALID,
            "list scan: needs QUANT4 / QUANT8, the prune on and a padded dim <= 768");
  if (scan_kind == 2) return true;
  return scan_kind == 0 && able && nq * (int64_t)P >= kListScanMinPairsPerList * K && n_total >= (int64_t)R * K;
}

int list_scan_cap(int R)
{
  int c = 2048;
  while (c < 2 * R) c <<= 1;
  return c;
}

// Search mode of query_bits (0 means 4): 4 / 8 = QUANT4 / QUANT8 (popcount estimator over 4- or
// 8-bit query codes), 16 / 32 = LUT16 / LUT32 (fp16 / fp32 tables of the float query).
int query_bits_of(int32_t bits)
{
  const int qb = bits == 0 ? 4 : bits;
  RBQ_CHECK(qb == 4 || qb == 8 || qb == 16 || qb == 32, RBQ_ERR_INVALID,
            "query bits must be 4 (QUANT4), 8 (QUANT8), 16 (LUT16) or 32 (LUT32)");
  return qb;
}

// Code width of the query preparation for a search mode: the LUT modes use only its k1 (and
// take the 4-bit planes it also makes).
int prep_bits_of(int qbits) { return qbits == 8 ? 8 : 4; }

// Scale constant of the query code width: t4 (const_scaling_factor_4bit, best rescale for 3
// extra bits) or t8 (const_scaling_factor_8bit, 7 extra bits; quantizer_gpu.cuh:81-85), the
// latter computed on first use unless an imported reference file supplied it.
float query_t(Index& ix, int qbits)
{
  if (qbits == 4) return ix.t4;
  if (std::isnan(ix.t8)) ix.t8 = query_scale(ix.Dp, ix.seed, 7);
  return ix.t8;
}

// Data scale of the extra-bit codes (construct_on_gpu, ivf_gpu.cu:629-644, fast quantize): the
// 4-bit query scale for 3 extra bits, the 8-bit one for 7, else the best-rescale mean for the
// extra-bit count (the reference computes that one from a time-seeded generator,
// quantizer_gpu.cu:1357-1435; here it comes from the index seed, so builds repeat).
float ex_scale_of(Index& ix)
{
  if (ix.ex_bits <= 0) return 0.0f;
  if (ix.ex_bits == 3) return ix.t4;
  if (ix.ex_bits == 7) return query_t(ix, 8);
  return query_scale(ix.Dp, ix.seed, ix.ex_bits);
}

SearchPlan plan_search(const Index& ix, const rbq_search_params_t& p, int64_t nq)
{
  RBQ_CHECK(p.k >= 1, RBQ_ERR_INVALID, "search: k must be >= 1");
  RBQ_CHECK(p.n_probes >= 1 && p.n_probes <= ix.K, RBQ_ERR_INVALID,
            "search: n_probes (" + std::to_string(p.n_probes) + ") must be in [1, n_lists = " +
                std::to_string(ix.K) + "]");
  RBQ_CHECK(p.rerank >= 0, RBQ_ERR_INVALID, "search: rerank must be >= 0");
  SearchPlan sp;
  sp.P = p.n_probes;
  sp.k = p.k;
  sp.R = p.rerank > 0 ? std::max(p.rerank, p.k) : p.k;
  RBQ_CHECK(sp.R <= 4096, RBQ_ERR_INVALID, "search: rerank depth / k must be <= 4096");
  sp.cap = p.cand_cap > 0 ? p.cand_cap : 1024;
  sp.cap = std::max(next_pow2(sp.cap), next_pow2(sp.R + kScanTile));
  int own = std::max(1, (sp.P + ix.shard_count - 1) / ix.shard_count);
  int sl = p.probe_split > 0 ? p.probe_split : (int)std::max<int64_t>(1, 512 / std::max<int64_t>(1, nq));
  sl = std::min(sl, own);
  sl = std::min(sl, std::max(1, 8192 / sp.R));
  sp.slices = std::max(1, sl);
  const int margin = p.coarse_margin > 0 ? p.coarse_margin : std::max(32, sp.P / 2);
  sp.m = std::min(ix.K, std::min(sp.P + margin, 1024));
  sp.prune = p.prune ? 1 : 0;
  sp.qbits = query_bits_of(p.query_bits);
  sp.seeded = sp.qbits < 16 && (p.seeded < 0 ? sp.slices > 1 : p.seeded > 0);  // no bound seed in LUT modes
  sp.lists = use_list_scan(p.scan_kind, sp.qbits, sp.prune, ix.Dp, nq, sp.P, ix.K, ix.n_total, sp.R);
  sp.lcap = list_scan_cap(sp.R);
  if (sp.lists) {  // two key rows per query: the nearest probe's tile scan and the list scan
    sp.slices = 2;
    sp.seeded = false;
  }
  return sp;
}

// Scan arguments of one query batch against this shard's lists (probes: [nq, nprobe]).
ScanArgs batch_scan_args(const Index& ix, const float* Qr, const uint32_t* planes, const float* delta,
                         const float* k1, int64_t nq, const int32_t* probes, const float* g, int nprobe, int R,
                         int cap, int prune, int slices, unsigned long long* out_keys, uint64_t* stats, int qbits)
{
  ScanArgs sa;
  sa.qbits = qbits;
  sa.list_off = ix.list_off;
  sa.ids = ix.ids;
  sa.codes = ix.codes;
  sa.fadd = ix.fadd;
  sa.frescale = ix.frescale;
  sa.ferr = ix.ferr;
  if (ix.ex_bits > 0) {
    sa.ex_codes = ix.ex_codes;
    sa.fexadd = ix.fexadd;
    sa.fexr = ix.fexr;
    sa.ex_bits = ix.ex_bits;
  }
  sa.n_slots = ix.n_rows;
  sa.Dp = ix.Dp;
  sa.W = ix.W;
  sa.Qr = Qr;
  sa.planes = planes;
  sa.delta = delta;
  sa.k1 = k1;
  sa.nq = nq;
  sa.probes = probes;
  sa.g = g;
  sa.nprobe = nprobe;
  sa.R = R;
  sa.cap = cap;
  sa.prune = prune ? 1 : 0;
  sa.slices = slices;
  sa.owner = ix.owner;
  sa.shard_rank = ix.shard_rank;
  sa.out_keys = out_keys;
  sa.stats = reinterpret_cast<unsigned long long*>(stats);
  return sa;
}

// The queries whose candidate row overflowed are few (at config 2, 50 of 10,000) but far: they
// admit up to every probed vector.  The tile scan answers them, each split into up to 16 slices
// of its probes, the slices of the listed queries spread over 8 blocks per SM.  The slices' keys
// [nq, slices, R] are held to 256 MiB (no fewer than 4 slices), and the merge of a query's
// slices must fit in shared memory.
constexpr int kListFallbackMaxSlices = 16;
constexpr int64_t kListFallbackBytes = 256ll << 20;
constexpr int kListFallbackBlocksPerSm = 8;

int list_fallback_slices(int64_t nq, int nprobe, int R)
{
  int fs = std::max(1, std::min(nprobe, kListFallbackMaxSlices));
  while (fs > 4 && (nq * fs * R * 8 > kListFallbackBytes || (int64_t)(fs + 1) * R * 8 > 200 * 1024))
    fs = std::max(4, fs / 2);
  return std::max(1, std::min(fs, nprobe));
}

// Scratch of a list scan over nq queries with P probe columns.
struct ListScanScratch {
  int8_t* qcodes;
  int32_t *list_start, *item_start, *cursor, *pair_q, *cand_cnt;
  float* pair_g;
  unsigned long long* cand;
  int fs;                    // slices of the overflowed queries' tile scan
  int32_t *over_list, *over_n;  // the overflowed queries, their count
  unsigned long long* fall;  // [nq, fs, R] keys of the overflowed queries' slices
};

ListScanScratch list_scan_scratch(Scratch& sc, const Index& ix, int64_t nq, int P, int cap, int R)
{
  ListScanScratch w;
  w.fs = list_fallback_slices(nq, P, R);
  w.over_list = sc.get<int32_t>((size_t)nq);
  w.over_n = sc.get<int32_t>(1);
  w.qcodes = sc.get<int8_t>((size_t)nq * ix.Dp);
  w.list_start = sc.get<int32_t>((size_t)ix.K + 1);
  w.item_start = sc.get<int32_t>((size_t)ix.K + 1);
  w.cursor = sc.get<int32_t>((size_t)ix.K + 1);
  w.pair_q = sc.get<int32_t>((size_t)nq * P);
  w.pair_g = sc.get<float>((size_t)nq * P);
  w.cand_cnt = sc.get<int32_t>((size_t)nq);
  w.cand = sc.get<unsigned long long>((size_t)nq * cap);
  w.fall = sc.get<unsigned long long>((size_t)nq * w.fs * R);
  return w;
}

// The list scan: fixed thresholds tau0 [nq] (every query admits while low < tau0), the
// tensor-core pass over all (list, query) pairs, the exact pass per query, and the
// fixed-threshold tile scan for queries whose candidate row overflowed.  out_keys [nq, R].
void list_scan(const Index& ix, const float* Qr, const uint32_t* planes, int qbits, const float* delta,
               const float* k1, int64_t nq, const int32_t* probes, const float* g, int nprobe, int pstride,
               const float* tau0, int R, int cap, const ListScanScratch& w, unsigned long long* out_keys,
               uint64_t* stats, cudaStream_t s, int out_slices = 1, int out_slice = 0)
{
  if (nq <= 0) return;
  launch_planes_to_codes(planes, nq, ix.W, qbits, w.qcodes, s);
  launch_list_pairs(probes, g, nq, nprobe, pstride, ix.owner, ix.shard_rank, ix.K, w.list_start, w.item_start,
                    w.cursor, w.pair_q, w.pair_g, s);
  RBQ_CUDA(cudaMemsetAsync(w.cand_cnt, 0, (size_t)nq * sizeof(int32_t), s));
  ListScanArgs la;
  la.list_off = ix.list_off;
  la.codes = ix.codes;
  la.fadd = ix.fadd;
  la.frescale = ix.frescale;
  la.ferr = ix.ferr;
  la.W = ix.W;
  la.Dp = ix.Dp;
  la.qcodes = w.qcodes;
  la.delta = delta;
  la.k1 = k1;
  la.tau0 = tau0;
  la.pair_q = w.pair_q;
  la.pair_g = w.pair_g;
  la.list_start = w.list_start;
  la.item_start = w.item_start;
  la.K = ix.K;
  la.cand = w.cand;
  la.cand_cnt = w.cand_cnt;
  la.cap = cap;
  la.stats = reinterpret_cast<unsigned long long*>(stats);
  la.err = ix.dev_err;
  // at most one partial item per list beyond nq * nprobe / 128 full ones
  const int64_t max_items = ix.K + (nq * nprobe) / kListScanRows + 1;
  launch_list_scan_tc(la, max_items, s);
  ExactArgs ea;
  ea.codes = ix.codes;
  ea.fadd = ix.fadd;
  ea.frescale = ix.frescale;
  ea.ids = ix.ids;
  if (ix.ex_bits > 0) {
    ea.ex_codes = ix.ex_codes;
    ea.fexadd = ix.fexadd;
    ea.fexr = ix.fexr;
    ea.ex_bits = ix.ex_bits;
  }
  ea.W = ix.W;
  ea.Qr = Qr;
  ea.k1 = k1;
  ea.tau0 = tau0;
  ea.cand = w.cand;
  ea.cand_cnt = w.cand_cnt;
  ea.cap = cap;
  ea.R = R;
  ea.nq = nq;
  ea.out_keys = out_keys;
  ea.out_slices = out_slices;
  ea.out_slice = out_slice;
  launch_exact_topr(ea, s);
  // rows that overflowed: listed on the device, then the tile scan with the same fixed
  // thresholds over the listed queries only, in slices merged into the query's row.  Slices
  // keep the answer: each holds the R best of its part of a set.
  const int fs = std::min(nprobe, w.fs);
  launch_over_list(w.cand_cnt, nq, cap, w.over_list, w.over_n, s);
  ScanArgs fa = batch_scan_args(ix, Qr, planes, delta, k1, nq, probes, g, nprobe, R,
                                std::max(next_pow2(1024), next_pow2(R + kScanTile)), 1, fs, w.fall, nullptr, qbits);
  fa.pstride = pstride;
  fa.tau0 = tau0;
  fa.fixed_tau = 1;
  fa.over_cnt = w.cand_cnt;
  fa.over_cap = cap;
  fa.qorder = w.over_list;
  fa.unit_count = w.over_n;
  fa.grid_blocks = kListFallbackBlocksPerSm * device_sm_count();
  launch_scan(fa, s);
  launch_merge_sorted_keys(w.fall, nq, fs, R, out_keys, out_slices, out_slice, w.cand_cnt, cap, s);
}

void search_scan(const Index& ix, const SearchPlan& sp, const float* Qr, const uint32_t* planes, const float* delta,
                 const float* k1, int64_t nq, const int32_t* probes, const float* g, float* tau_a,
                 unsigned long long* keys_s, unsigned long long* keys, uint64_t* stats, int32_t* qorder_buf,
                 const ListScanScratch* lw, cudaStream_t s)
{
  ScanArgs sa = batch_scan_args(ix, Qr, planes, delta, k1, nq, probes, g, sp.P, sp.R, sp.cap, sp.prune, sp.slices,
                                keys_s, stats, sp.qbits);
  if (sp.lists) {
    // 1. the bound seed over the leading probed lists holding >= R vectors; 2. the tile scan of
    //    the nearest probe from that seed -> keys_s[q][0] (a list scan of one probe column shares
    //    each list among too few queries to pay).  On one GPU whose every list holds R vectors
    //    the seed is the nearest list's, which the tile scan computes itself (and reports).
    ScanArgs aa = sa;
    aa.nprobe = 1;
    aa.pstride = sp.P;
    aa.slices = 1;
    aa.out_keys = keys_s;
    aa.out_slices = sp.P > 1 ? 2 : 1;
    if (ix.shard_count == 1 && ix.min_list >= sp.R) {
      aa.seed_out = tau_a;
    } else {
      ScanArgs a0 = sa;
      a0.slices = 1;
      a0.stats = nullptr;
      a0.tau_out = tau_a;
      launch_scan(a0, s);
      aa.tau0 = tau_a;
    }
    launch_scan(aa, s);
    if (sp.P == 1) {
      RBQ_CUDA(cudaMemcpyAsync(keys, keys_s, (size_t)nq * sp.R * 8, cudaMemcpyDeviceToDevice, s));
      return;
    }
    // 3. the threshold fixed for the other probes: the seed, or the nearest list's R-th distance
    launch_tighten_tau(keys_s, nq, 2 * sp.R, sp.R, tau_a, s);
    // 4. the list scan of probes 1..P-1 -> keys_s[q][1]; 5. the R smallest of both
    list_scan(ix, Qr, planes, sp.qbits, delta, k1, nq, probes + 1, g + 1, sp.P - 1, sp.P, tau_a, sp.R, sp.lcap,
              *lw, keys_s, stats, s, 2, 1);
    launch_merge_sorted_keys(keys_s, nq, 2, sp.R, keys, 1, 0, nullptr, 0, s);
    return;
  }
  if (qorder_buf && nq >= kQueryOrderMinBatch) {  // [K + 2] counts, then [nq] order
    launch_query_order(probes, nq, sp.P, ix.K, qorder_buf, qorder_buf + ix.K + 2, s);
    sa.qorder = qorder_buf + ix.K + 2;
  }
  if (sp.seeded && sp.prune) {
    ScanArgs a0 = sa;
    a0.nprobe = 1;
    a0.pstride = sp.P;
    a0.slices = 1;
    a0.stats = nullptr;
    a0.tau_out = tau_a;
    a0.qorder = sa.qorder;
    launch_scan(a0, s);
    sa.tau0 = tau_a;
  }
  launch_scan(sa, s);
  if (sp.slices > 1) launch_merge_keys(keys_s, nq, sp.slices, sp.R, keys, s);
}

// Qr_pre (optional): the batch already rotated ([nq, Dp]); the search then skips the rotation.
void run_search(Index& ix, const rbq_search_params_t& params, const float* Q, int64_t nq, float* dist, int64_t* ids,
                cudaStream_t s, uint64_t* stats, const float* Qr_pre = nullptr)
{
  RBQ_CHECK(nq >= 0, RBQ_ERR_INVALID, "search: negative query count");
  if (nq == 0) return;
  RBQ_CHECK(ix.trained, RBQ_ERR_STATE, "search called before train / set_centroids");
  RBQ_CHECK(params.rerank <= 0 || ix.has_raw, RBQ_ERR_STATE,
            "exact rerank needs the raw vectors; this index was imported without them (use rerank = 0)");
  const SearchPlan sp = plan_search(ix, params, nq);
  // The scan and rerank run over chunks bounded by the candidate keys (1 GiB); inside one, the
  // front end (rotation, coarse scores, top-m, refine) runs over sub-chunks bounded by the
  // [sub-chunk, K] score matrix (512 MiB), so a large K does not cut the scan into small grids.
  // (the list scan's candidate rows: 2 GiB)
  int64_t by_keys = std::max<int64_t>(1, (1ll << 30) / ((int64_t)sp.slices * sp.R * 8));
  if (sp.lists) by_keys = std::min<int64_t>(by_keys, std::max<int64_t>(1, (1ll << 31) / ((int64_t)sp.lcap * 8)));
  const int64_t chunk = std::min<int64_t>(nq, std::min<int64_t>(by_keys, 65535ll * 64));
  Scratch sc(s);
  float* Qr_buf = Qr_pre ? nullptr : sc.get<float>((size_t)chunk * ix.Dp);
  const int64_t fe_chunk = coarse_rows_per_call(Qr_pre ? Qr_pre : Qr_buf, ix.C_rot, ix.K, ix.Dp, sp.m, chunk);
  const CoarseScratch cs =
      coarse_scratch(sc, Qr_pre ? Qr_pre : Qr_buf, ix.C_rot, ix.K, ix.Dp, sp.m, fe_chunk);
  int32_t* probes = sc.get<int32_t>((size_t)chunk * sp.P);
  float* g = sc.get<float>((size_t)chunk * sp.P);
  const int pb = prep_bits_of(sp.qbits);
  uint32_t* planes = sc.get<uint32_t>((size_t)chunk * pb * ix.W);
  const float qt = query_t(ix, pb);
  float* delta = sc.get<float>(chunk);
  float* k1 = sc.get<float>(chunk);
  unsigned long long* keys_s = sc.get<unsigned long long>((size_t)chunk * sp.slices * sp.R);
  unsigned long long* keys = sp.slices > 1 ? sc.get<unsigned long long>((size_t)chunk * sp.R) : keys_s;
  float* tau_a = sp.seeded || sp.lists ? sc.get<float>((size_t)chunk) : nullptr;
  int32_t* qorder = chunk >= kQueryOrderMinBatch ? sc.get<int32_t>((size_t)ix.K + 2 + chunk) : nullptr;
  ListScanScratch lw{};
  if (sp.lists) lw = list_scan_scratch(sc, ix, chunk, sp.P, sp.lcap, sp.R);
  for (int64_t a = 0; a < nq; a += chunk) {
    const int64_t cn = std::min(chunk, nq - a);
    const float* Qc = Q + a * ix.D;
    const float* Qr = Qr_pre ? Qr_pre + a * ix.Dp : Qr_buf;
    for (int64_t b = 0; b < cn; b += fe_chunk) {
      Range r("rbq front end (rotate, coarse, top-m, refine)");
      const int64_t fn = std::min(fe_chunk, cn - b);
      const float* Qrb = Qr + b * ix.Dp;
      if (!Qr_pre) launch_rotate(Qc + b * ix.D, fn, ix.D, ix.Dp, ix.P, Qr_buf + b * ix.Dp, s);
      coarse_probes(ix, Qrb, fn, ix.C_rot, ix.C_rot_n2, ix.C_rot_n2_max, ix.K, ix.Dp, sp.m, sp.P, cs,
                    probes + b * sp.P, g + b * sp.P, s);
    }
    launch_query_prep(Qr, cn, ix.Dp, qt, pb, planes, delta, k1, s);
    {
      Range r("rbq scan");
      search_scan(ix, sp, Qr, planes, delta, k1, cn, probes, g, tau_a, keys_s, keys, stats, qorder, &lw, s);
    }
    Range r("rbq rerank / result");
    if (params.rerank > 0)
      launch_rerank(ix.X_r, ix.id2row, ix.D, Qc, cn, keys, sp.R, sp.k, dist + a * sp.k, ids + a * sp.k, s);
    else
      launch_keys_to_result(keys, cn, sp.R, sp.k, dist + a * sp.k, ids + a * sp.k, s);
  }
}

// The captured search of batch size nq and parameters p (p.graph ignored): found in the
// index's cache or captured now.  The capture runs run_search on a private stream into the
// graph's own buffers, so its scratch allocations become graph allocation / free nodes and
// every replay allocates and frees its own.
Index::SearchGraph& search_graph(Index& ix, const rbq_search_params_t& params, int64_t nq)
{
  rbq_search_params_t key = params;
  key.graph = 0;
  for (auto& g : ix.graphs)
    if (g.nq == nq && std::memcmp(&g.p, &key, sizeof key) == 0) return g;
  plan_search(ix, key, nq);  // argument errors before any allocation
  if (ix.graphs.size() >= 8) {
    Index::SearchGraph& old = ix.graphs.front();
    if (old.exec) cudaGraphExecDestroy(old.exec);
    if (old.done) cudaEventDestroy(old.done);
    dev_free(old.q);
    dev_free(old.d);
    dev_free(old.i);
    ix.graphs.erase(ix.graphs.begin());
  }
  Index::SearchGraph g;
  g.nq = nq;
  g.p = key;
  cudaStream_t cs = nullptr;
  cudaGraph_t graph = nullptr;
  try {
    g.q = dev_alloc<float>((size_t)nq * ix.D);
    g.d = dev_alloc<float>((size_t)nq * key.k);
    g.i = dev_alloc<int64_t>((size_t)nq * key.k);
    RBQ_CUDA(cudaEventCreateWithFlags(&g.done, cudaEventDisableTiming));
    RBQ_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
    RBQ_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeRelaxed));
    try {
      run_search(ix, key, g.q, nq, g.d, g.i, cs, nullptr);
    } catch (...) {
      cudaStreamEndCapture(cs, &graph);
      throw;
    }
    RBQ_CUDA(cudaStreamEndCapture(cs, &graph));
    RBQ_CUDA(cudaGraphInstantiate(&g.exec, graph, 0));
    cudaGraphDestroy(graph);
    graph = nullptr;
    cudaStreamDestroy(cs);
    cs = nullptr;
  } catch (...) {
    if (graph) cudaGraphDestroy(graph);
    if (cs) cudaStreamDestroy(cs);
    if (g.exec) cudaGraphExecDestroy(g.exec);
    if (g.done) cudaEventDestroy(g.done);
    cudaGetLastError();
    dev_free(g.q);
    dev_free(g.d);
    dev_free(g.i);
    throw;
  }
  ix.graphs.push_back(g);
  return ix.graphs.back();
}

// ---------------------------------------------------------------------------------------
// Persistence: "RBQB200\0", version, dims, seed, t4, P, C, then this shard's rows.
// ---------------------------------------------------------------------------------------
const char kMagic[8] = {'R', 'B', 'Q', 'B', '2', '0', '0', '\0'};
// 2 adds the shard policy and list -> rank map; 3 the extra-bit count and scale after the map and
// the extra-bit planes and factors after the 1-bit factors
constexpr uint32_t kFormatVersion = 3;

struct File {
  FILE* f = nullptr;
  std::string path;
  File(const char* p, const char* mode) : path(p ? p : "")
  {
    RBQ_CHECK(p != nullptr, RBQ_ERR_INVALID, "null path");
    f = std::fopen(p, mode);
    RBQ_CHECK(f != nullptr, RBQ_ERR_IO, "cannot open " + path);
  }
  ~File()
  {
    if (f) std::fclose(f);
  }
  void write(const void* d, size_t n)
  {
    if (n) RBQ_CHECK(std::fwrite(d, 1, n, f) == n, RBQ_ERR_IO, "write failed: " + path);
  }
  void read(void* d, size_t n)
  {
    if (n) RBQ_CHECK(std::fread(d, 1, n, f) == n, RBQ_ERR_FORMAT, "truncated index file: " + path);
  }
};

template <typename T>
void write_dev(File& f, const T* p, size_t count)
{
  std::vector<T> h(count);
  if (count) RBQ_CUDA(cudaMemcpy(h.data(), p, count * sizeof(T), cudaMemcpyDefault));  // device or mapped host
  f.write(h.data(), count * sizeof(T));
}

struct RefFile {
  uint64_t n = 0, D = 0, K = 0, ex_bits = 0;
  float t4 = 0.0f, t8 = 0.0f;
  std::vector<uint64_t> sizes;
  std::vector<float> P, Crot, fac, exfac;
  std::vector<uint32_t> codes, ids;
  std::vector<uint8_t> long_codes;  // n x Dp * ex_bits / 8
};

// The reference's long code of one vector (extra-bit codes of Dp dims, ex bits each, one
// MSB-first bit stream: exrabitq_fused_kernel_batch's packing, quantizer_gpu.cu:470-505, read
// back by extract_code, searcher_gpu_common.cuh:72-81) <-> this library's planes [ex, W].
void long_code_to_planes(const uint8_t* lc, int Dp, int ex, uint32_t* planes)
{
  const int W = Dp / 32;
  std::fill(planes, planes + (size_t)ex * W, 0u);
  for (int j = 0; j < Dp; ++j) {
    uint32_t x = 0;
    for (int b = 0; b < ex; ++b) {
      const size_t pos = (size_t)j * ex + b;
      x = (x << 1) | ((lc[pos >> 3] >> (7 - (pos & 7))) & 1u);
    }
    for (int p = 0; p < ex; ++p)
      if ((x >> p) & 1u) planes[(size_t)p * W + (j >> 5)] |= 1u << (31 - (j & 31));
  }
}

void planes_to_long_code(const uint32_t* planes, int Dp, int ex, uint8_t* lc)
{
  const int W = Dp / 32;
  std::fill(lc, lc + (size_t)Dp * ex / 8, (uint8_t)0);
  for (int j = 0; j < Dp; ++j) {
    uint32_t x = 0;
    for (int p = 0; p < ex; ++p) x |= ((planes[(size_t)p * W + (j >> 5)] >> (31 - (j & 31))) & 1u) << p;
    for (int b = 0; b < ex; ++b) {
      const size_t pos = (size_t)j * ex + b;
      if ((x >> (ex - 1 - b)) & 1u) lc[pos >> 3] |= (uint8_t)(1u << (7 - (pos & 7)));
    }
  }
}

RefFile read_ref_file(const char* path)
{
  File f(path, "rb");
  RefFile r;
  f.read(&r.n, 8);
  f.read(&r.D, 8);
  f.read(&r.K, 8);
  f.read(&r.ex_bits, 8);
  RBQ_CHECK(r.D >= 1 && r.D <= 2048 && r.K >= 1 && r.K <= (1u << 24) && r.n < 0xFFFFFFFFull, RBQ_ERR_FORMAT,
            "not a reference IVF-RaBitQ index (bad header): " + f.path);
  RBQ_CHECK(r.ex_bits <= 8, RBQ_ERR_FORMAT,
            "reference index with " + std::to_string(r.ex_bits) + " extra bits: at most 8 are supported");
  unsigned char flag = 0;
  f.read(&flag, 1);
  f.read(&r.t4, 4);
  f.read(&r.t8, 4);
  r.sizes.resize(r.K);
  f.read(r.sizes.data(), r.K * 8);
  uint64_t tot = 0;
  for (uint64_t c : r.sizes) tot += c;
  RBQ_CHECK(tot == r.n, RBQ_ERR_FORMAT, "cluster sizes do not sum to num_vectors: " + f.path);
  unsigned char kind = 0;
  f.read(&kind, 1);
  RBQ_CHECK(kind == 0, RBQ_ERR_FORMAT, "reference index uses the FHT-Kac rotator: only the matmul rotator is supported");
  const uint64_t Dp = (r.D + 31) / 32 * 32, W = Dp / 32;
  r.P.resize(Dp * Dp);
  f.read(r.P.data(), r.P.size() * 4);
  r.Crot.resize(r.K * Dp);
  f.read(r.Crot.data(), r.Crot.size() * 4);
  r.codes.resize(r.n * W);
  f.read(r.codes.data(), r.codes.size() * 4);
  r.fac.resize(r.n * 3);
  f.read(r.fac.data(), r.fac.size() * 4);
  r.long_codes.resize(r.n * (Dp * r.ex_bits / 8));
  f.read(r.long_codes.data(), r.long_codes.size());
  r.exfac.resize(r.n * 2);  // {f_ex_add, f_ex_rescale}; written but unused at 1 bit
  f.read(r.exfac.data(), r.exfac.size() * 4);
  r.ids.resize(r.n);
  f.read(r.ids.data(), r.n * 4);
  for (uint32_t id : r.ids) RBQ_CHECK(id < r.n, RBQ_ERR_FORMAT, "reference index id out of range: " + f.path);
  return r;
}

}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }

static std::atomic<uint64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

std::vector<int32_t> list_owners(int policy, const std::vector<int64_t>& sizes, int count)
{
  const int K = (int)sizes.size();
  std::vector<int32_t> own(K, 0);
  if (count <= 1) return own;
  if (policy == RBQ_SHARD_ROUND_ROBIN) {
    for (int l = 0; l < K; ++l) own[l] = l % count;
    return own;
  }
  // BALANCED: lists by decreasing size^2 (ties: smaller id), each to the least-loaded rank.
  std::vector<int> order(K);
  for (int l = 0; l < K; ++l) order[l] = l;
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return sizes[a] * sizes[a] > sizes[b] * sizes[b]; });
  std::vector<int64_t> load(count, 0);
  for (int l : order) {
    int r = 0;
    for (int j = 1; j < count; ++j)
      if (load[j] < load[r]) r = j;
    own[l] = r;
    load[r] += sizes[l] * sizes[l];
  }
  return own;
}

void install_owners(Index& ix, const std::vector<int32_t>& owners, bool fixed)
{
  RBQ_CHECK((int)owners.size() == ix.K, RBQ_ERR_INVALID, "owner map size mismatch");
  for (int32_t o : owners) RBQ_CHECK(o >= 0 && o < ix.shard_count, RBQ_ERR_INVALID, "owner out of range");
  if (!ix.owner) ix.owner = dev_alloc<int32_t>(ix.K);
  RBQ_CUDA(cudaMemcpy(ix.owner, owners.data(), (size_t)ix.K * 4, cudaMemcpyHostToDevice));
  ix.owner_host = owners;
  ix.owners_fixed = fixed;
}

void drop_graphs(Index& ix)
{
  for (auto& g : ix.graphs) {
    if (g.exec) cudaGraphExecDestroy(g.exec);
    if (g.done) cudaEventDestroy(g.done);
    dev_free(g.q);
    dev_free(g.d);
    dev_free(g.i);
  }
  ix.graphs.clear();
}

void free_index_memory(Index& ix)
{
  drop_graphs(ix);
  dev_free(ix.P);
  dev_free(ix.C);
  dev_free(ix.C_rot);
  dev_free(ix.C_rot_n2);
  dev_free(ix.C_rot_n2_max);
  dev_free(ix.C_n2);
  raw_free(ix, ix.X_r);
  dev_free(ix.codes_r);
  dev_free(ix.fadd_r);
  dev_free(ix.frescale_r);
  dev_free(ix.ferr_r);
  dev_free(ix.ex_codes_r);
  dev_free(ix.fexadd_r);
  dev_free(ix.fexr_r);
  dev_free(ix.labels_r);
  dev_free(ix.ids_r);
  dev_free(ix.id2row);
  dev_free(ix.dev_err);
  dev_free(ix.owner);
  if (ix.copy_stream) {
    cudaStreamDestroy(ix.copy_stream);
    ix.copy_stream = nullptr;
  }
  dev_free(ix.list_off);
  dev_free(ix.ids);
  dev_free(ix.codes);
  dev_free(ix.fadd);
  dev_free(ix.frescale);
  dev_free(ix.ferr);
  dev_free(ix.ex_codes);
  dev_free(ix.fexadd);
  dev_free(ix.fexr);
}

}  // namespace rbq

using namespace rbq;

extern "C" {

const char* rbq_last_error(void) { return g_last_error.c_str(); }

int rbq_version(void) { return 1; }

int rbq_debug_fail_alloc(int64_t after)
{
  g_fail_alloc_after.store(after < 0 ? -1 : after);
  return RBQ_OK;
}

uint64_t rbq_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

int rbq_scan_tile(void) { return rbq::kScanTile; }

void rbq_index_params_default(rbq_index_params_t* p)
{
  if (!p) return;
  p->dim = 0;
  p->n_lists = 1024;
  p->seed = 7;
  p->kmeans_n_iters = 20;
  p->max_train_points_per_cluster = 256;
  p->device = 0;
  p->shard_rank = 0;
  p->shard_count = 1;
  p->shard_policy = RBQ_SHARD_ROUND_ROBIN;
  p->kmeans_kind = RBQ_KMEANS_BALANCED;
  p->raw_store = RBQ_RAW_DEVICE;
  p->bits_per_dim = 1;
}

void rbq_search_params_default(rbq_search_params_t* p)
{
  if (!p) return;
  p->n_probes = 20;
  p->query_bits = 4;
  p->k = 10;
  p->rerank = 0;
  p->prune = 1;
  p->probe_split = 0;
  p->cand_cap = 0;
  p->coarse_margin = 0;
  p->seeded = -1;
  p->graph = 0;
  p->scan_kind = 0;
}

int rbq_make_rotation(int32_t padded_dim, uint64_t seed, float* P_host)
{
  return guarded([&] {
    RBQ_CHECK(P_host && padded_dim >= 32 && padded_dim % 32 == 0 && padded_dim <= 2048, RBQ_ERR_INVALID,
              "padded_dim must be a multiple of 32 in [32, 2048]");
    make_rotation(padded_dim, seed, P_host);
  });
}

int rbq_query_scale(int32_t padded_dim, uint64_t seed, int32_t ex_bits, float* t_out)
{
  return guarded([&] {
    RBQ_CHECK(t_out && padded_dim >= 1 && ex_bits >= 1 && ex_bits <= 8, RBQ_ERR_INVALID, "bad arguments");
    *t_out = query_scale(padded_dim, seed, ex_bits);
  });
}

int rbq_index_create(const rbq_index_params_t* params, rbq_index_t** out)
{
  return guarded([&] {
    RBQ_CHECK(params && out, RBQ_ERR_INVALID, "null argument");
    *out = nullptr;
    RBQ_CHECK(params->dim >= 1 && params->dim <= 2048, RBQ_ERR_INVALID, "dim must be in [1, 2048]");
    RBQ_CHECK(params->n_lists >= 1, RBQ_ERR_INVALID, "n_lists must be >= 1");
    RBQ_CHECK(params->shard_count >= 1 && params->shard_rank >= 0 && params->shard_rank < params->shard_count,
              RBQ_ERR_INVALID, "bad shard rank / count");
    RBQ_CHECK(params->kmeans_n_iters >= 0 && params->max_train_points_per_cluster >= 1, RBQ_ERR_INVALID,
              "bad k-means parameters");
    RBQ_CHECK(params->shard_policy == RBQ_SHARD_ROUND_ROBIN || params->shard_policy == RBQ_SHARD_BALANCED,
              RBQ_ERR_INVALID, "unknown shard policy");
    RBQ_CHECK(params->kmeans_kind == RBQ_KMEANS_BALANCED || params->kmeans_kind == RBQ_KMEANS_LLOYD,
              RBQ_ERR_INVALID, "unknown k-means kind");
    RBQ_CHECK(params->raw_store == RBQ_RAW_DEVICE || params->raw_store == RBQ_RAW_HOST, RBQ_ERR_INVALID,
              "unknown raw store (RBQ_RAW_DEVICE or RBQ_RAW_HOST)");
    RBQ_CHECK(params->bits_per_dim >= 1 && params->bits_per_dim <= 9, RBQ_ERR_INVALID,
              "bits_per_dim must be in [1, 9]");
    int ndev = 0;
    RBQ_CUDA(cudaGetDeviceCount(&ndev));
    RBQ_CHECK(params->device >= 0 && params->device < ndev, RBQ_ERR_INVALID, "device ordinal out of range");
    DeviceGuard dg(params->device);
    keep_pool_cached(params->device);
    rbq_index* h = new rbq_index();
    Index& ix = h->ix;
    ix.device = params->device;
    ix.D = params->dim;
    ix.Dp = (params->dim + 31) / 32 * 32;
    ix.W = ix.Dp / 32;
    ix.K = params->n_lists;
    ix.seed = params->seed;
    ix.kmeans_iters = params->kmeans_n_iters;
    ix.kmeans_kind = params->kmeans_kind;
    ix.raw_on_host = params->raw_store == RBQ_RAW_HOST;
    ix.max_train_per_list = params->max_train_points_per_cluster;
    ix.shard_rank = params->shard_rank;
    ix.shard_count = params->shard_count;
    ix.shard_policy = params->shard_policy;
    try {
      install_owners(ix, list_owners(RBQ_SHARD_ROUND_ROBIN, std::vector<int64_t>(ix.K, 0), ix.shard_count),
                     ix.shard_policy == RBQ_SHARD_ROUND_ROBIN || ix.shard_count == 1);
      ix.P_host.resize((size_t)ix.Dp * ix.Dp);
      make_rotation(ix.Dp, ix.seed, ix.P_host.data());
      ix.t4 = query_scale(ix.Dp, ix.seed, 3);
      ix.ex_bits = params->bits_per_dim - 1;
      ix.tex = ex_scale_of(ix);
      ix.P = dev_alloc<float>(ix.P_host.size());
      ix.dev_err = dev_alloc<int>(1);
      RBQ_CUDA(cudaMemset(ix.dev_err, 0, sizeof(int)));
      RBQ_CUDA(cudaMemcpy(ix.P, ix.P_host.data(), ix.P_host.size() * 4, cudaMemcpyHostToDevice));
      ix.off_host.assign(ix.K + 1, 0);
      ix.list_off = dev_alloc<int64_t>(ix.K + 1);
      RBQ_CUDA(cudaMemset(ix.list_off, 0, (ix.K + 1) * 8));
    } catch (...) {
      free_index_memory(ix);
      delete h;
      throw;
    }
    *out = h;
  });
}

int rbq_index_free(rbq_index_t* index)
{
  return guarded([&] {
    if (!index) return;
    {
      DeviceGuard dg(index->ix.device);
      free_index_memory(index->ix);
    }
    delete index;
  });
}

int rbq_index_info(rbq_index_t* index, rbq_index_info_t* out)
{
  return guarded([&] {
    RBQ_CHECK(index && out, RBQ_ERR_INVALID, "null argument");
    const Index& ix = index->ix;
    out->dim = ix.D;
    out->padded_dim = ix.Dp;
    out->n_lists = ix.K;
    out->shard_rank = ix.shard_rank;
    out->shard_count = ix.shard_count;
    out->trained = ix.trained ? 1 : 0;
    out->n_total = ix.n_total;
    out->n_local = ix.n_rows;
    out->query_scale = ix.t4;
    out->seed = ix.seed;
    const int64_t per_row = (int64_t)ix.D * 4 + (int64_t)ix.W * 4 * 2 + 12 * 2 + 4 * 3 +
                            ((int64_t)ix.ex_bits * ix.W * 4 + 8) * 2 * (ix.ex_bits > 0);
    out->device_bytes = ix.cap_rows * per_row + ix.cap_ids * 4 + (int64_t)ix.Dp * ix.Dp * 4 +
                        (int64_t)ix.K * (ix.D + ix.Dp + 3) * 4 + (ix.K + 1) * 8;
    out->shard_policy = ix.shard_policy;
    out->owners_fixed = ix.owners_fixed ? 1 : 0;
    out->kmeans_kind = ix.kmeans_kind;
    out->bits_per_dim = ix.ex_bits + 1;
    out->ex_scale = ix.tex;
  });
}

int rbq_get_list_owners(rbq_index_t* index, int32_t* owners)
{
  return guarded([&] {
    RBQ_CHECK(index && owners, RBQ_ERR_INVALID, "null argument");
    const Index& ix = index->ix;
    for (int l = 0; l < ix.K; ++l) owners[l] = ix.owners_fixed ? ix.owner_host[l] : -1;
  });
}

int rbq_train(rbq_index_t* index, const float* X_dev, int64_t n, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_train");
    RBQ_CHECK(index && X_dev, RBQ_ERR_INVALID, "null argument");
    DeviceGuard dg(index->ix.device);
    train_kmeans(index->ix, X_dev, n, as_stream(stream));
  });
}

int rbq_build(rbq_index_t* index, const float* X_dev, int64_t n, int32_t d, const float* C_host,
              const uint32_t* labels_dev, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_build");
    RBQ_CHECK(index && X_dev, RBQ_ERR_INVALID, "null argument");
    Index& ix = index->ix;
    RBQ_CHECK(d == ix.D, RBQ_ERR_INVALID, "build: dim " + std::to_string(d) + " != index dim " + std::to_string(ix.D));
    RBQ_CHECK(!labels_dev || C_host, RBQ_ERR_INVALID, "build: labels need the centroids they refer to");
    RBQ_CHECK(ix.n_total == 0, RBQ_ERR_STATE, "build: index already holds vectors");
    DeviceGuard dg(ix.device);
    cudaStream_t s = as_stream(stream);
    if (C_host) {
      ix.C_host.assign(C_host, C_host + (size_t)ix.K * ix.D);
      install_centroids(ix, s);
    } else {
      train_kmeans(ix, X_dev, n, s);
    }
    add_rows(ix, X_dev, n, labels_dev, s);
  });
}

int rbq_set_centroids(rbq_index_t* index, const float* C_host, int32_t n_lists)
{
  return guarded([&] {
    RBQ_CHECK(index && C_host, RBQ_ERR_INVALID, "null argument");
    Index& ix = index->ix;
    RBQ_CHECK(n_lists == ix.K, RBQ_ERR_INVALID, "set_centroids: n_lists mismatch");
    RBQ_CHECK(ix.n_total == 0, RBQ_ERR_STATE, "set_centroids: index already holds vectors");
    DeviceGuard dg(ix.device);
    ix.C_host.assign(C_host, C_host + (size_t)ix.K * ix.D);
    install_centroids(ix, 0);
  });
}

int rbq_add(rbq_index_t* index, const float* X_dev, int64_t n, const uint32_t* labels_dev, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_add");
    RBQ_CHECK(index && (X_dev || n == 0), RBQ_ERR_INVALID, "null argument");
    DeviceGuard dg(index->ix.device);
    add_rows(index->ix, X_dev, n, labels_dev, as_stream(stream));
  });
}

int rbq_search(rbq_index_t* index, const rbq_search_params_t* params, const float* Q_dev, int64_t nq,
               float* dist_dev, int64_t* ids_dev, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_search");
    RBQ_CHECK(index && params, RBQ_ERR_INVALID, "null argument");
    RBQ_CHECK(nq == 0 || (Q_dev && dist_dev && ids_dev), RBQ_ERR_INVALID, "null buffer");
    DeviceGuard dg(index->ix.device);
    Index& ix = index->ix;
    cudaStream_t s = as_stream(stream);
    if (params->graph && nq > 0) {
      Index::SearchGraph& g = search_graph(ix, *params, nq);
      RBQ_CUDA(cudaStreamWaitEvent(s, g.done, 0));  // the previous replay's results are out
      RBQ_CUDA(cudaMemcpyAsync(g.q, Q_dev, (size_t)nq * ix.D * 4, cudaMemcpyDeviceToDevice, s));
      RBQ_CUDA(cudaGraphLaunch(g.exec, s));
      RBQ_CUDA(cudaMemcpyAsync(dist_dev, g.d, (size_t)nq * params->k * 4, cudaMemcpyDeviceToDevice, s));
      RBQ_CUDA(cudaMemcpyAsync(ids_dev, g.i, (size_t)nq * params->k * 8, cudaMemcpyDeviceToDevice, s));
      RBQ_CUDA(cudaEventRecord(g.done, s));
      return;
    }
    run_search(ix, *params, Q_dev, nq, dist_dev, ids_dev, s, nullptr);
  });
}

int rbq_search_host(rbq_index_t* index, const rbq_search_params_t* params, const float* Q_host, int64_t nq,
                    float* dist_host, int64_t* ids_host, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_search_host");
    RBQ_CHECK(index && params, RBQ_ERR_INVALID, "null argument");
    RBQ_CHECK(nq == 0 || (Q_host && dist_host && ids_host), RBQ_ERR_INVALID, "null buffer");
    if (nq == 0) return;
    Index& ix = index->ix;
    DeviceGuard dg(ix.device);
    cudaStream_t s = as_stream(stream);
    const int k = params->k;
    RBQ_CHECK(k >= 1, RBQ_ERR_INVALID, "search: k must be >= 1");
    // Batches of >= 4096 queries are uploaded in two halves on a copy stream: the first half is
    // rotated while the second crosses PCIe, then the whole batch is searched at once (the same
    // plan and results as a device-side search of the batch).
    constexpr int64_t kMinHalf = 2048;
    if (params->graph) {  // the captured search reads and writes its own buffers
      Index::SearchGraph& g = search_graph(ix, *params, nq);
      RBQ_CUDA(cudaStreamWaitEvent(s, g.done, 0));  // the previous replay's results are out
      RBQ_CUDA(cudaMemcpyAsync(g.q, Q_host, (size_t)nq * ix.D * 4, cudaMemcpyHostToDevice, s));
      RBQ_CUDA(cudaGraphLaunch(g.exec, s));
      RBQ_CUDA(cudaMemcpyAsync(dist_host, g.d, (size_t)nq * k * 4, cudaMemcpyDeviceToHost, s));
      RBQ_CUDA(cudaMemcpyAsync(ids_host, g.i, (size_t)nq * k * 8, cudaMemcpyDeviceToHost, s));
      RBQ_CUDA(cudaEventRecord(g.done, s));
    } else {
      Scratch sc(s);
      float* q = sc.get<float>((size_t)nq * ix.D);
      float* d = sc.get<float>((size_t)nq * k);
      int64_t* i = sc.get<int64_t>((size_t)nq * k);
      if (nq < 2 * kMinHalf) {
        RBQ_CUDA(cudaMemcpyAsync(q, Q_host, (size_t)nq * ix.D * 4, cudaMemcpyHostToDevice, s));
        run_search(ix, *params, q, nq, d, i, s, nullptr);
      } else {
        if (!ix.copy_stream) RBQ_CUDA(cudaStreamCreateWithFlags(&ix.copy_stream, cudaStreamNonBlocking));
        cudaStream_t cs = ix.copy_stream;
        float* qr = sc.get<float>((size_t)nq * ix.Dp);
        cudaEvent_t ev[3];
        for (auto& e : ev) RBQ_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        try {
          const int64_t h = nq / 2;
          RBQ_CUDA(cudaEventRecord(ev[0], s));  // the scratch buffers exist on s
          RBQ_CUDA(cudaStreamWaitEvent(cs, ev[0], 0));
          RBQ_CUDA(cudaMemcpyAsync(q, Q_host, (size_t)h * ix.D * 4, cudaMemcpyHostToDevice, cs));
          RBQ_CUDA(cudaEventRecord(ev[1], cs));
          RBQ_CUDA(cudaMemcpyAsync(q + h * ix.D, Q_host + h * ix.D, (size_t)(nq - h) * ix.D * 4,
                                   cudaMemcpyHostToDevice, cs));
          RBQ_CUDA(cudaEventRecord(ev[2], cs));
          RBQ_CUDA(cudaStreamWaitEvent(s, ev[1], 0));
          launch_rotate(q, h, ix.D, ix.Dp, ix.P, qr, s);
          RBQ_CUDA(cudaStreamWaitEvent(s, ev[2], 0));
          launch_rotate(q + h * ix.D, nq - h, ix.D, ix.Dp, ix.P, qr + h * ix.Dp, s);
          run_search(ix, *params, q, nq, d, i, s, nullptr, qr);
        } catch (...) {
          cudaStreamSynchronize(cs);
          for (auto& e : ev) cudaEventDestroy(e);
          throw;
        }
        for (auto& e : ev) RBQ_CUDA(cudaEventDestroy(e));
      }
      RBQ_CUDA(cudaMemcpyAsync(dist_host, d, (size_t)nq * k * 4, cudaMemcpyDeviceToHost, s));
      RBQ_CUDA(cudaMemcpyAsync(ids_host, i, (size_t)nq * k * 8, cudaMemcpyDeviceToHost, s));
    }
    int code = 0;
    RBQ_CUDA(cudaMemcpyAsync(&code, ix.dev_err, sizeof(int), cudaMemcpyDeviceToHost, s));
    RBQ_CUDA(cudaStreamSynchronize(s));
    if (code) {
      RBQ_CUDA(cudaMemset(ix.dev_err, 0, sizeof(int)));
      throw Error{RBQ_ERR_CUDA, "a tensor-core pipeline wait timed out on the device (code " + std::to_string(code) + ")"};
    }
  });
}

int rbq_save(rbq_index_t* index, const char* path)
{
  return guarded([&] {
    Range nvtx_range("rbq_save");
    RBQ_CHECK(index, RBQ_ERR_INVALID, "null index");
    Index& ix = index->ix;
    DeviceGuard dg(ix.device);
    RBQ_CUDA(cudaDeviceSynchronize());
    File f(path, "wb");
    f.write(kMagic, 8);
    f.write(&kFormatVersion, 4);
    // hdr[7]: bit 0 trained, bit 1 no raw rows (an index imported without its vectors),
    // bit 2 Lloyd k-means (else balanced)
    int32_t hdr[8] = {ix.D, ix.Dp, ix.K, ix.kmeans_iters, ix.max_train_per_list, ix.shard_rank, ix.shard_count,
                      (ix.trained ? 1 : 0) | (ix.has_raw ? 0 : 2) | (ix.kmeans_kind == RBQ_KMEANS_LLOYD ? 4 : 0)};
    f.write(hdr, sizeof(hdr));
    f.write(&ix.seed, 8);
    f.write(&ix.t4, 4);
    f.write(&ix.n_total, 8);
    f.write(&ix.n_rows, 8);
    const int32_t pol[2] = {ix.shard_policy, ix.owners_fixed ? 1 : 0};
    f.write(pol, sizeof(pol));
    f.write(ix.owner_host.data(), (size_t)ix.K * 4);
    const int32_t exb = ix.ex_bits;
    f.write(&exb, 4);
    f.write(&ix.tex, 4);
    f.write(ix.P_host.data(), ix.P_host.size() * 4);
    if (ix.trained) f.write(ix.C_host.data(), ix.C_host.size() * 4);
    const size_t n = (size_t)ix.n_rows;
    write_dev(f, ix.labels_r, n);
    write_dev(f, ix.ids_r, n);
    write_dev(f, ix.codes_r, n * ix.W);
    write_dev(f, ix.fadd_r, n);
    write_dev(f, ix.frescale_r, n);
    write_dev(f, ix.ferr_r, n);
    if (ix.ex_bits > 0) {
      write_dev(f, ix.ex_codes_r, n * ix.ex_bits * ix.W);
      write_dev(f, ix.fexadd_r, n);
      write_dev(f, ix.fexr_r, n);
    }
    write_dev(f, ix.X_r, n * ix.D);
  });
}

int rbq_load(const char* path, int32_t device, int32_t shard_rank, int32_t shard_count, rbq_index_t** out)
{
  return guarded([&] {
    Range nvtx_range("rbq_load");
    RBQ_CHECK(out, RBQ_ERR_INVALID, "null argument");
    *out = nullptr;
    File f(path, "rb");
    char magic[8];
    f.read(magic, 8);
    RBQ_CHECK(std::memcmp(magic, kMagic, 8) == 0, RBQ_ERR_FORMAT, "not an RBQB200 index file: " + f.path);
    uint32_t ver = 0;
    f.read(&ver, 4);
    RBQ_CHECK(ver >= 1 && ver <= kFormatVersion, RBQ_ERR_FORMAT, "unsupported index file version");
    int32_t hdr[8];
    f.read(hdr, sizeof(hdr));
    uint64_t seed;
    float t4;
    int64_t n_total, n_rows;
    f.read(&seed, 8);
    f.read(&t4, 4);
    f.read(&n_total, 8);
    f.read(&n_rows, 8);
    const int D = hdr[0], Dp = hdr[1], K = hdr[2];
    RBQ_CHECK(D >= 1 && D <= 2048 && Dp == (D + 31) / 32 * 32 && K >= 1 && n_rows >= 0 && n_total >= n_rows,
              RBQ_ERR_FORMAT, "corrupt index header");
    const int file_rank = hdr[5], file_count = hdr[6];
    RBQ_CHECK(file_count >= 1 && file_rank >= 0 && file_rank < file_count, RBQ_ERR_FORMAT, "corrupt shard header");
    int32_t pol[2] = {RBQ_SHARD_ROUND_ROBIN, 1};  // version 1: round robin
    std::vector<int32_t> file_owner;
    if (ver >= 2) {
      f.read(pol, sizeof(pol));
      RBQ_CHECK(pol[0] == RBQ_SHARD_ROUND_ROBIN || pol[0] == RBQ_SHARD_BALANCED, RBQ_ERR_FORMAT,
                "corrupt shard policy");
      file_owner.resize(K);
      f.read(file_owner.data(), (size_t)K * 4);
    }
    int32_t exb = 0;
    float tex = 0.0f;
    if (ver >= 3) {
      f.read(&exb, 4);
      f.read(&tex, 4);
      RBQ_CHECK(exb >= 0 && exb <= 8, RBQ_ERR_FORMAT, "corrupt extra-bit count");
    }
    if (shard_count <= 0) {
      shard_count = file_count;
      shard_rank = file_rank;
    }
    RBQ_CHECK(file_count == 1 || (file_count == shard_count && file_rank == shard_rank), RBQ_ERR_INVALID,
              "index file holds shard " + std::to_string(file_rank) + "/" + std::to_string(file_count));
    rbq_index_params_t p;
    rbq_index_params_default(&p);
    p.dim = D;
    p.n_lists = K;
    p.seed = seed;
    p.kmeans_n_iters = hdr[3];
    p.max_train_points_per_cluster = hdr[4];
    p.device = device;
    p.shard_rank = shard_rank;
    p.shard_count = shard_count;
    RBQ_CHECK(p.shard_count >= 1 && p.shard_rank >= 0 && p.shard_rank < p.shard_count, RBQ_ERR_INVALID,
              "bad shard rank / count");
    int ndev = 0;
    RBQ_CUDA(cudaGetDeviceCount(&ndev));
    RBQ_CHECK(device >= 0 && device < ndev, RBQ_ERR_INVALID, "device ordinal out of range");
    DeviceGuard dg(device);
    keep_pool_cached(device);
    rbq_index* h = new rbq_index();
    Index& ix = h->ix;
    try {
      ix.device = device;
      ix.D = D;
      ix.Dp = Dp;
      ix.W = Dp / 32;
      ix.K = K;
      ix.seed = seed;
      ix.kmeans_iters = p.kmeans_n_iters;
      ix.kmeans_kind = (hdr[7] & 4) ? RBQ_KMEANS_LLOYD : RBQ_KMEANS_BALANCED;
      ix.max_train_per_list = p.max_train_points_per_cluster;
      ix.shard_rank = p.shard_rank;
      ix.shard_count = p.shard_count;
      ix.shard_policy = pol[0];
      ix.has_raw = (hdr[7] & 2) == 0;
      ix.t4 = t4;
      ix.ex_bits = exb;
      ix.tex = tex;
      ix.P_host.resize((size_t)Dp * Dp);
      f.read(ix.P_host.data(), ix.P_host.size() * 4);
      ix.P = dev_alloc<float>(ix.P_host.size());
      ix.dev_err = dev_alloc<int>(1);
      RBQ_CUDA(cudaMemset(ix.dev_err, 0, sizeof(int)));
      RBQ_CUDA(cudaMemcpy(ix.P, ix.P_host.data(), ix.P_host.size() * 4, cudaMemcpyHostToDevice));
      ix.off_host.assign(K + 1, 0);
      ix.list_off = dev_alloc<int64_t>(K + 1);
      RBQ_CUDA(cudaMemset(ix.list_off, 0, (K + 1) * 8));
      if (hdr[7] & 1) {
        ix.C_host.resize((size_t)K * D);
        f.read(ix.C_host.data(), ix.C_host.size() * 4);
        install_centroids(ix, 0);
      }
      const int W = ix.W;
      std::vector<uint32_t> lab(n_rows), ids(n_rows), codes((size_t)n_rows * W);
      std::vector<float> fa(n_rows), fr(n_rows), fe(n_rows), X((size_t)n_rows * D);
      f.read(lab.data(), lab.size() * 4);
      f.read(ids.data(), ids.size() * 4);
      f.read(codes.data(), codes.size() * 4);
      f.read(fa.data(), fa.size() * 4);
      f.read(fr.data(), fr.size() * 4);
      f.read(fe.data(), fe.size() * 4);
      const int EW = exb * W;
      std::vector<uint32_t> xc((size_t)n_rows * EW);
      std::vector<float> xa(exb ? n_rows : 0), xr(exb ? n_rows : 0);
      if (exb) {
        f.read(xc.data(), xc.size() * 4);
        f.read(xa.data(), xa.size() * 4);
        f.read(xr.data(), xr.size() * 4);
      }
      f.read(X.data(), X.size() * 4);
      for (int64_t i = 0; i < n_rows; ++i)
        RBQ_CHECK(lab[i] < (uint32_t)K && ids[i] < (uint64_t)n_total, RBQ_ERR_FORMAT, "corrupt row data");
      // The list -> rank map: the file's own when it is this shard's file (or unsharded);
      // re-derived from the file's list sizes when a full index is loaded as one shard.
      if (file_count == ix.shard_count && ver >= 2) {
        install_owners(ix, file_owner, pol[1] != 0);
      } else {
        std::vector<int64_t> sizes(K, 0);
        for (int64_t i = 0; i < n_rows; ++i) ++sizes[lab[i]];
        install_owners(ix, list_owners(pol[0], sizes, ix.shard_count), ix.shard_policy == RBQ_SHARD_ROUND_ROBIN ||
                                                                          n_rows > 0 || ix.shard_count == 1);
      }
      std::vector<int64_t> keep;
      for (int64_t i = 0; i < n_rows; ++i)
        if (ix.owner_host[lab[i]] == ix.shard_rank) keep.push_back(i);
      const int64_t m = (int64_t)keep.size();
      auto pick_u32 = [&](const std::vector<uint32_t>& src, int w) {
        std::vector<uint32_t> o((size_t)m * w);
        for (int64_t i = 0; i < m; ++i)
          std::memcpy(&o[(size_t)i * w], &src[(size_t)keep[i] * w], (size_t)w * 4);
        return o;
      };
      auto pick_f32 = [&](const std::vector<float>& src, int w) {
        std::vector<float> o((size_t)m * w);
        for (int64_t i = 0; i < m; ++i)
          std::memcpy(&o[(size_t)i * w], &src[(size_t)keep[i] * w], (size_t)w * 4);
        return o;
      };
      ensure_id_capacity(ix, std::max<int64_t>(n_total, 1));
      ensure_row_capacity(ix, std::max<int64_t>(m, 1));
      auto up = [&](void* dst, const void* src, size_t bytes) {
        if (bytes) RBQ_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
      };
      auto l2 = pick_u32(lab, 1), i2 = pick_u32(ids, 1), c2 = pick_u32(codes, W);
      auto fa2 = pick_f32(fa, 1), fr2 = pick_f32(fr, 1), fe2 = pick_f32(fe, 1), x2 = pick_f32(X, D);
      up(ix.labels_r, l2.data(), m * 4);
      up(ix.ids_r, i2.data(), m * 4);
      up(ix.codes_r, c2.data(), (size_t)m * W * 4);
      up(ix.fadd_r, fa2.data(), m * 4);
      up(ix.frescale_r, fr2.data(), m * 4);
      up(ix.ferr_r, fe2.data(), m * 4);
      if (exb) {
        const auto xc2 = pick_u32(xc, EW);
        const auto xa2 = pick_f32(xa, 1), xr2 = pick_f32(xr, 1);
        up(ix.ex_codes_r, xc2.data(), (size_t)m * EW * 4);
        up(ix.fexadd_r, xa2.data(), m * 4);
        up(ix.fexr_r, xr2.data(), m * 4);
      }
      up(ix.X_r, x2.data(), (size_t)m * D * 4);
      std::vector<uint32_t> id2row(n_total, 0xFFFFFFFFu);
      for (int64_t i = 0; i < m; ++i) id2row[i2[i]] = (uint32_t)i;
      up(ix.id2row, id2row.data(), (size_t)n_total * 4);
      ix.n_rows = m;
      ix.n_total = n_total;
      relayout(ix, 0);
    } catch (...) {
      free_index_memory(ix);
      delete h;
      throw;
    }
    *out = h;
  });
}

// ---------------------------------------------------------------------------------------
// The reference's index file (IVFGPU::save, gpu_index/ivf_gpu.cu:367-461, read back by
// load_transposed, :100-289), a format that has to be alike to exchange indexes:
//   size_t num_vectors, num_dimensions, num_centroids, ex_bits; bool legacy flag;
//   float const_scaling_factor_4bit, const_scaling_factor_8bit;  size_t cluster_sizes[K];
//   rotator: uint8 kind (0 = matmul) + Dp x Dp f32 row-major (rotator_gpu.cu:93-112);
//   rotated centroids K x Dp f32 (initializer_gpu.cu:54-64);
//   1-bit codes n x Dp/32 u32, clusters in order, vector-major inside a cluster;
//   factors n x {f_add, f_rescale, f_err} f32; long codes n x Dp*ex_bits/8 bytes;
//   extra-bit factors n x 2 f32; ids n x u32; optional "RPR1" representatives block.
// Files with up to 8 extra bits (bits_per_dim <= 9) and the matmul rotator are accepted; extra
// bits are converted between the long-code bit stream and this library's planes.
// ---------------------------------------------------------------------------------------
int rbq_import_reference(const char* path, int32_t device, const float* X_host, int64_t n_x, int32_t shard_rank,
                         int32_t shard_count, int32_t shard_policy, rbq_index_t** out)
{
  return guarded([&] {
    Range nvtx_range("rbq_import_reference");
    RBQ_CHECK(out, RBQ_ERR_INVALID, "null argument");
    *out = nullptr;
    RefFile r = read_ref_file(path);
    RBQ_CHECK(!X_host || n_x == (int64_t)r.n, RBQ_ERR_INVALID,
              "raw vectors: " + std::to_string(n_x) + " rows given, the index holds " + std::to_string(r.n));
    rbq_index_params_t p;
    rbq_index_params_default(&p);
    p.dim = (int32_t)r.D;
    p.n_lists = (int32_t)r.K;
    p.seed = 0;
    p.device = device;
    p.shard_rank = shard_rank;
    p.shard_count = shard_count;
    p.shard_policy = shard_policy;
    p.bits_per_dim = (int32_t)r.ex_bits + 1;
    rbq_index_t* h = nullptr;
    int st = rbq_index_create(&p, &h);
    if (st != RBQ_OK) throw Error{st, g_last_error};
    Index& ix = h->ix;
    try {
      DeviceGuard dg(ix.device);
      const int D = ix.D, Dp = ix.Dp, W = ix.W, K = ix.K;
      // the file's rotation, query constants and rotated centroids replace the seeded ones
      std::memcpy(ix.P_host.data(), r.P.data(), r.P.size() * 4);
      RBQ_CUDA(cudaMemcpy(ix.P, ix.P_host.data(), ix.P_host.size() * 4, cudaMemcpyHostToDevice));
      ix.t4 = r.t4;
      ix.t8 = r.t8;
      ix.tex = ex_scale_of(ix);
      // original-space centroids c = c_rot P^T (P orthogonal), first D columns, for assigning
      // later adds; the search keeps the file's rotated centroids bit for bit
      ix.C_host.assign((size_t)K * D, 0.0f);
      for (int c = 0; c < K; ++c)
        for (int d = 0; d < D; ++d) {
          double acc = 0.0;
          for (int j = 0; j < Dp; ++j) acc += (double)r.Crot[(size_t)c * Dp + j] * (double)r.P[(size_t)d * Dp + j];
          ix.C_host[(size_t)c * D + d] = (float)acc;
        }
      install_centroids(ix, 0);
      RBQ_CUDA(cudaMemcpy(ix.C_rot, r.Crot.data(), r.Crot.size() * 4, cudaMemcpyHostToDevice));
      launch_row_norms(ix.C_rot, K, Dp, ix.C_rot_n2, 0);
      launch_max_reduce(ix.C_rot_n2, K, ix.C_rot_n2_max, 0);
      RBQ_CUDA(cudaDeviceSynchronize());
      // owners from the file's cluster sizes; rows of owned clusters, in ascending id
      std::vector<int64_t> sizes(r.sizes.begin(), r.sizes.end());
      install_owners(ix, list_owners(ix.shard_policy, sizes, ix.shard_count), true);
      std::vector<std::pair<uint32_t, int64_t>> keep;  // (id, file row)
      std::vector<uint32_t> lab_of_row(r.n);
      int64_t row = 0;
      for (int c = 0; c < K; ++c)
        for (uint64_t i = 0; i < r.sizes[c]; ++i, ++row) {
          lab_of_row[row] = (uint32_t)c;
          if (ix.owner_host[c] == ix.shard_rank) keep.push_back({r.ids[row], row});
        }
      std::sort(keep.begin(), keep.end());
      const int64_t m = (int64_t)keep.size();
      std::vector<uint32_t> codes((size_t)m * W), ids(m), labs(m);
      std::vector<float> fa(m), fr(m), fe(m), X(X_host ? (size_t)m * D : 0);
      const int ex = ix.ex_bits;
      const size_t lcb = (size_t)Dp * ex / 8;
      std::vector<uint32_t> xc((size_t)m * ex * W);
      std::vector<float> xa(ex ? m : 0), xr(ex ? m : 0);
      for (int64_t i = 0; i < m; ++i) {
        const int64_t src = keep[i].second;
        if (ex) {
          long_code_to_planes(&r.long_codes[(size_t)src * lcb], Dp, ex, &xc[(size_t)i * ex * W]);
          xa[i] = r.exfac[src * 2 + 0];
          xr[i] = r.exfac[src * 2 + 1];
        }
        std::memcpy(&codes[(size_t)i * W], &r.codes[(size_t)src * W], (size_t)W * 4);
        ids[i] = keep[i].first;
        labs[i] = lab_of_row[src];
        fa[i] = r.fac[src * 3 + 0];
        fr[i] = r.fac[src * 3 + 1];
        fe[i] = r.fac[src * 3 + 2];
        if (X_host) std::memcpy(&X[(size_t)i * D], X_host + (size_t)keep[i].first * D, (size_t)D * 4);
      }
      ensure_id_capacity(ix, std::max<int64_t>((int64_t)r.n, 1));
      ensure_row_capacity(ix, std::max<int64_t>(m, 1));
      auto up = [&](void* dst, const void* src, size_t bytes) {
        if (bytes) RBQ_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
      };
      up(ix.codes_r, codes.data(), codes.size() * 4);
      up(ix.ids_r, ids.data(), (size_t)m * 4);
      up(ix.labels_r, labs.data(), (size_t)m * 4);
      up(ix.fadd_r, fa.data(), (size_t)m * 4);
      up(ix.frescale_r, fr.data(), (size_t)m * 4);
      up(ix.ferr_r, fe.data(), (size_t)m * 4);
      if (ex) {
        up(ix.ex_codes_r, xc.data(), xc.size() * 4);
        up(ix.fexadd_r, xa.data(), (size_t)m * 4);
        up(ix.fexr_r, xr.data(), (size_t)m * 4);
      }
      if (X_host) up(ix.X_r, X.data(), X.size() * 4);
      ix.has_raw = X_host != nullptr;
      std::vector<uint32_t> id2row(r.n, 0xFFFFFFFFu);
      for (int64_t i = 0; i < m; ++i) id2row[ids[i]] = (uint32_t)i;
      up(ix.id2row, id2row.data(), (size_t)r.n * 4);
      ix.n_rows = m;
      ix.n_total = (int64_t)r.n;
      relayout(ix, 0);
    } catch (...) {
      rbq_index_free(h);
      throw;
    }
    *out = h;
  });
}

int rbq_export_reference(rbq_index_t* index, const char* path)
{
  return guarded([&] {
    RBQ_CHECK(index, RBQ_ERR_INVALID, "null index");
    Index& ix = index->ix;
    RBQ_CHECK(ix.trained, RBQ_ERR_STATE, "index is not trained");
    RBQ_CHECK(ix.shard_count == 1, RBQ_ERR_STATE, "the reference format holds a whole index: export an unsharded one");
    DeviceGuard dg(ix.device);
    RBQ_CUDA(cudaDeviceSynchronize());
    const uint64_t n = (uint64_t)ix.n_rows, D = (uint64_t)ix.D, K = (uint64_t)ix.K, ex = (uint64_t)ix.ex_bits;
    File f(path, "wb");
    f.write(&n, 8);
    f.write(&D, 8);
    f.write(&K, 8);
    f.write(&ex, 8);
    const unsigned char flag = 1;
    f.write(&flag, 1);
    const float t8 = std::isnan(ix.t8) ? query_scale(ix.Dp, ix.seed, 7) : ix.t8;
    f.write(&ix.t4, 4);
    f.write(&t8, 4);
    std::vector<uint64_t> sizes(K);
    for (uint64_t c = 0; c < K; ++c) sizes[c] = (uint64_t)(ix.off_host[c + 1] - ix.off_host[c]);
    f.write(sizes.data(), K * 8);
    const unsigned char kind = 0;
    f.write(&kind, 1);
    f.write(ix.P_host.data(), ix.P_host.size() * 4);
    write_dev(f, ix.C_rot, (size_t)K * ix.Dp);
    write_dev(f, ix.codes, (size_t)n * ix.W);
    std::vector<float> fa(n), fr(n), fe(n), fac(n * 3);
    if (n) {
      RBQ_CUDA(cudaMemcpy(fa.data(), ix.fadd, n * 4, cudaMemcpyDeviceToHost));
      RBQ_CUDA(cudaMemcpy(fr.data(), ix.frescale, n * 4, cudaMemcpyDeviceToHost));
      RBQ_CUDA(cudaMemcpy(fe.data(), ix.ferr, n * 4, cudaMemcpyDeviceToHost));
    }
    for (uint64_t i = 0; i < n; ++i) {
      fac[i * 3 + 0] = fa[i];
      fac[i * 3 + 1] = fr[i];
      fac[i * 3 + 2] = fe[i];
    }
    f.write(fac.data(), fac.size() * 4);
    std::vector<float> exf(n * 2, 0.0f);
    if (ex && n) {
      const size_t EW = (size_t)ex * ix.W, lcb = (size_t)ix.Dp * ex / 8;
      std::vector<uint32_t> xc(n * EW);
      std::vector<uint8_t> lc(n * lcb);
      RBQ_CUDA(cudaMemcpy(xc.data(), ix.ex_codes, xc.size() * 4, cudaMemcpyDeviceToHost));
      for (uint64_t i = 0; i < n; ++i) planes_to_long_code(&xc[i * EW], ix.Dp, (int)ex, &lc[i * lcb]);
      f.write(lc.data(), lc.size());
      RBQ_CUDA(cudaMemcpy(fa.data(), ix.fexadd, n * 4, cudaMemcpyDeviceToHost));
      RBQ_CUDA(cudaMemcpy(fr.data(), ix.fexr, n * 4, cudaMemcpyDeviceToHost));
      for (uint64_t i = 0; i < n; ++i) {
        exf[i * 2 + 0] = fa[i];
        exf[i * 2 + 1] = fr[i];
      }
    }
    f.write(exf.data(), exf.size() * 4);
    write_dev(f, ix.ids, (size_t)n);
  });
}

int rbq_get_rotation(rbq_index_t* index, float* P_host)
{
  return guarded([&] {
    RBQ_CHECK(index && P_host, RBQ_ERR_INVALID, "null argument");
    std::memcpy(P_host, index->ix.P_host.data(), index->ix.P_host.size() * 4);
  });
}

int rbq_get_centroids(rbq_index_t* index, float* C_host, float* C_rot_host)
{
  return guarded([&] {
    RBQ_CHECK(index, RBQ_ERR_INVALID, "null argument");
    Index& ix = index->ix;
    RBQ_CHECK(ix.trained, RBQ_ERR_STATE, "index is not trained");
    if (C_host) std::memcpy(C_host, ix.C_host.data(), ix.C_host.size() * 4);
    if (C_rot_host) {
      DeviceGuard dg(ix.device);
      RBQ_CUDA(cudaMemcpy(C_rot_host, ix.C_rot, (size_t)ix.K * ix.Dp * 4, cudaMemcpyDeviceToHost));
    }
  });
}

int rbq_export_lists(rbq_index_t* index, int64_t* list_off, uint32_t* ids, uint32_t* codes, float* fadd,
                     float* frescale, float* ferr)
{
  return guarded([&] {
    RBQ_CHECK(index, RBQ_ERR_INVALID, "null argument");
    Index& ix = index->ix;
    DeviceGuard dg(ix.device);
    RBQ_CUDA(cudaDeviceSynchronize());
    const size_t n = (size_t)ix.n_rows;
    if (list_off) std::memcpy(list_off, ix.off_host.data(), (ix.K + 1) * 8);
    if (n == 0) return;
    if (ids) RBQ_CUDA(cudaMemcpy(ids, ix.ids, n * 4, cudaMemcpyDeviceToHost));
    if (codes) RBQ_CUDA(cudaMemcpy(codes, ix.codes, n * ix.W * 4, cudaMemcpyDeviceToHost));
    if (fadd) RBQ_CUDA(cudaMemcpy(fadd, ix.fadd, n * 4, cudaMemcpyDeviceToHost));
    if (frescale) RBQ_CUDA(cudaMemcpy(frescale, ix.frescale, n * 4, cudaMemcpyDeviceToHost));
    if (ferr) RBQ_CUDA(cudaMemcpy(ferr, ix.ferr, n * 4, cudaMemcpyDeviceToHost));
  });
}

int rbq_export_ex_lists(rbq_index_t* index, uint32_t* ex_codes, float* fexadd, float* fexr)
{
  return guarded([&] {
    RBQ_CHECK(index, RBQ_ERR_INVALID, "null argument");
    Index& ix = index->ix;
    RBQ_CHECK(ix.ex_bits > 0, RBQ_ERR_STATE, "the index has 1-bit codes only (bits_per_dim = 1)");
    DeviceGuard dg(ix.device);
    RBQ_CUDA(cudaDeviceSynchronize());
    const size_t n = (size_t)ix.n_rows;
    if (n == 0) return;
    if (ex_codes) RBQ_CUDA(cudaMemcpy(ex_codes, ix.ex_codes, n * ix.ex_bits * ix.W * 4, cudaMemcpyDeviceToHost));
    if (fexadd) RBQ_CUDA(cudaMemcpy(fexadd, ix.fexadd, n * 4, cudaMemcpyDeviceToHost));
    if (fexr) RBQ_CUDA(cudaMemcpy(fexr, ix.fexr, n * 4, cudaMemcpyDeviceToHost));
  });
}

int rbq_rotate(rbq_index_t* index, const float* X_dev, int64_t n, float* Y_dev, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_rotate");
    RBQ_CHECK(index && (n == 0 || (X_dev && Y_dev)), RBQ_ERR_INVALID, "null argument");
    Index& ix = index->ix;
    DeviceGuard dg(ix.device);
    launch_rotate(X_dev, n, ix.D, ix.Dp, ix.P, Y_dev, as_stream(stream));
  });
}

int rbq_query_prep(rbq_index_t* index, const float* Qr_dev, int64_t nq, uint32_t* planes_dev, float* delta_dev,
                   float* k1_dev, int32_t query_bits, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_query_prep");
    RBQ_CHECK(index && (nq == 0 || (Qr_dev && planes_dev && delta_dev && k1_dev)), RBQ_ERR_INVALID,
              "null argument");
    Index& ix = index->ix;
    DeviceGuard dg(ix.device);
    const int qb = prep_bits_of(query_bits_of(query_bits));
    launch_query_prep(Qr_dev, nq, ix.Dp, query_t(ix, qb), qb, planes_dev, delta_dev, k1_dev, as_stream(stream));
  });
}

int rbq_coarse_scores(rbq_index_t* index, const float* Qr_dev, int64_t nq, float* S_dev, int32_t tensor_cores,
                      void* stream)
{
  return guarded([&] {
    RBQ_CHECK(index && (nq == 0 || (Qr_dev && S_dev)), RBQ_ERR_INVALID, "null argument");
    Index& ix = index->ix;
    RBQ_CHECK(ix.trained, RBQ_ERR_STATE, "index is not trained");
    if (nq == 0) return;
    DeviceGuard dg(ix.device);
    if (tensor_cores)
      launch_coarse_scores_tc(Qr_dev, nq, ix.C_rot, ix.C_rot_n2, ix.K, ix.Dp, S_dev, ix.dev_err, as_stream(stream));
    else
      launch_coarse_scores(Qr_dev, nq, ix.C_rot, ix.C_rot_n2, ix.K, ix.Dp, S_dev, as_stream(stream));
  });
}

int rbq_check_errors(rbq_index_t* index)
{
  return guarded([&] {
    RBQ_CHECK(index, RBQ_ERR_INVALID, "null argument");
    Index& ix = index->ix;
    DeviceGuard dg(ix.device);
    RBQ_CUDA(cudaDeviceSynchronize());
    int code = 0;
    RBQ_CUDA(cudaMemcpy(&code, ix.dev_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (code) {
      RBQ_CUDA(cudaMemset(ix.dev_err, 0, sizeof(int)));
      throw Error{RBQ_ERR_CUDA, "a tensor-core pipeline wait timed out on the device (code " + std::to_string(code) +
                                    "); results of the affected search are invalid"};
    }
  });
}

int rbq_coarse(rbq_index_t* index, const float* Qr_dev, int64_t nq, int32_t nprobe, int32_t margin,
               int32_t* probes_dev, float* g_dev, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_coarse");
    RBQ_CHECK(index && (nq == 0 || (Qr_dev && probes_dev && g_dev)), RBQ_ERR_INVALID, "null argument");
    Index& ix = index->ix;
    RBQ_CHECK(ix.trained, RBQ_ERR_STATE, "index is not trained");
    RBQ_CHECK(nprobe >= 1 && nprobe <= ix.K, RBQ_ERR_INVALID, "nprobe must be in [1, n_lists]");
    if (nq == 0) return;
    DeviceGuard dg(ix.device);
    cudaStream_t s = as_stream(stream);
    const int m = std::min(ix.K, std::min(nprobe + (margin > 0 ? margin : std::max(32, nprobe / 2)), 1024));
    const int64_t chunk = coarse_rows_per_call(Qr_dev, ix.C_rot, ix.K, ix.Dp, m, nq);
    Scratch sc(s);
    const CoarseScratch cs = coarse_scratch(sc, Qr_dev, ix.C_rot, ix.K, ix.Dp, m, chunk);
    for (int64_t a = 0; a < nq; a += chunk) {
      const int64_t cn = std::min(chunk, nq - a);
      coarse_probes(ix, Qr_dev + a * ix.Dp, cn, ix.C_rot, ix.C_rot_n2, ix.C_rot_n2_max, ix.K, ix.Dp, m, nprobe, cs,
                    probes_dev + a * nprobe, g_dev + a * nprobe, s);
    }
  });
}

int rbq_scan(rbq_index_t* index, const float* Qr_dev, const uint32_t* planes_dev, const float* delta_dev,
             const float* k1_dev, int64_t nq, const int32_t* probes_dev, const float* g_dev, int32_t nprobe,
             int32_t probe_stride, const float* tau0_dev, const int64_t* init_ids_dev, const float* init_dist_dev, int32_t R, int32_t prune,
             int32_t slices, int32_t cand_cap, int64_t* cand_ids_dev, float* cand_dist_dev, uint64_t* stats_dev,
             int32_t query_bits, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_scan");
    RBQ_CHECK(index, RBQ_ERR_INVALID, "null argument");
    RBQ_CHECK(nq == 0 || (Qr_dev && planes_dev && delta_dev && k1_dev && probes_dev && g_dev && cand_ids_dev &&
                          cand_dist_dev),
              RBQ_ERR_INVALID, "null buffer");
    RBQ_CHECK(R >= 1 && R <= 4096 && nprobe >= 1 && slices >= 1 && (probe_stride == 0 || probe_stride >= nprobe),
              RBQ_ERR_INVALID, "bad scan parameters");
    RBQ_CHECK(!init_ids_dev == !init_dist_dev, RBQ_ERR_INVALID, "init_ids and init_dist go together");
    if (nq == 0) return;
    Index& ix = index->ix;
    DeviceGuard dg(ix.device);
    cudaStream_t s = as_stream(stream);
    const int cap = std::max(next_pow2(cand_cap > 0 ? cand_cap : 1024), next_pow2(R + kScanTile));
    Scratch sc(s);
    unsigned long long* ks = sc.get<unsigned long long>((size_t)nq * slices * R);
    unsigned long long* k2 = slices > 1 ? sc.get<unsigned long long>((size_t)nq * R) : ks;
    ScanArgs sa = batch_scan_args(ix, Qr_dev, planes_dev, delta_dev, k1_dev, nq, probes_dev, g_dev, nprobe, R, cap,
                                  prune, slices, ks, stats_dev, query_bits_of(query_bits));
    sa.tau0 = tau0_dev;
    sa.pstride = probe_stride;
    if (init_ids_dev) {
      unsigned long long* ik = sc.get<unsigned long long>((size_t)nq * R);
      launch_cands_to_keys(init_ids_dev, init_dist_dev, nq * R, ik, s);
      sa.init_keys = ik;
    }
    if (nq >= kQueryOrderMinBatch) {
      int32_t* qo = sc.get<int32_t>((size_t)ix.K + 2 + nq);
      launch_query_order(probes_dev, nq, probe_stride > 0 ? probe_stride : nprobe, ix.K, qo, qo + ix.K + 2, s);
      sa.qorder = qo + ix.K + 2;
    }
    launch_scan(sa, s);
    if (slices > 1) launch_merge_keys(ks, nq, slices, R, k2, s);
    launch_keys_to_ids(k2, nq * R, cand_ids_dev, cand_dist_dev, s);
  });
}

int rbq_scan_lists(rbq_index_t* index, const float* Qr_dev, const uint32_t* planes_dev, const float* delta_dev,
                   const float* k1_dev, int64_t nq, const int32_t* probes_dev, const float* g_dev, int32_t nprobe,
                   int32_t probe_stride, const float* tau0_dev, int32_t R, int64_t* cand_ids_dev, float* cand_dist_dev,
                   uint64_t* stats_dev, int32_t query_bits, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_scan_lists");
    RBQ_CHECK(index, RBQ_ERR_INVALID, "null argument");
    RBQ_CHECK(nq == 0 || (Qr_dev && planes_dev && delta_dev && k1_dev && probes_dev && g_dev && tau0_dev &&
                          cand_ids_dev && cand_dist_dev),
              RBQ_ERR_INVALID, "null buffer");
    RBQ_CHECK(R >= 1 && R <= 4096 && nprobe >= 1 && (probe_stride == 0 || probe_stride >= nprobe), RBQ_ERR_INVALID,
              "bad scan parameters");
    Index& ix = index->ix;
    const int qb = query_bits_of(query_bits);
    RBQ_CHECK((qb == 4 || qb == 8) && list_scan_tc_supported(ix.Dp), RBQ_ERR_INVALID,
              "list scan: needs QUANT4 / QUANT8 planes and a padded dim <= 768");
    if (nq == 0) return;
    DeviceGuard dg(ix.device);
    cudaStream_t s = as_stream(stream);
    const int cap = list_scan_cap(R);
    Scratch sc(s);
    unsigned long long* keys = sc.get<unsigned long long>((size_t)nq * R);
    const ListScanScratch w = list_scan_scratch(sc, ix, nq, nprobe, cap, R);
    list_scan(ix, Qr_dev, planes_dev, qb, delta_dev, k1_dev, nq, probes_dev, g_dev, nprobe,
              probe_stride > 0 ? probe_stride : nprobe, tau0_dev, R, cap, w, keys, stats_dev, s);
    launch_keys_to_ids(keys, nq * R, cand_ids_dev, cand_dist_dev, s);
  });
}

int rbq_bound_seed(rbq_index_t* index, const float* Qr_dev, const uint32_t* planes_dev, const float* delta_dev,
                   const float* k1_dev, int64_t nq, const int32_t* probes_dev, const float* g_dev, int32_t nprobe,
                   int32_t probe_stride, int32_t R, int32_t cand_cap, float* tau_dev, int32_t query_bits, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_bound_seed");
    RBQ_CHECK(index, RBQ_ERR_INVALID, "null argument");
    RBQ_CHECK(nq == 0 || (Qr_dev && planes_dev && delta_dev && k1_dev && probes_dev && g_dev && tau_dev),
              RBQ_ERR_INVALID, "null buffer");
    RBQ_CHECK(R >= 1 && R <= 4096 && nprobe >= 1 && (probe_stride == 0 || probe_stride >= nprobe), RBQ_ERR_INVALID,
              "bad seed parameters");
    if (nq == 0) return;
    Index& ix = index->ix;
    DeviceGuard dg(ix.device);
    const int cap = std::max(next_pow2(cand_cap > 0 ? cand_cap : 1024), next_pow2(R + kScanTile));
    ScanArgs sa = batch_scan_args(ix, Qr_dev, planes_dev, delta_dev, k1_dev, nq, probes_dev, g_dev, nprobe, R, cap,
                                  1, 1, nullptr, nullptr, query_bits_of(query_bits));
    sa.pstride = probe_stride;
    sa.tau_out = tau_dev;
    launch_scan(sa, as_stream(stream));
  });
}

int rbq_bound_seed_owned(rbq_index_t* index, const float* Qr_dev, const uint32_t* planes_dev, const float* delta_dev,
                         const float* k1_dev, int64_t nq, const int32_t* probes_dev, const float* g_dev, int32_t nprobe,
                         int32_t probe_stride, int32_t R, int32_t cand_cap, float* tau_dev, int32_t query_bits,
                         void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_bound_seed_owned");
    RBQ_CHECK(index, RBQ_ERR_INVALID, "null argument");
    RBQ_CHECK(nq == 0 || (Qr_dev && planes_dev && delta_dev && k1_dev && probes_dev && g_dev && tau_dev),
              RBQ_ERR_INVALID, "null buffer");
    RBQ_CHECK(R >= 1 && R <= 4096 && nprobe >= 1 && (probe_stride == 0 || probe_stride >= nprobe), RBQ_ERR_INVALID,
              "bad seed parameters");
    if (nq == 0) return;
    Index& ix = index->ix;
    DeviceGuard dg(ix.device);
    const int cap = std::max(next_pow2(cand_cap > 0 ? cand_cap : 1024), next_pow2(R + kScanTile));
    ScanArgs sa = batch_scan_args(ix, Qr_dev, planes_dev, delta_dev, k1_dev, nq, probes_dev, g_dev, nprobe, R, cap,
                                  1, 1, nullptr, nullptr, query_bits_of(query_bits));
    sa.pstride = probe_stride;
    sa.tau_out = tau_dev;
    sa.seed_nearest_owned = 1;
    launch_scan(sa, as_stream(stream));
  });
}

int rbq_list_estimates(rbq_index_t* index, const uint32_t* planes_dev, float delta, float k1, float g, int32_t list,
                       int32_t* acc_dev, float* est_dev, float* low_dev, int32_t query_bits, void* stream)
{
  return guarded([&] {
    RBQ_CHECK(index && planes_dev && acc_dev && est_dev && low_dev, RBQ_ERR_INVALID, "null argument");
    Index& ix = index->ix;
    RBQ_CHECK(list >= 0 && list < ix.K, RBQ_ERR_INVALID, "list out of range");
    DeviceGuard dg(ix.device);
    RBQ_CHECK(query_bits_of(query_bits) <= 8, RBQ_ERR_INVALID, "list estimates: popcount modes only (4 or 8)");
    launch_list_estimates(ix, planes_dev, query_bits_of(query_bits), delta, k1, g, list, acc_dev, est_dev, low_dev,
                          as_stream(stream));
  });
}

int rbq_rerank(rbq_index_t* index, const float* Q_dev, int64_t nq, const int64_t* cand_ids_dev, int32_t R, int32_t k,
               float* dist_dev, int64_t* ids_dev, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_rerank");
    RBQ_CHECK(index, RBQ_ERR_INVALID, "null argument");
    RBQ_CHECK(nq == 0 || (Q_dev && cand_ids_dev && dist_dev && ids_dev), RBQ_ERR_INVALID, "null buffer");
    RBQ_CHECK(R >= 1 && R <= 4096 && k >= 1, RBQ_ERR_INVALID, "bad rerank parameters");
    if (nq == 0) return;
    Index& ix = index->ix;
    RBQ_CHECK(ix.has_raw, RBQ_ERR_STATE, "exact rerank needs the raw vectors; this index was imported without them");
    DeviceGuard dg(ix.device);
    cudaStream_t s = as_stream(stream);
    Scratch sc(s);
    unsigned long long* keys = sc.get<unsigned long long>((size_t)nq * R);
    launch_ids_to_keys(cand_ids_dev, nq * R, keys, s);
    launch_rerank(ix.X_r, ix.id2row, ix.D, Q_dev, nq, keys, R, k, dist_dev, ids_dev, s);
  });
}

int rbq_merge_results(const float* dist_dev, const int64_t* ids_dev, int32_t parts, int64_t nq, int32_t k,
                      float* out_dist_dev, int64_t* out_ids_dev, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_merge_results");
    RBQ_CHECK(parts >= 1 && k >= 1 && nq >= 0, RBQ_ERR_INVALID, "bad merge parameters");
    RBQ_CHECK(nq == 0 || (dist_dev && ids_dev && out_dist_dev && out_ids_dev), RBQ_ERR_INVALID, "null buffer");
    launch_merge_results(dist_dev, ids_dev, parts, nq, k, out_dist_dev, out_ids_dev, as_stream(stream));
  });
}

int rbq_pack_results(const float* dist_dev, const int64_t* ids_dev, int64_t n, uint64_t* keys_dev, void* stream)
{
  return guarded([&] {
    RBQ_CHECK(n >= 0 && (n == 0 || (dist_dev && ids_dev && keys_dev)), RBQ_ERR_INVALID, "null buffer");
    launch_cands_to_keys(ids_dev, dist_dev, n, reinterpret_cast<unsigned long long*>(keys_dev), as_stream(stream));
  });
}

int rbq_merge_result_keys(const uint64_t* keys_dev, int32_t parts, int64_t nq, int32_t k, float* out_dist_dev,
                          int64_t* out_ids_dev, void* stream)
{
  return guarded([&] {
    Range nvtx_range("rbq_merge_result_keys");
    RBQ_CHECK(parts >= 1 && k >= 1 && nq >= 0, RBQ_ERR_INVALID, "bad merge parameters");
    RBQ_CHECK(nq == 0 || (keys_dev && out_dist_dev && out_ids_dev), RBQ_ERR_INVALID, "null buffer");
    launch_merge_results(nullptr, nullptr, parts, nq, k, out_dist_dev, out_ids_dev, as_stream(stream),
                         reinterpret_cast<const unsigned long long*>(keys_dev));
  });
}

int rbq_gen_mixture(float* X_dev, int64_t n, int32_t D, int32_t n_centres, float sigma, int32_t aniso,
                    int32_t normalize, uint64_t seed, void* stream)
{
  return guarded([&] {
    RBQ_CHECK(X_dev && n >= 0 && D >= 1 && n_centres >= 1, RBQ_ERR_INVALID, "bad generator arguments");
    cudaStream_t s = as_stream(stream);
    Scratch sc(s);
    float* cen = sc.get<float>((size_t)n_centres * D);
    launch_gen_mixture(X_dev, n, D, n_centres, sigma, aniso, normalize, seed, 10u, cen, s);
  });
}

int rbq_gen_queries(const float* X_dev, int64_t n, int32_t D, float* Q_dev, int64_t nq, float sigma,
                    int32_t normalize, uint64_t seed, int64_t* src_rows_dev, void* stream)
{
  return guarded([&] {
    RBQ_CHECK(X_dev && Q_dev && n >= 1 && D >= 1 && nq >= 0, RBQ_ERR_INVALID, "bad generator arguments");
    launch_gen_queries(X_dev, n, D, Q_dev, nq, sigma, normalize, seed, 20u, src_rows_dev, as_stream(stream));
  });
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Allocation-free scan (rbq_scan_noalloc).  Its scratch is this fixed device array; host code
// must never pass `rbq_noalloc_scratch` itself to a kernel (on the host the name is only a
// stand-in), so the device address is looked up once per device and cached.
// ---------------------------------------------------------------------------------------
static __device__ __align__(256) unsigned char rbq_noalloc_scratch[RBQ_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_noalloc_mu;
// Per device: the address and the unique id of the context it was looked up in.  A context
// destroyed and created again (cudaDeviceReset) has a new id, so the address is looked up again
// instead of being used stale.
struct NoallocSlot {
  unsigned long long ctx_id = 0;
  void* addr = nullptr;
};
NoallocSlot g_noalloc[64];

// Unique id of the calling thread's current context (cuCtxGetCurrent + cuCtxGetId through the
// runtime's driver entry points; no link-time libcuda).
unsigned long long current_context_id()
{
  typedef CUresult (*GetCurrentFn)(CUcontext*);
  typedef CUresult (*GetIdFn)(CUcontext, unsigned long long*);
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetIdFn>(p);
  });
  RBQ_CHECK(get_current && get_id, RBQ_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId are not available from the driver");
  CUcontext c = nullptr;
  RBQ_CHECK(get_current(&c) == CUDA_SUCCESS && c, RBQ_ERR_CUDA, "no current CUDA context");
  unsigned long long id = 0;
  RBQ_CHECK(get_id(c, &id) == CUDA_SUCCESS, RBQ_ERR_CUDA, "cuCtxGetId failed");
  return id;
}

// Device address of the scratch array on `device`, which must be the current device.
unsigned char* noalloc_scratch_address(int device)
{
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  RBQ_CHECK(device >= 0 && device < 64, RBQ_ERR_INVALID, "device ordinal out of range");
  const unsigned long long ctx = current_context_id();
  NoallocSlot& slot = g_noalloc[device];
  if (!slot.addr || slot.ctx_id != ctx) {
    void* p = nullptr;
    RBQ_CUDA(cudaGetSymbolAddress(&p, rbq_noalloc_scratch));
    slot.addr = p;
    slot.ctx_id = ctx;
  }
  return static_cast<unsigned char*>(slot.addr);
}

inline size_t round_up_256(size_t v) { return (v + 255) / 256 * 256; }
}  // namespace

extern "C" int rbq_scan_noalloc(rbq_index_t* index, const float* Qr_dev, const uint32_t* planes_dev,
                                const float* delta_dev, const float* k1_dev, int64_t nq, const int32_t* probes_dev,
                                const float* g_dev, int32_t nprobe, int32_t probe_stride, const float* tau0_dev,
                                int32_t R, int32_t prune,
                                int32_t slices, int32_t cand_cap, int64_t* cand_ids_dev, float* cand_dist_dev,
                                uint64_t* stats_dev, int32_t query_bits, void* stream)
{
  return guarded([&] {
    RBQ_CHECK(index, RBQ_ERR_INVALID, "null argument");
    RBQ_CHECK(nq == 0 || (Qr_dev && planes_dev && delta_dev && k1_dev && probes_dev && g_dev && cand_ids_dev &&
                          cand_dist_dev),
              RBQ_ERR_INVALID, "null buffer");
    RBQ_CHECK(nq >= 0 && R >= 1 && R <= 4096 && nprobe >= 1 && slices >= 1 &&
                  (probe_stride == 0 || probe_stride >= nprobe),
              RBQ_ERR_INVALID, "bad scan parameters");
    const size_t keys_bytes = round_up_256((size_t)nq * slices * R * 8);
    const size_t merged_bytes = slices > 1 ? round_up_256((size_t)nq * R * 8) : 0;
    RBQ_CHECK(keys_bytes + merged_bytes <= (size_t)RBQ_NOALLOC_SCRATCH_BYTES, RBQ_ERR_INVALID,
              "rbq_scan_noalloc: nq * slices * R needs " + std::to_string(keys_bytes + merged_bytes) +
                  " bytes of scratch; the static scratch holds " + std::to_string(RBQ_NOALLOC_SCRATCH_BYTES) +
                  " bytes (use rbq_scan, or split the batch)");
    if (nq == 0) return;
    Index& ix = index->ix;
    DeviceGuard dg(ix.device);
    cudaStream_t s = as_stream(stream);
    unsigned char* base = noalloc_scratch_address(ix.device);
    unsigned long long* ks = reinterpret_cast<unsigned long long*>(base);
    unsigned long long* k2 = slices > 1 ? reinterpret_cast<unsigned long long*>(base + keys_bytes) : ks;
    const int cap = std::max(next_pow2(cand_cap > 0 ? cand_cap : 1024), next_pow2(R + kScanTile));
    ScanArgs sa = batch_scan_args(ix, Qr_dev, planes_dev, delta_dev, k1_dev, nq, probes_dev, g_dev, nprobe, R, cap,
                                  prune, slices, ks, stats_dev, query_bits_of(query_bits));
    sa.tau0 = tau0_dev;
    sa.pstride = probe_stride;
    launch_scan(sa, s);
    if (slices > 1) launch_merge_keys(ks, nq, slices, R, k2, s);
    launch_keys_to_ids(k2, nq * R, cand_ids_dev, cand_dist_dev, s);
  });
}
