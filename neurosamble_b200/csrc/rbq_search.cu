// Search kernels for sm_100a: coarse quantiser (approximate pass + exact refine), 4-bit
// query quantisation, the list scan, candidate merges and the exact rerank.
//
// Compiled with -fmad=false.  The estimator, the prune test, the exact 1-bit distance and the
// rerank distance are evaluated in the operation order written here, which is also the order
// of the CPU oracle (oracle/rbq_oracle.cpp), so estimates and ids agree bit for bit.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "rbq_internal.cuh"

namespace rbq {

// ---------------------------------------------------------------------------------------
// Block-wide bitonic sort of n (power of two) u64 keys in shared memory, ascending.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void block_bitonic_sort(unsigned long long* keys, int n)
{
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long a = keys[i], b = keys[ixj];
          const bool up = (i & k) == 0;
          if ((a > b) == up) {
            keys[i] = b;
            keys[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------------------
// Approximate coarse scores S[q, c] = |c|^2 - 2 <a_q, c> (fp32, tiled SIMT GEMM).  Only
// used to shortlist lists; the final probes come from the exact refine below.
// Tiles: 64 queries x 64 centroids x 16 dims, 256 threads, 4x4 outputs per thread.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) coarse_scores_kernel(const float* __restrict__ A, int64_t nq,
                                                            const float* __restrict__ C,
                                                            const float* __restrict__ cn2, int K, int d,
                                                            float* __restrict__ S)
{
  __shared__ float As[16][64 + 4];
  __shared__ float Cs[16][64 + 4];
  const int64_t q0 = (int64_t)blockIdx.y * 64;
  const int c0 = blockIdx.x * 64;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  for (int k0 = 0; k0 < d; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int r = i >> 4, kk = i & 15;
      const int64_t q = q0 + r;
      const int c = c0 + r;
      const int k = k0 + kk;
      As[kk][r] = (q < nq && k < d) ? A[q * d + k] : 0.0f;
      Cs[kk][r] = (c < K && k < d) ? C[(size_t)c * d + k] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Cs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t q = q0 + ty * 4 + i;
    if (q >= nq) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = c0 + tx * 4 + j;
      if (c < K) S[q * K + c] = cn2[c] - 2.0f * acc[i][j];
    }
  }
}

void launch_coarse_scores(const float* A, int64_t nq, const float* C, const float* cn2, int K, int d, float* S,
                          cudaStream_t s)
{
  if (nq <= 0) return;
  RBQ_CHECK(ceil_div(nq, 64) <= 65535, RBQ_ERR_INVALID, "coarse: query chunk too large");
  dim3 grid((unsigned)ceil_div(K, 64), (unsigned)ceil_div(nq, 64));
  coarse_scores_kernel<<<grid, 256, 0, s>>>(A, nq, C, cn2, K, d, S);
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// Per row of S [nq, K]: the m smallest (score, column) keys.  The row streams through in rounds
// of 256 * KPER keys; a key is appended to the shared buffer only while it is below the m-th
// smallest key kept so far (keys are distinct, so no key at or above it can be among the m
// smallest), and a radix select (block_keep_smallest) cuts the buffer back to m keys when the
// next round might not fit.  After the first cut few keys pass, so a long row costs one read
// and about two selections.  Order of the m output columns is unspecified; the exact refine
// below ranks them.
// ---------------------------------------------------------------------------------------
constexpr int kTopmChunk = 4096;

__device__ unsigned long long block_keep_smallest(const unsigned long long* src, int n, int R,
                                                  unsigned long long* dst, unsigned* hist, int* misc,
                                                  unsigned long long* kmax, int* cnt);

template <int KPER>
__global__ void __launch_bounds__(256) topm_rows_kernel(const float* __restrict__ S, int K, int m, int buf,
                                                        int32_t* __restrict__ cand, int p, float2* __restrict__ bounds)
{
  extern __shared__ unsigned long long tk[];  // [2 * buf], buf >= m + 256 * KPER
  __shared__ unsigned s_hist[256];
  __shared__ int s_misc[3], s_cnt, s_fill;
  __shared__ unsigned long long s_kmax;
  unsigned long long* cur = tk;
  unsigned long long* nxt = tk + buf;
  const int64_t q = blockIdx.x;
  const float* row = S + q * K;
  const int lane = threadIdx.x & 31;
  const int step = 256 * KPER;
  unsigned long long thr = kEmptyKey;  // the m-th smallest key kept so far (none: all ones)
  int filled = 0;                      // keys at the front of `cur`
  bool cut = false;                    // a selection has run (thr is the m-th smallest so far)
  if (threadIdx.x == 0) s_fill = 0;
  __syncthreads();
  for (int c0 = 0; c0 < K; c0 += step) {
    if (filled + step > buf) {  // block-uniform; filled > m here because buf >= m + step
      thr = block_keep_smallest(cur, filled, m, nxt, s_hist, s_misc, &s_kmax, &s_cnt);
      cut = true;
      unsigned long long* t = cur;
      cur = nxt;
      nxt = t;
      filled = m;
      if (threadIdx.x == 0) s_fill = m;
      __syncthreads();
    }
    float v[KPER];
#pragma unroll
    for (int r = 0; r < KPER; ++r) {
      const int i = c0 + r * 256 + threadIdx.x;
      v[r] = i < K ? __ldg(row + i) : 0.0f;
    }
#pragma unroll
    for (int r = 0; r < KPER; ++r) {
      const int i = c0 + r * 256 + threadIdx.x;
      const unsigned long long key = make_key(v[r], (uint32_t)i);
      const bool keep = i < K && key < thr;
      const unsigned bal = __ballot_sync(0xffffffffu, keep);
      int base = 0;
      if (lane == 0 && bal) base = atomicAdd(&s_fill, __popc(bal));
      base = __shfl_sync(0xffffffffu, base, 0);
      if (keep) cur[base + __popc(bal & ((1u << lane) - 1u))] = key;
    }
    __syncthreads();
    filled = s_fill;
    __syncthreads();  // every thread has read s_fill before the next round appends
  }
  if (filled > m) {
    thr = block_keep_smallest(cur, filled, m, nxt, s_hist, s_misc, &s_kmax, &s_cnt);
    cut = true;
    unsigned long long* t = cur;
    cur = nxt;
    nxt = t;
    filled = m;
    __syncthreads();
  }
  for (int i = threadIdx.x; i < m; i += blockDim.x)
    cand[q * m + i] = i < filled ? (int32_t)(cur[i] & 0xFFFFFFFFu) : -1;
  // .y: the m-th smallest score (+inf when every column is kept); .x is not used
  if (bounds && threadIdx.x == 0)
    bounds[q] = make_float2(0.0f, cut ? from_ordered_bits((uint32_t)(thr >> 32)) : __int_as_float(0x7f800000));
}

void launch_topm_rows(const float* S, int64_t nq, int K, int m, int32_t* cand, cudaStream_t s, int p,
                      float2* bounds)
{
  if (nq <= 0) return;
  RBQ_CHECK(m >= 1 && m <= kTopmChunk / 2, RBQ_ERR_INVALID, "coarse: shortlist size out of range");
  if (K > kTopmChunk) {  // long rows: 2048 keys a round into a 4096-key buffer
    const int buf = kTopmChunk;
    const size_t smem = (size_t)buf * 2 * 8;
    RBQ_CUDA(cudaFuncSetAttribute(topm_rows_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    topm_rows_kernel<8><<<(unsigned)nq, 256, smem, s>>>(S, K, m, buf, cand, p, bounds);
  } else {  // rows of up to 4096 keys: 1024 a round, so K <= 1024 is one fill and one selection
    const int buf = std::max(std::max(2 * m, K), m + 1024);
    const size_t smem = (size_t)buf * 2 * 8;
    if (smem > 48 * 1024)
      RBQ_CUDA(cudaFuncSetAttribute(topm_rows_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    topm_rows_kernel<4><<<(unsigned)nq, 256, smem, s>>>(S, K, m, buf, cand, p, bounds);
  }
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// Exact refine of the shortlist: g = |a - c|^2 with lane l of a warp summing double(a_j - c_j)^2
// over j = l, l+32, ... and an xor butterfly (16..1) of double adds, rounded to float (the
// oracle's orc_coarse / orc_assign distance); keep the p smallest (g, list id), ascending.
// One CTA per query, one warp per candidate; with d = 32 * EPL the warp loads all EPL values
// of two candidates before the arithmetic (EPL = 0: the generic loop for other d).
// ---------------------------------------------------------------------------------------
// Bound on |tf32 score - exact score| for a query of squared norm qn2 against centroids of
// squared norm <= cmax2: the tensor core truncates each operand to tf32 (relative error 2^-10
// each, so 2^-9 per product), adds d products in fp32, and the score is |c|^2 - 2 <q, c>.  Twice
// that estimate, plus an absolute term for the float rounding of the exact distances.
__device__ __forceinline__ float tf32_score_bound(float qn2, float cmax2, int d)
{
  const float rel = 0.0078125f + (float)d * 4.76837158e-7f;  // 2^-7 + d * 2^-21
  return rel * sqrtf(qn2 * cmax2) + 1.90734863e-6f * (qn2 + cmax2);  // + 2^-19 (|q|^2 + |c|^2)
}

// The shortlist holds every column whose tf32 score is below its m-th smallest tf32 score sm, so a
// list outside it has exact score >= sm - E and exact distance >= |q|^2 + sm - E.  If that is above
// the p-th smallest exact distance gp found inside the shortlist (with slack for the float
// roundings of the distances), no outside list can be among the true p nearest.
__device__ __forceinline__ bool shortlist_is_safe(float qn2, float sm, float gp, float cmax2, int d)
{
  if (!(sm < __int_as_float(0x7f800000))) return true;  // every column was shortlisted
  if (!(gp < __int_as_float(0x7f800000))) return false;  // fewer than p candidates
  const float e = tf32_score_bound(qn2, cmax2, d);
  const float slack = 9.53674316e-7f * (qn2 + fabsf(sm) + gp);  // 2^-20 of the magnitudes
  return qn2 + sm - e - slack > gp;
}

template <int EPL>
__global__ void __launch_bounds__(256) refine_topp_kernel(const float* __restrict__ A, const float* __restrict__ C,
                                                          int d, const int32_t* __restrict__ cand, int m, int p,
                                                          int mp2, int32_t* __restrict__ probes,
                                                          float* __restrict__ gout, const float2* __restrict__ bounds,
                                                          const float* __restrict__ cmax2, int* __restrict__ unsafe)
{
  extern __shared__ unsigned char smem_raw[];
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_raw);
  float* a = reinterpret_cast<float*>(keys + mp2);
  const int64_t q = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int j = threadIdx.x; j < d; j += blockDim.x) a[j] = A[q * d + j];
  for (int i = threadIdx.x; i < mp2; i += blockDim.x) keys[i] = kEmptyKey;
  __syncthreads();
  auto finish = [&](int i, int c, double s) {
#pragma unroll
    for (int off = 16; off; off >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    if (lane == 0 && c >= 0) keys[i] = make_key((float)s, (uint32_t)c);
  };
  if constexpr (EPL > 0) {
    for (int i0 = warp * 2; i0 < m; i0 += nwarps * 2) {
      int c[2];
      float x[2][EPL];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        c[u] = i0 + u < m ? cand[q * m + i0 + u] : -1;
        const float* cr = C + (size_t)(c[u] < 0 ? 0 : c[u]) * d;
#pragma unroll
        for (int e = 0; e < EPL; ++e) x[u][e] = c[u] >= 0 ? __ldg(cr + lane + 32 * e) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        double s = 0.0;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float df = __fsub_rn(x[u][e], a[lane + 32 * e]);
          s = __dadd_rn(s, __dmul_rn((double)df, (double)df));
        }
        finish(i0 + u, c[u], s);
      }
    }
  } else {
    for (int i = warp; i < m; i += nwarps) {
      const int c = cand[q * m + i];
      double s = 0.0;
      if (c >= 0) {
        const float* cr = C + (size_t)c * d;
        for (int j = lane; j < d; j += 32) {
          const float df = __fsub_rn(__ldg(cr + j), a[j]);
          s = __dadd_rn(s, __dmul_rn((double)df, (double)df));
        }
      }
      finish(i, c, s);
    }
  }
  __syncthreads();
  block_bitonic_sort(keys, mp2);
  if (bounds && warp == 0) {  // queue the query for the exact pass if the shortlist may miss a probe
    double v = 0.0;
    for (int j = lane; j < d; j += 32) v = __dadd_rn(v, __dmul_rn((double)a[j], (double)a[j]));
#pragma unroll
    for (int off = 16; off; off >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (lane == 0) {
      const unsigned long long kp = p <= mp2 ? keys[p - 1] : kEmptyKey;
      const float gp = kp == kEmptyKey ? __int_as_float(0x7f800000) : from_ordered_bits((uint32_t)(kp >> 32));
      if (!shortlist_is_safe((float)v, bounds[q].y, gp, *cmax2, d)) unsafe[1 + atomicAdd(unsafe, 1)] = (int)q;
    }
  }
  for (int i = threadIdx.x; i < p; i += blockDim.x) {
    const unsigned long long key = keys[i];
    if (key == kEmptyKey) {
      probes[q * p + i] = -1;
      if (gout) gout[q * p + i] = __int_as_float(0x7f800000);
    } else {
      probes[q * p + i] = (int32_t)(key & 0xFFFFFFFFu);
      if (gout) gout[q * p + i] = from_ordered_bits((uint32_t)(key >> 32));
    }
  }
}

template <int EPL>
static void launch_refine_e(const float* A, int64_t nq, const float* C, int d, const int32_t* cand, int m, int p,
                            int mp2, size_t smem, int32_t* probes, float* g, const float2* bounds,
                            const float* cmax2, int* unsafe, cudaStream_t s)
{
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(refine_topp_kernel<EPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  refine_topp_kernel<EPL><<<(unsigned)nq, 256, smem, s>>>(A, C, d, cand, m, p, mp2, probes, g, bounds, cmax2,
                                                          unsafe);
  RBQ_LAUNCHED();
}

void launch_refine_topp(const float* A, int64_t nq, const float* C, int d, const int32_t* cand, int m, int p,
                        int32_t* probes, float* g, cudaStream_t s, const float2* bounds, const float* cmax2,
                        int* unsafe)
{
  if (nq <= 0) return;
  RBQ_CHECK(!bounds || (cmax2 && unsafe), RBQ_ERR_INVALID, "coarse: the shortlist check needs cmax2 and a queue");
  const int mp2 = next_pow2(m < 2 ? 2 : m);
  const size_t smem = (size_t)mp2 * 8 + (size_t)d * 4;
  RBQ_CHECK(smem <= 200 * 1024, RBQ_ERR_INVALID, "coarse: refine shortlist too large");
#define RBQ_REFINE_CASE(E) \
  launch_refine_e<E>(A, nq, C, d, cand, m, p, mp2, smem, probes, g, bounds, cmax2, unsafe, s)
  switch (d % 32 == 0 ? d / 32 : 0) {
    case 1: RBQ_REFINE_CASE(1); break;
    case 2: RBQ_REFINE_CASE(2); break;
    case 4: RBQ_REFINE_CASE(4); break;
    case 8: RBQ_REFINE_CASE(8); break;
    case 12: RBQ_REFINE_CASE(12); break;
    case 24: RBQ_REFINE_CASE(24); break;
    default: RBQ_REFINE_CASE(0); break;
  }
#undef RBQ_REFINE_CASE
}

// ---------------------------------------------------------------------------------------
// Exact probes of the queued queries (unsafe[0] = count, unsafe[1..] = query ids) over all K
// lists: the same per-centroid double distance as refine_topp_kernel (lane l sums j = l, l+32, ...,
// xor butterfly, rounded to float).  Lists stream through in chunks; a (g, list id) key is kept
// only while it is below the p-th smallest key kept so far, and a radix select cuts the buffer
// back to p keys when the next chunk might not fit, so a long row costs about one selection per
// few chunks.  The p kept keys are sorted and written.  Persistent blocks take queued queries in
// turn; a block with none left returns at once.
// ---------------------------------------------------------------------------------------
constexpr int kRefineAllChunk = 2048;

__global__ void __launch_bounds__(256) refine_all_kernel(const float* __restrict__ A, const float* __restrict__ C,
                                                         int d, int K, int p, int buf, const int* __restrict__ unsafe,
                                                         int32_t* __restrict__ probes, float* __restrict__ gout)
{
  extern __shared__ unsigned char smem_raw[];
  unsigned long long* const buf0 = reinterpret_cast<unsigned long long*>(smem_raw);  // [buf]
  unsigned long long* const buf1 = buf0 + buf;                                       // [buf]
  float* a = reinterpret_cast<float*>(buf1 + buf);                                    // [d]
  __shared__ unsigned s_hist[256];
  __shared__ int s_misc[3], s_cnt, s_fill;
  __shared__ unsigned long long s_kmax;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int n_unsafe = unsafe[0];
  for (int u = blockIdx.x; u < n_unsafe; u += gridDim.x) {
    const int64_t q = unsafe[1 + u];
    unsigned long long* cur = buf0;
    unsigned long long* nxt = buf1;
    __syncthreads();
    for (int j = threadIdx.x; j < d; j += blockDim.x) a[j] = A[q * d + j];
    if (threadIdx.x == 0) s_fill = 0;
    __syncthreads();
    unsigned long long thr = kEmptyKey;  // the p-th smallest key kept so far
    int filled = 0;
    for (int c0 = 0; c0 < K; c0 += kRefineAllChunk) {
      const int c1 = min(K, c0 + kRefineAllChunk);
      for (int c = c0 + warp; c < c1; c += nwarps) {
        const float* cr = C + (size_t)c * d;
        double sacc = 0.0;
        for (int j = lane; j < d; j += 32) {
          const float df = __fsub_rn(__ldg(cr + j), a[j]);
          sacc = __dadd_rn(sacc, __dmul_rn((double)df, (double)df));
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) sacc = __dadd_rn(sacc, __shfl_xor_sync(0xffffffffu, sacc, off));
        const unsigned long long key = make_key((float)sacc, (uint32_t)c);
        if (lane == 0 && key < thr) cur[atomicAdd(&s_fill, 1)] = key;
      }
      __syncthreads();
      filled = s_fill;
      if (filled > p && (filled + kRefineAllChunk > buf || c1 == K)) {
        thr = block_keep_smallest(cur, filled, p, nxt, s_hist, s_misc, &s_kmax, &s_cnt);
        unsigned long long* t = cur;
        cur = nxt;
        nxt = t;
        filled = p;
        if (threadIdx.x == 0) s_fill = p;
      }
      __syncthreads();
    }
    int n2 = 2;
    while (n2 < filled) n2 <<= 1;
    for (int i = filled + threadIdx.x; i < n2; i += blockDim.x) cur[i] = kEmptyKey;
    __syncthreads();
    block_bitonic_sort(cur, n2);
    for (int i = threadIdx.x; i < p; i += blockDim.x) {
      const unsigned long long key = i < filled ? cur[i] : kEmptyKey;
      probes[q * p + i] = key == kEmptyKey ? -1 : (int32_t)(key & 0xFFFFFFFFu);
      if (gout) gout[q * p + i] = key == kEmptyKey ? __int_as_float(0x7f800000) : from_ordered_bits((uint32_t)(key >> 32));
    }
  }
}

int device_sm_count()
{
  int dev = 0, n = 0;
  RBQ_CUDA(cudaGetDevice(&dev));
  RBQ_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  return n > 0 ? n : 1;
}

void launch_refine_all(const float* A, int64_t nq, const float* C, int d, int K, int p, const int* unsafe,
                       int32_t* probes, float* g, cudaStream_t s)
{
  if (nq <= 0) return;
  const int buf = std::max(next_pow2(p), p + kRefineAllChunk);  // room for a chunk and the final sort
  const size_t smem = (size_t)buf * 8 * 2 + (size_t)d * 4;
  RBQ_CHECK(smem <= 200 * 1024, RBQ_ERR_INVALID, "coarse: exact probe pass too large (nprobe / dim)");
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(refine_all_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const unsigned grid = (unsigned)std::min<int64_t>(nq, (int64_t)device_sm_count() * 4);
  refine_all_kernel<<<grid, 256, smem, s>>>(A, C, d, K, p, buf, unsafe, probes, g);
  RBQ_LAUNCHED();
}

// max_l C_n2[l] into *out (one block).
__global__ void __launch_bounds__(1024) max_reduce_kernel(const float* __restrict__ v, int n, float* __restrict__ out)
{
  __shared__ float s_m[32];
  float mx = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, v[i]);
#pragma unroll
  for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((threadIdx.x & 31) == 0) s_m[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    mx = threadIdx.x < (blockDim.x >> 5) ? s_m[threadIdx.x] : 0.0f;
#pragma unroll
    for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (threadIdx.x == 0) *out = mx;
  }
}

void launch_max_reduce(const float* v, int n, float* out, cudaStream_t s)
{
  max_reduce_kernel<<<1, 1024, 0, s>>>(v, n, out);
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// QB-bit query quantisation (exrabitq_quantize_query<256> with EX_BITS = num_bits = QB,
// searcher_gpu_quantize_query.cu:655-793; QUANT4: QB = 4, scale t4; QUANT8: QB = 8, scale t8)
// and k1 = -0.5 * sum q (ivf_gpu.cu:1451-1490).  One thread per query; sums are double
// accumulations in dimension order.  A block of 32 queries first stages its rows in shared
// memory (coalesced loads; rows padded by one float so that the 32 threads reading column j
// hit 32 banks).
//   code_j = clamp(rint(t * (q_j * (1/|q|))), -2^(QB-1), 2^(QB-1) - 1)
//   delta = (|q| / |code|) * (<q, code> / (|q| * |code|))   (0 if either norm <= 1e-6)
//   plane b, word w, bit 31-j = bit b of the QB-bit two's complement of code_{32w+j}
// ---------------------------------------------------------------------------------------
constexpr int kPrepQueries = 32;

template <int QB>
__global__ void __launch_bounds__(kPrepQueries) query_prep_kernel(const float* __restrict__ Qr, int64_t nq, int Dp,
                                                                  float t, uint32_t* __restrict__ planes,
                                                                  float* __restrict__ delta, float* __restrict__ k1)
{
  constexpr int kHi = (1 << (QB - 1)) - 1, kLo = -(1 << (QB - 1));
  constexpr uint32_t kMask = (1u << QB) - 1u;
  extern __shared__ float rows[];  // [kPrepQueries][Dp + 1]
  const int64_t q0 = (int64_t)blockIdx.x * kPrepQueries;
  const int nb = (int)(nq - q0 < kPrepQueries ? nq - q0 : kPrepQueries);
  const int ld = Dp + 1;
  for (int r = 0; r < nb; ++r)
    for (int j = threadIdx.x; j < Dp; j += kPrepQueries) rows[r * ld + j] = Qr[(q0 + r) * Dp + j];
  __syncthreads();
  if ((int)threadIdx.x >= nb) return;
  const int64_t q = q0 + threadIdx.x;
  const float* x = rows + threadIdx.x * ld;
  double s2 = 0.0, s1 = 0.0;
  for (int j = 0; j < Dp; ++j) {
    const double v = (double)x[j];
    s2 += v * v;
    s1 += v;
  }
  const float norm = sqrtf((float)s2);
  const float norm_inv = (norm > 0.0f) ? (1.0f / norm) : 0.0f;
  const int W = Dp >> 5;
  uint32_t* pl = planes + q * QB * W;
  double ipd = 0.0;
  long long xs = 0;
  for (int w = 0; w < W; ++w) {
    uint32_t p[QB];
#pragma unroll
    for (int b = 0; b < QB; ++b) p[b] = 0u;
    for (int j32 = 0; j32 < 32; ++j32) {
      const int j = (w << 5) + j32;
      const float val = x[j] * norm_inv;
      int cv = __float2int_rn(t * val);
      cv = cv > kHi ? kHi : (cv < kLo ? kLo : cv);
      ipd += (double)x[j] * (double)cv;
      xs += (long long)(cv * cv);
      const uint32_t u = (uint32_t)cv & kMask;
      const int sh = 31 - j32;
#pragma unroll
      for (int b = 0; b < QB; ++b) p[b] |= ((u >> b) & 1u) << sh;
    }
#pragma unroll
    for (int b = 0; b < QB; ++b) pl[b * W + w] = p[b];
  }
  const float ip = (float)ipd;
  const float xu_sq = (float)xs;
  const float norm_quan = sqrtf(fmaxf(xu_sq, 0.0f));
  float dl = 0.0f;
  if (norm > 1e-6f && norm_quan > 1e-6f) {
    const float cosv = ip / (norm * norm_quan);
    dl = (norm / norm_quan) * cosv;
  }
  delta[q] = dl;
  k1[q] = ((float)s1) * -0.5f;
}

void launch_query_prep(const float* Qr, int64_t nq, int Dp, float t, int qbits, uint32_t* planes, float* delta,
                       float* k1, cudaStream_t s)
{
  if (nq <= 0) return;
  RBQ_CHECK(qbits == 4 || qbits == 8, RBQ_ERR_INVALID, "query bits must be 4 (QUANT4) or 8 (QUANT8)");
  const size_t smem = (size_t)kPrepQueries * (Dp + 1) * sizeof(float);
  const unsigned grid = (unsigned)ceil_div(nq, kPrepQueries);
  if (qbits == 4) {
    if (smem > 48 * 1024)
      RBQ_CUDA(cudaFuncSetAttribute(query_prep_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    query_prep_kernel<4><<<grid, kPrepQueries, smem, s>>>(Qr, nq, Dp, t, planes, delta, k1);
  } else {
    if (smem > 48 * 1024)
      RBQ_CUDA(cudaFuncSetAttribute(query_prep_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    query_prep_kernel<8><<<grid, kPrepQueries, smem, s>>>(Qr, nq, Dp, t, planes, delta, k1);
  }
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// The list scan (computeInnerProductsWithBitwiseBlockSort<4, false, false>,
// searcher_gpu_quantize_query.cu:172-626, re-designed).  One CTA of 256 threads per
// (query, probe slice).  The slice's lists form one flat sequence of vectors (probe order,
// slot order inside a list) walked in tiles of kScanTile = 1024 vectors that run across list
// boundaries; thread t takes vectors t, t + 256, t + 512 and t + 768 of each tile (tiles of 512
// paid twice the barriers and threshold checks per vector; at 2048 the key buffers outgrow the
// shared memory of six resident blocks).
//   phase 1 (per thread; query planes broadcast from shared memory as 16-byte loads)
//            acc = sum_w [sum_{b<3} popc(P_b & c) << b  -  popc(P_3 & c) << 3]   (exact int)
//            summed by carry-save adders (two three-input logic ops each) and popcounts weighted
//            by integer multiply-adds, which keeps the logic pipe for the adders
//            est = (f_add + g) + f_rescale * (acc * delta + k1);  low = est - f_err * sqrt(g)
//            admit if !prune || low < tau
//   phase 2 (per warp)  right after each round of phase 1, the warp's admitted vectors are
//            taken one at a time by all 32 lanes (warp_exact_ip: per-byte sums, lane sums,
//            xor butterfly);
//            dist = (f_add + g) + f_rescale * (exact_ip + k1); keep (dist, id) if dist <= tau.
// tau (the R-th best kept distance) only changes between tiles: when the buffer holds more
// than cap - kScanTile keys, 2R keys, or R keys while tau is still +inf, it is cut to the R
// smallest.  A slice starts from tau0 (if given), slice 0 from the initial candidates (if
// given), and a pruning slice with neither from the bound seed below.  The schedule depends on
// the data alone, so results are deterministic and equal to the oracle's.
// ---------------------------------------------------------------------------------------
constexpr int kScanThreads = 256;
constexpr int kScanVpt = kScanTile / kScanThreads;
static_assert(kScanTile % kScanThreads == 0, "tile must be a multiple of the block size");

template <int W>
__device__ __forceinline__ void load_code(const uint32_t* __restrict__ codes, int64_t slot, uint32_t (&c)[W])
{
  if constexpr (W % 4 == 0) {
    const uint4* p = reinterpret_cast<const uint4*>(codes + slot * W);
#pragma unroll
    for (int i = 0; i < W / 4; ++i) {
      const uint4 v = __ldg(p + i);
      c[4 * i + 0] = v.x;
      c[4 * i + 1] = v.y;
      c[4 * i + 2] = v.z;
      c[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < W; ++i) c[i] = __ldg(codes + slot * W + i);
  }
}

// <bits of the vector at `slot`, q>, computed by the whole warp; every lane returns the value.
// Lane l adds bsum(j) for the code bytes j = l, l + 32, ... (bsum(j) = sum of q over the set
// bits of byte j of the MSB-first bit stream, dims 8j..8j+7, bit 7 first, from 0), then an xor
// butterfly (16, 8, 4, 2, 1) combines the lanes.  qsT is the query transposed by byte
// (qsT[jj * NB + j] = q[8 j + jj]), so the 32 lanes read 32 consecutive words.
template <int W>
__device__ __forceinline__ float warp_exact_ip(const uint32_t* __restrict__ codes, int64_t slot,
                                               const float* __restrict__ qsT, int lane)
{
  constexpr int NB = 4 * W;
  constexpr int M = (NB + 31) / 32;
  const unsigned char* cb = reinterpret_cast<const unsigned char*>(codes + slot * W);
  float v = 0.0f;
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const int j = lane + 32 * m;
    if (j < NB) {
      const uint32_t u8 = __ldg(cb + (j ^ 3));  // byte j of the MSB-first bit stream
      float b = 0.0f;
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const float q = qsT[jj * NB + j];
        b = ((u8 >> (7 - jj)) & 1u) ? __fadd_rn(b, q) : b;
      }
      v = __fadd_rn(v, b);
    }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// warp_exact_ip for four vectors at once, one per 8-lane group (lanes 8g..8g+7 take the vector
// at their own `slot`): lane k of a group forms the values that lanes k, k + 8, k + 16 and k + 24
// hold in warp_exact_ip, then adds them in that function's tree order (xor 16, then xor 8) and
// finishes with the xor 4, 2, 1 steps inside the group.  Every addition has the same operands,
// so the result equals warp_exact_ip's bit for bit; every lane of a group returns it.
template <int W>
__device__ __forceinline__ float group8_exact_ip(const uint32_t* __restrict__ codes, int64_t slot,
                                                 const float* __restrict__ qsT, int lane)
{
  constexpr int NB = 4 * W;
  constexpr int M = (NB + 31) / 32;
  const unsigned char* cb = reinterpret_cast<const unsigned char*>(codes + slot * W);
  const int k = lane & 7;
  float v[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    float acc = 0.0f;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const int j = k + 8 * h + 32 * m;
      if (j < NB) {
        const uint32_t u8 = __ldg(cb + (j ^ 3));
        float b = 0.0f;
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const float q = qsT[jj * NB + j];
          b = ((u8 >> (7 - jj)) & 1u) ? __fadd_rn(b, q) : b;
        }
        acc = __fadd_rn(acc, b);
      }
    }
    v[h] = acc;
  }
  float t = __fadd_rn(__fadd_rn(v[0], v[2]), __fadd_rn(v[1], v[3]));
#pragma unroll
  for (int off = 4; off; off >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, off));
  return t;
}

// <x, q> of the extra-bit code x at `slot` (planes [ex, W], plane p = bit p of every dim's
// code), computed by the whole warp: lane l takes code bytes j = l, l + 32, ...; per byte, planes
// p = ex-1 down to 0 add 2^p * bsum_p(j) (the sum of q over the set bits of byte j of plane p, bit
// 7 first, from 0) to the lane's value; an xor butterfly combines the lanes.
template <int W>
__device__ __forceinline__ float warp_ex_ip(const uint32_t* __restrict__ ex_codes, int64_t slot, int ex,
                                            const float* __restrict__ qsT, int lane)
{
  constexpr int NB = 4 * W;
  constexpr int M = (NB + 31) / 32;
  const unsigned char* cb = reinterpret_cast<const unsigned char*>(ex_codes + slot * ex * W);
  float v = 0.0f;
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const int j = lane + 32 * m;
    if (j < NB) {
      float qv[8];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) qv[jj] = qsT[jj * NB + j];
      for (int p = ex - 1; p >= 0; --p) {
        const uint32_t u8 = __ldg(cb + p * NB + (j ^ 3));
        float b = 0.0f;
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) b = ((u8 >> (7 - jj)) & 1u) ? __fadd_rn(b, qv[jj]) : b;
        v = __fadd_rn(v, __fmul_rn((float)(1 << p), b));
      }
    }
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// ---------------------------------------------------------------------------------------
// Signed 4-bit x 1-bit inner product with few popcounts.  The AND-ed plane words are summed
// bit-sliced with carry-save adders (Harley-Seal): a full adder turns three words of weight w
// into a sum word (weight w) and a carry word (weight 2w) in two logic ops, so eight words of
// a plane (and the carries of the plane below) collapse into one word per weight before any
// popcount.  The integer result equals sum_w [sum_{b<3} popc(P_b & c) << b - popc(P_3 & c) << 3].
// ---------------------------------------------------------------------------------------
// Any three-input bitwise function in one instruction: LUT is its truth table over the inputs
// a = 0xF0, b = 0xCC, c = 0xAA (PTX lop3.b32).
template <unsigned LUT>
__device__ __forceinline__ uint32_t lop3(uint32_t a, uint32_t b, uint32_t c)
{
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(d) : "r"(a), "r"(b), "r"(c), "n"(LUT));
  return d;
}
// Full adder: carry = majority(a, b, c), sum = a ^ b ^ c; two instructions.
__device__ __forceinline__ void csa(uint32_t& h, uint32_t& l, uint32_t a, uint32_t b, uint32_t c)
{
  h = lop3<0xE8>(a, b, c);
  l = lop3<0x96>(a, b, c);
}
__device__ __forceinline__ void hadd(uint32_t& h, uint32_t& l, uint32_t a, uint32_t b)
{
  h = a & b;
  l = a ^ b;
}
// Half adder of x and (p & c) with the AND folded in: carry x & p & c, sum x ^ (p & c).
__device__ __forceinline__ void hadd_and(uint32_t& h, uint32_t& l, uint32_t x, uint32_t p, uint32_t c)
{
  h = lop3<0x80>(x, p, c);
  l = lop3<0x78>(x, p, c);
}

// Weights of the popcounts of the adder outputs (weight 1, 2, 4, 8, 16, 32) and of plane 3 (-8).
// Held in constant memory and never written, so the weighted sum compiles to integer
// multiply-adds reading the weight from the constant bank (the multiply-add pipe), not to
// shifts and adds on the integer logic pipe that the adders keep busy.
__constant__ int32_t c_popc_weight[8] = {1, 2, 4, 8, 16, 32, -8, 0};

// Eight words: P(b, w) returns plane b word w of the chunk, c the chunk's code words.
template <typename PF>
__device__ __forceinline__ int32_t signed_dot8(const PF& P, const uint32_t (&c)[8])
{
  uint32_t a[8], b[8], d[8], e[8];
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    a[w] = P(0, w) & c[w];
    b[w] = P(1, w) & c[w];
    d[w] = P(2, w) & c[w];
    e[w] = P(3, w) & c[w];
  }
  uint32_t o1 = a[0], k0, k1, k2, k3;  // weight 1 (plane 0)
  csa(k0, o1, o1, a[1], a[2]);
  csa(k1, o1, o1, a[3], a[4]);
  csa(k2, o1, o1, a[5], a[6]);
  hadd(k3, o1, o1, a[7]);
  uint32_t o2 = k0, m0, m1, m2, m3, m4, m5;  // weight 2 (carries + plane 1)
  csa(m0, o2, o2, k1, k2);
  csa(m1, o2, o2, k3, b[0]);
  csa(m2, o2, o2, b[1], b[2]);
  csa(m3, o2, o2, b[3], b[4]);
  csa(m4, o2, o2, b[5], b[6]);
  hadd(m5, o2, o2, b[7]);
  uint32_t o4 = m0, n0, n1, n2, n3, n4, n5, n6;  // weight 4 (carries + plane 2)
  csa(n0, o4, o4, m1, m2);
  csa(n1, o4, o4, m3, m4);
  csa(n2, o4, o4, m5, d[0]);
  csa(n3, o4, o4, d[1], d[2]);
  csa(n4, o4, o4, d[3], d[4]);
  csa(n5, o4, o4, d[5], d[6]);
  hadd(n6, o4, o4, d[7]);
  uint32_t o8 = n0, r0, r1, r2;  // weight 8
  csa(r0, o8, o8, n1, n2);
  csa(r1, o8, o8, n3, n4);
  csa(r2, o8, o8, n5, n6);
  uint32_t o16 = r0, t0;  // weight 16, 32
  csa(t0, o16, o16, r1, r2);
  const int32_t pos = __popc(o1) + 2 * __popc(o2) + 4 * __popc(o4) + 8 * __popc(o8) + 16 * __popc(o16) +
                      32 * __popc(t0);
  // plane 3 (weight -8): one popcount per word keeps the popcount unit busy while the logic
  // unit does the adders above
  const int32_t neg = (__popc(e[0]) + __popc(e[1]) + __popc(e[2]) + __popc(e[3])) +
                      (__popc(e[4]) + __popc(e[5]) + __popc(e[6]) + __popc(e[7]));
  return pos - 8 * neg;
}

// The same eight-word sum with the plane words fetched as 16-byte groups G(b, h) (plane b,
// words 4h..4h+3) in the order the adders consume them, so at most one group of plane words is
// live at a time.
template <typename GF>
__device__ __forceinline__ int32_t signed_dot8_grouped(const GF& G, const uint32_t (&c)[8])
{
  uint4 g = G(0, 0);
  uint32_t o1 = g.x & c[0], k0, k1, k2, k3;  // weight 1 (plane 0)
  csa(k0, o1, o1, g.y & c[1], g.z & c[2]);
  uint32_t t = g.w & c[3];
  g = G(0, 1);
  csa(k1, o1, o1, t, g.x & c[4]);
  csa(k2, o1, o1, g.y & c[5], g.z & c[6]);
  hadd_and(k3, o1, o1, g.w, c[7]);
  g = G(1, 0);
  uint32_t o2 = k0, m0, m1, m2, m3, m4, m5;  // weight 2 (carries + plane 1)
  csa(m0, o2, o2, k1, k2);
  csa(m1, o2, o2, k3, g.x & c[0]);
  csa(m2, o2, o2, g.y & c[1], g.z & c[2]);
  t = g.w & c[3];
  g = G(1, 1);
  csa(m3, o2, o2, t, g.x & c[4]);
  csa(m4, o2, o2, g.y & c[5], g.z & c[6]);
  hadd_and(m5, o2, o2, g.w, c[7]);
  g = G(2, 0);
  uint32_t o4 = m0, n0, n1, n2, n3, n4, n5, n6;  // weight 4 (carries + plane 2)
  csa(n0, o4, o4, m1, m2);
  csa(n1, o4, o4, m3, m4);
  csa(n2, o4, o4, m5, g.x & c[0]);
  csa(n3, o4, o4, g.y & c[1], g.z & c[2]);
  t = g.w & c[3];
  g = G(2, 1);
  csa(n4, o4, o4, t, g.x & c[4]);
  csa(n5, o4, o4, g.y & c[5], g.z & c[6]);
  hadd_and(n6, o4, o4, g.w, c[7]);
  uint32_t o8 = n0, r0, r1, r2;  // weight 8
  csa(r0, o8, o8, n1, n2);
  csa(r1, o8, o8, n3, n4);
  csa(r2, o8, o8, n5, n6);
  uint32_t o16 = r0, t0;  // weight 16, 32
  csa(t0, o16, o16, r1, r2);
  const int32_t* wt = c_popc_weight;
  int32_t acc = __popc(o1) * wt[0];
  acc = __popc(o2) * wt[1] + acc;
  acc = __popc(o4) * wt[2] + acc;
  acc = __popc(o8) * wt[3] + acc;
  acc = __popc(o16) * wt[4] + acc;
  acc = __popc(t0) * wt[5] + acc;
  g = G(3, 0);  // plane 3 (weight -8): one popcount per word
  acc = __popc(g.x & c[0]) * wt[6] + acc;
  acc = __popc(g.y & c[1]) * wt[6] + acc;
  acc = __popc(g.z & c[2]) * wt[6] + acc;
  acc = __popc(g.w & c[3]) * wt[6] + acc;
  g = G(3, 1);
  acc = __popc(g.x & c[4]) * wt[6] + acc;
  acc = __popc(g.y & c[5]) * wt[6] + acc;
  acc = __popc(g.z & c[6]) * wt[6] + acc;
  acc = __popc(g.w & c[7]) * wt[6] + acc;
  return acc;
}

template <typename PF>
__device__ __forceinline__ int32_t signed_dot4(const PF& P, const uint32_t (&c)[4])
{
  uint32_t o1 = P(0, 0) & c[0], k0, k1;  // weight 1 (plane 0)
  csa(k0, o1, o1, P(0, 1) & c[1], P(0, 2) & c[2]);
  hadd_and(k1, o1, o1, P(0, 3), c[3]);
  uint32_t o2 = k0, m0, m1, m2;  // weight 2 (carries + plane 1)
  csa(m0, o2, o2, k1, P(1, 0) & c[0]);
  csa(m1, o2, o2, P(1, 1) & c[1], P(1, 2) & c[2]);
  hadd_and(m2, o2, o2, P(1, 3), c[3]);
  uint32_t o4 = m0, n0, n1, n2;  // weight 4 (carries + plane 2)
  csa(n0, o4, o4, m1, m2);
  csa(n1, o4, o4, P(2, 0) & c[0], P(2, 1) & c[1]);
  csa(n2, o4, o4, P(2, 2) & c[2], P(2, 3) & c[3]);
  uint32_t o8 = n0, r0;  // weight 8, 16
  csa(r0, o8, o8, n1, n2);
  const int32_t* wt = c_popc_weight;
  int32_t acc = __popc(o1) * wt[0];
  acc = __popc(o2) * wt[1] + acc;
  acc = __popc(o4) * wt[2] + acc;
  acc = __popc(o8) * wt[3] + acc;
  acc = __popc(r0) * wt[4] + acc;
#pragma unroll
  for (int w = 0; w < 4; ++w) acc = __popc(P(3, w) & c[w]) * wt[6] + acc;  // plane 3 (weight -8)
  return acc;
}

// Whole vector: chunks of 8 words (or one 4-word chunk), else one popcount per plane word.
// QB = 8 (QUANT8, searcher_gpu_quantize_query.cu:253-262 with NumBits = 8): one popcount per
// plane word, sum_w [sum_{b<7} popc(P_b & c) << b - popc(P_7 & c) << 7].
template <int W, int QB = 4, typename PF>
__device__ __forceinline__ int32_t signed_dot(const PF& P, const uint32_t (&c)[W])
{
  if constexpr (QB == 8) {
    int32_t acc = 0;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      int32_t pos = 0;
#pragma unroll
      for (int b = 0; b < 7; ++b) pos += __popc(P(b, w) & c[w]) << b;
      acc += pos - (__popc(P(7, w) & c[w]) << 7);
    }
    return acc;
  } else if constexpr (W % 8 == 0) {
    int32_t acc = 0;
#pragma unroll
    for (int k = 0; k < W / 8; ++k) {
      uint32_t cc[8];
#pragma unroll
      for (int w = 0; w < 8; ++w) cc[w] = c[8 * k + w];
      auto Pk = [&](int b, int w) { return P(b, 8 * k + w); };
      acc += signed_dot8(Pk, cc);
    }
    return acc;
  } else if constexpr (W == 4) {
    return signed_dot4(P, c);
  } else {
    int32_t s0 = 0, s1 = 0, s2 = 0, s3 = 0;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      s0 += __popc(P(0, w) & c[w]);
      s1 += __popc(P(1, w) & c[w]);
      s2 += __popc(P(2, w) & c[w]);
      s3 += __popc(P(3, w) & c[w]);
    }
    return s0 + 2 * s1 + 4 * s2 - 8 * s3;
  }
}

// The query's planes live at the start of the scan's shared memory (16-byte aligned), so when
// W % 4 == 0 each group of four plane words is one 16-byte shared load instead of four.
template <int W, int QB>
__device__ __forceinline__ int32_t dot_smem(const uint32_t* __restrict__ pl, const uint32_t (&c)[W])
{
  if constexpr (QB == 4 && W == 8) {
    int32_t acc = 0;
#pragma unroll
    for (int k = 0; k < W / 8; ++k) {
      uint32_t cc[8];
#pragma unroll
      for (int w = 0; w < 8; ++w) cc[w] = c[8 * k + w];
      auto G = [&](int b, int h) -> uint4 { return reinterpret_cast<const uint4*>(pl + b * W + 8 * k)[h]; };
      acc += signed_dot8_grouped(G, cc);
    }
    return acc;
  } else if constexpr (QB == 4 && W == 4) {
    const uint4 g0 = reinterpret_cast<const uint4*>(pl)[0], g1 = reinterpret_cast<const uint4*>(pl)[1];
    const uint4 g2 = reinterpret_cast<const uint4*>(pl)[2], g3 = reinterpret_cast<const uint4*>(pl)[3];
    auto P = [&](int b, int w) -> uint32_t {
      const uint4& v = b == 0 ? g0 : (b == 1 ? g1 : (b == 2 ? g2 : g3));
      return w == 0 ? v.x : (w == 1 ? v.y : (w == 2 ? v.z : v.w));
    };
    return signed_dot4(P, c);
  } else {
    auto P = [&](int b, int w) -> uint32_t { return pl[b * W + w]; };
    return signed_dot<W, QB>(P, c);
  }
}

// acc of the vector at `slot`.
template <int W, int QB>
__device__ __forceinline__ int32_t dot_vector(const uint32_t* __restrict__ codes, int64_t slot,
                                              const uint32_t* __restrict__ pl)
{
  uint32_t c[W];
  load_code<W>(codes, slot, c);
  return dot_smem<W, QB>(pl, c);
}

// ---------------------------------------------------------------------------------------
// Block-wide selection of the R smallest of n distinct keys src[0..n) (R <= n): a radix
// select, 8 bits per pass from the top, finds the threshold key T with exactly R keys <= T;
// those are copied to dst[0..R) (any order) and the largest of them (the R-th smallest key) is
// returned.  hist: 256 shared counters; misc: 3 shared ints; kmax, cnt: shared scratch.
// ---------------------------------------------------------------------------------------
// hist[bin] += 1 for every lane with `take`, one shared atomic per distinct bin of the warp:
// keys that share their leading bytes (close distances) would otherwise serialise up to 32
// atomics on one counter.
__device__ __forceinline__ void hist_add_aggregated(unsigned* hist, bool take, unsigned bin, int lane)
{
  const unsigned active = __ballot_sync(0xffffffffu, take);
  if (!take) return;
  const unsigned peers = __match_any_sync(active, bin);
  if (lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (unsigned)__popc(peers));
}

__device__ unsigned long long block_keep_smallest(const unsigned long long* src, int n, int R,
                                                  unsigned long long* dst, unsigned* hist, int* misc,
                                                  unsigned long long* kmax, int* cnt)
{
  const int tid = threadIdx.x, lane = tid & 31;
  unsigned long long prefix = 0, pmask = 0;
  int need = R;
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0u;
    __syncthreads();
    for (int i0 = tid - lane; i0 < n; i0 += blockDim.x) {  // warp-uniform trip count
      const int i = i0 + lane;
      const unsigned long long k = i < n ? src[i] : 0ull;
      hist_add_aggregated(hist, i < n && (k & pmask) == prefix, (unsigned)(k >> shift) & 255u, lane);
    }
    __syncthreads();
    if (tid < 32) {
      unsigned v[8], s = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[j] = hist[lane * 8 + j];
        s += v[j];
      }
      unsigned inc = s;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const unsigned t = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += t;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, inc >= (unsigned)need);
      if (lane == __ffs(hit) - 1) {
        unsigned cum = inc - s;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (cum + v[j] >= (unsigned)need) {
            misc[0] = lane * 8 + j;
            misc[1] = need - (int)cum;
            misc[2] = (int)v[j];
            break;
          }
          cum += v[j];
        }
      }
    }
    __syncthreads();
    const int bin = misc[0], nd = misc[1], inbin = misc[2];
    __syncthreads();
    prefix |= (unsigned long long)bin << shift;
    pmask |= 255ull << shift;
    need = nd;
    if (inbin == need) {  // the whole bin is kept: everything at or below its top
      if (shift > 0) prefix |= (1ull << shift) - 1;
      break;
    }
  }
  if (tid == 0) {
    *kmax = 0ull;
    *cnt = 0;
  }
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    const unsigned long long k = src[i];
    if (k <= prefix) {
      dst[atomicAdd(cnt, 1)] = k;
      atomicMax(kmax, k);
    }
  }
  __syncthreads();
  return *kmax;
}

#ifndef RBQ_SCAN_MINB8
#define RBQ_SCAN_MINB8 6
#endif
// Resident CTAs per SM the scan is compiled for: occupancy hides the L2 latency of the code
// loads, so vectors up to 256 dims get 6 CTAs (40 registers, no spill); wider ones 4.
template <int W>
constexpr int scan_min_blocks()
{
  return (W <= 4 || W == 8) ? RBQ_SCAN_MINB8 : (W < 8 ? 5 : 4);
}

// Bytes at the start of the scan's shared memory before the key buffers: the query planes
// (popcount modes) or the query tables (LUT16: fp16, LUT32: fp32 entries, 16 per 4-dim chunk),
// then the byte-transposed query (8 * 4W floats; in the LUT modes only filled for extra-bit
// codes).  All multiples of 16.
template <int W, int QB>
constexpr int scan_table_bytes()
{
  return QB == 16 ? 256 * W : (QB == 32 ? 512 * W : 4 * W * QB);
}
template <int W, int QB>
constexpr int scan_head_bytes()
{
  return scan_table_bytes<W, QB>() + 128 * W;
}

// <bits, q> by the query tables: words in order, nibbles from the top (bit 31) down, added one
// by one (computeInnerProductsWithLUT16Opt, searcher_gpu_shared_mem_opt.cu:165-177).
template <int W, int QB>
__device__ __forceinline__ float lut_ip(const unsigned char* __restrict__ tab, const uint32_t (&c)[W])
{
  float ip = 0.0f;
#pragma unroll
  for (int w = 0; w < W; ++w)
#pragma unroll
    for (int ci = 0; ci < 8; ++ci) {
      const int e = (w * 8 + ci) * 16 + (int)((c[w] >> (28 - 4 * ci)) & 0xFu);
      float v;
      if constexpr (QB == 16)
        v = __half2float(reinterpret_cast<const __half*>(tab)[e]);
      else
        v = reinterpret_cast<const float*>(tab)[e];
      ip = __fadd_rn(ip, v);
    }
  return ip;
}

// One unit of the tile scan: slice u % slices of query qorder[u / slices] (u / slices without
// an order).  Every early return is taken by the whole block.
template <int W, int QB>
__device__ __forceinline__ void scan_unit(const ScanArgs& a, const unsigned u)
{
  constexpr int NB = 4 * W;
  constexpr bool kLut = QB >= 16;    // LUT16 / LUT32: the table estimate is the distance
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // planes first (16-byte aligned); QB*W + 8*NB words = 4W(QB + 32) bytes keep the keys 8-aligned
  uint32_t* pl = reinterpret_cast<uint32_t*>(smem_raw);                        // [QB * W]
  unsigned char* tab = smem_raw;                                                // LUT modes
  float* qsT = reinterpret_cast<float*>(smem_raw + scan_table_bytes<W, QB>());  // [8 * NB]
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_raw + scan_head_bytes<W, QB>());  // [cap]
  unsigned long long* keys2 = keys + a.cap;                                    // [cap]
  int* pre = reinterpret_cast<int*>(keys2 + a.cap);                            // [nprobe + 1]
  int* lbase = pre + (a.nprobe + 1);                                            // [nprobe]
  float* lg = reinterpret_cast<float*>(lbase + a.nprobe);                       // [nprobe]
  float* lsq = lg + a.nprobe;                                                   // [nprobe]
  __shared__ int s_count, s_nl, s_misc[3], s_cnt2;
  __shared__ float s_tau;
  __shared__ unsigned s_hist[256];
  __shared__ unsigned long long s_kmax;

  const int64_t qi = u / (unsigned)a.slices;
  const int slice = (int)(u - (unsigned)qi * (unsigned)a.slices);
  const int64_t q = a.qorder ? (int64_t)a.qorder[qi] : qi;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (a.over_cnt && a.over_cnt[q] <= a.over_cap) return;  // only the list scan's overflowed rows
  if (a.tau_out && a.seed_nearest_owned) {
    const int l0 = a.probes[q * a.pstride];
    if (l0 < 0 || __ldg(a.owner + l0) != a.shard_rank) {
      if (tid == 0) a.tau_out[q] = __int_as_float(0x7f800000);
      return;
    }
  }
  // fixed-threshold scan: admission against tau0[q] throughout
  const float tau_fix = a.tau0 ? a.tau0[q] : __int_as_float(0x7f800000);

  if constexpr (kLut) {
    // query tables (precomputeAllLUTs / precomputeAllLUTs_fp16_simple, searcher_gpu.cu:65-108,
    // searcher_gpu_shared_mem_opt.cu:520-549): chunk c, pattern p -> fp32 sum from 0, in dimension
    // order, of q[4c + b] over the b with bit 3 - b of p set (LUT16: rounded to fp16)
    const float* qv = a.Qr + q * (32 * W);
    for (int i = tid; i < 8 * W * 16; i += kScanThreads) {
      const int c = i >> 4, pat = i & 15;
      float sum = 0.0f;
#pragma unroll
      for (int b = 0; b < 4; ++b)
        if (pat & (8 >> b)) sum = __fadd_rn(sum, qv[4 * c + b]);
      if constexpr (QB == 16)
        reinterpret_cast<__half*>(tab)[i] = __float2half_rn(sum);
      else
        reinterpret_cast<float*>(tab)[i] = sum;
    }
    if (a.ex_bits > 0)
      for (int i = tid; i < 8 * NB; i += kScanThreads) {
        const int jj = i / NB, j = i - jj * NB;
        qsT[i] = a.Qr[q * (8 * NB) + 8 * j + jj];
      }
  } else {
    for (int i = tid; i < 8 * NB; i += kScanThreads) {
      const int jj = i / NB, j = i - jj * NB;
      qsT[i] = a.Qr[q * (8 * NB) + 8 * j + jj];
    }
    for (int j = tid; j < QB * W; j += kScanThreads) pl[j] = a.planes[q * QB * W + j];
  }
  if (warp == 0) {
    // The slice's lists: owned probes (owner[l] == shard_rank) with owned-rank in
    // [pb, pe); per list its first slot, g, sqrt(g) and the running start pre[] of the flat
    // sequence.
    const int* prow = a.probes + q * a.pstride;
    int m = 0;
    for (int p0 = 0; p0 < a.nprobe; p0 += 32) {
      const int p = p0 + lane;
      const int l = p < a.nprobe ? prow[p] : -1;
      m += __popc(__ballot_sync(0xffffffffu, l >= 0 && __ldg(a.owner + l) == a.shard_rank));
    }
    const int pb = (int)(((int64_t)slice * m) / a.slices);
    const int pe = (int)(((int64_t)(slice + 1) * m) / a.slices);
    int o = 0;
    for (int p0 = 0; p0 < a.nprobe && o < pe; p0 += 32) {
      const int p = p0 + lane;
      const int l = p < a.nprobe ? prow[p] : -1;
      const bool own = l >= 0 && __ldg(a.owner + l) == a.shard_rank;
      const unsigned mask = __ballot_sync(0xffffffffu, own);
      const int rank = o + __popc(mask & ((1u << lane) - 1u));
      if (own && rank >= pb && rank < pe) {
        const int i = rank - pb;
        const int64_t b0 = a.list_off[l];
        const float g = a.g[q * a.pstride + p];
        lbase[i] = (int)b0;
        pre[i + 1] = (int)(a.list_off[l + 1] - b0);  // size, turned into a prefix below
        lg[i] = g;
        lsq[i] = sqrtf(g);
      }
      o += __popc(mask);
    }
    const int n = pe - pb;
    __syncwarp();
    int carry = 0;
    for (int c0 = 0; c0 < n; c0 += 32) {
      const int i = c0 + lane;
      int v = i < n ? pre[i + 1] : 0;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += t;
      }
      if (i < n) pre[i + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) {
      pre[0] = 0;
      if (n == 0) {
        lbase[0] = 0;
        lg[0] = 0.0f;
        lsq[0] = 0.0f;
      }
      s_nl = n;
      s_count = 0;
      s_kmax = 0ull;
      s_tau = a.tau0 ? a.tau0[q] : __int_as_float(0x7f800000);
    }
  }
  __syncthreads();
  if (a.init_keys && slice == 0) {
    for (int i = tid; i < a.R; i += kScanThreads) {
      const unsigned long long k = a.init_keys[q * a.R + i];
      if (k != kEmptyKey) {
        keys[atomicAdd(&s_count, 1)] = k;
        atomicMax(&s_kmax, k);
      }
    }
    __syncthreads();
    if (tid == 0 && s_count == a.R) s_tau = fminf(s_tau, from_ordered_bits((uint32_t)(s_kmax >> 32)));
    __syncthreads();
  }
  const int nl = s_nl;
  const int total = pre[nl];
  const float delta = a.delta[q];
  const float k1 = a.k1[q];
  // extra-bit estimator constants: 2^ex and kb = -(2^(ex+1) - 1)/2 * sum q = k1 * (2^(ex+1) - 1)
  // (computeQueryFactorsWarpKernel, ivf_gpu.cu:1450-1490)
  const float ex_scale = (float)(1 << a.ex_bits);
  const float kb = __fmul_rn(k1, (float)((2 << a.ex_bits) - 1));
  // Bound seed: a pruning slice with no threshold and no candidates yet starts from the R-th
  // smallest upper bound est + f_err * sqrt(g) over its leading whole lists holding at least R
  // vectors (the RaBitQ error bound: R of them are that close), instead of admitting its first
  // tile whole.  The bounds stream through the key buffer in tiles, cut to the R smallest
  // whenever the buffer would overflow.
  if (!kLut && a.prune && !a.fixed_tau && isinf(s_tau) && s_count == 0 && total >= a.R) {
    int nb = 0;
    for (int i = 1; i <= nl && nb < a.R; ++i) nb = pre[i];
    int c = 0, cnt = 0;
    for (int c0 = 0; c0 < nb; c0 += kScanTile) {
      const int c1 = min(nb, c0 + kScanTile);
      for (int f = c0 + tid; f < c1; f += kScanThreads) {
        while (pre[c + 1] <= f) ++c;
        const int slot = lbase[c] + (f - pre[c]);
        const int32_t acc = dot_vector<W, QB>(a.codes, slot, pl);
        const float base_d = __fadd_rn(__ldg(a.fadd + slot), lg[c]);
        const float ip = __fmul_rn((float)acc, delta);
        const float est = __fadd_rn(base_d, __fmul_rn(__ldg(a.frescale + slot), __fadd_rn(ip, k1)));
        const float up = __fadd_rn(est, __fmul_rn(__ldg(a.ferr + slot), lsq[c]));
        keys[cnt + (f - c0)] = make_key(up, (uint32_t)f);
      }
      cnt += c1 - c0;
      __syncthreads();
      if (cnt > a.cap - kScanTile || c1 == nb) {
        const unsigned long long kth = block_keep_smallest(keys, cnt, a.R, keys2, s_hist, s_misc, &s_kmax, &s_cnt2);
        unsigned long long* t = keys;
        keys = keys2;
        keys2 = t;
        cnt = a.R;
        if (c1 == nb && tid == 0) s_tau = from_ordered_bits((uint32_t)(kth >> 32));
      }
      __syncthreads();
    }
  }
  if (a.tau_out) {  // seed-only launch: the slice's starting threshold is the answer
    if (tid == 0) a.tau_out[q] = s_tau;
    return;
  }
  if (a.seed_out && slice == 0 && tid == 0) a.seed_out[q] = s_tau;  // the threshold the scan starts from
  unsigned n_admit = 0;
  // list cursor (monotone per thread): current list, end of it in the flat sequence, slot shift
  int cur = 0;
  int nxt = nl > 0 ? pre[1] : 0;
  int sadj = lbase[0];
  float gc = lg[0], sqc = lsq[0];

  for (int t0 = 0; t0 < total; t0 += kScanTile) {
    const float tau = s_tau;
    const float tau_adm = a.fixed_tau ? tau_fix : tau;
#pragma unroll
    for (int u = 0; u < kScanVpt; ++u) {
      const int f = t0 + u * kScanThreads + tid;
      bool surv = false;
      int sslot = 0;
      float sbase = 0.0f, sfr = 0.0f;
      if (f < total) {
        if (f >= nxt) {
          do {
            ++cur;
          } while (pre[cur + 1] <= f);
          nxt = pre[cur + 1];
          sadj = lbase[cur] - pre[cur];
          gc = lg[cur];
          sqc = lsq[cur];
        }
        const int slot = sadj + f;
        if constexpr (kLut) {
          uint32_t c[W];
          load_code<W>(a.codes, slot, c);
          const float ip = lut_ip<W, QB>(tab, c);
          const float est = __fadd_rn(__fadd_rn(__ldg(a.fadd + slot), gc),
                                      __fmul_rn(__ldg(a.frescale + slot), __fadd_rn(ip, k1)));
          if (a.ex_bits == 0) {
            if (est <= tau) {
              ++n_admit;
              keys[atomicAdd(&s_count, 1)] = make_key(est, __ldg(a.ids + slot));
            }
          } else {  // extra bits: the table estimate's error bound admits (sbase = g, sfr = ip)
            const float low = __fsub_rn(est, __fmul_rn(__ldg(a.ferr + slot), sqc));
            if (!a.prune || low < tau_adm) {
              ++n_admit;
              surv = true;
              sslot = slot;
              sbase = gc;
              sfr = ip;
            }
          }
        } else {
          const int32_t acc = dot_vector<W, QB>(a.codes, slot, pl);
          const float fr = __ldg(a.frescale + slot);
          const float base_d = __fadd_rn(__ldg(a.fadd + slot), gc);
          const float ip = __fmul_rn((float)acc, delta);
          const float est = __fadd_rn(base_d, __fmul_rn(fr, __fadd_rn(ip, k1)));
          const float low = __fsub_rn(est, __fmul_rn(__ldg(a.ferr + slot), sqc));
          if (!a.prune || low < tau_adm) {
            ++n_admit;
            surv = true;
            sslot = slot;
            sbase = a.ex_bits ? gc : base_d;  // extra bits: the distance starts from f_ex_add + g
            sfr = fr;
          }
        }
      }
      if constexpr (kLut) {
        if (a.ex_bits == 0) continue;  // no exact pass: the table estimate is the distance
      }
      // phase 2: the warp's admitted vectors of this round.
      unsigned mask = __ballot_sync(0xffffffffu, surv);
      if (!kLut && a.ex_bits == 0) {
        // four at a time, one per 8-lane group (group g takes the g-th lowest admitted lane)
        while (mask) {
          int src = -1;
#pragma unroll
          for (int gi = 0; gi < 4; ++gi) {
            const int sb = __ffs((int)mask) - 1;
            if ((lane >> 3) == gi) src = sb;
            mask &= mask - 1u;
          }
          const int from = src < 0 ? 0 : src;
          const int slot = __shfl_sync(0xffffffffu, sslot, from);
          const float base_d = __shfl_sync(0xffffffffu, sbase, from);
          const float fr = __shfl_sync(0xffffffffu, sfr, from);
          const float eip = group8_exact_ip<W>(a.codes, slot, qsT, lane);
          const float dist = __fadd_rn(base_d, __fmul_rn(fr, __fadd_rn(eip, k1)));
          if ((lane & 7) == 0 && src >= 0 && dist <= tau) {
            const int at = atomicAdd(&s_count, 1);
            keys[at] = make_key(dist, __ldg(a.ids + slot));
          }
        }
      }
      while (mask) {  // one at a time, all lanes (extra-bit codes)
        const int src = __ffs(mask) - 1;
        mask &= mask - 1;
        const int slot = __shfl_sync(0xffffffffu, sslot, src);
        const float base_d = __shfl_sync(0xffffffffu, sbase, src);
        const float fr = __shfl_sync(0xffffffffu, sfr, src);
        // the extra-bit distance (f_ex_add + g) + f_ex_rescale * ((2^ex ip + ip_x) + kb), ip the
        // 1-bit inner product: exact, or the table one (carried in fr) in the LUT modes
        float ip;
        if constexpr (kLut)
          ip = fr;
        else
          ip = warp_exact_ip<W>(a.codes, slot, qsT, lane);
        const float ipx = warp_ex_ip<W>(a.ex_codes, slot, a.ex_bits, qsT, lane);
        const float T = __fadd_rn(__fadd_rn(__fmul_rn(ex_scale, ip), ipx), kb);
        const float dist = __fadd_rn(__fadd_rn(__ldg(a.fexadd + slot), base_d), __fmul_rn(__ldg(a.fexr + slot), T));
        if (lane == 0 && dist <= tau) {
          const int at = atomicAdd(&s_count, 1);
          keys[at] = make_key(dist, __ldg(a.ids + slot));
        }
      }
    }
    __syncthreads();
    // Tighten tau after a tile when the buffer is nearly full, when it holds 2R keys, or as soon
    // as R keys exist while tau is still open.
    const int cnt = s_count;
    if (cnt > a.cap - kScanTile || cnt >= 2 * a.R || (cnt >= a.R && isinf(s_tau))) {
      const unsigned long long kth = block_keep_smallest(keys, cnt, a.R, keys2, s_hist, s_misc, &s_kmax, &s_cnt2);
      unsigned long long* t = keys;
      keys = keys2;
      keys2 = t;
      if (tid == 0) {
        s_count = a.R;
        s_tau = from_ordered_bits((uint32_t)(kth >> 32));
      }
    }
    __syncthreads();
  }
  // Final top-R: cut to R keys if needed, then sort only the next power of two >= the count.
  int cnt = s_count;
  if (cnt > a.R) {
    block_keep_smallest(keys, cnt, a.R, keys2, s_hist, s_misc, &s_kmax, &s_cnt2);
    keys = keys2;
    cnt = a.R;
  }
  int r2 = 2;
  while (r2 < cnt) r2 <<= 1;
  for (int i = cnt + tid; i < r2; i += kScanThreads) keys[i] = kEmptyKey;
  __syncthreads();
  block_bitonic_sort(keys, r2);
  unsigned long long* out =
      a.out_keys + ((size_t)q * (a.out_slices ? a.out_slices : a.slices) + a.out_slice + slice) * a.R;
  for (int i = tid; i < a.R; i += kScanThreads) out[i] = i < cnt ? keys[i] : kEmptyKey;
  if (a.stats) {  // every vector of the slice is scanned once: the block adds `total`
    unsigned long long s1 = n_admit;
    for (int off = 16; off; off >>= 1) s1 += __shfl_xor_sync(0xffffffffu, s1, off);
    if (lane == 0) atomicAdd(a.stats + 1, s1);
    if (tid == 0) atomicAdd(a.stats + 0, (unsigned long long)total);
  }
}

// One unit per block.
template <int W, int QB>
__global__ void __launch_bounds__(kScanThreads, scan_min_blocks<W>()) scan_kernel(const ScanArgs a)
{
  scan_unit<W, QB>(a, blockIdx.x);
}

// A grid-stride loop over the units of the first *unit_count queries of qorder (a list whose
// length only the device knows: the list scan's overflowed rows).  A kernel of its own, compiled
// for fewer resident blocks, so that the loop costs the one-unit scan no registers.
template <int W, int QB>
__global__ void __launch_bounds__(kScanThreads, 4) scan_listed_kernel(const ScanArgs a)
{
  const unsigned units = (unsigned)*a.unit_count * (unsigned)a.slices;
  for (unsigned u = blockIdx.x; u < units; u += gridDim.x) {
    scan_unit<W, QB>(a, u);
    __syncthreads();  // the unit's shared memory is free again
  }
}

template <int W, int QB>
static void launch_scan_wq(const ScanArgs& a, cudaStream_t s)
{
  const size_t smem = (size_t)a.cap * 8 * 2 + (size_t)(2 * a.nprobe + 1) * 4 + (size_t)2 * a.nprobe * 4 +
                      (size_t)scan_head_bytes<W, QB>();
  RBQ_CHECK(smem <= 200 * 1024, RBQ_ERR_INVALID, "scan: shared memory budget exceeded (cap/nprobe too large)");
  const int64_t blocks = a.nq * a.slices;
  RBQ_CHECK(blocks <= 0x7fffffff, RBQ_ERR_INVALID, "scan: grid too large");
  if constexpr (QB <= 8 && W <= 24) {  // the list scan's modes and dimensions
    if (a.unit_count) {
      if (smem > 48 * 1024)
        RBQ_CUDA(cudaFuncSetAttribute(scan_listed_kernel<W, QB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
      scan_listed_kernel<W, QB><<<(unsigned)std::min<int64_t>(blocks, a.grid_blocks), kScanThreads, smem, s>>>(a);
      RBQ_LAUNCHED();
      return;
    }
  }
  RBQ_CHECK(!a.unit_count, RBQ_ERR_INVALID, "scan: a listed-query scan takes 4- or 8-bit queries, dim <= 768");
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(scan_kernel<W, QB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  scan_kernel<W, QB><<<(unsigned)blocks, kScanThreads, smem, s>>>(a);
  RBQ_LAUNCHED();
}

template <int W>
static void launch_scan_w(const ScanArgs& a, cudaStream_t s)
{
  switch (a.qbits) {
    case 8: launch_scan_wq<W, 8>(a, s); break;
    case 16: launch_scan_wq<W, 16>(a, s); break;
    case 32: launch_scan_wq<W, 32>(a, s); break;
    default: launch_scan_wq<W, 4>(a, s); break;
  }
}

void launch_scan(const ScanArgs& args, cudaStream_t s)
{
  if (args.nq <= 0) return;
  ScanArgs a = args;
  if (a.pstride == 0) a.pstride = a.nprobe;
  RBQ_CHECK(a.nprobe >= 1 && a.pstride >= a.nprobe, RBQ_ERR_INVALID, "scan: bad probe stride");
  RBQ_CHECK(!a.tau_out || (a.slices == 1 && a.prune && !a.init_keys), RBQ_ERR_INVALID,
            "scan: a seed-only launch takes one slice, the prune on and no initial candidates");
  RBQ_CHECK(a.cap >= a.R + kScanTile && (a.cap & (a.cap - 1)) == 0, RBQ_ERR_INVALID,
            "scan: cap must be a power of two >= R + tile");
  RBQ_CHECK(a.Dp == 32 * a.W, RBQ_ERR_INVALID, "scan: padded dim mismatch");
  RBQ_CHECK(a.qbits == 4 || a.qbits == 8 || a.qbits == 16 || a.qbits == 32, RBQ_ERR_INVALID,
            "scan: query bits must be 4 (QUANT4), 8 (QUANT8), 16 (LUT16) or 32 (LUT32)");
  RBQ_CHECK(!(a.tau_out && a.qbits >= 16), RBQ_ERR_INVALID, "scan: the LUT modes have no bound seed");
  RBQ_CHECK(!a.fixed_tau || (!a.init_keys && !a.tau_out), RBQ_ERR_INVALID,
            "scan: a fixed-threshold scan takes no initial candidates");
  RBQ_CHECK(a.n_slots >= 0 && a.n_slots < (int64_t)0x7fffffff - 2 * kScanTile, RBQ_ERR_INVALID,
            "scan: more than 2^31 vectors on one shard");
  RBQ_CHECK(!a.unit_count || (a.qorder && a.grid_blocks >= 1), RBQ_ERR_INVALID,
            "scan: a listed-query scan needs the list (qorder) and a grid size");
  switch (a.W) {
    case 1: launch_scan_w<1>(a, s); break;
    case 2: launch_scan_w<2>(a, s); break;
    case 3: launch_scan_w<3>(a, s); break;
    case 4: launch_scan_w<4>(a, s); break;
    case 6: launch_scan_w<6>(a, s); break;
    case 8: launch_scan_w<8>(a, s); break;
    case 12: launch_scan_w<12>(a, s); break;
    case 16: launch_scan_w<16>(a, s); break;
    case 24: launch_scan_w<24>(a, s); break;
    case 32: launch_scan_w<32>(a, s); break;
    default: throw Error{RBQ_ERR_INVALID, "scan: unsupported padded dimension"};
  }
}

// ---------------------------------------------------------------------------------------
// Query visiting order for the scan: a counting sort of the queries by their nearest probe.
// counts[l] (l < K) counts queries whose nearest list is l, counts[K] those without a probe;
// an exclusive prefix sum turns the counts into bucket starts, and the scatter hands out slots
// inside a bucket in arrival order.
// ---------------------------------------------------------------------------------------
__global__ void query_order_hist_kernel(const int32_t* __restrict__ probes, int64_t nq, int pstride, int K,
                                        int32_t* __restrict__ counts)
{
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  const int32_t l = probes[q * pstride];
  atomicAdd(counts + (l >= 0 && l < K ? l : K), 1);
}

// Exclusive prefix sum of counts[0..n) in place, one block of 1024 threads: each thread sums a
// contiguous run, a block scan of the run totals gives each run's start.
__global__ void __launch_bounds__(1024) exclusive_scan_kernel(int32_t* __restrict__ counts, int n)
{
  __shared__ int32_t s_tot[1024];
  const int t = threadIdx.x;
  const int per = (n + 1023) / 1024;
  const int b = min(n, t * per), e = min(n, b + per);
  int32_t sum = 0;
  for (int i = b; i < e; ++i) sum += counts[i];
  s_tot[t] = sum;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const int32_t v = t >= off ? s_tot[t - off] : 0;
    __syncthreads();
    s_tot[t] += v;
    __syncthreads();
  }
  int32_t run = s_tot[t] - sum;
  for (int i = b; i < e; ++i) {
    const int32_t c = counts[i];
    counts[i] = run;
    run += c;
  }
}

__global__ void query_order_scatter_kernel(const int32_t* __restrict__ probes, int64_t nq, int pstride, int K,
                                           int32_t* __restrict__ starts, int32_t* __restrict__ qorder)
{
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  const int32_t l = probes[q * pstride];
  qorder[atomicAdd(starts + (l >= 0 && l < K ? l : K), 1)] = (int32_t)q;
}

void launch_query_order(const int32_t* probes, int64_t nq, int pstride, int K, int32_t* counts, int32_t* qorder,
                        cudaStream_t s)
{
  if (nq <= 0) return;
  RBQ_CHECK(nq < 0x7fffffff && K >= 1, RBQ_ERR_INVALID, "query order: bad sizes");
  RBQ_CUDA(cudaMemsetAsync(counts, 0, (size_t)(K + 1) * sizeof(int32_t), s));
  const unsigned grid = (unsigned)ceil_div(nq, 256);
  query_order_hist_kernel<<<grid, 256, 0, s>>>(probes, nq, pstride, K, counts);
  RBQ_LAUNCHED();
  exclusive_scan_kernel<<<1, 1024, 0, s>>>(counts, K + 1);
  RBQ_LAUNCHED();
  query_order_scatter_kernel<<<grid, 256, 0, s>>>(probes, nq, pstride, K, counts, qorder);
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// List-scan plan.  codes[q, 32w + j] = the query's signed code of dim 32w + j read back from its
// planes (sum_{b < QB-1} bit_b << b - bit_{QB-1} << (QB-1)), one thread per (query, word).
// ---------------------------------------------------------------------------------------
__global__ void planes_to_codes_kernel(const uint32_t* __restrict__ planes, int64_t nq, int W, int QB,
                                       int8_t* __restrict__ codes)
{
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq * W) return;
  const int64_t q = i / W;
  const int w = (int)(i - q * W);
  uint32_t p[8];
#pragma unroll
  for (int b = 0; b < 8; ++b) p[b] = b < QB ? __brev(planes[(q * QB + b) * W + w]) : 0u;  // bit j = dim j
  uint32_t o[8];
#pragma unroll
  for (int j4 = 0; j4 < 8; ++j4) {
    uint32_t word = 0u;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 4 * j4 + k;
      int v = 0;
#pragma unroll
      for (int b = 0; b < 8; ++b)
        if (b < QB) v += (int)((p[b] >> j) & 1u) << b;
      if ((p[QB - 1] >> j) & 1u) v -= 2 << (QB - 1);  // the top plane weighs -2^(QB-1)
      word |= ((uint32_t)v & 0xFFu) << (8 * k);
    }
    o[j4] = word;
  }
  uint4* dst = reinterpret_cast<uint4*>(codes + q * (32 * W) + 32 * w);
  dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
  dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

void launch_planes_to_codes(const uint32_t* planes, int64_t nq, int W, int QB, int8_t* codes, cudaStream_t s)
{
  if (nq <= 0) return;
  RBQ_CHECK(QB == 4 || QB == 8, RBQ_ERR_INVALID, "query codes: 4- or 8-bit planes");
  planes_to_codes_kernel<<<(unsigned)ceil_div(nq * W, 256), 256, 0, s>>>(planes, nq, W, QB, codes);
  RBQ_LAUNCHED();
}

// The (list, query) pairs of this shard's probed lists, bucketed by list: counts, their
// exclusive prefix sum (list_start), work items of up to kListScanRows pairs per list and their
// prefix sum (item_start), then the pairs (query, g) in arrival order inside a list.
__global__ void list_pairs_hist_kernel(const int32_t* __restrict__ probes, int64_t nq, int nprobe, int pstride,
                                       const int32_t* __restrict__ owner, int rank, int K, int32_t* __restrict__ cnt)
{
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq * nprobe) return;
  const int64_t q = i / nprobe;
  const int l = probes[q * pstride + (i - q * nprobe)];
  if (l >= 0 && l < K && __ldg(owner + l) == rank) atomicAdd(cnt + l, 1);
}

__global__ void list_items_kernel(const int32_t* __restrict__ list_start, int K, int32_t* __restrict__ item_cnt)
{
  const int l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l < K) item_cnt[l] = (list_start[l + 1] - list_start[l] + kListScanRows - 1) / kListScanRows;
  if (l == K) item_cnt[K] = 0;
}

__global__ void list_pairs_scatter_kernel(const int32_t* __restrict__ probes, const float* __restrict__ g, int64_t nq,
                                          int nprobe, int pstride, const int32_t* __restrict__ owner, int rank, int K,
                                          int32_t* __restrict__ cursor, int32_t* __restrict__ pair_q,
                                          float* __restrict__ pair_g)
{
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq * nprobe) return;
  const int64_t q = i / nprobe;
  const int64_t e = q * pstride + (i - q * nprobe);
  const int l = probes[e];
  if (l < 0 || l >= K || __ldg(owner + l) != rank) return;
  const int pos = atomicAdd(cursor + l, 1);
  pair_q[pos] = (int32_t)q;
  pair_g[pos] = g[e];
}

void launch_list_pairs(const int32_t* probes, const float* g, int64_t nq, int nprobe, int pstride,
                       const int32_t* owner, int rank, int K, int32_t* list_start, int32_t* item_start,
                       int32_t* cursor, int32_t* pair_q, float* pair_g, cudaStream_t s)
{
  if (nq <= 0) return;
  RBQ_CHECK(nq * nprobe < 0x7fffffff && K >= 1, RBQ_ERR_INVALID, "list scan: too many (list, query) pairs");
  RBQ_CUDA(cudaMemsetAsync(list_start, 0, (size_t)(K + 1) * sizeof(int32_t), s));
  const unsigned grid = (unsigned)ceil_div(nq * nprobe, 256);
  list_pairs_hist_kernel<<<grid, 256, 0, s>>>(probes, nq, nprobe, pstride, owner, rank, K, list_start);
  RBQ_LAUNCHED();
  exclusive_scan_kernel<<<1, 1024, 0, s>>>(list_start, K + 1);
  RBQ_LAUNCHED();
  list_items_kernel<<<(unsigned)ceil_div(K + 1, 256), 256, 0, s>>>(list_start, K, item_start);
  RBQ_LAUNCHED();
  exclusive_scan_kernel<<<1, 1024, 0, s>>>(item_start, K + 1);
  RBQ_LAUNCHED();
  RBQ_CUDA(cudaMemcpyAsync(cursor, list_start, (size_t)(K + 1) * sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
  list_pairs_scatter_kernel<<<grid, 256, 0, s>>>(probes, g, nq, nprobe, pstride, owner, rank, K, cursor, pair_q,
                                                  pair_g);
  RBQ_LAUNCHED();
}

// The queries whose candidate row overflowed (cnt[q] > cap), in no particular order: list[0..*n).
__global__ void over_list_kernel(const int32_t* __restrict__ cnt, int64_t nq, int cap, int32_t* __restrict__ list,
                                 int32_t* __restrict__ n)
{
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool over = q < nq && cnt[q] > cap;
  const unsigned m = __ballot_sync(0xffffffffu, over);
  if (!m) return;
  const int lane = threadIdx.x & 31;
  int base = 0;
  if (lane == 0) base = atomicAdd(n, __popc(m));
  base = __shfl_sync(0xffffffffu, base, 0);
  if (over) list[base + __popc(m & ((1u << lane) - 1u))] = (int32_t)q;
}

void launch_over_list(const int32_t* cnt, int64_t nq, int cap, int32_t* list, int32_t* n, cudaStream_t s)
{
  RBQ_CUDA(cudaMemsetAsync(n, 0, sizeof(int32_t), s));
  if (nq <= 0) return;
  over_list_kernel<<<(unsigned)ceil_div(nq, 256), 256, 0, s>>>(cnt, nq, cap, list, n);
  RBQ_LAUNCHED();
}

// Exact pass of the list scan, one block per query: the candidates of its row, taken four at a
// time by a warp, one per 8-lane group (the exact 1-bit inner product of the tile scan), or one
// at a time with extra bits (the extra-bit distance), kept while dist <= tau0[q]; the R smallest keys, ascending, go to out_keys.  The admitted set
// does not depend on the order the list scan found it in, so neither does the result.
constexpr int kExactThreads = 256;

__global__ void __launch_bounds__(kExactThreads) exact_topr_kernel(const ExactArgs a)
{
  const int64_t q = blockIdx.x;
  const int n = a.cand_cnt[q];
  if (n > a.cap) return;  // overflowed row: the fixed-threshold tile scan answers this query
  extern __shared__ __align__(16) unsigned char ex_smem_raw[];
  const int W = a.W, NB = 4 * W;
  float* qsT = reinterpret_cast<float*>(ex_smem_raw);                                  // [8 * NB]
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(ex_smem_raw + 128 * W);  // [cap]
  unsigned long long* keys2 = keys + a.cap;                                            // [cap]
  __shared__ int s_count, s_misc[3], s_cnt2;
  __shared__ unsigned s_hist[256];
  __shared__ unsigned long long s_kmax;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 8 * NB; i += kExactThreads) {
    const int jj = i / NB, j = i - jj * NB;
    qsT[i] = a.Qr[q * (8 * NB) + 8 * j + jj];
  }
  if (tid == 0) s_count = 0;
  __syncthreads();
  const float k1 = a.k1[q];
  const float tau = a.tau0[q];
  const float ex_scale = (float)(1 << a.ex_bits);
  const float kb = __fmul_rn(k1, (float)((2 << a.ex_bits) - 1));
  const unsigned long long* row = a.cand + q * a.cap;
  if (a.ex_bits == 0) {
    // four candidates per warp at a time, one per 8-lane group
    const int grp = lane >> 3;
    for (int c0 = 4 * warp; c0 < n; c0 += 4 * (kExactThreads / 32)) {
      const int c = c0 + grp;
      const bool has = c < n;
      const unsigned long long e = row[has ? c : c0];
      const int slot = (int)(uint32_t)e;
      const float g = __uint_as_float((uint32_t)(e >> 32));
      float eip;
      switch (W) {
#define RBQ_EXACT_W(w) \
  case w: eip = group8_exact_ip<w>(a.codes, slot, qsT, lane); break;
        RBQ_EXACT_W(1) RBQ_EXACT_W(2) RBQ_EXACT_W(3) RBQ_EXACT_W(4) RBQ_EXACT_W(6) RBQ_EXACT_W(8) RBQ_EXACT_W(12)
        RBQ_EXACT_W(16) RBQ_EXACT_W(24)
#undef RBQ_EXACT_W
        default: eip = 0.0f;
      }
      if ((lane & 7) == 0 && has) {
        const float dist =
            __fadd_rn(__fadd_rn(__ldg(a.fadd + slot), g), __fmul_rn(__ldg(a.frescale + slot), __fadd_rn(eip, k1)));
        if (dist <= tau) keys[atomicAdd(&s_count, 1)] = make_key(dist, __ldg(a.ids + slot));
      }
    }
  }
  for (int c = warp; a.ex_bits > 0 && c < n; c += kExactThreads / 32) {
    const unsigned long long e = row[c];
    const int slot = (int)(uint32_t)e;
    const float g = __uint_as_float((uint32_t)(e >> 32));
    float eip;
    switch (W) {  // the exact inner product is unrolled per word count
#define RBQ_EXACT_W(w) \
  case w: eip = warp_exact_ip<w>(a.codes, slot, qsT, lane); break;
      RBQ_EXACT_W(1) RBQ_EXACT_W(2) RBQ_EXACT_W(3) RBQ_EXACT_W(4) RBQ_EXACT_W(6) RBQ_EXACT_W(8) RBQ_EXACT_W(12)
      RBQ_EXACT_W(16) RBQ_EXACT_W(24)
#undef RBQ_EXACT_W
      default: eip = 0.0f;
    }
    float ipx;
    switch (W) {
#define RBQ_EX_W(w) \
  case w: ipx = warp_ex_ip<w>(a.ex_codes, slot, a.ex_bits, qsT, lane); break;
      RBQ_EX_W(1) RBQ_EX_W(2) RBQ_EX_W(3) RBQ_EX_W(4) RBQ_EX_W(6) RBQ_EX_W(8) RBQ_EX_W(12) RBQ_EX_W(16) RBQ_EX_W(24)
#undef RBQ_EX_W
      default: ipx = 0.0f;
    }
    const float T = __fadd_rn(__fadd_rn(__fmul_rn(ex_scale, eip), ipx), kb);
    const float dist = __fadd_rn(__fadd_rn(__ldg(a.fexadd + slot), g), __fmul_rn(__ldg(a.fexr + slot), T));
    if (lane == 0 && dist <= tau) keys[atomicAdd(&s_count, 1)] = make_key(dist, __ldg(a.ids + slot));
  }
  __syncthreads();
  int cnt = s_count;
  if (cnt > a.R) {
    block_keep_smallest(keys, cnt, a.R, keys2, s_hist, s_misc, &s_kmax, &s_cnt2);
    keys = keys2;
    cnt = a.R;
  }
  int r2 = 2;
  while (r2 < cnt) r2 <<= 1;
  for (int i = cnt + tid; i < r2; i += kExactThreads) keys[i] = kEmptyKey;
  __syncthreads();
  block_bitonic_sort(keys, r2);
  unsigned long long* out = a.out_keys + ((size_t)q * a.out_slices + a.out_slice) * a.R;
  for (int i = tid; i < a.R; i += kExactThreads) out[i] = i < cnt ? keys[i] : kEmptyKey;
}

__global__ void tighten_tau_kernel(const unsigned long long* __restrict__ keys, int64_t nq, int stride, int R,
                                   float* __restrict__ tau)
{
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  const unsigned long long k = keys[q * stride + R - 1];
  if (k != kEmptyKey) tau[q] = fminf(tau[q], from_ordered_bits((uint32_t)(k >> 32)));
}

void launch_tighten_tau(const unsigned long long* keys, int64_t nq, int stride, int R, float* tau, cudaStream_t s)
{
  if (nq <= 0) return;
  tighten_tau_kernel<<<(unsigned)ceil_div(nq, 256), 256, 0, s>>>(keys, nq, stride, R, tau);
  RBQ_LAUNCHED();
}

void launch_exact_topr(const ExactArgs& a, cudaStream_t s)
{
  if (a.nq <= 0) return;
  RBQ_CHECK(a.W >= 1 && a.W <= 24, RBQ_ERR_INVALID, "list scan: padded dim above 768");
  RBQ_CHECK(a.cap >= a.R && a.cap <= 8192, RBQ_ERR_INVALID, "list scan: candidate row size");
  // keys2 holds the cut (R keys) and the sort pads to a power of two: 2 * cap keys suffice
  const size_t smem = (size_t)128 * a.W + (size_t)a.cap * 16;
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(exact_topr_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  exact_topr_kernel<<<(unsigned)a.nq, kExactThreads, smem, s>>>(a);
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// Merge [nq, parts, R] key lists -> the R smallest of their union, ascending.  The non-empty
// keys are gathered into shared memory, cut to R by the radix select, and only those R are
// sorted (a query split into 32 slices holds 6,400 keys; sorting all of them took 0.2 ms).
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) merge_keys_kernel(const unsigned long long* __restrict__ in, int parts, int R,
                                                         int r2, unsigned long long* __restrict__ out)
{
  extern __shared__ unsigned long long mk[];  // [parts * R] gathered keys, then [r2] result
  unsigned long long* res = mk + (size_t)parts * R;
  __shared__ int s_n, s_misc[3], s_cnt;
  __shared__ unsigned s_hist[256];
  __shared__ unsigned long long s_kmax;
  const int64_t q = blockIdx.x;
  const int tot = parts * R;
  if (threadIdx.x == 0) s_n = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < tot; i += blockDim.x) {
    const unsigned long long k = in[q * tot + i];
    if (k != kEmptyKey) mk[atomicAdd(&s_n, 1)] = k;
  }
  __syncthreads();
  int n = s_n;
  if (n > R) {
    block_keep_smallest(mk, n, R, res, s_hist, s_misc, &s_kmax, &s_cnt);
    n = R;
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) res[i] = mk[i];
  }
  for (int i = n + threadIdx.x; i < r2; i += blockDim.x) res[i] = kEmptyKey;
  __syncthreads();
  block_bitonic_sort(res, r2);
  for (int i = threadIdx.x; i < R; i += blockDim.x) out[q * R + i] = res[i];
}

// The R smallest keys of `parts` ascending rows of R keys per query (in [nq, parts, R]), without a
// sort: a key at rank r of row p lands at r plus, per other row, its count of keys below (rows
// after p) or up to (rows before p) the key, found by binary search in shared memory.  The result
// row of query q is out + (q * out_rows + out_row) * R.  With over_cnt, only queries whose
// over_cnt[q] exceeds over_cap are merged (the others' rows are left as they are).
__global__ void __launch_bounds__(256) merge_sorted_keys_kernel(const unsigned long long* __restrict__ in,
                                                                int parts, int R, unsigned long long* __restrict__ out,
                                                                int out_rows, int out_row,
                                                                const int32_t* __restrict__ over_cnt, int over_cap)
{
  extern __shared__ unsigned long long ms[];  // [parts * R] rows, then [R] result
  const int64_t q = blockIdx.x;
  if (over_cnt && over_cnt[q] <= over_cap) return;
  unsigned long long* res = ms + (size_t)parts * R;
  const int tot = parts * R;
  for (int i = threadIdx.x; i < tot; i += blockDim.x) ms[i] = in[q * tot + i];
  for (int i = threadIdx.x; i < R; i += blockDim.x) res[i] = kEmptyKey;
  __syncthreads();
  for (int i = threadIdx.x; i < tot; i += blockDim.x) {
    const unsigned long long e = ms[i];
    if (e == kEmptyKey) continue;
    const int p = i / R;
    int pos = i - p * R;
    for (int o = 0; o < parts && pos < R; ++o) {
      if (o == p) continue;
      const unsigned long long* row = ms + o * R;
      int lo = 0, hi = R;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (row[mid] < e || (o < p && row[mid] == e))
          lo = mid + 1;
        else
          hi = mid;
      }
      pos += lo;
    }
    if (pos < R) res[pos] = e;
  }
  __syncthreads();
  unsigned long long* dst = out + ((size_t)q * out_rows + out_row) * R;
  for (int i = threadIdx.x; i < R; i += blockDim.x) dst[i] = res[i];
}

void launch_merge_sorted_keys(const unsigned long long* in, int64_t nq, int parts, int R, unsigned long long* out,
                              int out_rows, int out_row, const int32_t* over_cnt, int over_cap, cudaStream_t s)
{
  if (nq <= 0) return;
  const size_t smem = ((size_t)parts + 1) * R * 8;
  RBQ_CHECK(smem <= 200 * 1024, RBQ_ERR_INVALID, "merge: too many candidates per query");
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(merge_sorted_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  merge_sorted_keys_kernel<<<(unsigned)nq, 256, smem, s>>>(in, parts, R, out, out_rows, out_row, over_cnt, over_cap);
  RBQ_LAUNCHED();
}

void launch_merge_keys(const unsigned long long* in, int64_t nq, int parts, int R, unsigned long long* out,
                       cudaStream_t s)
{
  if (nq <= 0) return;
  const int r2 = next_pow2(R < 2 ? 2 : R);
  const size_t smem = ((size_t)parts * R + r2) * 8;
  RBQ_CHECK(smem <= 200 * 1024, RBQ_ERR_INVALID, "merge: too many candidates per query");
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(merge_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  merge_keys_kernel<<<(unsigned)nq, 256, smem, s>>>(in, parts, R, r2, out);
  RBQ_LAUNCHED();
}

__global__ void keys_to_result_kernel(const unsigned long long* __restrict__ keys, int64_t nq, int R, int k,
                                      float* __restrict__ dist, int64_t* __restrict__ ids)
{
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq * k) return;
  const int64_t q = i / k;
  const int r = (int)(i - q * k);
  const unsigned long long key = (r < R) ? keys[q * R + r] : kEmptyKey;
  if (key == kEmptyKey) {
    dist[i] = __int_as_float(0x7f800000);
    ids[i] = -1;
  } else {
    dist[i] = from_ordered_bits((uint32_t)(key >> 32));
    ids[i] = (int64_t)(key & 0xFFFFFFFFu);
  }
}

void launch_keys_to_result(const unsigned long long* keys, int64_t nq, int R, int k, float* dist, int64_t* ids,
                           cudaStream_t s)
{
  if (nq <= 0) return;
  keys_to_result_kernel<<<(unsigned)ceil_div(nq * k, 256), 256, 0, s>>>(keys, nq, R, k, dist, ids);
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// Exact rerank (semantics of cuvs::neighbors::refine, refine/refine_device.cuh:31-150): for
// each candidate, |x - q|^2 over the original D dims: lane l sums double(x_d - q_d)^2 over
// d = l, l+32, ... ascending, then an xor butterfly (16, 8, 4, 2, 1) of double adds, rounded
// to float.  Top-k by (distance, id).  One CTA per query; each warp takes kRerankInFlight
// candidates at a time and issues all their row loads before the arithmetic (EPL = D / 32
// values per lane; EPL = 0 is the generic loop for other D).
// ---------------------------------------------------------------------------------------
constexpr int kRerankInFlight = 2;

template <int EPL>
__global__ void __launch_bounds__(256) rerank_kernel(const float* __restrict__ Xrows,
                                                     const uint32_t* __restrict__ id2row, int D,
                                                     const float* __restrict__ Q,
                                                     const unsigned long long* __restrict__ cand, int R, int k,
                                                     int r2, float* __restrict__ dist, int64_t* __restrict__ ids)
{
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_raw);  // [r2]
  float* qs = reinterpret_cast<float*>(keys + r2);                           // [D]
  const int64_t q = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  __shared__ int s_nv;
  if (threadIdx.x == 0) s_nv = 0;
  for (int j = threadIdx.x; j < D; j += blockDim.x) qs[j] = Q[q * D + j];
  __syncthreads();
  // Candidates stored on this shard, compacted to keys[0, nv) as (row << 32 | id): a shard of a
  // seeded sharded search holds only a few of the R slots, and the work follows nv, not R.
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const unsigned long long ck = cand[q * R + r];
    if (ck != kEmptyKey) {
      const uint32_t id = (uint32_t)(ck & 0xFFFFFFFFu);
      const uint32_t row = id2row[id];
      if (row != 0xFFFFFFFFu) keys[atomicAdd(&s_nv, 1)] = ((unsigned long long)row << 32) | id;
    }
  }
  __syncthreads();
  const int nv = s_nv;
  for (int r0 = warp * kRerankInFlight; r0 < nv; r0 += nwarps * kRerankInFlight) {
    const float* xp[kRerankInFlight];
    uint32_t idv[kRerankInFlight];
    bool ok[kRerankInFlight];
#pragma unroll
    for (int c = 0; c < kRerankInFlight; ++c) {  // warp-uniform: every lane reads the same slot
      const int r = r0 + c;
      ok[c] = r < nv;
      const unsigned long long e = ok[c] ? keys[r] : 0ull;
      xp[c] = Xrows + (size_t)(uint32_t)(e >> 32) * D;
      idv[c] = (uint32_t)(e & 0xFFFFFFFFu);
    }
    __syncwarp();
    if constexpr (EPL > 0) {
      float xv[kRerankInFlight][EPL];
#pragma unroll
      for (int c = 0; c < kRerankInFlight; ++c)
#pragma unroll
        for (int i = 0; i < EPL; ++i) xv[c][i] = ok[c] ? __ldg(xp[c] + lane + 32 * i) : 0.0f;
#pragma unroll
      for (int c = 0; c < kRerankInFlight; ++c) {
        double s = 0.0;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
          const float df = __fsub_rn(xv[c][i], qs[lane + 32 * i]);
          s = __dadd_rn(s, __dmul_rn((double)df, (double)df));
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
        if (lane == 0 && ok[c]) keys[r0 + c] = make_key((float)s, idv[c]);
      }
    } else {
#pragma unroll
      for (int c = 0; c < kRerankInFlight; ++c) {
        double s = 0.0;
        if (ok[c]) {
          for (int d = lane; d < D; d += 32) {
            const float df = __fsub_rn(__ldg(xp[c] + d), qs[d]);
            s = __dadd_rn(s, __dmul_rn((double)df, (double)df));
          }
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
        if (lane == 0 && ok[c]) keys[r0 + c] = make_key((float)s, idv[c]);
      }
    }
  }
  __syncthreads();
  int n2 = 2;
  while (n2 < nv) n2 <<= 1;
  for (int i = nv + threadIdx.x; i < n2; i += blockDim.x) keys[i] = kEmptyKey;
  __syncthreads();
  block_bitonic_sort(keys, n2);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const unsigned long long key = (i < nv) ? keys[i] : kEmptyKey;
    if (key == kEmptyKey) {
      dist[q * k + i] = __int_as_float(0x7f800000);
      ids[q * k + i] = -1;
    } else {
      dist[q * k + i] = from_ordered_bits((uint32_t)(key >> 32));
      ids[q * k + i] = (int64_t)(key & 0xFFFFFFFFu);
    }
  }
}

template <int EPL>
static void launch_rerank_e(const float* Xrows, const uint32_t* id2row, int D, const float* Q, int64_t nq,
                            const unsigned long long* cand, int R, int k, int r2, size_t smem, float* dist,
                            int64_t* ids, cudaStream_t s)
{
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(rerank_kernel<EPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  rerank_kernel<EPL><<<(unsigned)nq, 256, smem, s>>>(Xrows, id2row, D, Q, cand, R, k, r2, dist, ids);
  RBQ_LAUNCHED();
}

void launch_rerank(const float* Xrows, const uint32_t* id2row, int D, const float* Q, int64_t nq,
                   const unsigned long long* cand, int R, int k, float* dist, int64_t* ids, cudaStream_t s)
{
  if (nq <= 0) return;
  const int r2 = next_pow2(R < 2 ? 2 : R);
  const size_t smem = (size_t)r2 * 8 + (size_t)D * 4;
  RBQ_CHECK(smem <= 200 * 1024, RBQ_ERR_INVALID, "rerank: depth too large");
  const int epl = (D % 32 == 0) ? D / 32 : 0;
  switch (epl) {
    case 1: launch_rerank_e<1>(Xrows, id2row, D, Q, nq, cand, R, k, r2, smem, dist, ids, s); break;
    case 2: launch_rerank_e<2>(Xrows, id2row, D, Q, nq, cand, R, k, r2, smem, dist, ids, s); break;
    case 4: launch_rerank_e<4>(Xrows, id2row, D, Q, nq, cand, R, k, r2, smem, dist, ids, s); break;
    case 8: launch_rerank_e<8>(Xrows, id2row, D, Q, nq, cand, R, k, r2, smem, dist, ids, s); break;
    case 12: launch_rerank_e<12>(Xrows, id2row, D, Q, nq, cand, R, k, r2, smem, dist, ids, s); break;
    case 24: launch_rerank_e<24>(Xrows, id2row, D, Q, nq, cand, R, k, r2, smem, dist, ids, s); break;
    default: launch_rerank_e<0>(Xrows, id2row, D, Q, nq, cand, R, k, r2, smem, dist, ids, s); break;
  }
}

__global__ void ids_to_keys_kernel(const int64_t* __restrict__ ids, int64_t n, unsigned long long* __restrict__ keys)
{
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) keys[i] = ids[i] < 0 ? kEmptyKey : (unsigned long long)(uint32_t)ids[i];
}

void launch_ids_to_keys(const int64_t* ids, int64_t n, unsigned long long* keys, cudaStream_t s)
{
  if (n <= 0) return;
  ids_to_keys_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(ids, n, keys);
  RBQ_LAUNCHED();
}

__global__ void cands_to_keys_kernel(const int64_t* __restrict__ ids, const float* __restrict__ dist, int64_t n,
                                     unsigned long long* __restrict__ keys)
{
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) keys[i] = ids[i] < 0 ? kEmptyKey : make_key(dist[i], (uint32_t)ids[i]);
}

void launch_cands_to_keys(const int64_t* ids, const float* dist, int64_t n, unsigned long long* keys, cudaStream_t s)
{
  if (n <= 0) return;
  cands_to_keys_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(ids, dist, n, keys);
  RBQ_LAUNCHED();
}

__global__ void keys_to_ids_kernel(const unsigned long long* __restrict__ keys, int64_t n, int64_t* __restrict__ ids,
                                   float* __restrict__ dist)
{
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const unsigned long long key = keys[i];
  if (key == kEmptyKey) {
    ids[i] = -1;
    if (dist) dist[i] = __int_as_float(0x7f800000);
  } else {
    ids[i] = (int64_t)(key & 0xFFFFFFFFu);
    if (dist) dist[i] = from_ordered_bits((uint32_t)(key >> 32));
  }
}

void launch_keys_to_ids(const unsigned long long* keys, int64_t n, int64_t* ids, float* dist, cudaStream_t s)
{
  if (n <= 0) return;
  keys_to_ids_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(keys, n, ids, dist);
  RBQ_LAUNCHED();
}

// Per-shard results [parts, nq, k] as keys: from (dist, id) pairs (id < 0 = empty), or already
// packed (keys != nullptr; what a sharded search all-gathers, 8 bytes a result instead of 12).
struct ResultSource {
  const float* dist;
  const int64_t* ids;
  const unsigned long long* keys;
  __device__ __forceinline__ unsigned long long at(size_t i) const
  {
    if (keys) return keys[i];
    return ids[i] >= 0 ? make_key(dist[i], (uint32_t)ids[i]) : kEmptyKey;
  }
};

// k-way merge of per-shard results [parts, nq, k] by (distance, id): the on-device merge that
// follows the all-gather of a list-sharded search.  Shard results arrive sorted (a search returns
// its rows ascending); then an element at rank r of part p lands at r plus, per other part, the
// number of its keys below (parts after p) or up to (parts before p) the element, found by binary
// search in shared memory, and only the elements landing below k are written (one barrier
// instead of a sort).  Rows that are not ascending take the block-wide bitonic sort.
__device__ __forceinline__ int keys_below(const unsigned long long* row, int k, unsigned long long e, bool or_equal)
{
  int lo = 0, hi = k;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (row[mid] < e || (or_equal && row[mid] == e))
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

__global__ void __launch_bounds__(256) merge_results_kernel(const ResultSource src, int parts, int64_t nq, int k,
                                                            int n2, float* __restrict__ out_dist,
                                                            int64_t* __restrict__ out_ids)
{
  extern __shared__ unsigned long long mr[];
  __shared__ int s_unsorted;
  const int64_t q = blockIdx.x;
  const int n = parts * k;
  if (threadIdx.x == 0) s_unsorted = 0;
  for (int i = threadIdx.x; i < n2; i += blockDim.x) {
    unsigned long long key = kEmptyKey;
    if (i < n) {
      const int p = i / k, r = i - p * k;
      key = src.at(((size_t)p * nq + q) * k + r);
    }
    mr[i] = key;
  }
  __syncthreads();
  bool bad = false;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    if (i % k != 0 && mr[i - 1] > mr[i]) bad = true;
  if (bad) s_unsorted = 1;
  __syncthreads();
  if (!s_unsorted) {
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
      out_ids[q * k + i] = -1;
      out_dist[q * k + i] = __int_as_float(0x7f800000);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const unsigned long long e = mr[i];
      if (e == kEmptyKey) continue;
      const int p = i / k;
      int pos = i - p * k;
      for (int o = 0; o < parts && pos < k; ++o)
        if (o != p) pos += keys_below(mr + o * k, k, e, o < p);
      if (pos < k) {
        out_ids[q * k + pos] = (int64_t)(e & 0xFFFFFFFFu);
        out_dist[q * k + pos] = from_ordered_bits((uint32_t)(e >> 32));
      }
    }
    return;
  }
  block_bitonic_sort(mr, n2);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const unsigned long long key = mr[i];
    out_ids[q * k + i] = key == kEmptyKey ? -1 : (int64_t)(key & 0xFFFFFFFFu);
    out_dist[q * k + i] = key == kEmptyKey ? __int_as_float(0x7f800000) : from_ordered_bits((uint32_t)(key >> 32));
  }
}

// Small merges (parts * k <= 32 * L): one warp per query holds the candidates in registers and
// takes the k smallest keys by k rounds of a warp-wide minimum; the lowest lane holding the
// minimum drops one copy of it, so the result equals the sort's first k.
template <int L>
__global__ void __launch_bounds__(256) merge_results_warp_kernel(const ResultSource src, int parts, int64_t nq,
                                                                 int k, float* __restrict__ out_dist,
                                                                 int64_t* __restrict__ out_ids)
{
  const int64_t q = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (q >= nq) return;
  const int n = parts * k;
  unsigned long long v[L];
#pragma unroll
  for (int i = 0; i < L; ++i) {
    const int e = lane + 32 * i;
    v[i] = kEmptyKey;
    if (e < n) {
      const int p = e / k, r = e - p * k;
      v[i] = src.at(((size_t)p * nq + q) * k + r);
    }
  }
  for (int o = 0; o < k; ++o) {
    unsigned long long m = v[0];
#pragma unroll
    for (int i = 1; i < L; ++i) m = v[i] < m ? v[i] : m;
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, m, off);
      m = t < m ? t : m;
    }
    if (m != kEmptyKey) {
      bool has = false;
#pragma unroll
      for (int i = 0; i < L; ++i) has |= v[i] == m;
      const unsigned who = __ballot_sync(0xffffffffu, has);
      if (lane == __ffs(who) - 1) {
        bool done = false;
#pragma unroll
        for (int i = 0; i < L; ++i)
          if (!done && v[i] == m) {
            v[i] = kEmptyKey;
            done = true;
          }
      }
    }
    if (lane == 0) {
      out_ids[q * k + o] = m == kEmptyKey ? -1 : (int64_t)(m & 0xFFFFFFFFu);
      out_dist[q * k + o] = m == kEmptyKey ? __int_as_float(0x7f800000) : from_ordered_bits((uint32_t)(m >> 32));
    }
  }
}

void launch_merge_results(const float* dist, const int64_t* ids, int parts, int64_t nq, int k, float* out_dist,
                          int64_t* out_ids, cudaStream_t s, const unsigned long long* keys)
{
  if (nq <= 0) return;
  const ResultSource src{dist, ids, keys};
  if ((int64_t)parts * k <= 32 * 8) {
    const unsigned grid = (unsigned)ceil_div(nq * 32, 256);
    if (parts * k <= 32 * 2)
      merge_results_warp_kernel<2><<<grid, 256, 0, s>>>(src, parts, nq, k, out_dist, out_ids);
    else if (parts * k <= 32 * 4)
      merge_results_warp_kernel<4><<<grid, 256, 0, s>>>(src, parts, nq, k, out_dist, out_ids);
    else
      merge_results_warp_kernel<8><<<grid, 256, 0, s>>>(src, parts, nq, k, out_dist, out_ids);
    RBQ_LAUNCHED();
    return;
  }
  const int n2 = next_pow2(parts * k < 2 ? 2 : parts * k);
  const size_t smem = (size_t)n2 * 8;
  RBQ_CHECK(smem <= 200 * 1024, RBQ_ERR_INVALID, "merge: parts * k too large");
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(merge_results_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  merge_results_kernel<<<(unsigned)nq, 256, smem, s>>>(src, parts, nq, k, n2, out_dist, out_ids);
  RBQ_LAUNCHED();
}

// Phase-1 dump (inspection / parity): same arithmetic as the scan's phase 1.
template <int W>
__global__ void list_estimates_kernel(const uint32_t* __restrict__ codes, const float* __restrict__ fadd,
                                      const float* __restrict__ frescale, const float* __restrict__ ferr,
                                      int64_t base, int64_t n, const uint32_t* __restrict__ planes, int qbits,
                                      float delta, float k1, float g, int32_t* __restrict__ acc_out,
                                      float* __restrict__ est_out, float* __restrict__ low_out)
{
  const int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= n) return;
  const int64_t slot = base + v;
  uint32_t c[W];
  load_code<W>(codes, slot, c);
  int32_t acc = 0;
  for (int w = 0; w < W; ++w) {
    for (int b = 0; b < qbits - 1; ++b) acc += __popc(planes[b * W + w] & c[w]) << b;
    acc -= __popc(planes[(qbits - 1) * W + w] & c[w]) << (qbits - 1);
  }
  const float base_d = __fadd_rn(fadd[slot], g);
  const float ip = __fmul_rn((float)acc, delta);
  const float est = __fadd_rn(base_d, __fmul_rn(frescale[slot], __fadd_rn(ip, k1)));
  const float low = __fsub_rn(est, __fmul_rn(ferr[slot], sqrtf(g)));
  acc_out[v] = acc;
  est_out[v] = est;
  low_out[v] = low;
}

void launch_list_estimates(const Index& ix, const uint32_t* planes, int qbits, float delta, float k1, float g,
                           int list, int32_t* acc, float* est, float* low, cudaStream_t s)
{
  RBQ_CHECK(qbits == 4 || qbits == 8, RBQ_ERR_INVALID, "estimates: query bits must be 4 or 8");
  const int64_t base = ix.off_host[list], n = ix.off_host[list + 1] - base;
  if (n <= 0) return;
  const unsigned grid = (unsigned)ceil_div(n, 128);
#define RBQ_LE_CASE(WW)                                                                                     \
  case WW:                                                                                                  \
    list_estimates_kernel<WW><<<grid, 128, 0, s>>>(ix.codes, ix.fadd, ix.frescale, ix.ferr, base, n, planes, \
                                                   qbits, delta, k1, g, acc, est, low);                     \
    break;
  switch (ix.W) {
    RBQ_LE_CASE(1)
    RBQ_LE_CASE(2)
    RBQ_LE_CASE(3)
    RBQ_LE_CASE(4)
    RBQ_LE_CASE(6)
    RBQ_LE_CASE(8)
    RBQ_LE_CASE(12)
    RBQ_LE_CASE(16)
    RBQ_LE_CASE(24)
    RBQ_LE_CASE(32)
    default: throw Error{RBQ_ERR_INVALID, "estimates: unsupported padded dimension"};
  }
#undef RBQ_LE_CASE
  RBQ_LAUNCHED();
}

}  // namespace rbq
