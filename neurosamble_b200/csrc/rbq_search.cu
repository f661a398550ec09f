// Search kernels for sm_100a: coarse quantiser (approximate pass + exact refine), 4-bit
// query quantisation, the list scan, candidate merges and the exact rerank.
//
// Compiled with -fmad=false.  The estimator, the prune test, the exact 1-bit distance and the
// rerank distance are evaluated in the operation order written here, which is also the order
// of the CPU oracle (oracle/rbq_oracle.cpp), so estimates and ids agree bit for bit.
#include <cuda_runtime.h>
#include <stdint.h>

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
// Per row of S [nq, K]: the m smallest (score, column) keys, ascending.  Chunks of the row
// are appended behind the running top-m and the buffer is re-sorted.
// ---------------------------------------------------------------------------------------
constexpr int kTopmBuf = 2048;

__global__ void __launch_bounds__(256) topm_rows_kernel(const float* __restrict__ S, int K, int m,
                                                        int32_t* __restrict__ cand)
{
  __shared__ unsigned long long keys[kTopmBuf];
  const int64_t q = blockIdx.x;
  const float* row = S + q * K;
  int filled = 0;  // valid running entries at the front
  for (int c0 = 0; c0 < K;) {
    const int take = min(kTopmBuf - filled, K - c0);
    for (int i = threadIdx.x; i < kTopmBuf - filled; i += blockDim.x)
      keys[filled + i] = (i < take) ? make_key(row[c0 + i], (uint32_t)(c0 + i)) : kEmptyKey;
    __syncthreads();
    block_bitonic_sort(keys, kTopmBuf);
    c0 += take;
    filled = min(m, filled + take);
  }
  for (int i = threadIdx.x; i < m; i += blockDim.x)
    cand[q * m + i] = (keys[i] == kEmptyKey) ? -1 : (int32_t)(keys[i] & 0xFFFFFFFFu);
}

void launch_topm_rows(const float* S, int64_t nq, int K, int m, int32_t* cand, cudaStream_t s)
{
  if (nq <= 0) return;
  RBQ_CHECK(m >= 1 && m <= kTopmBuf / 2, RBQ_ERR_INVALID, "coarse: shortlist size out of range");
  topm_rows_kernel<<<(unsigned)nq, 256, 0, s>>>(S, K, m, cand);
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// Exact refine of the shortlist: g = float(sum_j double(a_j - c_j)^2), j ascending; keep the
// p smallest (g, list id).  Same distance as the oracle's orc_coarse / orc_assign.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) refine_topp_kernel(const float* __restrict__ A, const float* __restrict__ C,
                                                          int d, const int32_t* __restrict__ cand, int m, int p,
                                                          int mp2, int32_t* __restrict__ probes,
                                                          float* __restrict__ gout)
{
  extern __shared__ unsigned char smem_raw[];
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_raw);
  float* a = reinterpret_cast<float*>(keys + mp2);
  const int64_t q = blockIdx.x;
  for (int j = threadIdx.x; j < d; j += blockDim.x) a[j] = A[q * d + j];
  __syncthreads();
  for (int i = threadIdx.x; i < mp2; i += blockDim.x) {
    unsigned long long key = kEmptyKey;
    if (i < m) {
      const int c = cand[q * m + i];
      if (c >= 0) {
        const float* cr = C + (size_t)c * d;
        double s = 0.0;
        for (int j = 0; j < d; ++j) {
          const float df = a[j] - cr[j];
          s += (double)df * (double)df;
        }
        key = make_key((float)s, (uint32_t)c);
      }
    }
    keys[i] = key;
  }
  __syncthreads();
  block_bitonic_sort(keys, mp2);
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

void launch_refine_topp(const float* A, int64_t nq, const float* C, int d, const int32_t* cand, int m, int p,
                        int32_t* probes, float* g, cudaStream_t s)
{
  if (nq <= 0) return;
  const int mp2 = next_pow2(m < 2 ? 2 : m);
  const size_t smem = (size_t)mp2 * 8 + (size_t)d * 4;
  RBQ_CHECK(smem <= 200 * 1024, RBQ_ERR_INVALID, "coarse: refine shortlist too large");
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(refine_topp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  refine_topp_kernel<<<(unsigned)nq, 256, smem, s>>>(A, C, d, cand, m, p, mp2, probes, g);
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// 4-bit query quantisation (exrabitq_quantize_query<256> with EX_BITS = 4,
// searcher_gpu_quantize_query.cu:655-793) and k1 = -0.5 * sum q (ivf_gpu.cu:1451-1490).
// One thread per query; sums are double accumulations in dimension order.
//   code_j = clamp(rint(t4 * (q_j * (1/|q|))), -8, 7)
//   delta = (|q| / |code|) * (<q, code> / (|q| * |code|))   (0 if either norm <= 1e-6)
//   plane b, word w, bit 31-j = bit b of (code_{32w+j} & 0xF)
// ---------------------------------------------------------------------------------------
__global__ void query_prep_kernel(const float* __restrict__ Qr, int64_t nq, int Dp, float t4,
                                  uint32_t* __restrict__ planes, float* __restrict__ delta, float* __restrict__ k1)
{
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  const float* x = Qr + q * Dp;
  double s2 = 0.0, s1 = 0.0;
  for (int j = 0; j < Dp; ++j) {
    const double v = (double)x[j];
    s2 += v * v;
    s1 += v;
  }
  const float norm = sqrtf((float)s2);
  const float norm_inv = (norm > 0.0f) ? (1.0f / norm) : 0.0f;
  const int W = Dp >> 5;
  uint32_t* pl = planes + q * 4 * W;
  double ipd = 0.0;
  long long xs = 0;
  for (int w = 0; w < W; ++w) {
    uint32_t p0 = 0, p1 = 0, p2 = 0, p3 = 0;
    for (int b = 0; b < 32; ++b) {
      const int j = (w << 5) + b;
      const float val = x[j] * norm_inv;
      int cv = __float2int_rn(t4 * val);
      cv = cv > 7 ? 7 : (cv < -8 ? -8 : cv);
      ipd += (double)x[j] * (double)cv;
      xs += (long long)(cv * cv);
      const uint32_t u = (uint32_t)cv & 0xFu;
      const int sh = 31 - b;
      p0 |= (u & 1u) << sh;
      p1 |= ((u >> 1) & 1u) << sh;
      p2 |= ((u >> 2) & 1u) << sh;
      p3 |= ((u >> 3) & 1u) << sh;
    }
    pl[0 * W + w] = p0;
    pl[1 * W + w] = p1;
    pl[2 * W + w] = p2;
    pl[3 * W + w] = p3;
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

void launch_query_prep(const float* Qr, int64_t nq, int Dp, float t4, uint32_t* planes, float* delta, float* k1,
                       cudaStream_t s)
{
  if (nq <= 0) return;
  query_prep_kernel<<<(unsigned)ceil_div(nq, 128), 128, 0, s>>>(Qr, nq, Dp, t4, planes, delta, k1);
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// The list scan (computeInnerProductsWithBitwiseBlockSort<4, false, false>,
// searcher_gpu_quantize_query.cu:172-626, re-designed).  One CTA per (query, probe slice):
// the CTA walks its slice's lists in probe order in tiles of kScanTile vectors, one vector
// per thread:
//   phase 1  acc = sum_w [sum_{b<3} popc(P_b & c) << b  -  popc(P_3 & c) << 3]   (exact int)
//            est = (f_add + g) + f_rescale * (acc * delta + k1);  low = est - f_err * sqrt(g)
//            admit if !prune || low < tau
//   phase 2  exact_ip = sum over set bits of q (per byte from 0, per word ((b0+b1)+b2)+b3,
//            words in order); dist = (f_add + g) + f_rescale * (exact_ip + k1);
//            keep (dist, id) if dist <= tau.
// tau (the R-th best kept distance) only changes at tile boundaries: when the buffer holds
// more than cap - kScanTile keys it is sorted and cut to R.  The schedule is a function of
// the data alone, so results are deterministic and equal to the oracle's.
// ---------------------------------------------------------------------------------------
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

template <int W>
__device__ __forceinline__ float exact_ip_bits(const float* __restrict__ qs, const uint32_t (&c)[W])
{
  float acc = 0.0f;
#pragma unroll
  for (int w = 0; w < W; ++w) {
    const uint32_t cw = c[w];
    float part[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float v = qs[32 * w + 8 * i + j];
        s = ((cw >> (31 - (8 * i + j))) & 1u) ? __fadd_rn(s, v) : s;
      }
      part[i] = s;
    }
    const float pw = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), part[2]), part[3]);
    acc = __fadd_rn(acc, pw);
  }
  return acc;
}

template <int W>
__global__ void __launch_bounds__(kScanTile) scan_kernel(const ScanArgs a)
{
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_raw);          // [cap]
  float* qs = reinterpret_cast<float*>(keys + a.cap);                                  // [Dp]
  uint32_t* pl = reinterpret_cast<uint32_t*>(qs + W * 32);                             // [4W]
  int32_t* own_l = reinterpret_cast<int32_t*>(pl + 4 * W);                             // [nprobe]
  float* own_g = reinterpret_cast<float*>(own_l + a.nprobe);                           // [nprobe]
  __shared__ int s_count, s_m;
  __shared__ float s_tau;

  const int64_t q = blockIdx.x / a.slices;
  const int slice = blockIdx.x - (int)(q * a.slices);
  const int tid = threadIdx.x;

  for (int j = tid; j < W * 32; j += blockDim.x) qs[j] = a.Qr[q * (W * 32) + j];
  for (int j = tid; j < 4 * W; j += blockDim.x) pl[j] = a.planes[q * 4 * W + j];
  if (tid == 0) {
    int m = 0;
    for (int p = 0; p < a.nprobe; ++p) {
      const int l = a.probes[q * a.nprobe + p];
      if (l >= 0 && l % a.shard_count == a.shard_rank) {
        own_l[m] = l;
        own_g[m] = a.g[q * a.nprobe + p];
        ++m;
      }
    }
    s_m = m;
    s_count = 0;
    s_tau = __int_as_float(0x7f800000);
  }
  __syncthreads();
  const int m = s_m;
  const int p_begin = (int)(((int64_t)slice * m) / a.slices);
  const int p_end = (int)(((int64_t)(slice + 1) * m) / a.slices);
  const float delta = a.delta[q];
  const float k1 = a.k1[q];
  unsigned long long n_scan = 0, n_admit = 0;

  for (int pi = p_begin; pi < p_end; ++pi) {
    const int l = own_l[pi];
    const float g = own_g[pi];
    const float sqrt_g = sqrtf(g);
    const int64_t base = a.list_off[l];
    const int64_t n = a.list_off[l + 1] - base;
    for (int64_t t0 = 0; t0 < n; t0 += kScanTile) {
      const float tau = s_tau;
      const int64_t v = t0 + tid;
      if (v < n) {
        const int64_t slot = base + v;
        uint32_t c[W];
        load_code<W>(a.codes, slot, c);
        int32_t acc = 0;
#pragma unroll
        for (int w = 0; w < W; ++w) {
          acc += __popc(pl[0 * W + w] & c[w]);
          acc += __popc(pl[1 * W + w] & c[w]) << 1;
          acc += __popc(pl[2 * W + w] & c[w]) << 2;
          acc -= __popc(pl[3 * W + w] & c[w]) << 3;
        }
        const float fr = __ldg(a.frescale + slot);
        const float base_d = __fadd_rn(__ldg(a.fadd + slot), g);
        const float ip = __fmul_rn((float)acc, delta);
        const float est = __fadd_rn(base_d, __fmul_rn(fr, __fadd_rn(ip, k1)));
        const float low = __fsub_rn(est, __fmul_rn(__ldg(a.ferr + slot), sqrt_g));
        ++n_scan;
        if (!a.prune || low < tau) {
          ++n_admit;
          const float eip = exact_ip_bits<W>(qs, c);
          const float dist = __fadd_rn(base_d, __fmul_rn(fr, __fadd_rn(eip, k1)));
          if (dist <= tau) {
            const int at = atomicAdd(&s_count, 1);
            keys[at] = make_key(dist, __ldg(a.ids + slot));
          }
        }
      }
      __syncthreads();
      const int cnt = s_count;
      if (cnt > a.cap - kScanTile) {
        for (int i = cnt + tid; i < a.cap; i += blockDim.x) keys[i] = kEmptyKey;
        __syncthreads();
        block_bitonic_sort(keys, a.cap);
        if (tid == 0) {
          s_count = a.R;
          s_tau = from_ordered_bits((uint32_t)(keys[a.R - 1] >> 32));
        }
      }
      __syncthreads();
    }
  }
  const int cnt = s_count;
  for (int i = cnt + tid; i < a.cap; i += blockDim.x) keys[i] = kEmptyKey;
  __syncthreads();
  block_bitonic_sort(keys, a.cap);
  unsigned long long* out = a.out_keys + ((size_t)q * a.slices + slice) * a.R;
  for (int i = tid; i < a.R; i += blockDim.x) out[i] = keys[i];
  if (a.stats) {
    for (int off = 16; off; off >>= 1) {
      n_scan += __shfl_xor_sync(0xffffffffu, n_scan, off);
      n_admit += __shfl_xor_sync(0xffffffffu, n_admit, off);
    }
    if ((tid & 31) == 0) {
      atomicAdd(a.stats + 0, n_scan);
      atomicAdd(a.stats + 1, n_admit);
    }
  }
}

template <int W>
static void launch_scan_w(const ScanArgs& a, cudaStream_t s)
{
  const size_t smem = (size_t)a.cap * 8 + (size_t)W * 32 * 4 + (size_t)4 * W * 4 + (size_t)a.nprobe * 8;
  RBQ_CHECK(smem <= 200 * 1024, RBQ_ERR_INVALID, "scan: shared memory budget exceeded (cap/nprobe too large)");
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(scan_kernel<W>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t blocks = a.nq * a.slices;
  RBQ_CHECK(blocks <= 0x7fffffff, RBQ_ERR_INVALID, "scan: grid too large");
  scan_kernel<W><<<(unsigned)blocks, kScanTile, smem, s>>>(a);
  RBQ_LAUNCHED();
}

void launch_scan(const ScanArgs& a, cudaStream_t s)
{
  if (a.nq <= 0) return;
  RBQ_CHECK(a.cap >= a.R + kScanTile && (a.cap & (a.cap - 1)) == 0, RBQ_ERR_INVALID,
            "scan: cap must be a power of two >= R + 256");
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
// Merge [nq, parts, R] ascending key lists -> first R of the union, ascending.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) merge_keys_kernel(const unsigned long long* __restrict__ in, int parts, int R,
                                                         int n2, unsigned long long* __restrict__ out)
{
  extern __shared__ unsigned long long mk[];
  const int64_t q = blockIdx.x;
  const int tot = parts * R;
  for (int i = threadIdx.x; i < n2; i += blockDim.x) mk[i] = (i < tot) ? in[q * tot + i] : kEmptyKey;
  __syncthreads();
  block_bitonic_sort(mk, n2);
  for (int i = threadIdx.x; i < R; i += blockDim.x) out[q * R + i] = mk[i];
}

void launch_merge_keys(const unsigned long long* in, int64_t nq, int parts, int R, unsigned long long* out,
                       cudaStream_t s)
{
  if (nq <= 0) return;
  const int n2 = next_pow2(parts * R);
  const size_t smem = (size_t)n2 * 8;
  RBQ_CHECK(smem <= 200 * 1024, RBQ_ERR_INVALID, "merge: too many candidates per query");
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(merge_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  merge_keys_kernel<<<(unsigned)nq, 256, smem, s>>>(in, parts, R, n2, out);
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
// to float.  Top-k by (distance, id).  One CTA per query, one warp per candidate.
// ---------------------------------------------------------------------------------------
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
  for (int j = threadIdx.x; j < D; j += blockDim.x) qs[j] = Q[q * D + j];
  for (int i = threadIdx.x; i < r2; i += blockDim.x) keys[i] = kEmptyKey;
  __syncthreads();
  for (int r = warp; r < R; r += nwarps) {
    const unsigned long long ck = cand[q * R + r];
    if (ck == kEmptyKey) continue;
    const uint32_t id = (uint32_t)(ck & 0xFFFFFFFFu);
    const uint32_t row = id2row[id];
    if (row == 0xFFFFFFFFu) continue;
    const float* x = Xrows + (size_t)row * D;
    double s = 0.0;
    for (int d = lane; d < D; d += 32) {
      const float df = __fsub_rn(__ldg(x + d), qs[d]);
      s = __dadd_rn(s, __dmul_rn((double)df, (double)df));
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    if (lane == 0) keys[r] = make_key((float)s, id);
  }
  __syncthreads();
  block_bitonic_sort(keys, r2);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const unsigned long long key = (i < r2) ? keys[i] : kEmptyKey;
    if (key == kEmptyKey) {
      dist[q * k + i] = __int_as_float(0x7f800000);
      ids[q * k + i] = -1;
    } else {
      dist[q * k + i] = from_ordered_bits((uint32_t)(key >> 32));
      ids[q * k + i] = (int64_t)(key & 0xFFFFFFFFu);
    }
  }
}

void launch_rerank(const float* Xrows, const uint32_t* id2row, int D, const float* Q, int64_t nq,
                   const unsigned long long* cand, int R, int k, float* dist, int64_t* ids, cudaStream_t s)
{
  if (nq <= 0) return;
  const int r2 = next_pow2(R < 2 ? 2 : R);
  const size_t smem = (size_t)r2 * 8 + (size_t)D * 4;
  RBQ_CHECK(smem <= 200 * 1024, RBQ_ERR_INVALID, "rerank: depth too large");
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(rerank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  rerank_kernel<<<(unsigned)nq, 256, smem, s>>>(Xrows, id2row, D, Q, cand, R, k, r2, dist, ids);
  RBQ_LAUNCHED();
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

// k-way merge of per-shard results [parts, nq, k] by (distance, id): the on-device merge that
// follows the all-gather of a list-sharded search.
__global__ void __launch_bounds__(256) merge_results_kernel(const float* __restrict__ dist,
                                                            const int64_t* __restrict__ ids, int parts, int64_t nq,
                                                            int k, int n2, float* __restrict__ out_dist,
                                                            int64_t* __restrict__ out_ids)
{
  extern __shared__ unsigned long long mr[];
  const int64_t q = blockIdx.x;
  for (int i = threadIdx.x; i < n2; i += blockDim.x) {
    unsigned long long key = kEmptyKey;
    if (i < parts * k) {
      const int p = i / k, r = i - p * k;
      const size_t at = ((size_t)p * nq + q) * k + r;
      if (ids[at] >= 0) key = make_key(dist[at], (uint32_t)ids[at]);
    }
    mr[i] = key;
  }
  __syncthreads();
  block_bitonic_sort(mr, n2);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const unsigned long long key = mr[i];
    out_ids[q * k + i] = key == kEmptyKey ? -1 : (int64_t)(key & 0xFFFFFFFFu);
    out_dist[q * k + i] = key == kEmptyKey ? __int_as_float(0x7f800000) : from_ordered_bits((uint32_t)(key >> 32));
  }
}

void launch_merge_results(const float* dist, const int64_t* ids, int parts, int64_t nq, int k, float* out_dist,
                          int64_t* out_ids, cudaStream_t s)
{
  if (nq <= 0) return;
  const int n2 = next_pow2(parts * k < 2 ? 2 : parts * k);
  const size_t smem = (size_t)n2 * 8;
  RBQ_CHECK(smem <= 200 * 1024, RBQ_ERR_INVALID, "merge: parts * k too large");
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(merge_results_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  merge_results_kernel<<<(unsigned)nq, 256, smem, s>>>(dist, ids, parts, nq, k, n2, out_dist, out_ids);
  RBQ_LAUNCHED();
}

// Phase-1 dump (inspection / parity): same arithmetic as the scan's phase 1.
template <int W>
__global__ void list_estimates_kernel(const uint32_t* __restrict__ codes, const float* __restrict__ fadd,
                                      const float* __restrict__ frescale, const float* __restrict__ ferr,
                                      int64_t base, int64_t n, const uint32_t* __restrict__ planes, float delta,
                                      float k1, float g, int32_t* __restrict__ acc_out, float* __restrict__ est_out,
                                      float* __restrict__ low_out)
{
  const int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= n) return;
  const int64_t slot = base + v;
  uint32_t c[W];
  load_code<W>(codes, slot, c);
  int32_t acc = 0;
#pragma unroll
  for (int w = 0; w < W; ++w) {
    acc += __popc(planes[0 * W + w] & c[w]);
    acc += __popc(planes[1 * W + w] & c[w]) << 1;
    acc += __popc(planes[2 * W + w] & c[w]) << 2;
    acc -= __popc(planes[3 * W + w] & c[w]) << 3;
  }
  const float base_d = __fadd_rn(fadd[slot], g);
  const float ip = __fmul_rn((float)acc, delta);
  const float est = __fadd_rn(base_d, __fmul_rn(frescale[slot], __fadd_rn(ip, k1)));
  const float low = __fsub_rn(est, __fmul_rn(ferr[slot], sqrtf(g)));
  acc_out[v] = acc;
  est_out[v] = est;
  low_out[v] = low;
}

void launch_list_estimates(const Index& ix, const uint32_t* planes, float delta, float k1, float g, int list,
                           int32_t* acc, float* est, float* low, cudaStream_t s)
{
  const int64_t base = ix.off_host[list], n = ix.off_host[list + 1] - base;
  if (n <= 0) return;
  const unsigned grid = (unsigned)ceil_div(n, 128);
#define RBQ_LE_CASE(WW)                                                                                     \
  case WW:                                                                                                  \
    list_estimates_kernel<WW><<<grid, 128, 0, s>>>(ix.codes, ix.fadd, ix.frescale, ix.ferr, base, n, planes, \
                                                   delta, k1, g, acc, est, low);                            \
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
