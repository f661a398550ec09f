// Index-build kernels for sm_100a: rotation, 1-bit quantiser + RaBitQ factors, k-means
// centroid update, row gathers and the synthetic-data generators used by the benchmarks.
//
// Compiled with -fmad=false: every float/double expression below is evaluated exactly as
// written (no FMA contraction), which is what makes the codes and factors bit-identical to
// the CPU oracle's.
#include <cuda_runtime.h>
#include <stdint.h>

#include "rbq_internal.cuh"

namespace rbq {

// ---------------------------------------------------------------------------------------
// Rotation: Y[n, Dp] = pad(X[n, D]) * P, P row-major [Dp, Dp] (RotatorGPU::rotate,
// gpu_index/rotator_gpu.cu:162-176 computes the same product with cuBLAS sgemm).
// Each output is float(sum_k double(x_k) * double(P[k][j])) accumulated for k = 0..Dp-1;
// the float*float product is exact in double, so DFMA and DMUL+DADD give the same bits.
// Block: RB rows x all Dp columns; thread t owns columns t, t+blockDim, ...  The block's rows
// are staged in shared memory already widened to double (read two k at a time, 16-byte
// broadcasts); the thread's P values stream from L2 four k ahead of their use, so the DFMAs of
// one step overlap the loads of the next.
template <int RB, int CPT>
__global__ void __launch_bounds__(256, (CPT <= 2 ? 3 : 2)) rotate_kernel(const float* __restrict__ X, int64_t n, int D, int Dp,
                                                     const float* __restrict__ P, float* __restrict__ Y)
{
  constexpr int KU = 4;  // k per step (Dp is a multiple of 32)
  extern __shared__ __align__(16) double xs[];  // [RB][Dp]
  const int64_t r0 = (int64_t)blockIdx.x * RB;
  for (int i = threadIdx.x; i < RB * Dp; i += blockDim.x) {
    const int r = i / Dp, k = i - r * Dp;
    const int64_t row = r0 + r;
    xs[i] = (row < n && k < D) ? (double)X[row * D + k] : 0.0;
  }
  __syncthreads();
  double acc[RB][CPT];
#pragma unroll
  for (int r = 0; r < RB; ++r)
#pragma unroll
    for (int c = 0; c < CPT; ++c) acc[r][c] = 0.0;
  float pn[KU][CPT];
  auto load_p = [&](int k0) {
#pragma unroll
    for (int u = 0; u < KU; ++u)
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        const int j = threadIdx.x + c * blockDim.x;
        pn[u][c] = (j < Dp && k0 + u < Dp) ? __ldg(P + (size_t)(k0 + u) * Dp + j) : 0.0f;
      }
  };
  load_p(0);
  for (int k = 0; k < Dp; k += KU) {
    double p[KU][CPT];
#pragma unroll
    for (int u = 0; u < KU; ++u)
#pragma unroll
      for (int c = 0; c < CPT; ++c) p[u][c] = (double)pn[u][c];
    load_p(k + KU);
#pragma unroll
    for (int r = 0; r < RB; ++r) {
#pragma unroll
      for (int u = 0; u < KU; u += 2) {
        const double2 xv = *reinterpret_cast<const double2*>(xs + r * Dp + k + u);
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          acc[r][c] = __fma_rn(xv.x, p[u][c], acc[r][c]);
          acc[r][c] = __fma_rn(xv.y, p[u + 1][c], acc[r][c]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RB; ++r) {
    const int64_t row = r0 + r;
    if (row >= n) break;
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      const int j = threadIdx.x + c * blockDim.x;
      if (j < Dp) Y[row * Dp + j] = (float)acc[r][c];
    }
  }
}

template <int RB, int CPT>
static void launch_rotate_rc(const float* X, int64_t n, int D, int Dp, const float* P, float* Y, int threads,
                             cudaStream_t s)
{
  const size_t smem = (size_t)RB * Dp * sizeof(double);
  if (smem > 48 * 1024)
    RBQ_CUDA(cudaFuncSetAttribute(rotate_kernel<RB, CPT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  rotate_kernel<RB, CPT><<<(unsigned)ceil_div(n, RB), threads, smem, s>>>(X, n, D, Dp, P, Y);
  RBQ_LAUNCHED();
}

void launch_rotate(const float* X, int64_t n, int D, int Dp, const float* P, float* Y, cudaStream_t s)
{
  if (n <= 0) return;
  const int threads = Dp < 256 ? Dp : 256;
  const int cpt = (Dp + threads - 1) / threads;
  // Rows per block: at most 8 (RB * CPT double accumulators per thread), sized so that the
  // thread's accumulators and four k of prefetched P fit three (CPT <= 2) or two blocks per SM.
  switch (cpt) {
    case 1: launch_rotate_rc<8, 1>(X, n, D, Dp, P, Y, threads, s); break;
    case 2: launch_rotate_rc<4, 2>(X, n, D, Dp, P, Y, threads, s); break;
    case 3: launch_rotate_rc<4, 3>(X, n, D, Dp, P, Y, threads, s); break;
    case 4: launch_rotate_rc<4, 4>(X, n, D, Dp, P, Y, threads, s); break;
    case 6: launch_rotate_rc<2, 6>(X, n, D, Dp, P, Y, threads, s); break;
    case 8: launch_rotate_rc<1, 8>(X, n, D, Dp, P, Y, threads, s); break;
    default: throw Error{RBQ_ERR_INVALID, "rotation: padded dim must be <= 2048 with Dp/256 in {1,2,3,4,6,8}"};
  }
}

// ---------------------------------------------------------------------------------------
// 1-bit quantiser + factors (subtract_normalize_binarize_Kernel and
// pack_and_compute_factors_kernel, gpu_index/quantizer_gpu.cu:109-172 and 251-338).
// One thread per vector; every sum is a double accumulation in dimension order, rounded to
// float once, so the block-reduction order of the reference does not enter.
//   r = y - c_rot[label];  bit_j = (|r| > 0 && r_j > 0);  dim 32w+j -> bit 31-j of word w
//   xu = bit - 0.5;  l2 = |r|^2;  ip = <r, xu> (0 -> +inf);  ipc = <c_rot, xu>;  xu2 = Dp/4
//   f_add = l2 + 2 l2 * (ipc / ip);  f_rescale = -2 l2 / ip
//   f_err = 2 * (|r| * 1.9) * sqrt(max(0, (l2 * xu2 / ip^2 - 1) / max(Dp - 1, 1)))
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) quantize_kernel(const float* __restrict__ Y, int64_t n, int Dp,
                                                       const float* __restrict__ C_rot,
                                                       const uint32_t* __restrict__ labels,
                                                       uint32_t* __restrict__ codes, float* __restrict__ fadd,
                                                       float* __restrict__ frescale, float* __restrict__ ferr)
{
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float* y = Y + i * Dp;
  const float* c = C_rot + (size_t)labels[i] * Dp;
  double l2d = 0.0;
  for (int j = 0; j < Dp; ++j) {
    const float r = y[j] - c[j];
    l2d += (double)r * (double)r;
  }
  const float l2_sqr = (float)l2d;
  const float norm = sqrtf(l2_sqr);
  double ipr = 0.0, ipc = 0.0;
  const int W = Dp >> 5;
  for (int w = 0; w < W; ++w) {
    uint32_t word = 0u;
    for (int b = 0; b < 32; ++b) {
      const int j = (w << 5) + b;
      const float r = y[j] - c[j];
      const int bit = (norm > 0.0f && r > 0.0f) ? 1 : 0;
      word |= (uint32_t)bit << (31 - b);
      const double xu = bit ? 0.5 : -0.5;
      ipr += (double)r * xu;
      ipc += (double)c[j] * xu;
    }
    codes[i * W + w] = word;
  }
  float ip_resi = (float)ipr;
  const float ip_cent = (float)ipc;
  const float xu_sq = 0.25f * (float)Dp;
  if (ip_resi == 0.0f) ip_resi = __int_as_float(0x7f800000);
  const float l2_norm = sqrtf(fmaxf(l2_sqr, 0.0f));
  const float denom = ip_resi;
  fadd[i] = l2_sqr + (2.0f * l2_sqr) * (ip_cent / denom);
  frescale[i] = (-2.0f * l2_sqr) / denom;
  const float ratio = (l2_sqr * xu_sq) / (denom * denom);
  float inner = (ratio - 1.0f) / fmaxf((float)(Dp - 1), 1.0f);
  inner = fmaxf(inner, 0.0f);
  ferr[i] = 2.0f * ((l2_norm * 1.9f) * sqrtf(inner));
}

void launch_quantize(const float* Y, int64_t n, int Dp, const float* C_rot, const uint32_t* labels,
                     uint32_t* codes, float* fadd, float* frescale, float* ferr, cudaStream_t s)
{
  if (n <= 0) return;
  quantize_kernel<<<(unsigned)ceil_div(n, 128), 128, 0, s>>>(Y, n, Dp, C_rot, labels, codes, fadd, frescale,
                                                             ferr);
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// ExRaBitQ extra bits (bits_per_dim = ex + 1), one thread per row: the fast-quantize branch of
// quantize_batch_opt (exrabitq_fused_kernel_batch, quantizer_gpu.cu:347-468) on the normalised
// residual xn = r / |r| of subtract_normalize_binarize_Kernel (:109-172).  Per dim:
//   e = min(int(t * |xn| + 1e-5), 2^ex - 1); stored x = e where the 1-bit code is 1, else
//   2^ex - 1 - e; centred code xu = (bit * 2^ex + x) - (2^ex - 1/2);
//   ip_norm = sum (e + 1/2) |xn|, ip_resi = sum r xu, ip_cent = sum c xu (double, dim order);
//   f_ex_add = |r|^2 + (2 |r|^2 ip_cent) / ip_resi (0 -> +inf); f_ex_rescale = -2 |r| / ip_norm.
// The top bit of the code is the stored 1-bit code (r > 0) in the factors too; the reference
// uses r >= 0 there, which differs only where a residual coordinate is exactly zero.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) quantize_ex_kernel(const float* __restrict__ Y, int64_t n, int Dp,
                                                          const float* __restrict__ C_rot,
                                                          const uint32_t* __restrict__ labels, int ex, float t,
                                                          uint32_t* __restrict__ planes, float* __restrict__ fexadd,
                                                          float* __restrict__ fexr)
{
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float* y = Y + i * Dp;
  const float* c = C_rot + (size_t)labels[i] * Dp;
  double l2d = 0.0;
  for (int j = 0; j < Dp; ++j) {
    const float r = __fsub_rn(y[j], c[j]);
    l2d += (double)r * (double)r;
  }
  const float l2_sqr = (float)l2d;
  const float norm = sqrtf(l2_sqr);
  const int W = Dp >> 5;
  const int mask = (1 << ex) - 1;
  const float shift = __fsub_rn((float)(1 << ex), 0.5f);
  double ipn = 0.0, ipr = 0.0, ipc = 0.0;
  uint32_t* out = planes + (size_t)i * ex * W;
  for (int w = 0; w < W; ++w) {
    uint32_t pw[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    for (int b = 0; b < 32; ++b) {
      const int j = (w << 5) + b;
      const float r = __fsub_rn(y[j], c[j]);
      const int bit = (norm > 0.0f && r > 0.0f) ? 1 : 0;
      const float xn = norm > 0.0f ? __fdiv_rn(r, norm) : 0.0f;
      const float a = fabsf(xn);
      int e = (int)__fadd_rn(__fmul_rn(t, a), 1e-5f);
      if (e > mask) e = mask;
      ipn += (double)__fmul_rn(__fadd_rn((float)e, 0.5f), a);
      const int x = bit ? e : mask - e;
#pragma unroll
      for (int p = 0; p < 8; ++p) pw[p] |= (uint32_t)((x >> p) & 1) << (31 - b);
      const float xu = __fsub_rn((float)((bit << ex) | x), shift);
      ipr += (double)r * (double)xu;
      ipc += (double)c[j] * (double)xu;
    }
#pragma unroll
    for (int p = 0; p < 8; ++p)
      if (p < ex) out[p * W + w] = pw[p];
  }
  const float ip_resi = (float)ipr, ip_cent = (float)ipc, ip_norm = (float)ipn;
  const float denom = ip_resi == 0.0f ? __int_as_float(0x7f800000) : ip_resi;
  const float l2_norm = sqrtf(fmaxf(l2_sqr, 0.0f));
  fexadd[i] = __fadd_rn(l2_sqr, __fdiv_rn(__fmul_rn(__fmul_rn(2.0f, l2_sqr), ip_cent), denom));
  float inv = __fdiv_rn(1.0f, ip_norm);
  if (!isfinite(inv)) inv = 1.0f;
  fexr[i] = __fmul_rn(__fmul_rn(-2.0f, l2_norm), inv);
}

void launch_quantize_ex(const float* Y, int64_t n, int Dp, const float* C_rot, const uint32_t* labels, int ex,
                        float t, uint32_t* planes, float* fexadd, float* fexr, cudaStream_t s)
{
  if (n <= 0 || ex <= 0) return;
  quantize_ex_kernel<<<(unsigned)ceil_div(n, 128), 128, 0, s>>>(Y, n, Dp, C_rot, labels, ex, t, planes, fexadd,
                                                                fexr);
  RBQ_LAUNCHED();
}

// Row squared norms (float accumulation; only used to rank candidates approximately).
__global__ void row_norms_kernel(const float* __restrict__ A, int64_t n, int d, float* __restrict__ out)
{
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  float s = 0.0f;
  for (int j = lane; j < d; j += 32) {
    const float v = A[row * d + j];
    s = __fmaf_rn(v, v, s);
  }
  for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) out[row] = s;
}

void launch_row_norms(const float* A, int64_t n, int d, float* out, cudaStream_t s)
{
  if (n <= 0) return;
  row_norms_kernel<<<(unsigned)ceil_div(n, 8), 256, 0, s>>>(A, n, d, out);
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// k-means centroid update: C[c] = mean of member rows, members in the order given by
// `order` (host counting sort), double accumulation.  Empty lists keep their centroid
// (Lloyd) or become the zero vector (balanced k-means: the reference's division by a zero
// size yields 0, kmeans_balanced.cuh:295-300).
// ---------------------------------------------------------------------------------------
__global__ void centroid_update_kernel(const float* __restrict__ X, int D, const int64_t* __restrict__ off,
                                       const uint32_t* __restrict__ order, float* __restrict__ C, int zero_empty)
{
  const int c = blockIdx.x;
  const int64_t a = off[c], b = off[c + 1];
  if (b <= a) {
    if (zero_empty)
      for (int j = threadIdx.x; j < D; j += blockDim.x) C[(size_t)c * D + j] = 0.0f;
    return;
  }
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    double s = 0.0;
    for (int64_t m = a; m < b; ++m) s += (double)X[(size_t)order[m] * D + j];
    C[(size_t)c * D + j] = (float)(s / (double)(b - a));
  }
}

void launch_centroid_update(const float* X, int64_t /*n*/, int D, const uint32_t* /*labels*/, const int64_t* off,
                            const uint32_t* order, int K, float* C, bool zero_empty, cudaStream_t s)
{
  if (K <= 0) return;
  centroid_update_kernel<<<K, 128, 0, s>>>(X, D, off, order, C, zero_empty ? 1 : 0);
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// Balanced k-means rebalancing (kmeans_balanced.cuh:443-496): a small cluster's centre moves
// towards a row of a large cluster, C[l] = (wc * C[li] + 1 * X[i]) / (wc + 1), evaluated in
// that order in round-to-nearest float arithmetic.  adj[4a .. 4a+3] = {l, li, i, wc}; the
// host picked them (li is never an adjusted cluster, so the reads do not race the writes).
// ---------------------------------------------------------------------------------------
__global__ void adjust_centers_kernel(float* __restrict__ C, int D, const float* __restrict__ X,
                                      const int64_t* __restrict__ adj)
{
  const int64_t* e = adj + 4 * (size_t)blockIdx.x;
  const int64_t l = e[0], li = e[1], i = e[2];
  const float wc = (float)e[3];
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    float v = 0.0f;
    v = __fadd_rn(v, __fmul_rn(wc, C[(size_t)li * D + j]));
    v = __fadd_rn(v, __fmul_rn(1.0f, X[(size_t)i * D + j]));
    C[(size_t)l * D + j] = __fdiv_rn(v, __fadd_rn(wc, 1.0f));
  }
}

void launch_adjust_centers(float* C, int D, const float* X, const int64_t* adj, int n_adj, cudaStream_t s)
{
  if (n_adj <= 0) return;
  adjust_centers_kernel<<<n_adj, 128, 0, s>>>(C, D, X, adj);
  RBQ_LAUNCHED();
}

__global__ void gather_rows_kernel(const float* __restrict__ src, int64_t rows, int cols,
                                   const int64_t* __restrict__ src_row, float* __restrict__ dst)
{
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int64_t sr = src_row[r];
  for (int j = threadIdx.x & 31; j < cols; j += 32) dst[r * cols + j] = src[sr * cols + j];
}

void launch_gather_rows_f32(const float* src, int64_t rows, int cols, const int64_t* src_row, float* dst,
                            cudaStream_t s)
{
  if (rows <= 0) return;
  gather_rows_kernel<<<(unsigned)ceil_div(rows, 8), 256, 0, s>>>(src, rows, cols, src_row, dst);
  RBQ_LAUNCHED();
}

// ---------------------------------------------------------------------------------------
// Synthetic data for the benchmark configurations (configs 1, 2, 4, 5).
// Philox-4x32-10 counters; normals by Box-Muller in double (CUDA's log/sincos).
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void philox_dev(uint32_t k0, uint32_t k1, uint32_t c[4])
{
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c[0]), lo0 = 0xD2511F53u * c[0];
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]), lo1 = 0xCD9E8D57u * c[2];
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

__device__ __forceinline__ double normal_dev(uint64_t seed, uint32_t stream, uint64_t i)
{
  const uint64_t blk = i >> 1;
  uint32_t c[4] = {(uint32_t)blk, (uint32_t)(blk >> 32), stream, 0x52425142u};
  philox_dev((uint32_t)seed, (uint32_t)(seed >> 32), c);
  const double scale = 1.0 / 9007199254740992.0;
  const double u1 = ((double)(((uint64_t)c[0] << 21) ^ (c[1] >> 11)) + 0.5) * scale;
  const double u2 = ((double)(((uint64_t)c[2] << 21) ^ (c[3] >> 11)) + 0.5) * scale;
  const double radius = sqrt(-2.0 * log(u1));
  double sv, cv;
  sincospi(2.0 * u2, &sv, &cv);
  return (i & 1) ? radius * sv : radius * cv;
}

__device__ __forceinline__ uint64_t hash64_dev(uint64_t seed, uint32_t stream, uint64_t i)
{
  uint32_t c[4] = {(uint32_t)i, (uint32_t)(i >> 32), stream, 0x48534831u};
  philox_dev((uint32_t)seed, (uint32_t)(seed >> 32), c);
  return ((uint64_t)c[0] << 32) | c[1];
}

__device__ __forceinline__ float dim_scale(int d, int aniso)
{
  return aniso ? (float)sqrt(1.0 / (1.0 + (double)d / 64.0)) : 1.0f;
}

__global__ void gen_centres_kernel(float* __restrict__ C, int nc, int D, int aniso, uint64_t seed, uint32_t stream)
{
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)nc * D) return;
  const int d = (int)(i % D);
  C[i] = (float)normal_dev(seed, stream, (uint64_t)i) * dim_scale(d, aniso);
}

// One warp per row.
__global__ void gen_rows_kernel(float* __restrict__ X, int64_t n, int D, const float* __restrict__ C, int nc,
                                float sigma, int aniso, int normalize, uint64_t seed, uint32_t stream)
{
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  const int cen = (int)(hash64_dev(seed, stream, (uint64_t)row) % (uint64_t)nc);
  float ss = 0.0f;
  for (int d = lane; d < D; d += 32) {
    const float v = C[(size_t)cen * D + d] +
                    sigma * dim_scale(d, aniso) * (float)normal_dev(seed, stream + 1u, (uint64_t)row * D + d);
    X[row * D + d] = v;
    ss = __fmaf_rn(v, v, ss);
  }
  if (!normalize) return;
  for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float inv = ss > 0.0f ? 1.0f / sqrtf(ss) : 0.0f;
  for (int d = lane; d < D; d += 32) X[row * D + d] *= inv;
}

void launch_gen_mixture(float* X, int64_t n, int D, int n_centres, float sigma, int aniso, int normalize,
                        uint64_t seed, uint32_t stream, float* centres, cudaStream_t s)
{
  const int64_t cn = (int64_t)n_centres * D;
  gen_centres_kernel<<<(unsigned)ceil_div(cn, 256), 256, 0, s>>>(centres, n_centres, D, aniso, seed, stream);
  RBQ_LAUNCHED();
  gen_rows_kernel<<<(unsigned)ceil_div(n, 8), 256, 0, s>>>(X, n, D, centres, n_centres, sigma, aniso, normalize,
                                                          seed, stream + 1u);
  RBQ_LAUNCHED();
}

__global__ void gen_queries_kernel(const float* __restrict__ X, int64_t n, int D, float* __restrict__ Q, int64_t nq,
                                   float sigma, int normalize, uint64_t seed, uint32_t stream,
                                   int64_t* __restrict__ src_rows)
{
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= nq) return;
  const int64_t src = (int64_t)(hash64_dev(seed, stream, (uint64_t)row) % (uint64_t)n);
  if (src_rows && lane == 0) src_rows[row] = src;
  float ss = 0.0f;
  for (int d = lane; d < D; d += 32) {
    const float v = X[src * D + d] + sigma * (float)normal_dev(seed, stream + 1u, (uint64_t)row * D + d);
    Q[row * D + d] = v;
    ss = __fmaf_rn(v, v, ss);
  }
  if (!normalize) return;
  for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float inv = ss > 0.0f ? 1.0f / sqrtf(ss) : 0.0f;
  for (int d = lane; d < D; d += 32) Q[row * D + d] *= inv;
}

void launch_gen_queries(const float* X, int64_t n, int D, float* Q, int64_t nq, float sigma, int normalize,
                        uint64_t seed, uint32_t stream, int64_t* src_rows, cudaStream_t s)
{
  if (nq <= 0) return;
  gen_queries_kernel<<<(unsigned)ceil_div(nq, 8), 256, 0, s>>>(X, n, D, Q, nq, sigma, normalize, seed, stream,
                                                              src_rows);
  RBQ_LAUNCHED();
}

__global__ void gather_rows_u32_kernel(const uint32_t* __restrict__ src, int64_t rows, int cols,
                                       const int64_t* __restrict__ src_row, uint32_t* __restrict__ dst)
{
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const int64_t r = i / cols;
  const int j = (int)(i - r * cols);
  dst[i] = src[src_row[r] * cols + j];
}

void launch_gather_rows_u32(const uint32_t* src, int64_t rows, int cols, const int64_t* src_row, uint32_t* dst,
                            cudaStream_t s)
{
  if (rows <= 0) return;
  gather_rows_u32_kernel<<<(unsigned)ceil_div(rows * cols, 256), 256, 0, s>>>(src, rows, cols, src_row, dst);
  RBQ_LAUNCHED();
}

__global__ void scatter_id2row_kernel(const uint32_t* __restrict__ ids, int64_t n, uint32_t* __restrict__ id2row)
{
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r < n) id2row[ids[r]] = (uint32_t)r;
}

void launch_scatter_id2row(const uint32_t* ids, int64_t n, uint32_t* id2row, cudaStream_t s)
{
  if (n <= 0) return;
  scatter_id2row_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(ids, n, id2row);
  RBQ_LAUNCHED();
}

}  // namespace rbq
