// Coarse-quantiser scores on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// S[q, c] = |c|^2 - 2 <q, c> for a block of 128 rotated queries against all K rotated centroids
// (the query x centroid GEMM of PrepareClusterSearchInputs, gpu_index/ivf_gpu.cu:1531-1570,
// which the reference runs with cuBLAS sgemm).  kind::tf32 MMAs with fp32 accumulators in
// tensor memory; the scores only rank a shortlist of P + margin lists per query, the exact
// double-precision refine (refine_topp_kernel) decides the probes.
//
// CTA: 256 threads, 128 queries; centroids in chunks of 256 (one 128 x 256 fp32 accumulator =
// 256 TMEM columns); the reduction dimension in chunks of 32 tf32 values (128-byte rows),
// stored K-major with the 128-byte swizzle (16-byte unit u of row r of an 8-row atom lives at
// u ^ r).  Two shared-memory stages: threads fill one stage while the tensor core consumes the
// other; one elected thread issues the MMAs and commits them to a per-stage mbarrier.  The
// epilogue reads the accumulator with tcgen05.ld (warp w: TMEM lanes 32*(w%4).., columns half
// w/4) and writes the scores.  Every mbarrier wait is bounded: on time-out the kernel records
// an error code in err[0] and stops issuing work, it never spins forever.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "rbq_internal.cuh"

namespace rbq {
namespace {

constexpr int kTcM = 128;        // queries per CTA (accumulator rows = TMEM lanes)
constexpr int kTcN = 256;        // centroids per accumulator (TMEM columns)
constexpr int kTcKc = 32;        // tf32 values per 128-byte smem row
constexpr int kTcThreads = 256;
constexpr int kTcStageBytes = (kTcM + kTcN) * 128;  // A chunk (16 KB) + B chunk (32 KB)
constexpr uint32_t kWaitLimit = 1u << 26;           // bounded mbarrier polling

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// 64-bit shared-memory matrix descriptor (K-major, 128-byte swizzle): start address, leading
// byte offset (unused for this layout, 16 B), stride byte offset (1024 B between 8-row atoms),
// descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16u >> 4) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor for kind::tf32: D f32, A/B tf32, both K-major, N = kTcN, M = kTcM.
constexpr uint32_t kTcIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kTcN >> 3) << 17) |
                              ((uint32_t)(kTcM >> 4) << 24);

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

// Polls mbarrier phase `parity`; false if it did not complete within kWaitLimit polls.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity)
{
  for (uint32_t it = 0; it < kWaitLimit; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

__device__ __forceinline__ void tc_mma(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc)
{
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}" ::"r"(dtmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void tc_commit(uint32_t bar)
{
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 consecutive fp32 accumulator columns of the warp's 32 TMEM lanes.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32])
{
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Copy `rows` rows x 32 values (columns [k0, k0+32) of a row-major [nrows_src, ld] matrix,
// rows from r0) into a 128-byte-swizzled K-major block; rows past nrows_src are zeros.
__device__ __forceinline__ void fill_sw128(unsigned char* blk, int rows, const float* __restrict__ src, int r0,
                                           int nrows_src, int ld, int k0)
{
  for (int e = threadIdx.x; e < rows * 8; e += kTcThreads) {
    const int r = e >> 3, u = e & 7;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r0 + r < nrows_src) v = __ldg(reinterpret_cast<const float4*>(src + (size_t)(r0 + r) * ld + k0) + u);
    unsigned char* dst = blk + (r >> 3) * 1024 + (r & 7) * 128 + ((u ^ (r & 7)) << 4);
    *reinterpret_cast<float4*>(dst) = v;
  }
}

__global__ void __launch_bounds__(kTcThreads, 1) coarse_tc_kernel(const float* __restrict__ Qr, int nq,
                                                                  const float* __restrict__ Cr,
                                                                  const float* __restrict__ cn2, int K, int dp,
                                                                  float* __restrict__ S, int* __restrict__ err)
{
  extern __shared__ unsigned char tc_smem_raw[];
  // 1024-byte aligned stages (the swizzle pattern is taken from the address bits).
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
  unsigned char* stage[2] = {base, base + kTcStageBytes};
  __shared__ __align__(8) unsigned long long s_bar[2];
  __shared__ uint32_t s_tmem;
  __shared__ int s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = blockIdx.x * kTcM;  // blockIdx.y: the first centroid chunk of this CTA
  const uint32_t bar0 = smem_u32(&s_bar[0]), bar1 = smem_u32(&s_bar[1]);
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"((uint32_t)kTcN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bar0, 1);
    mbar_init(bar1, 1);
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem;

  // Stage s = it & 1 of k-chunk `it` (counted over the whole kernel) is reused by chunk it + 2
  // only after the MMAs of chunk it completed: completion number (it >> 1) of barrier s, i.e.
  // mbarrier phase parity (it >> 1) & 1.  Only thread 0 polls; the block reads s_fail after a
  // barrier, so every thread takes the same path.
  const int nkc = dp / kTcKc;
  int it = 0;
  for (int n0 = blockIdx.y * kTcN; n0 < K; n0 += gridDim.y * kTcN) {
    for (int kc = 0; kc < nkc; ++kc, ++it) {
      const int sidx = it & 1;
      const uint32_t bar = sidx ? bar1 : bar0;
      if (it >= 2 && tid == 0) {
        if (!mbar_wait(bar, (uint32_t)((it - 2) >> 1) & 1u)) {
          s_fail = 1;
          atomicExch(err, 1);
        }
      }
      __syncthreads();
      if (s_fail) break;
      unsigned char* a_blk = stage[sidx];
      unsigned char* b_blk = stage[sidx] + kTcM * 128;
      fill_sw128(a_blk, kTcM, Qr, q0, nq, dp, kc * kTcKc);
      fill_sw128(b_blk, kTcN, Cr, n0, K, dp, kc * kTcKc);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncthreads();
      if (tid == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_addr = smem_u32(a_blk), b_addr = smem_u32(b_blk);
#pragma unroll
        for (int ks = 0; ks < kTcKc / 8; ++ks)  // 8 tf32 (32 bytes) per MMA
          tc_mma(tmem, sw128_desc(a_addr + ks * 32), sw128_desc(b_addr + ks * 32), kTcIdesc,
                 (kc > 0 || ks > 0) ? 1u : 0u);
        tc_commit(bar);
      }
    }
    if (s_fail) break;
    // The last chunk's commit covers every MMA issued before it.
    if (tid == 0) {
      const int last = it - 1;
      if (!mbar_wait((last & 1) ? bar1 : bar0, (uint32_t)(last >> 1) & 1u)) {
        s_fail = 1;
        atomicExch(err, 2);
      }
    }
    __syncthreads();
    if (s_fail) break;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    {
      const int quarter = warp & 3, half = warp >> 2;
      const int row = quarter * 32 + lane;
      const int q = q0 + row;
#pragma unroll 1
      for (int j = 0; j < (kTcN / 2) / 32; ++j) {
        const int col = half * (kTcN / 2) + j * 32;
        float v[32];
        tc_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)col, v);
        if (q < nq) {
          float* out = S + (size_t)q * K + n0 + col;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int c = n0 + col + i;
            if (c < K) out[i] = __ldg(cn2 + c) - 2.0f * v[i];
          }
        }
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
  }
  // On failure, give the MMAs already issued a bounded chance to finish before freeing TMEM.
  if (s_fail && tid == 0 && it > 0) {
    const int last = it - 1;
    mbar_wait((last & 1) ? bar1 : bar0, (uint32_t)(last >> 1) & 1u);
  }
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)kTcN));
  }
}

}  // namespace

bool coarse_tc_supported(int dp) { return dp % kTcKc == 0 && dp >= kTcKc && dp <= 4096; }

void launch_coarse_scores_tc(const float* A, int64_t nq, const float* C, const float* cn2, int K, int dp, float* S,
                             int* err, cudaStream_t s)
{
  if (nq <= 0) return;
  RBQ_CHECK(coarse_tc_supported(dp), RBQ_ERR_INVALID, "coarse (tensor cores): padded dim must be a multiple of 32");
  RBQ_CHECK(nq <= 0x7fffffff && K >= 1, RBQ_ERR_INVALID, "coarse (tensor cores): bad sizes");
  const size_t smem = (size_t)2 * kTcStageBytes + 1024;
  RBQ_CUDA(cudaFuncSetAttribute(coarse_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  // one CTA per (128 queries, 256-centroid chunk)
  const dim3 grid((unsigned)ceil_div(nq, kTcM), (unsigned)std::min<int64_t>(ceil_div(K, kTcN), 65535));
  coarse_tc_kernel<<<grid, kTcThreads, smem, s>>>(A, (int)nq, C, cn2, K, dp, S, err);
  RBQ_LAUNCHED();
}

}  // namespace rbq
