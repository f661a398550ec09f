// Coarse-quantiser scores on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// S[q, c] = |c|^2 - 2 <q, c> for a block of 128 rotated queries against all K rotated centroids
// (the query x centroid GEMM of PrepareClusterSearchInputs, gpu_index/ivf_gpu.cu:1531-1570,
// which the reference runs with cuBLAS sgemm).  kind::tf32 MMAs with fp32 accumulators in
// tensor memory; the scores only rank a shortlist of P + margin lists per query, the exact
// double-precision refine (refine_topp_kernel) decides the probes.
//
// CTA: 256 threads, 128 queries x one chunk of 256 centroids (a 128 x 256 fp32 accumulator =
// 256 TMEM columns); the reduction dimension in chunks of 32 tf32 values (128-byte rows),
// stored K-major with the 128-byte swizzle (16-byte unit u of row r of an 8-row atom lives at
// u ^ r).  The operand tiles arrive by TMA (cp.async.bulk.tensor, 2-D tiles of the row-major
// query and centroid matrices, zero fill past the last row; no multicast) into a ring of four
// shared-memory stages, so up to three k-chunks are in flight while the tensor core works.  One
// thread issues the loads and the MMAs: a stage is refilled once the MMAs that read it have
// committed to its "empty" mbarrier.  The epilogue reads the accumulator with tcgen05.ld
// (warp w: TMEM lanes 32*(w%4).., columns half w/4; lane = query row) and turns each 32 x 32
// block through shared memory, so that every store writes 32 consecutive scores of one row.  Every mbarrier
// wait is bounded: on time-out the kernel records an error code in err[0], waits (bounded)
// for its copies and MMAs in flight, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "rbq_internal.cuh"

namespace rbq {
namespace {

constexpr int kTcM = 128;        // queries per CTA (accumulator rows = TMEM lanes)
constexpr int kTcN = 256;        // centroids per accumulator (TMEM columns)
constexpr int kTcKc = 32;        // tf32 values per 128-byte smem row
constexpr int kTcThreads = 256;
constexpr int kTcStageBytes = (kTcM + kTcN) * 128;  // A chunk (16 KB) + B chunk (32 KB)
constexpr int kTcStages = 3;
constexpr int kTcEpiPitch = 33;  // floats per row of a warp's 32 x 32 epilogue tile (bank-conflict free)
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

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// 2-D tile load of the tensor map's box at element coordinates (x, y) into shared memory.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar)
{
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__global__ void __launch_bounds__(kTcThreads, 1) coarse_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                                  const __grid_constant__ CUtensorMap tmC, int nq,
                                                                  const float* __restrict__ cn2, int K, int dp,
                                                                  float* __restrict__ S, int* __restrict__ err)
{
  extern __shared__ unsigned char tc_smem_raw[];
  // 1024-byte aligned stages (the swizzle pattern is taken from the address bits).
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
  float* epi = reinterpret_cast<float*>(base + kTcStages * kTcStageBytes);  // [8 warps][32][kTcEpiPitch]
  __shared__ __align__(8) unsigned long long s_full[kTcStages], s_empty[kTcStages];
  __shared__ uint32_t s_tmem;
  __shared__ int s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = blockIdx.x * kTcM;  // blockIdx.y: the first centroid chunk of this CTA
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"((uint32_t)kTcN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int i = 0; i < kTcStages; ++i) {
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&s_empty[i]), 1);
    }
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmQ)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmC)) : "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem;

  // k-chunks are numbered over the CTA's whole run: chunk c = (n0 index, kc), stage c % 4.
  // The j-th load into a stage completes phase j of its "full" barrier, the j-th MMA group
  // that read it commits phase j of its "empty" barrier (parity j & 1).  Thread 0 alone
  // issues loads and MMAs; the block learns of a failed wait through s_fail after a barrier.
  const int nkc = dp / kTcKc;
  int n_n0 = 0;
  for (int n0 = blockIdx.y * kTcN; n0 < K; n0 += gridDim.y * kTcN) ++n_n0;
  const int total = n_n0 * nkc;
  int issued = 0, consumed = 0;
  auto stage_of = [&](int c) { return base + (c % kTcStages) * kTcStageBytes; };
  auto issue = [&](int c) -> bool {  // thread 0: load chunk c once its stage is free
    const int st = c % kTcStages;
    if (c >= kTcStages && !mbar_wait(smem_u32(&s_empty[st]), (uint32_t)((c / kTcStages - 1) & 1))) return false;
    const int n0 = (blockIdx.y + (c / nkc) * gridDim.y) * kTcN, kc = c % nkc;
    unsigned char* a_blk = stage_of(c);
    const uint32_t full = smem_u32(&s_full[st]);
    mbar_expect_tx(full, (uint32_t)kTcStageBytes);
    tma_load_2d(smem_u32(a_blk), &tmQ, kc * kTcKc, q0, full);
    tma_load_2d(smem_u32(a_blk + kTcM * 128), &tmC, kc * kTcKc, n0, full);
    return true;
  };
  if (tid == 0)
    for (; issued < total && issued < kTcStages; ++issued) issue(issued);

  for (int t = 0; t < n_n0; ++t) {
    const int n0 = (blockIdx.y + t * gridDim.y) * kTcN;
    if (tid == 0) {
      bool ok = true;
      for (int kc = 0; kc < nkc && ok; ++kc) {
        const int c = consumed;
        const int st = c % kTcStages;
        if (!mbar_wait(smem_u32(&s_full[st]), (uint32_t)((c / kTcStages) & 1))) {
          ok = false;
          atomicExch(err, 1);
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_addr = smem_u32(stage_of(c)), b_addr = a_addr + kTcM * 128;
#pragma unroll
        for (int ks = 0; ks < kTcKc / 8; ++ks)  // 8 tf32 (32 bytes) per MMA
          tc_mma(tmem, sw128_desc(a_addr + ks * 32), sw128_desc(b_addr + ks * 32), kTcIdesc,
                 (kc > 0 || ks > 0) ? 1u : 0u);
        tc_commit(smem_u32(&s_empty[st]));
        ++consumed;
        if (issued < total) {
          if (!issue(issued)) {
            ok = false;
            atomicExch(err, 3);
            break;
          }
          ++issued;
        }
      }
      // The last commit covers every MMA issued before it: the accumulator is complete.
      if (ok) {
        const int last = consumed - 1;
        if (!mbar_wait(smem_u32(&s_empty[last % kTcStages]), (uint32_t)((last / kTcStages) & 1))) {
          ok = false;
          atomicExch(err, 2);
        }
      }
      if (!ok) s_fail = 1;
    }
    __syncthreads();
    if (s_fail) break;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    {
      const int quarter = warp & 3, half = warp >> 2;
      float* tile = epi + warp * 32 * kTcEpiPitch;
#pragma unroll 1
      for (int j = 0; j < (kTcN / 2) / 32; ++j) {
        const int col = half * (kTcN / 2) + j * 32;
        float v[32];
        tc_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)col, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) tile[lane * kTcEpiPitch + i] = v[i];
        __syncwarp();
        const int c = n0 + col + lane;
        const float cn = c < K ? __ldg(cn2 + c) : 0.0f;
#pragma unroll 4
        for (int r = 0; r < 32; ++r) {
          const int q = q0 + quarter * 32 + r;
          if (q < nq && c < K) S[(size_t)q * K + c] = cn - 2.0f * tile[r * kTcEpiPitch + lane];
        }
        __syncwarp();
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
  }
  // On failure: wait (bounded) for the copies and MMAs still in flight, then free TMEM.
  if (s_fail && tid == 0) {
    for (int c = consumed; c < issued; ++c)
      mbar_wait(smem_u32(&s_full[c % kTcStages]), (uint32_t)((c / kTcStages) & 1));
    if (consumed > 0) {
      const int last = consumed - 1;
      mbar_wait(smem_u32(&s_empty[last % kTcStages]), (uint32_t)((last / kTcStages) & 1));
    }
  }
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)kTcN));
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder()
{
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  RBQ_CHECK(fn != nullptr, RBQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  return fn;
}

// Row-major fp32 [rows, dp] matrix, box = [box_rows, 32 values], 128-byte swizzle, zero fill.
CUtensorMap row_major_map(const float* ptr, int64_t rows, int dp, int box_rows)
{
  RBQ_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15u) == 0, RBQ_ERR_INVALID,
            "coarse (tensor cores): operands must be 16-byte aligned");
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)dp, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)dp * sizeof(float)};
  const cuuint32_t box[2] = {(cuuint32_t)kTcKc, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims,
                                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  RBQ_CHECK(r == CUDA_SUCCESS, RBQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return m;
}

}  // namespace

bool coarse_tc_supported(int dp) { return dp % kTcKc == 0 && dp >= kTcKc && dp <= 4096; }

void launch_coarse_scores_tc(const float* A, int64_t nq, const float* C, const float* cn2, int K, int dp, float* S,
                             int* err, cudaStream_t s)
{
  if (nq <= 0) return;
  RBQ_CHECK(coarse_tc_supported(dp), RBQ_ERR_INVALID, "coarse (tensor cores): padded dim must be a multiple of 32");
  RBQ_CHECK(nq <= 0x7fffffff && K >= 1, RBQ_ERR_INVALID, "coarse (tensor cores): bad sizes");
  const size_t smem = (size_t)kTcStages * kTcStageBytes + (size_t)(kTcThreads / 32) * 32 * kTcEpiPitch * 4 + 1024;
  RBQ_CUDA(cudaFuncSetAttribute(coarse_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const CUtensorMap tmQ = row_major_map(A, nq, dp, kTcM);
  const CUtensorMap tmC = row_major_map(C, K, dp, kTcN);
  // one CTA per (128 queries, 256-centroid chunk)
  const dim3 grid((unsigned)ceil_div(nq, kTcM), (unsigned)std::min<int64_t>(ceil_div(K, kTcN), 65535));
  coarse_tc_kernel<<<grid, kTcThreads, smem, s>>>(tmQ, tmC, (int)nq, cn2, K, dp, S, err);
  RBQ_LAUNCHED();
}

}  // namespace rbq
