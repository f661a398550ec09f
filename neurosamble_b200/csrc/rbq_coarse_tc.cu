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

// ---------------------------------------------------------------------------------------
// Fused scores + shortlist for large K (the [queries, K] score matrix never leaves the SM).
//
// CTA: 192 threads, 128 queries against all K centroids in chunks of kTcN = 256.  Warp 4 (one
// lane) streams the operand k-chunks by TMA into a ring of four stages; warp 5 (one lane) issues
// the tf32 MMAs of chunk t into accumulator t % 2 (two accumulators, all 512 TMEM columns), so
// the MMAs of one chunk overlap the epilogue of the previous one; warps 0-3 are the epilogue,
// thread r owning query row r (TMEM lane r).  Per chunk an epilogue thread reads its 256 scores
// S = |c|^2 - 2 <q, c> (the same arithmetic as coarse_tc_kernel), and appends the (score,
// column) key to its row's buffer in global memory only when it is below the row's threshold
// (the m-th smallest key kept so far).  When a buffer could overflow, its warp cuts it to the m
// smallest by a cooperative radix select and the threshold tightens; a threshold is never below
// the final m-th smallest key, so the result is the m smallest keys of the row, as
// topm_rows_kernel's.  At the end each row writes its m columns (ascending) and its m-th smallest
// score.  Every wait is bounded and a failed wait makes all roles stop.
// ---------------------------------------------------------------------------------------
constexpr int kFtThreads = 192;
constexpr int kFtStages = 4;
constexpr int kFtProducerWarp = 4, kFtMmaWarp = 5;

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// mbar_wait that also gives up as soon as another role has reported a failure.
__device__ __forceinline__ bool mbar_wait_or_fail(uint32_t bar, uint32_t parity, volatile int* fail)
{
  for (uint32_t it = 0; it < kWaitLimit; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((it & 1023u) == 1023u && *fail) return false;
  }
  return false;
}

// Ascending bitonic sort of the 32 * KPL keys a warp holds in registers: element e = lane * KPL + j
// lives in k[j] of lane `lane`.  Partners closer than KPL are in the same lane; farther ones are
// exchanged by shuffles.
template <int KPL>
__device__ __forceinline__ void warp_bitonic_sort(unsigned long long (&k)[KPL], int lane)
{
  constexpr int N = 32 * KPL;
#pragma unroll
  for (int size = 2; size <= N; size <<= 1) {
#pragma unroll
    for (int dist = size >> 1; dist > 0; dist >>= 1) {
      if (dist >= KPL) {
        const int lx = dist / KPL;
#pragma unroll
        for (int j = 0; j < KPL; ++j) {
          const int e = lane * KPL + j;
          const unsigned long long o = __shfl_xor_sync(0xffffffffu, k[j], lx);
          const bool up = (e & size) == 0, lower = (lane & lx) == 0;
          const bool take_min = lower == up;
          k[j] = take_min ? (o < k[j] ? o : k[j]) : (o > k[j] ? o : k[j]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < KPL; ++j) {
          const int jp = j ^ dist;
          if (jp > j) {
            const int e = lane * KPL + j;
            const bool up = (e & size) == 0;
            const unsigned long long a = k[j], b = k[jp];
            const bool sw = up ? (a > b) : (a < b);
            k[j] = sw ? b : a;
            k[jp] = sw ? a : b;
          }
        }
      }
    }
  }
}

// Sorts the n <= 32 * KPL distinct keys buf[0..n) (global memory) by the whole warp and writes back
// the `keep` smallest, ascending, to buf[0..keep); returns the `want`-th smallest key
// (kEmptyKey if n < want).
template <int KPL>
__device__ unsigned long long warp_sort_keys(unsigned long long* buf, int n, int keep, int want, int lane)
{
  unsigned long long k[KPL];
#pragma unroll
  for (int j = 0; j < KPL; ++j) {
    const int e = lane * KPL + j;
    k[j] = e < n ? buf[e] : kEmptyKey;
  }
  warp_bitonic_sort<KPL>(k, lane);
  __syncwarp();  // every lane has read its keys before any is overwritten
  unsigned long long r = kEmptyKey;
#pragma unroll
  for (int j = 0; j < KPL; ++j) {
    const int e = lane * KPL + j;
    if (e < keep && e < n) buf[e] = k[j];
    if (e == want - 1) r = k[j];
  }
  const int src = (want - 1) / KPL;
  return want >= 1 && want <= n ? __shfl_sync(0xffffffffu, r, src) : kEmptyKey;
}

template <int KPL>
__global__ void __launch_bounds__(kFtThreads, 1)
    coarse_topm_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmC, int nq,
                          const float* __restrict__ cn2, int K, int dp, int m, int p, int cap,
                          unsigned long long* __restrict__ rowbuf, int32_t* __restrict__ cand,
                          float2* __restrict__ bounds, int* __restrict__ err)
{
  extern __shared__ unsigned char tc_smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
  float* cn2s = reinterpret_cast<float*>(base + kFtStages * kTcStageBytes);  // [2][kTcN]
  __shared__ __align__(8) unsigned long long s_full[kFtStages], s_empty[kFtStages], s_accf[2], s_acce[2];
  __shared__ uint32_t s_tmem;
  __shared__ volatile int s_fail;
  __shared__ int s_issued, s_consumed;
  __shared__ int s_ok[2][4];  // epilogue warps' wait results, by chunk parity

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = blockIdx.x * kTcM;
  const int nkc = dp / kTcKc;
  const int n_chunks = (K + kTcN - 1) / kTcN;
  const int total = n_chunks * nkc;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"((uint32_t)(2 * kTcN)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == kFtProducerWarp * 32) {
    for (int i = 0; i < kFtStages; ++i) {
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&s_empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&s_accf[i]), 1);
      mbar_init(smem_u32(&s_acce[i]), 4);
    }
    s_fail = 0;
    s_issued = 0;
    s_consumed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmQ)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmC)) : "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem;

  if (warp == kFtProducerWarp) {
    if (lane == 0) {
      int c = 0;
      for (; c < total; ++c) {
        const int st = c % kFtStages;
        if (c >= kFtStages &&
            !mbar_wait_or_fail(smem_u32(&s_empty[st]), (uint32_t)((c / kFtStages - 1) & 1), &s_fail)) {
          atomicExch(err, 11);
          s_fail = 1;
          break;
        }
        const int t = c / nkc, kc = c - t * nkc;
        unsigned char* a_blk = base + st * kTcStageBytes;
        const uint32_t full = smem_u32(&s_full[st]);
        mbar_expect_tx(full, (uint32_t)kTcStageBytes);
        tma_load_2d(smem_u32(a_blk), &tmQ, kc * kTcKc, q0, full);
        tma_load_2d(smem_u32(a_blk + kTcM * 128), &tmC, kc * kTcKc, t * kTcN, full);
      }
      s_issued = c;
    }
  } else if (warp == kFtMmaWarp) {
    if (lane == 0) {
      int c = 0;
      bool ok = true;
      for (int t = 0; t < n_chunks && ok; ++t) {
        const int b = t & 1;
        if (t >= 2 && !mbar_wait_or_fail(smem_u32(&s_acce[b]), (uint32_t)(((t >> 1) - 1) & 1), &s_fail)) {
          ok = false;
          atomicExch(err, 12);
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc = tmem + (uint32_t)(b * kTcN);
        for (int kc = 0; kc < nkc; ++kc, ++c) {
          const int st = c % kFtStages;
          if (!mbar_wait_or_fail(smem_u32(&s_full[st]), (uint32_t)((c / kFtStages) & 1), &s_fail)) {
            ok = false;
            atomicExch(err, 13);
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_addr = smem_u32(base + st * kTcStageBytes), b_addr = a_addr + kTcM * 128;
#pragma unroll
          for (int ks = 0; ks < kTcKc / 8; ++ks)
            tc_mma(acc, sw128_desc(a_addr + ks * 32), sw128_desc(b_addr + ks * 32), kTcIdesc,
                   (kc > 0 || ks > 0) ? 1u : 0u);
          tc_commit(smem_u32(&s_empty[st]));
        }
        if (ok) tc_commit(smem_u32(&s_accf[b]));
      }
      s_consumed = c;
      if (!ok) s_fail = 1;
    }
  } else {
    // epilogue: thread r of warps 0-3 owns query row r
    const int row = warp * 32 + lane;
    const int64_t q = (int64_t)q0 + row;
    const bool active = q < nq;
    unsigned long long* rb = rowbuf + ((size_t)blockIdx.x * kTcM + row) * cap;
    // thr: the m-th smallest key kept so far (kEmptyKey: none yet); thr_s its score.  A column
    // is appended when its score is <= thr_s: that keeps every key below thr, and the ties
    // above it only add keys a later cut removes.
    unsigned long long thr = kEmptyKey;
    float thr_s = __int_as_float(0x7f800000);
    int cnt = 0;
    bool cut = false;
    for (int t = 0; t < n_chunks; ++t) {
      const int b = t & 1, n0 = t * kTcN;
      // stage |c|^2 of the chunk (two buffers: a buffer is rewritten two chunks later, after every
      // epilogue thread has passed the next chunk's barrier)
      for (int i = row; i < kTcN; i += 128) cn2s[b * kTcN + i] = n0 + i < K ? __ldg(cn2 + n0 + i) : 0.0f;
      if (lane == 0) {
        const bool okw = mbar_wait_or_fail(smem_u32(&s_accf[b]), (uint32_t)((t >> 1) & 1), &s_fail);
        s_ok[b][warp] = okw ? 1 : 0;
        if (!okw) atomicExch(err, 14);
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      // every epilogue warp takes the same decision (a lone warp leaving would strand the others
      // at the next named barrier); s_ok[b] is rewritten two chunks later, after the next barrier
      if (!(s_ok[b][0] && s_ok[b][1] && s_ok[b][2] && s_ok[b][3])) {
        s_fail = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const float* cs = cn2s + b * kTcN;
#pragma unroll 1
      for (int j = 0; j < kTcN / 32; ++j) {
        float v[32];
        tc_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(b * kTcN + 32 * j), v);
        // score = |c|^2 - 2 acc, one rounding (2 acc is exact): the arithmetic of coarse_tc_kernel
        const int cb = n0 + 32 * j;
        unsigned pm = 0u;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v[i] = __fmaf_rn(-2.0f, v[i], cs[32 * j + i]);
          pm |= (v[i] <= thr_s ? 1u : 0u) << i;
        }
        if (!active || cb >= K) pm = 0u;
        else if (cb + 32 > K) pm &= (1u << (K - cb)) - 1u;
        // append the passing columns: only the columns some lane of the warp passes are visited
        unsigned any = __reduce_or_sync(0xffffffffu, pm);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (any & (1u << i)) {
            if ((pm >> i) & 1u) rb[cnt++] = make_key(v[i], (uint32_t)(cb + i));
          }
        }
        unsigned full = __ballot_sync(0xffffffffu, cnt > cap - 32);
        while (full) {  // cut each full row of the warp to its m smallest keys
          const int L = __ffs(full) - 1;
          full &= full - 1;
          const int n = __shfl_sync(0xffffffffu, cnt, L);
          unsigned long long* lb = rowbuf + ((size_t)blockIdx.x * kTcM + warp * 32 + L) * cap;
          const unsigned long long kth = warp_sort_keys<KPL>(lb, n, m, m, lane);
          if (lane == L) {
            thr = kth;
            thr_s = from_ordered_bits((uint32_t)(kth >> 32));
            cnt = m;
            cut = true;
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s_acce[b]));
    }
    if (!s_fail) {
      // final cut to m, then the p-th smallest of the m (not compacted)
      // final: each row sorted, its m smallest kept (ascending); the p-th and m-th scores
      unsigned act = __ballot_sync(0xffffffffu, active);
      while (act) {
        const int L = __ffs(act) - 1;
        act &= act - 1;
        const int n = __shfl_sync(0xffffffffu, cnt, L);
        unsigned long long* lb = rowbuf + ((size_t)blockIdx.x * kTcM + warp * 32 + L) * cap;
        const int64_t qL = (int64_t)q0 + warp * 32 + L;
        warp_sort_keys<KPL>(lb, n, m, m, lane);
        __syncwarp();
        const int kept = n < m ? n : m;
        for (int i = lane; i < m; i += 32) cand[qL * m + i] = i < kept ? (int32_t)(lb[i] & 0xFFFFFFFFu) : -1;
        // the m-th smallest key: when more than m columns were ever kept (cut or n > m) the row
        // dropped columns above it; a row that saw every column keeps +inf
        const bool cutL = (__shfl_sync(0xffffffffu, (int)cut, L) != 0) || n > m;
        const unsigned long long km = n >= m ? lb[m - 1] : kEmptyKey;
        if (lane == 0)
          bounds[qL] = make_float2(0.0f, cutL ? from_ordered_bits((uint32_t)(km >> 32)) : __int_as_float(0x7f800000));
      }
    }
  }
  __syncthreads();
  // On failure: wait (bounded) for the copies and MMAs still in flight, then free TMEM.
  if (s_fail && tid == kFtProducerWarp * 32) {
    for (int c = s_consumed; c < s_issued; ++c)
      mbar_wait(smem_u32(&s_full[c % kFtStages]), (uint32_t)((c / kFtStages) & 1));
    if (s_consumed > 0) {
      const int last = s_consumed - 1;
      mbar_wait(smem_u32(&s_empty[last % kFtStages]), (uint32_t)((last / kFtStages) & 1));
    }
  }
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(2 * kTcN)));
  }
}

// ---------------------------------------------------------------------------------------
// List scan on the tensor cores.  One CTA (256 threads) per work item: up to 128 queries
// probing one list (the accumulator's 128 rows = TMEM lanes) against all of the list's vectors,
// in tiles of N vectors (accumulator columns; N = 128, or 64 above 512 padded dims).  Operands
// are int8 in shared memory, K-major with the 128-byte swizzle, one 128-byte chunk of dimensions
// per [rows x 128 B] region: A holds the queries' codes (copied once), B a tile's code bits
// expanded to bytes 0 / 1.  The tiles are pipelined with one block barrier each: in step t every
// thread expands tile t + 1 into the other B buffer (from code words it loaded during step t - 1)
// and issues the loads of tile t + 2; after the barrier one thread issues tile t + 1's kind::i8
// MMAs into the other TMEM accumulator, and every thread waits for tile t's MMAs and reads its
// accumulator (warp w: TMEM lanes 32 (w % 4).., column half w / 4), forms the estimate and its
// lower bound from the integer exactly as the popcount scan does, and appends admitted vectors
// (low < tau0[q]) to their query's candidate row.  Column data (factors, slot) is kept for three
// tiles, so the single barrier separates every writer from its readers.  Every mbarrier wait is
// bounded; on time-out the kernel records an error code, stops, waits (bounded) for the MMAs it
// issued, frees its TMEM and returns.
// ---------------------------------------------------------------------------------------
constexpr int kLsM = kListScanRows;  // queries per work item
constexpr int kLsThreads = 256;
constexpr int kLsMaxChunks = 6;      // padded dimension <= 768

// kind::i8: D s32 (2), A s8 (1), B s8 (1), both K-major, N, M = 128.
template <int N>
constexpr uint32_t ls_idesc()
{
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kLsM >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_i8(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t acc)
{
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(dtmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void tc_ld32_u(uint32_t taddr, uint32_t (&r)[32])
{
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The 32 code bits of one word (dim 32w + j -> bit 31 - j) as 32 bytes 0 / 1, byte j = dim 32w + j:
// after the bit reversal bit j is dim j, and a multiply spreads each nibble's 4 bits into the low
// bits of 4 bytes (the products do not overlap, so nothing carries).
__device__ __forceinline__ void expand_word(uint32_t c, uint32_t (&o)[8])
{
  const uint32_t r = __brev(c);
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = (((r >> (4 * i)) & 0xFu) * 0x00204081u) & 0x01010101u;
}

template <int N>
__global__ void __launch_bounds__(kLsThreads, N == 128 ? 2 : 1) list_scan_tc_kernel(const ListScanArgs a)
{
  constexpr int kWpt = N * 24 / kLsThreads;  // code words per thread per tile (W <= 24)
  extern __shared__ __align__(16) unsigned char ls_smem_raw[];
  // 1024-byte aligned by an offset from the shared array itself, so that every access through
  // these pointers stays a shared-memory access
  unsigned char* base = ls_smem_raw + ((1024u - (smem_u32(ls_smem_raw) & 1023u)) & 1023u);
  const int Kc = (a.Dp + 127) >> 7;
  unsigned char* As = base;                           // [Kc][kLsM rows][128 B]
  unsigned char* Bs0 = base + Kc * kLsM * 128;        // [2][Kc][N rows][128 B]
  const int b_stride = Kc * N * 128;
  __shared__ int s_q[kLsM];
  __shared__ float s_g[kLsM], s_sg[kLsM], s_dl[kLsM], s_k1[kLsM], s_tau[kLsM];
  __shared__ float4 s_col[3][N];  // per tile column: f_add, f_rescale, f_err, slot bits
  __shared__ __align__(8) unsigned long long s_bar[2];
  __shared__ uint32_t s_tmem;
  __shared__ int s_fail, s_l, s_p0, s_rows;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {  // work item -> list (the last list whose first item is <= blockIdx.x), pairs
    const int b = blockIdx.x;
    int l = -1;
    if (b < a.item_start[a.K]) {
      int lo = 0, hi = a.K - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.item_start[mid] <= b)
          lo = mid;
        else
          hi = mid - 1;
      }
      l = lo;
      const int p0 = a.list_start[l] + (b - a.item_start[l]) * kLsM;
      s_p0 = p0;
      s_rows = min(kLsM, a.list_start[l + 1] - p0);
    }
    s_l = l;
  }
  __syncthreads();
  const int l = s_l;
  if (l < 0) return;
  const int rows = s_rows, p0 = s_p0;
  const int64_t lb = a.list_off[l];
  const int nl = (int)(a.list_off[l + 1] - lb);
  const int W = a.W;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"((uint32_t)(2 * N)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(smem_u32(&s_bar[0]), 1);
    mbar_init(smem_u32(&s_bar[1]), 1);
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int r = tid; r < kLsM; r += kLsThreads) {
    if (r < rows) {
      const int q = a.pair_q[p0 + r];
      const float g = a.pair_g[p0 + r];
      s_q[r] = q;
      s_g[r] = g;
      s_sg[r] = sqrtf(g);
      s_dl[r] = a.delta[q];
      s_k1[r] = a.k1[q];
      s_tau[r] = a.tau0[q];
    } else {
      s_q[r] = 0;
      s_g[r] = s_sg[r] = s_dl[r] = s_k1[r] = 0.0f;
      s_tau[r] = -__int_as_float(0x7f800000);  // admits nothing
    }
  }
  __syncthreads();
  // A: the queries' codes; rows past `rows` and bytes past Dp are zero.
  for (int i = tid; i < kLsM * Kc * 8; i += kLsThreads) {
    const int r = i / (Kc * 8), u = i - r * (Kc * 8);
    const int byte = u << 4;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < rows && byte < a.Dp) v = __ldg(reinterpret_cast<const uint4*>(a.qcodes + (size_t)s_q[r] * a.Dp + byte));
    *reinterpret_cast<uint4*>(As + (u >> 3) * (kLsM * 128) + r * 128 + (((u & 7) ^ (r & 7)) << 4)) = v;
  }
  // B: the padding past Dp in the last chunk stays zero in both buffers.
  if (a.Dp < Kc * 128)
    for (int i = tid; i < 2 * N * 8; i += kLsThreads) {
      const int bb = i / (N * 8), v = (i >> 3) % N, u = i & 7;
      if ((Kc - 1) * 128 + (u << 4) >= a.Dp)
        *reinterpret_cast<uint4*>(Bs0 + bb * b_stride + (Kc - 1) * (N * 128) + v * 128 + ((u ^ (v & 7)) << 4)) =
            make_uint4(0u, 0u, 0u, 0u);
    }
  const int ntiles = (nl + N - 1) / N;
  // i / W for i < N * 24 as a multiply-high by ceil(2^32 / W) (exact in that range)
  const unsigned long long w_magic = (0xFFFFFFFFull + (unsigned)W) / (unsigned)W;
  auto div_w = [&](int i) { return (int)(((unsigned long long)(unsigned)i * w_magic) >> 32); };
  uint32_t cw[kWpt];
  float cf0 = 0.0f, cf1 = 0.0f, cf2 = 0.0f;  // column data of the tile being loaded (threads < N)
  auto load_codes = [&](int t) {  // code words and column data of tile t into registers
    const int t0 = t * N;
#pragma unroll
    for (int j = 0; j < kWpt; ++j) {
      const int i = tid + j * kLsThreads;
      cw[j] = (i < N * W && t0 + div_w(i) < nl) ? __ldg(a.codes + (lb + t0) * W + i) : 0u;
    }
    if (tid < N && t0 + tid < nl) {
      const int64_t slot = lb + t0 + tid;
      cf0 = __ldg(a.fadd + slot);
      cf1 = __ldg(a.frescale + slot);
      cf2 = __ldg(a.ferr + slot);
    }
  };
  auto store_tile = [&](int t) {  // expand tile t into B[t % 2], its column data into s_col[t % 3]
    unsigned char* Bs = Bs0 + (t & 1) * b_stride;
    const int t0 = t * N;
#pragma unroll
    for (int j = 0; j < kWpt; ++j) {
      const int i = tid + j * kLsThreads;
      if (i < N * W) {
        const int v = div_w(i), w = i - v * W;
        uint32_t o[8];
        expand_word(cw[j], o);
        const int byte = w << 5, u0 = (byte & 127) >> 4;
        unsigned char* rowp = Bs + (byte >> 7) * (N * 128) + v * 128;
        // words of odd 128-byte chunks store their second unit first: the 8 threads of a
        // quarter warp then cover 8 different 16-byte units (all 32 banks) in each store
        const int sw = (w >> 2) & 1;
        const uint4 lo = make_uint4(o[0], o[1], o[2], o[3]), hi = make_uint4(o[4], o[5], o[6], o[7]);
        *reinterpret_cast<uint4*>(rowp + (((u0 + sw) ^ (v & 7)) << 4)) = sw ? hi : lo;
        *reinterpret_cast<uint4*>(rowp + (((u0 + 1 - sw) ^ (v & 7)) << 4)) = sw ? lo : hi;
      }
    }
    if (tid < N && t0 + tid < nl)
      s_col[t % 3][tid] = make_float4(cf0, cf1, cf2, __uint_as_float((uint32_t)(lb + t0 + tid)));
  };
  auto issue = [&](int t) {  // thread 0: tile t's MMAs into accumulator t % 2, committed to s_bar[t % 2]
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t a_addr = smem_u32(As), b_addr = smem_u32(Bs0 + (t & 1) * b_stride);
    const uint32_t d = s_tmem + (uint32_t)((t & 1) * N);
    for (int c = 0; c < Kc; ++c)
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)  // 32 int8 values (32 bytes) per MMA
        tc_mma_i8(d, sw128_desc(a_addr + c * (kLsM * 128) + ks * 32), sw128_desc(b_addr + c * (N * 128) + ks * 32),
                  ls_idesc<N>(), (c > 0 || ks > 0) ? 1u : 0u);
    tc_commit(smem_u32(&s_bar[t & 1]));
  };
  static_assert(N <= kLsThreads, "one column per thread");
  if (ntiles > 0) {
    load_codes(0);
    store_tile(0);
    if (ntiles > 1) load_codes(1);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy stores -> MMA reads
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem;
  if (tid == 0 && ntiles > 0) issue(0);
  const int quarter = warp & 3, half = warp >> 2;
  const int row = quarter * 32 + lane;
  const bool row_ok = row < rows;
  const int q = s_q[row];
  const float g = s_g[row], sg = s_sg[row], dl = s_dl[row], kk = s_k1[row], tau = s_tau[row];
  const unsigned long long gbits = (unsigned long long)__float_as_uint(g) << 32;
  unsigned long long n_admit = 0;
  int issued = ntiles > 0 ? 1 : 0;
  for (int t = 0; t < ntiles; ++t) {
    if (t + 1 < ntiles) {
      store_tile(t + 1);  // B[(t+1) % 2] was read by tile t - 1's MMAs, which every thread waited for
      if (t + 2 < ntiles) load_codes(t + 2);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (s_fail) break;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (tid == 0 && t + 1 < ntiles) {
      issue(t + 1);  // accumulator (t+1) % 2 was last read in step t - 1, before this barrier
      ++issued;
    }
    if (!mbar_wait(smem_u32(&s_bar[t & 1]), (uint32_t)((t >> 1) & 1))) {
      s_fail = 1;
      atomicExch(a.err, 4);
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int tn = min(N, nl - t * N);
    const float4* col = s_col[t % 3];
#pragma unroll 1
    for (int j = 0; j < N / 64; ++j) {
      const int col0 = half * (N / 2) + j * 32;
      uint32_t acc[32];
      tc_ld32_u(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)((t & 1) * N + col0), acc);
      if (row_ok && col0 < tn) {
        // admission of the 32 columns as a bit mask (no branch per pair); the few admitted
        // vectors are appended afterwards
        uint32_t adm = 0u;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float4 c = col[col0 + i];
          const float ip = __fmul_rn((float)(int32_t)acc[i], dl);
          const float base_d = __fadd_rn(c.x, g);
          const float est = __fadd_rn(base_d, __fmul_rn(c.y, __fadd_rn(ip, kk)));
          const float low = __fsub_rn(est, __fmul_rn(c.z, sg));
          adm |= (low < tau ? 1u : 0u) << i;
        }
        if (tn - col0 < 32) adm &= (1u << (tn - col0)) - 1u;  // columns past the list
        while (adm) {
          const int i = __ffs((int)adm) - 1;
          adm &= adm - 1u;
          ++n_admit;
          const int pos = atomicAdd(a.cand_cnt + q, 1);
          if (pos < a.cap) a.cand[(size_t)q * a.cap + pos] = gbits | __float_as_uint(col[col0 + i].w);
        }
      }
    }
  }
  // on failure: wait (bounded) for the last MMAs issued before freeing the accumulators
  __syncthreads();
  if (s_fail && tid == 0 && issued > 0) mbar_wait(smem_u32(&s_bar[(issued - 1) & 1]), (uint32_t)(((issued - 1) >> 1) & 1));
  if (a.stats) {
    unsigned long long s1 = n_admit;
    for (int off = 16; off; off >>= 1) s1 += __shfl_xor_sync(0xffffffffu, s1, off);
    if (lane == 0 && s1) atomicAdd(a.stats + 1, s1);
    if (tid == 0) atomicAdd(a.stats + 0, (unsigned long long)rows * (unsigned long long)nl);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)(2 * N)));
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

// Candidate keys per row the fused shortlist keeps: room for m keys, as many new ones and one
// 32-column group, rounded to the warp (a cut sorts the row's keys in registers, cap / 32 per
// lane).  Twice that buffer halved the cuts but cost more in appends and larger sorts.
int coarse_topm_row_cap(int m) { return (2 * m + 64 + 31) / 32 * 32; }
constexpr int kFtMaxCap = 32 * 32;  // m <= 480

void launch_coarse_topm_tc(const float* A, int64_t nq, const float* C, const float* cn2, int K, int dp, int m, int p,
                           unsigned long long* rowbuf, int32_t* cand, float2* bounds, int* err, cudaStream_t s)
{
  if (nq <= 0) return;
  RBQ_CHECK(coarse_tc_supported(dp), RBQ_ERR_INVALID, "coarse (tensor cores): padded dim must be a multiple of 32");
  RBQ_CHECK(nq <= 0x7fffffff && K >= 1 && m >= 1 && m <= K && p >= 1 && p <= m, RBQ_ERR_INVALID,
            "coarse (fused shortlist): bad sizes");
  const int cap = coarse_topm_row_cap(m);
  RBQ_CHECK(cap <= kFtMaxCap, RBQ_ERR_INVALID, "coarse (fused shortlist): shortlist too long");
  const size_t smem = (size_t)kFtStages * kTcStageBytes + (size_t)2 * kTcN * 4 + 1024;
  const CUtensorMap tmQ = row_major_map(A, nq, dp, kTcM);
  const CUtensorMap tmC = row_major_map(C, K, dp, kTcN);
  const unsigned grid = (unsigned)ceil_div(nq, kTcM);
#define RBQ_FT_LAUNCH(KPL)                                                                                        \
  {                                                                                                               \
    RBQ_CUDA(cudaFuncSetAttribute(coarse_topm_tc_kernel<KPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,       \
                                  (int)smem));                                                                    \
    coarse_topm_tc_kernel<KPL><<<grid, kFtThreads, smem, s>>>(tmQ, tmC, (int)nq, cn2, K, dp, m, p, cap, rowbuf,  \
                                                             cand, bounds, err);                                  \
  }
  if (cap <= 8 * 32)
    RBQ_FT_LAUNCH(8)
  else if (cap <= 16 * 32)
    RBQ_FT_LAUNCH(16)
  else
    RBQ_FT_LAUNCH(32)
#undef RBQ_FT_LAUNCH
  RBQ_LAUNCHED();
}

int coarse_topm_max_shortlist() { return (kFtMaxCap - 64) / 2; }

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

bool list_scan_tc_supported(int dp) { return dp % 32 == 0 && dp >= 32 && dp <= kLsMaxChunks * 128; }

template <int N>
static void launch_list_scan_tc_n(const ListScanArgs& a, int64_t max_items, cudaStream_t s)
{
  const int Kc = (a.Dp + 127) / 128;
  // A, two B buffers; at least a quarter of the shared memory per CTA, so that at most two CTAs
  // (2 x 2N <= 512 TMEM columns) share an SM
  const size_t smem = std::max<size_t>((size_t)Kc * (kLsM + 2 * N) * 128 + 1024, 80 * 1024);
  RBQ_CUDA(cudaFuncSetAttribute(list_scan_tc_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  list_scan_tc_kernel<N><<<(unsigned)max_items, kLsThreads, smem, s>>>(a);
  RBQ_LAUNCHED();
}

void launch_list_scan_tc(const ListScanArgs& a, int64_t max_items, cudaStream_t s)
{
  if (max_items <= 0) return;
  RBQ_CHECK(list_scan_tc_supported(a.Dp), RBQ_ERR_INVALID, "list scan: padded dim must be a multiple of 32, <= 768");
  RBQ_CHECK(max_items <= 0x7fffffff, RBQ_ERR_INVALID, "list scan: too many work items");
  if (a.Dp <= 512)
    launch_list_scan_tc_n<128>(a, max_items, s);
  else
    launch_list_scan_tc_n<64>(a, max_items, s);
}

}  // namespace rbq
