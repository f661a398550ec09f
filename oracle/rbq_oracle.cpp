// rbq_oracle.cpp -- CPU oracle for the IVF-RaBitQ retrieval hot path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker, never the product: only tests/,
// __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs load it.
// The product path (neurosamble_b200) never links, imports or calls anything here.
//
// It restates, statement for statement where the reference is deterministic, the
// reference's 1-bit IVF-RaBitQ build and QUANT4 search (vendored cuVS fork, paths relative
// to third-party/cuvs_rabitq/cpp/src/neighbors/ivf_rabitq/):
//   * residual / sign / pack / factors   gpu_index/quantizer_gpu.cu:109-172, 251-338
//   * query scaling constant t4           gpu_index/quantizer_gpu.cu:887-980
//   * 4-bit query quantisation + planes   gpu_index/searcher_gpu_quantize_query.cu:655-793
//   * popcount estimator + error prune    gpu_index/searcher_gpu_quantize_query.cu:233-281
//   * exact 1-bit distance of survivors   gpu_index/searcher_gpu_quantize_query.cu:540-604
//   * k1xSumq                             gpu_index/ivf_gpu.cu:1451-1490
//   * coarse distance + top-nprobe        gpu_index/ivf_gpu.cu:1526-1628
//   * rotation X_rot = X * P (row-major)  gpu_index/rotator_gpu.cu:162-176
// Where the reference is nondeterministic or sits behind RAFT/cuSOLVER (Philox normal
// generator, QR, reduction trees, atomicMin threshold, atomic in-list order) this file
// follows the fixed-order schedule that the CUDA library implements too, so the two agree
// bit for bit on codes, factors, popcount sums, estimates and ids:
//   * every reduction is a double accumulation in index order, rounded to float once;
//   * the prune threshold only tightens at tile boundaries (tile = TILE vectors), when the
//     per-query candidate buffer passes CAP - TILE entries, reaches 2R, or reaches R while
//     the threshold is still +inf; a pruning slice that starts with no threshold and no
//     candidates takes the R-th smallest upper bound est + f_err * sqrt(g) over its leading
//     whole lists holding at least R vectors;
//   * candidates are ordered by the 64-bit key (order-preserving float bits << 32 | id).
// Parity with the reference itself is UNPINNED at those boundaries (the reference ships no
// golden vectors and cannot be built here); the known-answer tests in tests/ pin the
// formulas instead.
//
// Build: oracle/Makefile (g++ -O3 -fopenmp -ffp-contract=off); ctypes wrapper oracle/oracle.py.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <queue>
#include <utility>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// ---------------------------------------------------------------------------------------
// Philox-4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11), restated from the published spec.
// ---------------------------------------------------------------------------------------
inline void philox4x32_10(const uint32_t key_in[2], const uint32_t ctr_in[4], uint32_t out[4])
{
  uint32_t k0 = key_in[0], k1 = key_in[1];
  uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c0;
    uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
    uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    uint32_t n0 = hi1 ^ c1 ^ k0;
    uint32_t n2 = hi0 ^ c3 ^ k1;
    c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
    k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

// Standard normal number `i` of stream `stream` under `seed` (Box-Muller in double).
inline double gaussian_at(uint64_t seed, uint32_t stream, uint64_t i)
{
  uint64_t blk = i >> 1;
  uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  uint32_t ctr[4] = {(uint32_t)blk, (uint32_t)(blk >> 32), stream, 0x52425142u};
  uint32_t r[4];
  philox4x32_10(key, ctr, r);
  const double inv53 = 1.0 / 9007199254740992.0;
  double u1 = ((double)(((uint64_t)r[0] << 21) ^ (r[1] >> 11)) + 0.5) * inv53;
  double u2 = ((double)(((uint64_t)r[2] << 21) ^ (r[3] >> 11)) + 0.5) * inv53;
  double rad = std::sqrt(-2.0 * std::log(u1));
  double th = 6.283185307179586 * u2;
  return (i & 1) ? rad * std::sin(th) : rad * std::cos(th);
}

inline uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// Order-preserving map float -> uint32 (ascending floats give ascending keys).
inline uint32_t ordered_bits(float f)
{
  uint32_t u = f2u(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
inline float from_ordered_bits(uint32_t o)
{
  return (o & 0x80000000u) ? u2f(o & 0x7FFFFFFFu) : u2f(~o);
}
inline uint64_t make_key(float d, uint32_t id) { return ((uint64_t)ordered_bits(d) << 32) | id; }
constexpr uint64_t kEmptyKey = ~0ull;

// Rotation of one row: y[j] = float( sum_k double(x[k]) * double(P[k][j]) ), k ascending.
// x has Dp entries (zero padded).  Every product of two floats is exact in double, so the
// result does not depend on FMA contraction.
inline void rotate_row(const float* x, const float* P, int Dp, float* y, double* acc)
{
  for (int j = 0; j < Dp; ++j) acc[j] = 0.0;
  for (int k = 0; k < Dp; ++k) {
    const double xk = (double)x[k];
    const float* prow = P + (size_t)k * Dp;
    for (int j = 0; j < Dp; ++j) acc[j] += xk * (double)prow[j];
  }
  for (int j = 0; j < Dp; ++j) y[j] = (float)acc[j];
}

// kTightStart of the reference (quantizer_gpu.cu:875-885): the start fraction of the
// rescale search per extra-bit count.  A table that has to be alike.
// float, as the reference's std::array<float, 9>: t_end is multiplied by (double)0.15f.
const float kTightStart[9] = {0.0f, 0.15f, 0.20f, 0.52f, 0.59f, 0.71f, 0.75f, 0.77f, 0.81f};

// Restatement of best_rescale_factor (quantizer_gpu.cu:887-943): the scale t that maximises
// <o_bar, o> / |o_bar| over the codes o_bar = floor(t*o) (ex_bits magnitude levels).
double best_rescale(const double* o, int dim, int ex_bits)
{
  const double eps = 1e-5;
  const int n_enum = 10;
  double max_o = *std::max_element(o, o + dim);
  double t_end = (double)(((1 << ex_bits) - 1) + n_enum) / max_o;
  double t_start = t_end * kTightStart[ex_bits];
  std::vector<int> cur(dim);
  double sqr_den = (double)dim * 0.25;
  double num = 0;
  for (int i = 0; i < dim; ++i) {
    int c = (int)((t_start * o[i]) + eps);
    cur[i] = c;
    sqr_den += c * c + c;
    num += (c + 0.5) * o[i];
  }
  typedef std::pair<double, size_t> E;
  std::priority_queue<E, std::vector<E>, std::greater<E>> heap;
  for (int i = 0; i < dim; ++i) heap.emplace((double)(cur[i] + 1) / o[i], (size_t)i);
  double max_ip = 0, t = 0;
  while (!heap.empty()) {
    double ct = heap.top().first;
    size_t id = heap.top().second;
    heap.pop();
    cur[id]++;
    int u = cur[id];
    sqr_den += 2 * u;
    num += o[id];
    double ip = num / std::sqrt(sqr_den);
    if (ip > max_ip) { max_ip = ip; t = ct; }
    if (u < (1 << ex_bits) - 1) {
      double tn = (double)(u + 1) / o[id];
      if (tn < t_end) heap.emplace(tn, id);
    }
  }
  return t;
}

}  // namespace

extern "C" {

int orc_version(void) { return 1; }

// Standard normals, for golden tests of the generator.
void orc_gaussian(uint64_t seed, uint32_t stream, uint64_t start, int64_t n, double* out)
{
  for (int64_t i = 0; i < n; ++i) out[i] = gaussian_at(seed, stream, start + (uint64_t)i);
}

void orc_philox(const uint32_t* key, const uint32_t* ctr, uint32_t* out) { philox4x32_10(key, ctr, out); }

// Seeded random orthogonal Dp x Dp matrix, row-major float (a1; replaces RAFT normal +
// cuSOLVER QR of rotator_gpu.cu:52-59).  G[i][j] = gaussian(seed, stream 1, i*Dp + j);
// Householder QR in double with index-order sums; Q's columns are multiplied by sign(R_kk)
// so the result is Haar distributed.
void orc_make_rotation(int Dp, uint64_t seed, float* P_out)
{
  const int n = Dp;
  std::vector<double> A((size_t)n * n), Q((size_t)n * n, 0.0), V((size_t)n * n, 0.0);
  std::vector<double> beta(n, 0.0), rdiag(n, 0.0);
  for (size_t i = 0; i < (size_t)n * n; ++i) A[i] = gaussian_at(seed, 1u, i);
  for (int k = 0; k < n; ++k) {
    double s = 0.0;
    for (int i = k; i < n; ++i) s += A[(size_t)i * n + k] * A[(size_t)i * n + k];
    double nrm = std::sqrt(s);
    double x0 = A[(size_t)k * n + k];
    double alpha = (x0 >= 0.0) ? -nrm : nrm;
    double* v = &V[(size_t)k * n];
    for (int i = k; i < n; ++i) v[i] = A[(size_t)i * n + k];
    v[k] = x0 - alpha;
    double vn = 0.0;
    for (int i = k; i < n; ++i) vn += v[i] * v[i];
    double b = (vn == 0.0) ? 0.0 : 2.0 / vn;
    beta[k] = b;
    for (int j = k; j < n; ++j) {
      double d = 0.0;
      for (int i = k; i < n; ++i) d += v[i] * A[(size_t)i * n + j];
      double f = b * d;
      for (int i = k; i < n; ++i) A[(size_t)i * n + j] -= f * v[i];
    }
    rdiag[k] = A[(size_t)k * n + k];
  }
  for (int i = 0; i < n; ++i) Q[(size_t)i * n + i] = 1.0;
  for (int k = n - 1; k >= 0; --k) {
    const double* v = &V[(size_t)k * n];
    double b = beta[k];
    for (int j = 0; j < n; ++j) {
      double d = 0.0;
      for (int i = k; i < n; ++i) d += v[i] * Q[(size_t)i * n + j];
      double f = b * d;
      for (int i = k; i < n; ++i) Q[(size_t)i * n + j] -= f * v[i];
    }
  }
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < n; ++j) {
      double q = Q[(size_t)i * n + j];
      if (rdiag[j] < 0.0) q = -q;
      P_out[(size_t)i * n + j] = (float)q;
    }
}

// Query scaling constant t4 (a6; restates get_const_scaling_factors(D, 3),
// quantizer_gpu.cu:947-980, with this project's generator in place of RAFT's):
// mean over 100 rows of best_rescale(|g|/|g|_2, Dp, 3), g = gaussian(seed, stream 2).
float orc_query_scale(int Dp, uint64_t seed, int ex_bits)
{
  const int rows = 100;
  std::vector<double> g(Dp), o(Dp);
  double sum = 0.0;
  for (int r = 0; r < rows; ++r) {
    double s = 0.0;
    for (int j = 0; j < Dp; ++j) {
      g[j] = gaussian_at(seed, 2u, (uint64_t)r * Dp + j);
      s += g[j] * g[j];
    }
    double nrm = std::sqrt(s);
    for (int j = 0; j < Dp; ++j) o[j] = std::fabs(g[j] / nrm);
    sum += best_rescale(o.data(), Dp, ex_bits);
  }
  return (float)(sum / rows);
}

double orc_best_rescale(const double* o, int dim, int ex_bits) { return best_rescale(o, dim, ex_bits); }

// Pad rows of X [n, D] to Dp with zeros and rotate: Y [n, Dp].
void orc_rotate(const float* X, int64_t n, int D, int Dp, const float* P, float* Y)
{
#pragma omp parallel
  {
    std::vector<float> x(Dp, 0.0f);
    std::vector<double> acc(Dp);
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      for (int j = 0; j < Dp; ++j) x[j] = (j < D) ? X[(size_t)i * D + j] : 0.0f;
      rotate_row(x.data(), P, Dp, Y + (size_t)i * Dp, acc.data());
    }
  }
}

// 1-bit code and the three factors of one rotated vector y against rotated centroid c
// (a3 + a4; quantizer_gpu.cu:109-172 and 251-338).  W = Dp/32 words, dim 32w+j -> bit 31-j.
void orc_quantize_one(const float* y, const float* c, int Dp, uint32_t* code, float* f3)
{
  double l2d = 0.0;
  for (int j = 0; j < Dp; ++j) {
    float r = y[j] - c[j];
    l2d += (double)r * (double)r;
  }
  float l2_sqr = (float)l2d;
  float norm = sqrtf(l2_sqr);
  double ipr = 0.0, ipc = 0.0;
  const int W = Dp / 32;
  for (int w = 0; w < W; ++w) code[w] = 0u;
  for (int j = 0; j < Dp; ++j) {
    float r = y[j] - c[j];
    int bit = (norm > 0.0f && r > 0.0f) ? 1 : 0;
    if (bit) code[j >> 5] |= (1u << (31 - (j & 31)));
    double xu = bit ? 0.5 : -0.5;
    ipr += (double)r * xu;
    ipc += (double)c[j] * xu;
  }
  float ip_resi = (float)ipr;
  float ip_cent = (float)ipc;
  float xu_sq = 0.25f * (float)Dp;
  if (ip_resi == 0.0f) ip_resi = INFINITY;
  float l2_norm = sqrtf(fmaxf(l2_sqr, 0.0f));
  float denom = ip_resi;
  float fadd = l2_sqr + (2.0f * l2_sqr) * (ip_cent / denom);
  float frescale = (-2.0f * l2_sqr) / denom;
  float ratio = (l2_sqr * xu_sq) / (denom * denom);
  float inner = (ratio - 1.0f) / fmaxf((float)(Dp - 1), 1.0f);
  inner = fmaxf(inner, 0.0f);
  float tmp_err = (l2_norm * 1.9f) * sqrtf(inner);
  f3[0] = fadd;
  f3[1] = frescale;
  f3[2] = 2.0f * tmp_err;
}

// ExRaBitQ extra bits (bits_per_dim = ex + 1 > 1) of one rotated vector y against rotated
// centroid c: the fast-quantize branch of quantize_batch_opt (exrabitq_fused_kernel_batch,
// quantizer_gpu.cu:347-468) on the normalised residual of subtract_normalize_binarize_Kernel
// (:109-172).  t is the data scale (construct_on_gpu, ivf_gpu.cu:629-644: the 4-bit query scale
// for ex = 3, the 8-bit one for ex = 7).  Per dim j, with r = y - c, xn = r / |r| (0 if |r| = 0):
//   e_j = min(int(t * |xn_j| + 1e-5), 2^ex - 1);   stored x_j = e_j if bit_j else 2^ex - 1 - e_j
//   (bit_j is the 1-bit code), so the whole (ex+1)-bit code u_j = bit_j * 2^ex + x_j and its
//   centred value xu_j = u_j - (2^ex - 1/2);
//   ip_norm = sum (e_j + 1/2) |xn_j|,  ip_resi = sum r_j xu_j,  ip_cent = sum c_j xu_j  (double
//   sums in dim order, rounded to float);
//   f_ex_add = |r|^2 + (2 |r|^2 ip_cent) / ip_resi  (ip_resi = 0 -> +inf);
//   f_ex_rescale = -2 |r| / ip_norm  (1 / ip_norm not finite -> 1).
// The reference sets the code's top bit from r_j >= 0 in the factors and from r_j > 0 in the
// 1-bit code; here both use bit_j, so an exactly zero residual coordinate counts the same in
// both.  planes [ex, W]: plane p word w, dim 32w+j -> bit 31-j = bit p of x_j.
void orc_quantize_ex_one(const float* y, const float* c, int Dp, int ex, float t, uint32_t* planes, float* f2)
{
  double l2d = 0.0;
  for (int j = 0; j < Dp; ++j) {
    float r = y[j] - c[j];
    l2d += (double)r * (double)r;
  }
  const float l2_sqr = (float)l2d;
  const float norm = sqrtf(l2_sqr);
  const int W = Dp / 32;
  const int mask = (1 << ex) - 1;
  const float shift = (float)(1 << ex) - 0.5f;
  for (int i = 0; i < ex * W; ++i) planes[i] = 0u;
  double ipn = 0.0, ipr = 0.0, ipc = 0.0;
  for (int j = 0; j < Dp; ++j) {
    const float r = y[j] - c[j];
    const int bit = (norm > 0.0f && r > 0.0f) ? 1 : 0;
    const float xn = norm > 0.0f ? r / norm : 0.0f;
    const float a = fabsf(xn);
    const float ta = t * a;
    int e = (int)(ta + 1e-5f);
    if (e > mask) e = mask;
    const float en = (float)e + 0.5f;
    ipn += (double)(en * a);
    const int x = bit ? e : mask - e;
    for (int b = 0; b < ex; ++b)
      if ((x >> b) & 1) planes[b * W + (j >> 5)] |= 1u << (31 - (j & 31));
    const float xu = (float)((bit << ex) | x) - shift;
    ipr += (double)r * (double)xu;
    ipc += (double)c[j] * (double)xu;
  }
  const float ip_resi = (float)ipr, ip_cent = (float)ipc, ip_norm = (float)ipn;
  const float denom = ip_resi == 0.0f ? INFINITY : ip_resi;
  const float l2_norm = sqrtf(fmaxf(l2_sqr, 0.0f));
  const float num = (2.0f * l2_sqr) * ip_cent;
  f2[0] = l2_sqr + num / denom;
  float inv = 1.0f / ip_norm;
  if (!std::isfinite(inv)) inv = 1.0f;
  f2[1] = (-2.0f * l2_norm) * inv;
}

// Extra-bit codes of n rotated rows Y [n, Dp] against the rotated centroids of their labels:
// planes [n, ex, W], f_ex_add [n], f_ex_rescale [n].
void orc_quantize_ex(const float* Y, int64_t n, int Dp, const float* c_rot, const uint32_t* labels, int ex,
                     float t, uint32_t* planes, float* fexadd, float* fexr)
{
  const int W = Dp / 32;
#pragma omp parallel for schedule(dynamic, 256)
  for (int64_t i = 0; i < n; ++i) {
    float f2[2];
    orc_quantize_ex_one(Y + (size_t)i * Dp, c_rot + (size_t)labels[i] * Dp, Dp, ex, t,
                        planes + (size_t)i * ex * W, f2);
    fexadd[i] = f2[0];
    fexr[i] = f2[1];
  }
}

// Build (a2 inputs, a3-a5): labels/centroids given.  Lists are a stable counting sort of
// the labels (ids ascending inside a list).  Outputs are in list-slot order:
//   list_off [K+1], ids [n] (global ids), codes [n*W] (vector-major), f_add/f_rescale/f_err [n],
//   c_rot [K*Dp] (rotated centroids).
void orc_build(const float* X, int64_t n, int D, int Dp, const float* P, const float* C, int K,
               const uint32_t* labels, int64_t* list_off, uint32_t* ids, uint32_t* codes,
               float* fadd, float* frescale, float* ferr, float* c_rot)
{
  const int W = Dp / 32;
  orc_rotate(C, K, D, Dp, P, c_rot);
  std::vector<int64_t> cnt(K + 1, 0);
  for (int64_t i = 0; i < n; ++i) cnt[labels[i] + 1]++;
  for (int k = 0; k < K; ++k) cnt[k + 1] += cnt[k];
  for (int k = 0; k <= K; ++k) list_off[k] = cnt[k];
  std::vector<int64_t> pos(cnt.begin(), cnt.end() - 1);
  for (int64_t i = 0; i < n; ++i) ids[pos[labels[i]]++] = (uint32_t)i;
#pragma omp parallel
  {
    std::vector<float> x(Dp, 0.0f), y(Dp);
    std::vector<double> acc(Dp);
#pragma omp for schedule(dynamic, 256)
    for (int64_t s = 0; s < n; ++s) {
      uint32_t id = ids[s];
      for (int j = 0; j < Dp; ++j) x[j] = (j < D) ? X[(size_t)id * D + j] : 0.0f;
      rotate_row(x.data(), P, Dp, y.data(), acc.data());
      float f3[3];
      orc_quantize_one(y.data(), c_rot + (size_t)labels[id] * Dp, Dp, codes + (size_t)s * W, f3);
      fadd[s] = f3[0];
      frescale[s] = f3[1];
      ferr[s] = f3[2];
    }
  }
}

// Query preparation (a8 + k1xSumq) with B = qbits-bit codes (QUANT4: B = 4 and t = t4;
// QUANT8: B = 8 and t = t8; exrabitq_quantize_query with EX_BITS = num_bits,
// searcher_gpu_quantize_query.cu:716-723, 774-791).  Input: rotated queries [nq, Dp].
// Outputs: planes [nq, B, W] (plane b word w, dim 32w+j -> bit 31-j of the B-bit two's
// complement of code_j, shifted right by b), delta [nq], k1 [nq] (= -0.5 * sum q), codes_out
// [nq, Dp] int8 (optional).
void orc_query_prep(const float* Qr, int64_t nq, int Dp, float t4, int qbits, uint32_t* planes, float* delta,
                    float* k1, int8_t* codes_out)
{
  const int W = Dp / 32;
  const int hi = (1 << (qbits - 1)) - 1, lo = -(1 << (qbits - 1));
  const uint32_t mask = (1u << qbits) - 1u;
#pragma omp parallel
  {
    std::vector<int> code(Dp);
#pragma omp for schedule(static)
    for (int64_t q = 0; q < nq; ++q) {
      const float* x = Qr + (size_t)q * Dp;
      double s2 = 0.0, s1 = 0.0;
      for (int j = 0; j < Dp; ++j) {
        s2 += (double)x[j] * (double)x[j];
        s1 += (double)x[j];
      }
      float norm = sqrtf((float)s2);
      float norm_inv = (norm > 0.0f) ? (1.0f / norm) : 0.0f;
      double ipd = 0.0;
      long long xs = 0;
      for (int j = 0; j < Dp; ++j) {
        float val = x[j] * norm_inv;
        float tv = t4 * val;
        int cv = (int)std::nearbyint(tv);  // round half to even (default FE_TONEAREST)
        if (cv > hi) cv = hi;
        if (cv < lo) cv = lo;
        code[j] = cv;
        ipd += (double)x[j] * (double)cv;
        xs += (long long)cv * cv;
      }
      float ip = (float)ipd;
      float xu_sq = (float)xs;
      float norm_quan = sqrtf(fmaxf(xu_sq, 0.0f));
      float dl;
      if (norm > 1e-6f && norm_quan > 1e-6f) {
        float cosv = ip / (norm * norm_quan);
        dl = (norm / norm_quan) * cosv;
      } else {
        dl = 0.0f;
      }
      delta[q] = dl;
      k1[q] = ((float)s1) * -0.5f;
      uint32_t* pl = planes + (size_t)q * qbits * W;
      for (int i = 0; i < qbits * W; ++i) pl[i] = 0u;
      for (int j = 0; j < Dp; ++j) {
        uint32_t u = (uint32_t)code[j] & mask;
        for (int b = 0; b < qbits; ++b)
          if ((u >> b) & 1u) pl[b * W + (j >> 5)] |= (1u << (31 - (j & 31)));
      }
      if (codes_out)
        for (int j = 0; j < Dp; ++j) codes_out[(size_t)q * Dp + j] = (int8_t)code[j];
    }
  }
}

// Squared L2 in the order of a CUDA warp: lane l (0..31) sums double(x_d - q_d)^2 over
// d = l, l+32, ... ascending; the 32 lane sums are combined by an xor butterfly (offsets
// 16, 8, 4, 2, 1: v[l] = v[l] + v[l ^ off]); lane 0's value is rounded to float.
static inline float l2_lanes(const float* x, const float* q, int D)
{
  double v[32];
  for (int l = 0; l < 32; ++l) {
    double s = 0.0;
    for (int d = l; d < D; d += 32) {
      float df = x[d] - q[d];
      s += (double)df * (double)df;
    }
    v[l] = s;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    double nv[32];
    for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ off];
    for (int l = 0; l < 32; ++l) v[l] = nv[l];
  }
  return (float)v[0];
}

// Exact coarse distance g = |q - c|^2 (rotated space) in the warp order of l2_lanes.
static inline float coarse_dist(const float* q, const float* c, int Dp) { return l2_lanes(c, q, Dp); }

// Coarse quantiser (a7): top-nprobe lists per query by (g, list id) ascending.
void orc_coarse(const float* Qr, int64_t nq, const float* Cr, int K, int Dp, int nprobe,
                int32_t* probes, float* gout)
{
#pragma omp parallel
  {
    std::vector<uint64_t> keys(K);
#pragma omp for schedule(dynamic, 16)
    for (int64_t q = 0; q < nq; ++q) {
      for (int c = 0; c < K; ++c)
        keys[c] = make_key(coarse_dist(Qr + (size_t)q * Dp, Cr + (size_t)c * Dp, Dp), (uint32_t)c);
      std::partial_sort(keys.begin(), keys.begin() + nprobe, keys.end());
      for (int p = 0; p < nprobe; ++p) {
        probes[q * nprobe + p] = (int32_t)(keys[p] & 0xFFFFFFFFu);
        gout[q * nprobe + p] = from_ordered_bits((uint32_t)(keys[p] >> 32));
      }
    }
  }
}

// Signed B-bit x 1-bit popcount inner product of one vector (a10 phase 1,
// searcher_gpu_quantize_query.cu:253-262 with NumBits = B = qbits):
// sum_w sum_{b<B-1} popc(P_b & c) << b - popc(P_{B-1} & c) << (B-1).
int32_t orc_popcount_ip(const uint32_t* planes, const uint32_t* code, int W, int qbits)
{
  int32_t acc = 0;
  for (int w = 0; w < W; ++w) {
    uint32_t c = code[w];
    for (int b = 0; b < qbits - 1; ++b) acc += __builtin_popcount(planes[b * W + w] & c) << b;
    acc -= __builtin_popcount(planes[(qbits - 1) * W + w] & c) << (qbits - 1);
  }
  return acc;
}

// Estimator of one vector (a10 phase 1, searcher_gpu_quantize_query.cu:264-266):
// est = (f_add + g) + f_rescale * (acc * delta + k1);  low = est - f_err * sqrt(g).
void orc_estimate(const float* f3, float g, int32_t acc, float delta, float k1, float* est_low)
{
  float base_d = f3[0] + g;
  float ip = (float)acc * delta;
  float est = base_d + f3[1] * (ip + k1);
  est_low[0] = est;
  est_low[1] = est - f3[2] * sqrtf(g);
}

// Sum of q over the set bits of code byte j (byte j of the MSB-first bit stream = dims
// 8j .. 8j+7, bit 7 first), a float sum starting from 0.
static inline float byte_sum(const float* q, const uint32_t* code, int j)
{
  const uint32_t byte = (code[j >> 2] >> (24 - 8 * (j & 3))) & 0xFFu;
  float s = 0.0f;
  for (int jj = 0; jj < 8; ++jj)
    if ((byte >> (7 - jj)) & 1u) s = s + q[8 * j + jj];
  return s;
}

// Exact 1-bit inner product <bits, q> in the order of the CUDA scan's warp: lane l (0..31)
// adds byte_sum(j) for j = l, l+32, ... (< 4W) in order from 0; the 32 lane values are
// combined by an xor butterfly (16, 8, 4, 2, 1: v[l] = v[l] + v[l ^ off]); lane 0's value.
float orc_exact_ip(const float* q, const uint32_t* code, int W)
{
  const int NB = 4 * W;
  float v[32];
  for (int l = 0; l < 32; ++l) {
    float s = 0.0f;
    for (int j = l; j < NB; j += 32) s = s + byte_sum(q, code, j);
    v[l] = s;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    float nv[32];
    for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ off];
    for (int l = 0; l < 32; ++l) v[l] = nv[l];
  }
  return v[0];
}

// <x, q> of a vector's extra-bit code x (planes [ex, W]) in the order of the CUDA scan's warp:
// lane l takes code bytes j = l, l+32, ... (< 4W); per byte, planes p = ex-1 down to 0 add
// 2^p * byte_sum(plane p, j) to the lane's value; xor butterfly; lane 0's value.  The extra-bit
// distance of the scan (the WithEx branch, searcher_gpu_quantize_query.cu:405-473):
//   d = (f_ex_add + g) + f_ex_rescale * ((2^ex * ip + ip_x) + kb),  kb = k1 * (2^(ex+1) - 1)
// with ip the vector's 1-bit inner product (exact, or the table one in the LUT modes) and
// kb = -(2^(ex+1) - 1)/2 * sum q (computeQueryFactorsWarpKernel, ivf_gpu.cu:1450-1490).
float orc_ex_ip(const float* q, const uint32_t* planes, int W, int ex)
{
  const int NB = 4 * W;
  float v[32];
  for (int l = 0; l < 32; ++l) {
    float s = 0.0f;
    for (int j = l; j < NB; j += 32)
      for (int p = ex - 1; p >= 0; --p) s = s + (float)(1 << p) * byte_sum(q, planes + (size_t)p * W, j);
    v[l] = s;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    float nv[32];
    for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ off];
    for (int l = 0; l < 32; ++l) v[l] = nv[l];
  }
  return v[0];
}

static inline float ex_distance(float fexadd, float fexr, float g, float ip, float ipx, int ex, float k1)
{
  const float kb = k1 * (float)((2 << ex) - 1);
  const float T = ((float)(1 << ex) * ip + ipx) + kb;
  return (fexadd + g) + fexr * T;
}

// fp32 -> IEEE binary16, round to nearest, ties to even (the rounding of CUDA's __float2half),
// and back (exact).  Written from the IEEE 754 encodings.
static uint16_t float_to_half_rn(float f)
{
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ex = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (ex == 0xFFu) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u | (man >> 13) : 0u));  // inf / nan
  const int e = (int)ex - 127 + 15;  // half exponent
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);  // overflow -> inf
  if (e <= 0) {  // half subnormal or zero
    if (e < -10) return (uint16_t)sign;  // rounds to zero
    man |= 0x800000u;  // implicit bit
    const int shift = 14 - e;  // bits dropped: 13 + (1 - e)
    const uint32_t half_man = man >> shift;
    const uint32_t rem = man & ((1u << shift) - 1u), halfway = 1u << (shift - 1);
    uint32_t r = half_man;
    if (rem > halfway || (rem == halfway && (half_man & 1u))) ++r;
    return (uint16_t)(sign | r);  // a carry into the exponent field gives the smallest normal: correct
  }
  uint32_t r = ((uint32_t)e << 10) | (man >> 13);
  const uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;  // a carry may reach the exponent / inf: correct
  return (uint16_t)(sign | r);
}

static float half_to_float(uint16_t h)
{
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t ex = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t x;
  if (ex == 0) {
    if (man == 0) {
      x = sign;
    } else {  // subnormal: normalise
      int e = -1;
      do {
        man <<= 1;
        ++e;
      } while (!(man & 0x400u));
      x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (ex == 0x1Fu) {
    x = sign | 0x7F800000u | (man << 13);
  } else {
    x = sign | ((ex - 15 + 127) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

// LUT16 / LUT32 query tables (precomputeAllLUTs and precomputeAllLUTs_fp16_simple,
// searcher_gpu.cu:65-108 and searcher_gpu_shared_mem_opt.cu:520-549): for chunk c (dims
// 4c..4c+3) and 4-bit pattern p, the fp32 sum from 0, in dimension order, of q[4c + b] over the b
// with bit 3-b of p set; LUT16 stores it rounded to fp16.  Returned as floats.
static void lut_tables(const float* qr, int Dp, bool half, std::vector<float>& lut)
{
  const int chunks = Dp / 4;
  lut.assign((size_t)chunks * 16, 0.0f);
  for (int c = 0; c < chunks; ++c)
    for (int p = 0; p < 16; ++p) {
      float sum = 0.0f;
      for (int b = 0; b < 4; ++b)
        if (p & (1 << (3 - b))) sum += qr[4 * c + b];
      lut[(size_t)c * 16 + p] = half ? half_to_float(float_to_half_rn(sum)) : sum;
    }
}

// <bits, q> by the tables: words in order, nibbles from the top (bit 31) down, added one by one
// (computeInnerProductsWithLUT16Opt, searcher_gpu_shared_mem_opt.cu:165-177).
static float lut_ip(const std::vector<float>& lut, const uint32_t* code, int W)
{
  float ip = 0.0f;
  for (int w = 0; w < W; ++w)
    for (int ci = 0; ci < 8; ++ci) {
      const int pattern = (int)((code[w] >> (28 - 4 * ci)) & 0xFu);
      ip += lut[(size_t)(w * 8 + ci) * 16 + pattern];
    }
  return ip;
}

inline bool is_lut_mode(int qbits) { return qbits == 16 || qbits == 32; }

// The fp16 conversions on their own, for checking them against another implementation.
void orc_float_to_half(const float* x, int64_t n, uint16_t* out)
{
  for (int64_t i = 0; i < n; ++i) out[i] = float_to_half_rn(x[i]);
}
void orc_half_to_float(const uint16_t* h, int64_t n, float* out)
{
  for (int64_t i = 0; i < n; ++i) out[i] = half_to_float(h[i]);
}

struct ScanIndex {
  const int64_t* list_off;
  const uint32_t* ids;
  const uint32_t* codes;
  const float* fadd;
  const float* frescale;
  const float* ferr;
  int qbits;  // query code width (planes per query)
  // ExRaBitQ extra bits (ex = 0: 1-bit codes only): planes [n, ex, W], f_ex_add, f_ex_rescale
  const uint32_t* ex_codes;
  const float* fexadd;
  const float* fexr;
  int ex;
};

// One slice of one query's probes.  Mirrors the CUDA scan kernel's schedule exactly.
static void scan_slice(const ScanIndex& ix, int W, const float* qr, const uint32_t* pl, float delta,
                       float k1, const int32_t* probe_l, const float* probe_g, int np, float tau0,
                       const std::vector<uint64_t>& init, int R, int tile, int cap, int prune,
                       std::vector<uint64_t>& keys, int64_t* stats)
{
  // The slice starts from the candidates `init` (an earlier scan's, possibly none) and from
  // tau0, lowered to their largest distance when all R are present.
  keys.assign(init.begin(), init.end());
  float tau = tau0;
  if ((int)keys.size() == R) {
    const uint64_t kmax = *std::max_element(keys.begin(), keys.end());
    tau = std::fmin(tau, from_ordered_bits((uint32_t)(kmax >> 32)));
  }
  int64_t n_scanned = 0, n_admit = 0;
  // The slice's lists form one flat sequence of vectors (probe order, slot order inside a
  // list); tiles of `tile` vectors run across list boundaries.
  std::vector<int64_t> pre(np + 1, 0);
  for (int p = 0; p < np; ++p) pre[p + 1] = pre[p] + (ix.list_off[probe_l[p] + 1] - ix.list_off[probe_l[p]]);
  const int64_t total = pre[np];
  // Bound seed: a pruning slice with no threshold and no candidates yet starts from the R-th
  // smallest upper bound est + f_err * sqrt(g) over its leading whole lists holding >= R vectors.
  const bool lut = is_lut_mode(ix.qbits);
  std::vector<float> table;
  if (lut) lut_tables(qr, W * 32, ix.qbits == 16, table);
  if (!lut && prune && std::isinf(tau) && keys.empty() && total >= R) {
    int64_t nb = 0;
    for (int i = 1; i <= np && nb < R; ++i) nb = pre[i];
    std::vector<uint64_t> ub((size_t)nb);
    int c = 0;
    for (int64_t f = 0; f < nb; ++f) {
      while (pre[c + 1] <= f) ++c;
      const float g = probe_g[c];
      const int64_t s = ix.list_off[probe_l[c]] + (f - pre[c]);
      const int32_t acc = orc_popcount_ip(pl, ix.codes + (size_t)s * W, W, ix.qbits);
      const float ip = (float)acc * delta;
      const float base_d = ix.fadd[s] + g;
      const float est = base_d + ix.frescale[s] * (ip + k1);
      const float up = est + ix.ferr[s] * sqrtf(g);
      ub[(size_t)f] = make_key(up, (uint32_t)f);
    }
    std::nth_element(ub.begin(), ub.begin() + (R - 1), ub.end());
    tau = from_ordered_bits((uint32_t)(ub[(size_t)R - 1] >> 32));
  }
  int cur = 0;
  for (int64_t t0 = 0; t0 < total; t0 += tile) {
    const int64_t t1 = std::min<int64_t>(total, t0 + tile);
    for (int64_t f = t0; f < t1; ++f) {
      while (pre[cur + 1] <= f) ++cur;
      const float g = probe_g[cur];
      const float sqrt_g = sqrtf(g);
      const int64_t s = ix.list_off[probe_l[cur]] + (f - pre[cur]);
      const uint32_t* code = ix.codes + (size_t)s * W;
      ++n_scanned;
      if (lut) {  // LUT16 / LUT32: the table estimate is the candidate's distance
        const float ip = lut_ip(table, code, W);
        const float est = (ix.fadd[s] + g) + ix.frescale[s] * (ip + k1);
        if (ix.ex == 0) {
          if (est <= tau) {
            ++n_admit;
            keys.push_back(make_key(est, ix.ids[s]));
          }
          continue;
        }
        // with extra bits the table estimate's error bound admits, the extra-bit distance ranks
        // (searcher_gpu_shared_mem_opt.cu:303-310, 359-420)
        const float low = est - ix.ferr[s] * sqrt_g;
        if (!prune || low < tau) {
          ++n_admit;
          const float ipx = orc_ex_ip(qr, ix.ex_codes + (size_t)s * ix.ex * W, W, ix.ex);
          const float dist = ex_distance(ix.fexadd[s], ix.fexr[s], g, ip, ipx, ix.ex, k1);
          if (dist <= tau) keys.push_back(make_key(dist, ix.ids[s]));
        }
        continue;
      }
      int32_t acc = orc_popcount_ip(pl, code, W, ix.qbits);
      float ip = (float)acc * delta;
      float base_d = ix.fadd[s] + g;
      float est = base_d + ix.frescale[s] * (ip + k1);
      float low = est - ix.ferr[s] * sqrt_g;
      if (!prune || low < tau) {
        ++n_admit;
        float eip = orc_exact_ip(qr, code, W);
        float dist;
        if (ix.ex > 0) {
          const float ipx = orc_ex_ip(qr, ix.ex_codes + (size_t)s * ix.ex * W, W, ix.ex);
          dist = ex_distance(ix.fexadd[s], ix.fexr[s], g, eip, ipx, ix.ex, k1);
        } else {
          dist = base_d + ix.frescale[s] * (eip + k1);
        }
        if (dist <= tau) keys.push_back(make_key(dist, ix.ids[s]));
      }
    }
    // Tighten tau after a tile when the buffer is nearly full, when it holds 2R keys, or as soon
    // as R keys exist while tau is still open.
    const int cnt = (int)keys.size();
    if (cnt > cap - tile || cnt >= 2 * R || (cnt >= R && std::isinf(tau))) {
      std::sort(keys.begin(), keys.end());
      keys.resize(R);
      tau = from_ordered_bits((uint32_t)(keys[R - 1] >> 32));
    }
  }
  std::sort(keys.begin(), keys.end());
  if ((int)keys.size() > R) keys.resize(R);
  if (stats) {
    stats[0] += n_scanned;
    stats[1] += n_admit;
  }
}

// Bound seed per query (rbq_bound_seed): the R-th smallest upper bound over the leading whole
// owned lists of the given probes holding >= R vectors, +inf if they hold fewer.
void orc_bound_seed(const int64_t* list_off, const uint32_t* codes, const float* fadd, const float* frescale,
                    const float* ferr, int Dp, const uint32_t* planes, const float* delta, const float* k1, int64_t nq,
                    const int32_t* probes, const float* gq, int nprobe, int R, int shard_rank, int shard_count,
                    const int32_t* owner, float* tau_out, int qbits)
{
  const int W = Dp / 32;
#pragma omp parallel for schedule(dynamic, 16)
  for (int64_t q = 0; q < nq; ++q) {
    std::vector<int32_t> own_l;
    std::vector<float> own_g;
    for (int p = 0; p < nprobe; ++p) {
      const int l = probes[q * nprobe + p];
      if ((owner ? owner[l] : l % shard_count) == shard_rank) {
        own_l.push_back(l);
        own_g.push_back(gq[q * nprobe + p]);
      }
    }
    std::vector<uint64_t> ub;
    int64_t have = 0;
    for (size_t i = 0; i < own_l.size() && have < R; ++i) {
      const int l = own_l[i];
      const float g = own_g[i];
      for (int64_t s = list_off[l]; s < list_off[l + 1]; ++s, ++have) {
        const int32_t acc = orc_popcount_ip(planes + (size_t)q * qbits * W, codes + (size_t)s * W, W, qbits);
        const float ip = (float)acc * delta[q];
        const float est = (fadd[s] + g) + frescale[s] * (ip + k1[q]);
        ub.push_back(make_key(est + ferr[s] * sqrtf(g), (uint32_t)have));
      }
    }
    if ((int64_t)ub.size() < R) {
      tau_out[q] = INFINITY;
    } else {
      std::nth_element(ub.begin(), ub.begin() + (R - 1), ub.end());
      tau_out[q] = from_ordered_bits((uint32_t)(ub[(size_t)R - 1] >> 32));
    }
  }
}

// Scan (a9-a11): for every query the top-R candidates by (estimated distance, id).
// probes/g: [nq, nprobe] from orc_coarse.  tau0 (optional, [nq]): every slice of query q starts
// with threshold tau0[q] instead of +inf (a threshold seeded by an earlier scan).  init_ids /
// init_dist (optional, [nq, R], id -1 = none): candidates of an earlier scan that slice 0
// starts from.
// Lists owned by this shard: owner[l] == shard_rank (owner NULL: l % shard_count), taken in
// probe order and split into `slices` contiguous ranges (slice s gets
// owned[floor(s*m/S) : floor((s+1)*m/S)]), each scanned with its own threshold, then merged.
// Outputs out_ids [nq, R] (int64, -1 pad) and out_dist [nq, R] (+inf pad).
// stats (optional, int64[2]): vectors scanned, vectors admitted by the prune.
// ex_codes / fexadd / fexr (optional, ExRaBitQ index with ex_bits extra bits, slot order): an
// admitted vector's distance is the extra-bit distance (orc_ex_ip) instead of the 1-bit one.
void orc_scan(const int64_t* list_off, const uint32_t* ids, const uint32_t* codes, const float* fadd,
              const float* frescale, const float* ferr, int Dp, const float* Qr, const uint32_t* planes,
              const float* delta, const float* k1, int64_t nq, const int32_t* probes, const float* gq,
              int nprobe, const float* tau0, const int64_t* init_ids, const float* init_dist, int R, int tile,
              int cap, int prune, int slices, int shard_rank, int shard_count, const int32_t* owner,
              int64_t* out_ids, float* out_dist, int64_t* stats, int qbits, const uint32_t* ex_codes,
              const float* fexadd, const float* fexr, int ex_bits)
{
  const int W = Dp / 32;
  ScanIndex ix{list_off, ids, codes, fadd, frescale, ferr, qbits, ex_codes, fexadd, fexr, ex_codes ? ex_bits : 0};
  int64_t tot[2] = {0, 0};
#pragma omp parallel
  {
    std::vector<uint64_t> keys, all, init;
    const std::vector<uint64_t> none;
    std::vector<int32_t> own_l;
    std::vector<float> own_g;
    int64_t loc[2] = {0, 0};
#pragma omp for schedule(dynamic, 4)
    for (int64_t q = 0; q < nq; ++q) {
      own_l.clear();
      own_g.clear();
      for (int p = 0; p < nprobe; ++p) {
        int l = probes[q * nprobe + p];
        if ((owner ? owner[l] : l % shard_count) == shard_rank) {
          own_l.push_back(l);
          own_g.push_back(gq[q * nprobe + p]);
        }
      }
      const int m = (int)own_l.size();
      all.clear();
      init.clear();
      if (init_ids)
        for (int r = 0; r < R; ++r)
          if (init_ids[q * R + r] >= 0)
            init.push_back(make_key(init_dist[q * R + r], (uint32_t)init_ids[q * R + r]));
      for (int s = 0; s < slices; ++s) {
        int a = (int)(((int64_t)s * m) / slices), b = (int)(((int64_t)(s + 1) * m) / slices);
        scan_slice(ix, W, Qr + (size_t)q * Dp, planes + (size_t)q * (is_lut_mode(qbits) ? 4 : qbits) * W, delta[q], k1[q],
                   own_l.data() + a, own_g.data() + a, b - a, tau0 ? tau0[q] : INFINITY, s == 0 ? init : none,
                   R, tile, cap, prune, keys, loc);
        all.insert(all.end(), keys.begin(), keys.end());
      }
      std::sort(all.begin(), all.end());
      for (int r = 0; r < R; ++r) {
        if (r < (int)all.size()) {
          out_ids[q * R + r] = (int64_t)(all[r] & 0xFFFFFFFFu);
          out_dist[q * R + r] = from_ordered_bits((uint32_t)(all[r] >> 32));
        } else {
          out_ids[q * R + r] = -1;
          out_dist[q * R + r] = INFINITY;
        }
      }
    }
#pragma omp critical
    {
      tot[0] += loc[0];
      tot[1] += loc[1];
    }
  }
  if (stats) {
    stats[0] = tot[0];
    stats[1] = tot[1];
  }
}

// Exact squared L2 of two unrotated D-dim rows, in the order the CUDA rerank uses: lane l
// (0..31) sums double(x_d - q_d)^2 over d = l, l+32, ... ascending; the 32 lane sums are
// combined by a butterfly (offsets 16, 8, 4, 2, 1: v[l] = v[l] + v[l ^ off]); lane 0's value
// is rounded to float.
float orc_l2_exact(const float* x, const float* q, int D) { return l2_lanes(x, q, D); }

// Exact rerank (a13): candidates [nq, R] (-1 = empty) -> top-k by (exact L2^2, id).
void orc_rerank(const float* X, int D, const float* Q, int64_t nq, const int64_t* cand, int R, int k,
                float* out_dist, int64_t* out_ids)
{
#pragma omp parallel
  {
    std::vector<uint64_t> keys;
#pragma omp for schedule(dynamic, 16)
    for (int64_t q = 0; q < nq; ++q) {
      keys.clear();
      for (int r = 0; r < R; ++r) {
        int64_t id = cand[q * R + r];
        if (id < 0) continue;
        float d = orc_l2_exact(X + (size_t)id * D, Q + (size_t)q * D, D);
        keys.push_back(make_key(d, (uint32_t)id));
      }
      std::sort(keys.begin(), keys.end());
      for (int i = 0; i < k; ++i) {
        if (i < (int)keys.size()) {
          out_ids[q * k + i] = (int64_t)(keys[i] & 0xFFFFFFFFu);
          out_dist[q * k + i] = from_ordered_bits((uint32_t)(keys[i] >> 32));
        } else {
          out_ids[q * k + i] = -1;
          out_dist[q * k + i] = INFINITY;
        }
      }
    }
  }
}

// Brute-force exact k-NN (ground truth for recall), same distance as the rerank.
void orc_knn_exact(const float* X, int64_t n, int D, const float* Q, int64_t nq, int k, float* out_dist,
                   int64_t* out_ids)
{
#pragma omp parallel
  {
    std::vector<uint64_t> keys(n);
#pragma omp for schedule(dynamic, 1)
    for (int64_t q = 0; q < nq; ++q) {
      for (int64_t i = 0; i < n; ++i)
        keys[i] = make_key(orc_l2_exact(X + (size_t)i * D, Q + (size_t)q * D, D), (uint32_t)i);
      std::partial_sort(keys.begin(), keys.begin() + k, keys.end());
      for (int i = 0; i < k; ++i) {
        out_ids[q * k + i] = (int64_t)(keys[i] & 0xFFFFFFFFu);
        out_dist[q * k + i] = from_ordered_bits((uint32_t)(keys[i] >> 32));
      }
    }
  }
}

// Nearest-centroid labels in the original space (k-means assignment), ties -> lower id.
void orc_assign(const float* X, int64_t n, int D, const float* C, int K, uint32_t* labels)
{
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    uint64_t best = kEmptyKey;
    for (int c = 0; c < K; ++c) {
      uint64_t key = make_key(coarse_dist(X + (size_t)i * D, C + (size_t)c * D, D), (uint32_t)c);
      if (key < best) best = key;
    }
    labels[i] = (uint32_t)(best & 0xFFFFFFFFu);
  }
}

// Number of OpenMP threads this library will use.
int orc_threads(void)
{
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_threads(int n)
{
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

}  // extern "C"
