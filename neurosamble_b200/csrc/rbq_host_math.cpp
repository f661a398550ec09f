// Host-side index constants: the seeded orthogonal rotation P and the query scale t4.
//
// Both are one-off O(Dp^3) / O(100 * Dp log Dp) computations done once per index in double
// precision with index-order sums (compiled with -ffp-contract=off), so every machine that
// builds an index from the same seed gets the same bytes.  They replace
//   * RotatorGPU::init_matmul (gpu_index/rotator_gpu.cu:52-59): RAFT Philox normal + cuSOLVER
//     QR, which cannot be reproduced outside RAPIDS;
//   * DataQuantizerGPU::get_const_scaling_factors (gpu_index/quantizer_gpu.cu:947-980) with its
//     best_rescale_factor search (:887-943), fed by this library's generator instead of RAFT's.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <queue>
#include <utility>
#include <vector>

#include "rbq_internal.cuh"

namespace rbq {
namespace {

// Philox-4x32-10, from the published description (Salmon et al., SC'11).
void philox(uint32_t k0, uint32_t k1, uint32_t c[4])
{
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    c[1] = (uint32_t)p1;
    c[3] = (uint32_t)p0;
    c[0] = n0;
    c[2] = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

// Normal number i of stream `stream`: Box-Muller over two 53-bit uniforms in (0, 1).
double normal_at(uint64_t seed, uint32_t stream, uint64_t i)
{
  uint64_t blk = i >> 1;
  uint32_t c[4] = {(uint32_t)blk, (uint32_t)(blk >> 32), stream, 0x52425142u};
  philox((uint32_t)seed, (uint32_t)(seed >> 32), c);
  const double scale = 1.0 / 9007199254740992.0;
  double u1 = ((double)(((uint64_t)c[0] << 21) ^ (c[1] >> 11)) + 0.5) * scale;
  double u2 = ((double)(((uint64_t)c[2] << 21) ^ (c[3] >> 11)) + 0.5) * scale;
  double radius = std::sqrt(-2.0 * std::log(u1));
  double angle = 6.283185307179586 * u2;
  return (i & 1) ? radius * std::sin(angle) : radius * std::cos(angle);
}

// Start fraction of the rescale search per extra-bit count; the reference's table
// (quantizer_gpu.cu:875-885), which must be alike for t4 to mean the same thing.
// Held as float like the reference's std::array<float, 9>, so t_end is multiplied by the
// double value of each float constant (0.15f, not 0.15).
const float kStartFraction[9] = {0.0f, 0.15f, 0.20f, 0.52f, 0.59f, 0.71f, 0.75f, 0.77f, 0.81f};

// Scale t maximising <floor(t*o)+0.5, o> / |floor(t*o)+0.5| over the critical points where a
// coordinate's level steps up (levels capped at 2^ex_bits - 1).  Same search as the
// reference's best_rescale_factor: start at t_end*fraction, walk the next critical t in
// ascending order with a min-heap.
double best_scale(const std::vector<double>& o, int ex_bits)
{
  const int dim = (int)o.size();
  const int top_level = (1 << ex_bits) - 1;
  const double max_o = *std::max_element(o.begin(), o.end());
  const double t_end = (double)(top_level + 10) / max_o;
  const double t_start = t_end * kStartFraction[ex_bits];
  std::vector<int> level(dim);
  double den2 = 0.25 * (double)dim;
  double num = 0.0;
  for (int i = 0; i < dim; ++i) {
    int lv = (int)((t_start * o[i]) + 1e-5);
    level[i] = lv;
    den2 += lv * lv + lv;
    num += (lv + 0.5) * o[i];
  }
  typedef std::pair<double, size_t> Step;
  std::priority_queue<Step, std::vector<Step>, std::greater<Step>> next;
  for (int i = 0; i < dim; ++i) next.emplace((double)(level[i] + 1) / o[i], (size_t)i);
  double best_ip = 0.0, best_t = 0.0;
  while (!next.empty()) {
    const Step s = next.top();
    next.pop();
    int lv = ++level[s.second];
    den2 += 2 * lv;
    num += o[s.second];
    double ip = num / std::sqrt(den2);
    if (ip > best_ip) {
      best_ip = ip;
      best_t = s.first;
    }
    if (lv < top_level) {
      double tn = (double)(lv + 1) / o[s.second];
      if (tn < t_end) next.emplace(tn, s.second);
    }
  }
  return best_t;
}

}  // namespace

// P = Q(G) * diag(sign(R_jj)), G[i][j] = normal(seed, stream 1, i*Dp + j), by Householder
// reflections in double; rows of A are eliminated column by column, Q accumulated backwards.
void make_rotation(int Dp, uint64_t seed, float* P_out)
{
  const int n = Dp;
  const size_t nn = (size_t)n * n;
  std::vector<double> A(nn), Qm(nn, 0.0), V(nn, 0.0), beta(n, 0.0), rdiag(n, 0.0);
  for (size_t i = 0; i < nn; ++i) A[i] = normal_at(seed, 1u, i);
  for (int k = 0; k < n; ++k) {
    double ss = 0.0;
    for (int i = k; i < n; ++i) ss += A[(size_t)i * n + k] * A[(size_t)i * n + k];
    const double col_norm = std::sqrt(ss);
    const double x0 = A[(size_t)k * n + k];
    const double alpha = (x0 >= 0.0) ? -col_norm : col_norm;
    double* v = &V[(size_t)k * n];
    for (int i = k; i < n; ++i) v[i] = A[(size_t)i * n + k];
    v[k] = x0 - alpha;
    double vv = 0.0;
    for (int i = k; i < n; ++i) vv += v[i] * v[i];
    const double b = (vv == 0.0) ? 0.0 : 2.0 / vv;
    beta[k] = b;
    for (int j = k; j < n; ++j) {
      double dot = 0.0;
      for (int i = k; i < n; ++i) dot += v[i] * A[(size_t)i * n + j];
      const double f = b * dot;
      for (int i = k; i < n; ++i) A[(size_t)i * n + j] -= f * v[i];
    }
    rdiag[k] = A[(size_t)k * n + k];
  }
  for (int i = 0; i < n; ++i) Qm[(size_t)i * n + i] = 1.0;
  for (int k = n - 1; k >= 0; --k) {
    const double* v = &V[(size_t)k * n];
    const double b = beta[k];
    for (int j = 0; j < n; ++j) {
      double dot = 0.0;
      for (int i = k; i < n; ++i) dot += v[i] * Qm[(size_t)i * n + j];
      const double f = b * dot;
      for (int i = k; i < n; ++i) Qm[(size_t)i * n + j] -= f * v[i];
    }
  }
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < n; ++j) {
      double q = Qm[(size_t)i * n + j];
      P_out[(size_t)i * n + j] = (float)(rdiag[j] < 0.0 ? -q : q);
    }
}

// t4 = mean over 100 rows of best_scale(|g| / |g|_2), g = normal(seed, stream 2, r*Dp + j).
float query_scale(int Dp, uint64_t seed, int ex_bits)
{
  const int rows = 100;
  std::vector<double> g(Dp), o(Dp);
  double total = 0.0;
  for (int r = 0; r < rows; ++r) {
    double ss = 0.0;
    for (int j = 0; j < Dp; ++j) {
      g[j] = normal_at(seed, 2u, (uint64_t)r * Dp + j);
      ss += g[j] * g[j];
    }
    const double nrm = std::sqrt(ss);
    for (int j = 0; j < Dp; ++j) o[j] = std::fabs(g[j] / nrm);
    total += best_scale(o, ex_bits);
  }
  return (float)(total / rows);
}

}  // namespace rbq
