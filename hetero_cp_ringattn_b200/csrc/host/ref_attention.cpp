// Double-precision attention oracle (the reference's f64 ring-attention correctness check,
// rust/src/smoke/reference_algo.rs: ring == full attention over uneven chunks and blocks),
// extended with causal masking on global positions, GQA and the log-sum-exp output.
//
// The ring model is the algorithm the GPU kernels implement: each rank keeps (m, l, acc) per
// (query, head), visits every source chunk in ring order in blocks, skips a block whose first
// key position is past the rank's last query position, and rescales by exp(m_old - m_new).
#include <cmath>
#include <limits>

#include "hcp_host.h"

namespace hcp::host {

namespace {

constexpr double kNegInf = -std::numeric_limits<double>::infinity();

void CheckShapes(const std::vector<double>& q, const std::vector<double>& k,
                 const std::vector<double>& v, int64_t L, int64_t H, int64_t Hkv, int64_t D) {
  if (L < 0 || H <= 0 || Hkv <= 0 || D <= 0 || H % Hkv)
    throw RingError("attention oracle: bad shape");
  if (int64_t(q.size()) != L * H * D || int64_t(k.size()) != L * Hkv * D ||
      int64_t(v.size()) != L * Hkv * D)
    throw RingError("attention oracle: tensor sizes do not match [L, H, D] / [L, Hkv, D]");
}

double Dot(const double* a, const double* b, int64_t D) {
  double s = 0.0;
  for (int64_t d = 0; d < D; ++d) s += a[d] * b[d];
  return s;
}

}  // namespace

AttnResult FullAttentionF64(const std::vector<double>& q, const std::vector<double>& k,
                            const std::vector<double>& v, int64_t L, int64_t H, int64_t Hkv,
                            int64_t D, bool causal) {
  CheckShapes(q, k, v, L, H, Hkv, D);
  const double scale = 1.0 / std::sqrt(double(D));
  const int64_t G = H / Hkv;
  AttnResult r;
  r.o.assign(size_t(L * H * D), 0.0);
  r.lse.assign(size_t(H * L), kNegInf);
  std::vector<double> s(static_cast<size_t>(L));
  for (int64_t i = 0; i < L; ++i)
    for (int64_t h = 0; h < H; ++h) {
      const double* qi = &q[size_t((i * H + h) * D)];
      const int64_t kh = h / G;
      const int64_t nk = causal ? i + 1 : L;
      double m = kNegInf;
      for (int64_t j = 0; j < nk; ++j) {
        s[size_t(j)] = Dot(qi, &k[size_t((j * Hkv + kh) * D)], D) * scale;
        m = std::max(m, s[size_t(j)]);
      }
      if (nk == 0) continue;
      double l = 0.0;
      double* oi = &r.o[size_t((i * H + h) * D)];
      for (int64_t j = 0; j < nk; ++j) {
        const double p = std::exp(s[size_t(j)] - m);
        l += p;
        const double* vj = &v[size_t((j * Hkv + kh) * D)];
        for (int64_t d = 0; d < D; ++d) oi[d] += p * vj[d];
      }
      for (int64_t d = 0; d < D; ++d) oi[d] /= l;
      r.lse[size_t(h * L + i)] = m + std::log(l);
    }
  return r;
}

AttnResult RingAttentionF64(const std::vector<double>& q, const std::vector<double>& k,
                            const std::vector<double>& v, int64_t L, int64_t H, int64_t Hkv,
                            int64_t D, const std::vector<std::vector<int64_t>>& positions,
                            const std::vector<int64_t>& block_sizes, bool causal) {
  CheckShapes(q, k, v, L, H, Hkv, D);
  const int64_t N = int64_t(positions.size());
  if (N == 0 || int64_t(block_sizes.size()) != N)
    throw RingError("ring oracle: one block size per rank");
  int64_t covered = 0;
  for (const auto& p : positions) {
    covered += int64_t(p.size());
    for (int64_t x : p)
      if (x < 0 || x >= L) throw RingError("ring oracle: position out of range");
  }
  if (covered != L) throw RingError("ring oracle: positions must partition the sequence");
  const double scale = 1.0 / std::sqrt(double(D));
  const int64_t G = H / Hkv;
  AttnResult r;
  r.o.assign(size_t(L * H * D), 0.0);
  r.lse.assign(size_t(H * L), kNegInf);
  for (int64_t t = 0; t < N; ++t) {
    const auto& qpos = positions[size_t(t)];
    const int64_t Tq = int64_t(qpos.size());
    int64_t qmax = -1;
    for (int64_t x : qpos) qmax = std::max(qmax, x);
    // running state per (local query, head), initialised like the reference (finite -1e4)
    std::vector<double> m(size_t(Tq * H), -1e4), l(size_t(Tq * H), 0.0), acc(size_t(Tq * H * D), 0.0);
    for (int64_t step = 0; step < N; ++step) {
      const int64_t src = (t + step) % N;
      const auto& kpos = positions[size_t(src)];
      const int64_t bs = std::max<int64_t>(1, block_sizes[size_t(src)]);
      for (int64_t b0 = 0; b0 < int64_t(kpos.size()); b0 += bs) {
        const int64_t b1 = std::min<int64_t>(int64_t(kpos.size()), b0 + bs);
        int64_t kmin = L;
        for (int64_t j = b0; j < b1; ++j) kmin = std::min(kmin, kpos[size_t(j)]);
        if (causal && kmin > qmax) continue;  // fully-future block
        for (int64_t i = 0; i < Tq; ++i)
          for (int64_t h = 0; h < H; ++h) {
            const int64_t gi = qpos[size_t(i)];
            const double* qi = &q[size_t((gi * H + h) * D)];
            const int64_t kh = h / G;
            double bm = kNegInf;
            std::vector<double> sc(size_t(b1 - b0), kNegInf);
            for (int64_t j = b0; j < b1; ++j) {
              const int64_t gj = kpos[size_t(j)];
              if (causal && gj > gi) continue;
              sc[size_t(j - b0)] = Dot(qi, &k[size_t((gj * Hkv + kh) * D)], D) * scale;
              bm = std::max(bm, sc[size_t(j - b0)]);
            }
            const size_t st = size_t(i * H + h);
            const double mn = std::max(m[st], bm);
            const double alpha = std::exp(m[st] - mn);
            double* a = &acc[st * size_t(D)];
            for (int64_t d = 0; d < D; ++d) a[d] *= alpha;
            double lsum = l[st] * alpha;
            for (int64_t j = b0; j < b1; ++j) {
              if (sc[size_t(j - b0)] == kNegInf) continue;
              const double p = std::exp(sc[size_t(j - b0)] - mn);
              lsum += p;
              const double* vj = &v[size_t((kpos[size_t(j)] * Hkv + kh) * D)];
              for (int64_t d = 0; d < D; ++d) a[d] += p * vj[d];
            }
            m[st] = mn;
            l[st] = lsum;
          }
      }
    }
    for (int64_t i = 0; i < Tq; ++i)
      for (int64_t h = 0; h < H; ++h) {
        const size_t st = size_t(i * H + h);
        const int64_t gi = qpos[size_t(i)];
        if (l[st] <= 0.0) continue;  // no visible key: o = 0, lse = -inf
        double* oi = &r.o[size_t((gi * H + h) * D)];
        for (int64_t d = 0; d < D; ++d) oi[d] = acc[st * size_t(D) + size_t(d)] / l[st];
        r.lse[size_t(h * L + gi)] = m[st] + std::log(l[st]);
      }
  }
  return r;
}

}  // namespace hcp::host
