// Ring layouts: which rank owns which global token position.
//
// The three layouts are those of rust/src/model/attention/strategy.rs:16-146, kept exactly
// because the coordinator, every rank's RoPE positions and the attention kernels' causal skip all
// derive from the same assignment:
//   vanilla: contiguous chunks in rank order;
//   striped: weighted round robin, one slot per rank that still has quota, repeated;
//   zigzag:  rank i owns a prefix segment of ceil(c_i / 2) tokens (prefixes in rank order) and a
//            suffix segment of floor(c_i / 2) tokens (suffixes in reverse rank order).
#include "hcp_host.h"

#include <algorithm>

namespace hcp::host {

RingStrategy ParseStrategy(const std::string& name) {
  std::string s;
  for (char c : name) s.push_back(char(c >= 'A' && c <= 'Z' ? c - 'A' + 'a' : c));
  if (s == "vanilla") return RingStrategy::kVanilla;
  if (s == "striped") return RingStrategy::kStriped;
  if (s == "zigzag") return RingStrategy::kZigzag;
  throw std::invalid_argument("unknown ring strategy '" + name + "' (vanilla|striped|zigzag)");
}

std::vector<int64_t> BuildAssignment(const std::vector<int64_t>& chunks, RingStrategy s) {
  const int64_t n = int64_t(chunks.size());
  int64_t total = 0;
  for (int64_t c : chunks) {
    if (c < 0) throw RingError("chunk sizes must be non-negative");
    total += c;
  }
  std::vector<int64_t> out;
  out.reserve(size_t(total));
  switch (s) {
    case RingStrategy::kVanilla:
      for (int64_t d = 0; d < n; ++d) out.insert(out.end(), size_t(chunks[d]), d);
      break;
    case RingStrategy::kStriped: {
      std::vector<int64_t> left(chunks);
      while (int64_t(out.size()) < total) {
        for (int64_t d = 0; d < n; ++d) {
          if (left[d] > 0) {
            out.push_back(d);
            --left[d];
          }
        }
      }
      break;
    }
    case RingStrategy::kZigzag:
      for (int64_t d = 0; d < n; ++d) out.insert(out.end(), size_t(chunks[d] - chunks[d] / 2), d);
      for (int64_t d = n - 1; d >= 0; --d) out.insert(out.end(), size_t(chunks[d] / 2), d);
      break;
  }
  return out;
}

std::vector<std::vector<int64_t>> BuildDomainPositions(const std::vector<int64_t>& assignment,
                                                       int64_t num_domains) {
  if (num_domains < 0) {
    num_domains = 0;
    for (int64_t a : assignment) num_domains = std::max(num_domains, a + 1);
  }
  std::vector<std::vector<int64_t>> pos(static_cast<size_t>(num_domains));
  for (size_t p = 0; p < assignment.size(); ++p) {
    const int64_t d = assignment[p];
    if (d < 0 || d >= num_domains) throw RingError("assignment names a rank out of range");
    pos[size_t(d)].push_back(int64_t(p));
  }
  return pos;
}

std::vector<int64_t> BuildInversePerm(const std::vector<int64_t>& assignment) {
  const auto pos = BuildDomainPositions(assignment, -1);
  std::vector<int64_t> inv(assignment.size());
  int64_t off = 0;
  for (const auto& v : pos)
    for (int64_t p : v) inv[size_t(p)] = off++;
  return inv;
}

}  // namespace hcp::host
