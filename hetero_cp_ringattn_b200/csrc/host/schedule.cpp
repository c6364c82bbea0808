// Frozen KV-growth assignee schedule and stationary layer starters.
//
// Behaviour of rust/src/model/self_driving.rs:12-144, kept exactly: the coordinator and every
// rank derive the same owner for each decoded (token, layer) KV row from the capacity tickets
// alone, without exchanging messages.
//   quotas:   total * ticket / sum(tickets) rounded down, the remaining units to the largest
//             fractional parts (ties to the lower rank);
//   sequence: smooth weighted round robin over the quotas (each step every rank's score grows by
//             its quota, the highest score takes the unit, ties to the lower rank, and pays back
//             `total`), which spreads each rank's units evenly over the sequence;
//   phase:    request_id % total, so concurrent requests do not all start on the same rank.
#include "hcp_host.h"

#include <algorithm>

namespace hcp::host {

FrozenKvAssigneeSchedule::FrozenKvAssigneeSchedule(const std::vector<uint64_t>& tickets,
                                                   uint64_t request_id, uint64_t total_units) {
  if (tickets.empty()) throw RingError("KV assignee schedule requires at least one worker");
  if (total_units == 0) throw RingError("KV assignee schedule requires at least one KV unit");
  unsigned __int128 cap_sum = 0;
  for (uint64_t t : tickets) cap_sum += t;
  if (cap_sum == 0) throw RingError("KV assignee schedule requires non-zero capacity");
  const int64_t n = int64_t(tickets.size());
  const int64_t total = int64_t(total_units);
  counts_.assign(size_t(n), 0);
  std::vector<std::pair<int64_t, unsigned __int128>> rems;
  int64_t assigned = 0;
  for (int64_t d = 0; d < n; ++d) {
    const unsigned __int128 num = (unsigned __int128)total * tickets[size_t(d)];
    counts_[size_t(d)] = int64_t(num / cap_sum);
    assigned += counts_[size_t(d)];
    rems.emplace_back(d, num % cap_sum);
  }
  std::stable_sort(rems.begin(), rems.end(),
                   [](const auto& a, const auto& b) { return a.second > b.second; });
  for (int64_t k = 0; k < total - assigned && k < n; ++k) ++counts_[size_t(rems[size_t(k)].first)];
  std::vector<int64_t> score(size_t(n), 0);
  seq_.reserve(size_t(total));
  for (int64_t u = 0; u < total; ++u) {
    int64_t best = 0;
    for (int64_t d = 0; d < n; ++d) {
      score[size_t(d)] += counts_[size_t(d)];
      if (score[size_t(d)] > score[size_t(best)]) best = d;
    }
    score[size_t(best)] -= total;
    seq_.push_back(best);
  }
  phase_ = request_id % total_units;
}

int64_t FrozenKvAssigneeSchedule::AssigneeFor(int64_t token_offset, int64_t layer,
                                              int64_t num_layers) const {
  if (num_layers <= 0 || layer < 0 || layer >= num_layers || token_offset < 0) return -1;
  const int64_t ordinal = token_offset * num_layers + layer;
  if (ordinal >= int64_t(seq_.size())) return -1;
  return seq_[size_t((phase_ + uint64_t(ordinal)) % seq_.size())];
}

std::vector<int64_t> FrozenKvAssigneeSchedule::PerRankUnits(int64_t num_ranks, int64_t first_token,
                                                            int64_t last_token,
                                                            int64_t num_layers) const {
  std::vector<int64_t> out(size_t(std::max<int64_t>(num_ranks, 0)), 0);
  for (int64_t t = first_token; t < last_token; ++t)
    for (int64_t l = 0; l < num_layers; ++l) {
      const int64_t a = AssigneeFor(t, l, num_layers);
      if (a >= 0 && a < num_ranks) ++out[size_t(a)];
    }
  return out;
}

std::vector<int64_t> AssigneeTable(const std::vector<uint64_t>& tickets, uint64_t request_id,
                                   int64_t horizon, int64_t layers) {
  if (horizon <= 0 || layers <= 0) return {};
  const uint64_t units = uint64_t(horizon) * uint64_t(layers);
  FrozenKvAssigneeSchedule s(tickets, request_id, units);
  const auto& seq = s.Sequence();
  std::vector<int64_t> out(static_cast<size_t>(units));
  for (uint64_t k = 0; k < units; ++k) out[size_t(k)] = seq[size_t((s.Phase() + k) % units)];
  return out;
}

std::vector<int64_t> StationaryLayerStarters(int64_t initial_starter, int64_t layers,
                                             int64_t domains) {
  if (domains <= 0) throw RingError("stationary ring requires at least one domain");
  if (initial_starter < 0 || initial_starter >= domains)
    throw RingError("stationary ring starter " + std::to_string(initial_starter) + " out of " +
                    std::to_string(domains) + " domains");
  std::vector<int64_t> out;
  int64_t s = initial_starter;
  for (int64_t l = 0; l < layers; ++l) {
    out.push_back(s);
    s = (s + domains - 1) % domains;
  }
  return out;
}

}  // namespace hcp::host
