// Capacity-weighted chunking and KV byte admission.
//
// AllocateByCapacity is the largest-remainder method of rust/src/capacity.rs:67-150, step for
// step, because chunk boundaries must agree with the reference for the same capacities: the floor
// of each proportional share, at least one token per rank, any excess trimmed one token at a time
// from the largest chunk (the last one on ties), then the remainder handed out by descending
// fractional share (ties in rank order). AdmitReservedKvBytes follows capacity.rs:227-297 and
// CapacityMbToBytes capacity.rs:200-225. ChunkSizes is the coordinator's chooser
// (coordinator.rs:900-960) plus the integer ratio override ("5:5:1").
#include "hcp_host.h"

#include <algorithm>
#include <numeric>

namespace hcp::host {

namespace {
using u128 = unsigned __int128;

std::string Str(uint64_t v) { return std::to_string(v); }
}  // namespace

std::vector<int64_t> AllocateByCapacity(int64_t prompt_len, const std::vector<uint64_t>& caps) {
  const int64_t n = int64_t(caps.size());
  if (n == 0) throw RingError("capacities must not be empty");
  if (prompt_len < n)
    throw RingError("prompt_len (" + std::to_string(prompt_len) + ") must be >= num_domains (" +
                    std::to_string(n) + ") to give each domain at least 1 token");
  u128 total = 0;
  for (uint64_t c : caps) total += c;
  std::vector<int64_t> chunks(size_t(n), 0);
  if (total == 0) {
    for (int64_t i = 0; i < n; ++i) chunks[size_t(i)] = prompt_len / n + (i < prompt_len % n ? 1 : 0);
    return chunks;
  }
  int64_t consumed = 0;
  for (int64_t i = 0; i < n; ++i) {
    int64_t c = int64_t(u128(prompt_len) * caps[size_t(i)] / total);
    if (c == 0) c = 1;
    chunks[size_t(i)] = c;
    consumed += c;
  }
  if (consumed > prompt_len) {
    int64_t excess = consumed - prompt_len;
    while (excess > 0) {
      const int64_t mx = *std::max_element(chunks.begin(), chunks.end());
      int64_t idx = 0;
      for (int64_t i = 0; i < n; ++i)
        if (chunks[size_t(i)] == mx) idx = i;  // the last maximal element
      if (chunks[size_t(idx)] <= 1) break;
      --chunks[size_t(idx)];
      --excess;
    }
  }
  int64_t rem = prompt_len - std::accumulate(chunks.begin(), chunks.end(), int64_t(0));
  if (rem > 0) {
    // fractional share of each rank, as the double quotient of the exact integer product
    std::vector<std::pair<int64_t, double>> fr;
    for (int64_t i = 0; i < n; ++i) {
      const double share = double(u128(prompt_len) * caps[size_t(i)]) / double(total);
      fr.emplace_back(i, share - double(chunks[size_t(i)]));
    }
    std::stable_sort(fr.begin(), fr.end(),
                     [](const auto& a, const auto& b) { return a.second > b.second; });
    for (int64_t k = 0; k < rem && k < n; ++k) ++chunks[size_t(fr[size_t(k)].first)];
  }
  if (std::accumulate(chunks.begin(), chunks.end(), int64_t(0)) != prompt_len)
    throw RingError("capacity allocation does not sum to the prompt length");
  return chunks;
}

std::vector<int64_t> EqualChunks(int64_t prompt_len, int64_t n) {
  if (n <= 0) throw RingError("need at least one domain");
  if (prompt_len < n)
    throw RingError("prompt_len (" + std::to_string(prompt_len) + ") must be >= num_domains (" +
                    std::to_string(n) + ")");
  const int64_t size = (prompt_len + n - 1) / n;
  std::vector<int64_t> out;
  int64_t left = prompt_len;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t c = std::min(size, left - (n - i - 1));
    out.push_back(c);
    left -= c;
  }
  return out;
}

std::vector<int64_t> ChunkSizes(int64_t prompt_len, int64_t num_domains,
                                const std::vector<int64_t>& explicit_sizes,
                                const std::vector<uint64_t>& capacities_mb, bool capacity_aware,
                                const std::vector<uint64_t>& ratio, int64_t activation_reserve_mb) {
  if (!explicit_sizes.empty()) {
    if (int64_t(explicit_sizes.size()) != num_domains)
      throw RingError("--chunk-sizes has " + std::to_string(explicit_sizes.size()) +
                      " entries for " + std::to_string(num_domains) + " domains");
    int64_t sum = 0;
    for (int64_t x : explicit_sizes) sum += x;
    if (sum != prompt_len)
      throw RingError("--chunk-sizes sum " + std::to_string(sum) + " != prompt length " +
                      std::to_string(prompt_len));
    for (int64_t x : explicit_sizes)
      if (x < 1) throw RingError("every domain needs at least one token");
    return explicit_sizes;
  }
  if (!ratio.empty()) {
    if (int64_t(ratio.size()) != num_domains)
      throw RingError("ratio has " + std::to_string(ratio.size()) + " entries for " +
                      std::to_string(num_domains) + " domains");
    return AllocateByCapacity(prompt_len, ratio);
  }
  if (capacity_aware && !capacities_mb.empty()) {
    std::vector<uint64_t> caps;
    for (uint64_t c : capacities_mb) {
      if (c == kUnknownCapacity) {
        caps.push_back(0);
      } else {
        const int64_t r = int64_t(c) - activation_reserve_mb;
        caps.push_back(r > 0 ? uint64_t(r) : 0);
      }
    }
    return AllocateByCapacity(prompt_len, caps);
  }
  return EqualChunks(prompt_len, num_domains);
}

std::vector<int64_t> ContinuationSplit(int64_t segment_len, const std::vector<uint64_t>& tickets) {
  const int64_t n = int64_t(tickets.size());
  if (segment_len >= n) return AllocateByCapacity(segment_len, tickets);
  std::vector<int64_t> order(static_cast<size_t>(n));
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(),
                   [&](int64_t a, int64_t b) { return tickets[size_t(a)] > tickets[size_t(b)]; });
  std::vector<int64_t> out(size_t(n), 0);
  for (int64_t k = 0; k < segment_len; ++k) out[size_t(order[size_t(k)])] = 1;
  return out;
}

std::vector<uint64_t> CapacityMbToBytes(const std::vector<uint64_t>& capacity_mb) {
  std::vector<uint64_t> out;
  for (size_t d = 0; d < capacity_mb.size(); ++d) {
    const uint64_t mb = capacity_mb[d];
    if (mb == kUnknownCapacity)
      throw CapacityError("KV byte admission domain " + std::to_string(d) +
                          " reported unknown capacity");
    if (u128(mb) * 1024 * 1024 >= (u128(1) << 64))
      throw CapacityError("KV byte admission domain " + std::to_string(d) + " capacity " + Str(mb) +
                          " MB cannot be represented in bytes");
    out.push_back(mb * 1024 * 1024);
  }
  return out;
}

KvByteAdmission AdmitReservedKvBytes(const std::vector<std::vector<uint64_t>>& layer_caps,
                                     const std::vector<uint64_t>& budget_bytes,
                                     uint64_t num_kv_heads, uint64_t head_dim,
                                     uint64_t element_size_bytes) {
  const size_t domains = layer_caps.size();
  if (domains == 0) throw CapacityError("KV byte admission requires at least one domain");
  if (budget_bytes.size() != domains)
    throw CapacityError("KV byte admission has " + std::to_string(domains) + " domains but " +
                        std::to_string(budget_bytes.size()) + " byte budgets");
  const size_t layers = layer_caps[0].size();
  if (layers == 0) throw CapacityError("KV byte admission requires at least one layer");
  for (size_t d = 0; d < domains; ++d)
    if (layer_caps[d].size() != layers)
      throw CapacityError("KV byte admission domain " + std::to_string(d) + " has " +
                          std::to_string(layer_caps[d].size()) + " layers, expected " +
                          std::to_string(layers));
  if (num_kv_heads == 0 || head_dim == 0 || element_size_bytes == 0)
    throw CapacityError(
        "KV byte admission requires non-zero KV heads, head dimension, and element bytes");
  KvByteAdmission a;
  const u128 bpt = u128(2) * num_kv_heads * head_dim * element_size_bytes;
  if (bpt >= (u128(1) << 64)) throw CapacityError("KV byte admission arithmetic overflow");
  a.bytes_per_token_per_layer = uint64_t(bpt);
  for (size_t d = 0; d < domains; ++d) {
    u128 rows = 0;
    for (uint64_t c : layer_caps[d]) rows += c;
    const u128 need = rows * bpt;
    if (need >= (u128(1) << 64)) throw CapacityError("KV byte admission arithmetic overflow");
    if (need > budget_bytes[d])
      throw CapacityError("KV byte admission domain " + std::to_string(d) + " requires " +
                          Str(uint64_t(need)) + " bytes, budget is " + Str(budget_bytes[d]) +
                          " bytes");
    a.required_bytes_per_domain.push_back(uint64_t(need));
  }
  return a;
}

KvLedger::KvLedger(std::vector<uint64_t> budgets)
    : budgets_(std::move(budgets)), used_(budgets_.size(), 0) {}

void KvLedger::TryReserve(uint64_t request_id, const std::vector<uint64_t>& bytes) {
  if (bytes.size() != budgets_.size()) throw CapacityError("reservation domain count mismatch");
  for (size_t d = 0; d < bytes.size(); ++d)
    if (u128(used_[d]) + bytes[d] > budgets_[d])
      throw CapacityError("KV reservation for request " + Str(request_id) + " exceeds domain " +
                          std::to_string(d) + " budget: used " + Str(used_[d]) + " + " +
                          Str(bytes[d]) + " > " + Str(budgets_[d]));
  auto& held = by_request_[request_id];
  held.resize(budgets_.size(), 0);
  for (size_t d = 0; d < bytes.size(); ++d) {
    used_[d] += bytes[d];
    held[d] += bytes[d];
  }
}

std::vector<uint64_t> KvLedger::Release(uint64_t request_id) {
  auto it = by_request_.find(request_id);
  if (it == by_request_.end()) return std::vector<uint64_t>(budgets_.size(), 0);
  std::vector<uint64_t> held = std::move(it->second);
  by_request_.erase(it);
  for (size_t d = 0; d < held.size(); ++d) used_[d] -= held[d];
  return held;
}

std::vector<uint64_t> KvLedger::FreeBytes() const {
  std::vector<uint64_t> out;
  for (size_t d = 0; d < budgets_.size(); ++d) out.push_back(budgets_[d] - used_[d]);
  return out;
}

}  // namespace hcp::host
