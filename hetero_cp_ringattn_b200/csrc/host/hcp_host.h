// Host-side runtime library: the context-parallel planning and bookkeeping that every rank and
// the coordinator run on the CPU. No CUDA here; it is built into its own Python module
// (`hetero_cp_ringattn_b200._host`) and linked into the native tests.
//
//   * ring layouts (vanilla / striped / zigzag): token -> rank assignment, per-rank positions,
//     inverse permutation (reference: rust/src/model/attention/strategy.rs:16-146);
//   * capacity-weighted chunking, equal splits, ratio overrides, continuation splits, KV byte
//     admission and the per-rank KV byte ledger (rust/src/capacity.rs:67-297,
//     rust/src/distributed/coordinator.rs:784-960);
//   * the frozen KV-growth assignee schedule and the stationary layer starters
//     (rust/src/model/self_driving.rs:12-144);
//   * the paged KV arena's page allocator (rust/src/model/cache.rs block tables,
//     self_driving.rs:146-331 reserved slabs);
//   * the iterative batch scheduler's queue / active-set core (rust/src/distributed/scheduler.rs);
//   * the binary frames of the coordinator <-> rank control protocol
//     (rust/src/distributed/protocol.rs:14-192 message set);
//   * a float64 attention / ring-attention oracle (rust/src/smoke/reference_algo.rs).
#pragma once

#include <condition_variable>
#include <cstdint>
#include <deque>
#include <map>
#include <mutex>
#include <optional>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace hcp::host {

// Errors map onto the Python package's RingError / CapacityError in the bindings.
struct RingError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct CapacityError : RingError {
  using RingError::RingError;
};

// ----------------------------------------------------------------------------- ring layouts
enum class RingStrategy { kVanilla = 0, kStriped = 1, kZigzag = 2 };

RingStrategy ParseStrategy(const std::string& name);
// a[p] = rank that owns global position p; rank i owns chunks[i] positions.
std::vector<int64_t> BuildAssignment(const std::vector<int64_t>& chunks, RingStrategy s);
// Ordered global positions owned by each of `num_domains` ranks.
std::vector<std::vector<int64_t>> BuildDomainPositions(const std::vector<int64_t>& assignment,
                                                       int64_t num_domains);
// inverse[p] = index of position p inside concat(rank 0 positions, rank 1 positions, ...).
std::vector<int64_t> BuildInversePerm(const std::vector<int64_t>& assignment);

// ----------------------------------------------------------------------------- capacity
constexpr uint64_t kUnknownCapacity = ~uint64_t(0);

std::vector<int64_t> AllocateByCapacity(int64_t prompt_len, const std::vector<uint64_t>& caps);
std::vector<int64_t> EqualChunks(int64_t prompt_len, int64_t n);
// The coordinator's chooser: explicit sizes, ratio override, capacity-aware (capacities minus the
// activation reserve), else equal splits.
std::vector<int64_t> ChunkSizes(int64_t prompt_len, int64_t num_domains,
                                const std::vector<int64_t>& explicit_sizes,
                                const std::vector<uint64_t>& capacities_mb, bool capacity_aware,
                                const std::vector<uint64_t>& ratio, int64_t activation_reserve_mb);
// Continuation segment cut into contiguous per-rank pieces by capacity tickets.
std::vector<int64_t> ContinuationSplit(int64_t segment_len, const std::vector<uint64_t>& tickets);
std::vector<uint64_t> CapacityMbToBytes(const std::vector<uint64_t>& capacity_mb);

struct KvByteAdmission {
  uint64_t bytes_per_token_per_layer = 0;
  std::vector<uint64_t> required_bytes_per_domain;
};
KvByteAdmission AdmitReservedKvBytes(const std::vector<std::vector<uint64_t>>& layer_caps,
                                     const std::vector<uint64_t>& budget_bytes,
                                     uint64_t num_kv_heads, uint64_t head_dim,
                                     uint64_t element_size_bytes);

// Per-rank KV byte ledger: all-or-nothing reservations keyed by request, released as a whole.
class KvLedger {
 public:
  explicit KvLedger(std::vector<uint64_t> budgets);
  void TryReserve(uint64_t request_id, const std::vector<uint64_t>& bytes_per_domain);
  std::vector<uint64_t> Release(uint64_t request_id);  // zeros if the request holds nothing
  std::vector<uint64_t> FreeBytes() const;
  const std::vector<uint64_t>& Used() const { return used_; }
  const std::vector<uint64_t>& Budgets() const { return budgets_; }
  bool Holds(uint64_t request_id) const { return by_request_.count(request_id) != 0; }

 private:
  std::vector<uint64_t> budgets_, used_;
  std::unordered_map<uint64_t, std::vector<uint64_t>> by_request_;
};

// ----------------------------------------------------------------------------- KV growth schedule
// Every (decoded token, layer) KV row is stored by exactly one rank. The rank is fixed up front
// from capacity tickets: per-rank quotas by largest remainder, interleaved by smooth weighted
// round robin, started at phase request_id % total so that requests spread their first rows.
class FrozenKvAssigneeSchedule {
 public:
  FrozenKvAssigneeSchedule(const std::vector<uint64_t>& tickets, uint64_t request_id,
                           uint64_t total_units);
  // -1 when out of range (the reference returns None).
  int64_t AssigneeFor(int64_t token_offset, int64_t layer, int64_t num_layers) const;
  std::vector<int64_t> PerRankUnits(int64_t num_ranks, int64_t first_token, int64_t last_token,
                                    int64_t num_layers) const;
  const std::vector<int64_t>& Sequence() const { return seq_; }
  const std::vector<int64_t>& Counts() const { return counts_; }
  uint64_t Phase() const { return phase_; }

 private:
  std::vector<int64_t> seq_, counts_;
  uint64_t phase_ = 0;
};

// [horizon x layers] owner table of a request's decode rows: the frozen schedule over
// horizon * layers units (row t = t-th decoded token).
std::vector<int64_t> AssigneeTable(const std::vector<uint64_t>& tickets, uint64_t request_id,
                                   int64_t horizon, int64_t layers);
std::vector<int64_t> StationaryLayerStarters(int64_t initial_starter, int64_t layers,
                                             int64_t domains);

// ----------------------------------------------------------------------------- KV pages
class PageAllocator {
 public:
  PageAllocator(int64_t num_pages, int64_t page_size);
  std::vector<int64_t> Alloc(int64_t n, int64_t request_id);  // lowest never-used ids first
  void Free(const std::vector<int64_t>& pages);
  int64_t FreePages() const { return int64_t(free_.size()); }
  int64_t NumPages() const { return num_pages_; }
  int64_t PageSize() const { return page_size_; }
  int64_t OwnerOf(int64_t page) const;  // -1 when free

 private:
  int64_t num_pages_, page_size_;
  std::vector<int64_t> free_;  // stack: the next page handed out is at the back
  std::unordered_map<int64_t, int64_t> owner_;
};

// ----------------------------------------------------------------------------- batch scheduler
// FIFO of pending request ids plus the active set (insertion ordered), bounded by
// max_batch_size. Thread safe: HTTP threads enqueue while the coordinator loop pops.
class BatchSchedulerCore {
 public:
  explicit BatchSchedulerCore(int64_t max_batch_size);
  void Enqueue(uint64_t request_id);
  std::optional<uint64_t> PopPending();  // only while the active set has room
  void RequeueFront(uint64_t request_id);
  void Activate(uint64_t request_id);
  bool Complete(uint64_t request_id);
  bool HasCapacity() const;
  std::vector<uint64_t> Active() const;
  int64_t Queued() const;
  int64_t NumActive() const;
  // Blocks up to timeout_s while there is neither pending nor active work.
  void WaitForWork(double timeout_s);
  int64_t MaxBatchSize() const { return max_batch_; }

 private:
  int64_t max_batch_;
  mutable std::mutex mu_;
  std::condition_variable cv_;
  std::deque<uint64_t> pending_;
  std::vector<uint64_t> active_;
};

// ----------------------------------------------------------------------------- control protocol
// Binary frames of the coordinator <-> rank control messages:
//   [u32 payload bytes][u8 version][u8 message type][fields ...], all little endian.
// Each message type has a fixed field list (kinds below); arrays carry a u64 count, strings a u32
// byte count, optionals a u8 presence flag. Token arrays travel as raw int64, so a 128k-token
// prompt costs one memcpy instead of a text encoding.
enum class FieldKind : char {
  kI64 = 'i',        // int64
  kF64 = 'f',        // double
  kBool = 'b',       // u8 0/1
  kStr = 's',        // u32 length + utf-8 bytes
  kI64Array = 'A',   // u64 count + int64[count]
  kPairs = 'P',      // u64 count + int64[2 * count] (rows of two)
  kOptI64 = 'o',     // u8 present + int64
  kOptI64Array = 'O',// u8 present + array
  kOptF32Array = 'G',// u8 present + u64 count + float[count]
};

struct Field {
  FieldKind kind = FieldKind::kI64;
  bool present = true;             // optionals
  int64_t i = 0;
  double f = 0.0;
  std::string s;
  std::vector<int64_t> a;          // arrays and pairs (row-major)
  std::vector<float> fa;
};

constexpr uint8_t kProtocolVersion = 1;
// Field kinds of a message type ("" if unknown).
const char* MessageSchema(int type);
std::string EncodeFrame(int type, const std::vector<Field>& fields);
// Throws ProtocolError on a short, partial, oversized, unknown-type or wrong-version frame.
std::vector<Field> DecodeFrame(const std::string& frame, int* type);

struct ProtocolError : RingError {
  using RingError::RingError;
};

// ----------------------------------------------------------------------------- f64 oracle
// Double-precision attention oracle on the CPU (the reference's f64 ring algorithm check):
// q [L, H, D], k / v [L, Hkv, D] row-major; GQA by head // (H / Hkv); causal compares positions.
struct AttnResult {
  std::vector<double> o;    // [L, H, D]
  std::vector<double> lse;  // [H, L] natural log; -inf for a row with no visible key
};
AttnResult FullAttentionF64(const std::vector<double>& q, const std::vector<double>& k,
                            const std::vector<double>& v, int64_t L, int64_t H, int64_t Hkv,
                            int64_t D, bool causal);
// Ring attention with uneven chunks: rank t owns positions[t] (global positions, any layout) and
// folds the sources (t + step) % N in blocks of block_sizes[source] rows with an online softmax;
// fully-future blocks are skipped when causal. Returns the same layout as FullAttentionF64.
AttnResult RingAttentionF64(const std::vector<double>& q, const std::vector<double>& k,
                            const std::vector<double>& v, int64_t L, int64_t H, int64_t Hkv,
                            int64_t D, const std::vector<std::vector<int64_t>>& positions,
                            const std::vector<int64_t>& block_sizes, bool causal);

}  // namespace hcp::host
