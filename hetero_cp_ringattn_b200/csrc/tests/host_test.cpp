// Native tests of the host runtime library (no Python, no GPU): golden vectors from the
// reference's own unit tests (strategy.rs:154-202, capacity.rs:445-668, self_driving.rs:1066-1105)
// plus the page allocator, the KV ledger and the batch scheduler core under concurrent producers.
// Exit status 0 and "host_test ok" on success; the first failed check prints its line.
#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <random>
#include <thread>

#include "../host/hcp_host.h"

using namespace hcp::host;
using V = std::vector<int64_t>;

static int g_checks = 0;
#define CHECK(cond)                                                   \
  do {                                                                \
    ++g_checks;                                                       \
    if (!(cond)) {                                                    \
      std::fprintf(stderr, "host_test: CHECK failed at line %d: %s\n", __LINE__, #cond); \
      std::exit(1);                                                   \
    }                                                                 \
  } while (0)

template <class E, class F>
static bool Throws(F f) {
  try {
    f();
  } catch (const E&) {
    return true;
  } catch (...) {
    return false;
  }
  return false;
}

static void Layouts() {
  CHECK((BuildAssignment({3, 1}, RingStrategy::kVanilla) == V{0, 0, 0, 1}));
  CHECK((BuildAssignment({3, 1}, RingStrategy::kStriped) == V{0, 1, 0, 0}));
  CHECK((BuildAssignment({3, 1}, RingStrategy::kZigzag) == V{0, 0, 1, 0}));
  CHECK((BuildAssignment({4, 4}, RingStrategy::kZigzag) == V{0, 0, 1, 1, 1, 1, 0, 0}));
  const auto pos = BuildDomainPositions(BuildAssignment({4, 4}, RingStrategy::kZigzag), -1);
  CHECK(pos.size() == 2 && (pos[0] == V{0, 1, 6, 7}) && (pos[1] == V{2, 3, 4, 5}));
  CHECK((BuildInversePerm(BuildAssignment({3, 1}, RingStrategy::kStriped)) == V{0, 3, 1, 2}));
  CHECK(Throws<std::invalid_argument>([] { ParseStrategy("ring"); }));
  CHECK(ParseStrategy("ZigZag") == RingStrategy::kZigzag);
  // every layout partitions the positions
  for (auto s : {RingStrategy::kVanilla, RingStrategy::kStriped, RingStrategy::kZigzag}) {
    const V chunks{5, 5, 5, 5, 2, 2, 1, 1};
    const auto a = BuildAssignment(chunks, s);
    const auto p = BuildDomainPositions(a, 8);
    for (size_t d = 0; d < 8; ++d) CHECK(int64_t(p[d].size()) == chunks[d]);
  }
}

static void Capacity() {
  CHECK((AllocateByCapacity(10, {4096, 4096}) == V{5, 5}));
  CHECK((AllocateByCapacity(9, {8192, 4096}) == V{6, 3}));
  CHECK((AllocateByCapacity(14, {4096, 2048, 1024}) == V{8, 4, 2}));
  CHECK((AllocateByCapacity(5, {0, 4096}) == V{1, 4}));
  CHECK((AllocateByCapacity(3, {100, 100, 100}) == V{1, 1, 1}));
  CHECK((AllocateByCapacity(8, {0, 0, 0}) == V{3, 3, 2}));
  CHECK((AllocateByCapacity(11, {8192, 12288}) == V{4, 7}));
  CHECK((AllocateByCapacity(11, {8192, 12288, 6144}) == V{3, 5, 3}));
  CHECK((AllocateByCapacity(16, {8192, 20480, 16384}) == V{3, 7, 6}));
  CHECK(Throws<RingError>([] { AllocateByCapacity(2, {1, 1, 1}); }));
  CHECK(Throws<RingError>([] { AllocateByCapacity(2, {}); }));
  CHECK((EqualChunks(10, 3) == V{4, 4, 2}));
  CHECK((ChunkSizes(12, 2, {}, {1536 + 100, 1536 + 300}, true, {}, 1536) == V{3, 9}));
  CHECK((ChunkSizes(10, 2, {7, 3}, {}, false, {}, 1536) == V{7, 3}));
  CHECK(Throws<RingError>([] { ChunkSizes(10, 2, {7, 4}, {}, false, {}, 1536); }));
  const auto c8 = ChunkSizes(65536, 8, {}, {}, false, {5, 5, 5, 5, 2, 2, 1, 1}, 1536);
  CHECK(c8[0] == c8[3] && c8[4] == c8[5] && c8[6] == c8[7]);
  CHECK((ContinuationSplit(2, {1, 3, 3}) == V{0, 1, 1}));
  CHECK((ContinuationSplit(5, {3, 1}) == V{4, 1}));
  const auto adm = AdmitReservedKvBytes({{10, 10}, {5, 5}}, {1 << 20, 1 << 20}, 2, 64, 2);
  CHECK(adm.bytes_per_token_per_layer == 512);
  CHECK((adm.required_bytes_per_domain == std::vector<uint64_t>{20 * 512, 10 * 512}));
  CHECK(Throws<CapacityError>([] { AdmitReservedKvBytes({{10}}, {100}, 2, 64, 2); }));
  CHECK(Throws<CapacityError>([] { CapacityMbToBytes({kUnknownCapacity}); }));
  KvLedger led({100, 100});
  led.TryReserve(1, {60, 10});
  CHECK(Throws<CapacityError>([&] { led.TryReserve(2, {50, 10}); }));
  CHECK((led.FreeBytes() == std::vector<uint64_t>{40, 90}));
  CHECK((led.Release(1) == std::vector<uint64_t>{60, 10}));
  CHECK((led.Release(1) == std::vector<uint64_t>{0, 0}));
}

static void Schedule() {
  CHECK((FrozenKvAssigneeSchedule({1, 2, 3}, 75, 4).Counts() == V{1, 1, 2}));
  CHECK((FrozenKvAssigneeSchedule({1, 2, 3}, 75, 24).Counts() == V{4, 8, 12}));
  FrozenKvAssigneeSchedule s({1, 3, 2}, 41, 24);
  CHECK((s.Counts() == V{4, 12, 8}));
  CHECK((s.PerRankUnits(3, 0, 8, 3) == s.Counts()));
  CHECK(s.AssigneeFor(0, 3, 3) == -1 && s.AssigneeFor(8, 0, 3) == -1);
  CHECK(Throws<RingError>([] { FrozenKvAssigneeSchedule({0, 0}, 1, 4); }));
  // any prefix of the sequence stays within each rank's quota
  for (uint64_t rid = 0; rid < 19; ++rid) {
    FrozenKvAssigneeSchedule q({2, 5, 1, 4}, rid, 19);
    V used(4, 0);
    for (int64_t o = 0; o < 19; ++o) {
      const int64_t a = q.AssigneeFor(o, 0, 1);
      ++used[size_t(a)];
      for (size_t d = 0; d < 4; ++d) CHECK(used[d] <= q.Counts()[d]);
    }
  }
  const auto tab = AssigneeTable({1, 3, 2}, 41, 8, 3);
  for (int64_t t = 0; t < 8; ++t)
    for (int64_t l = 0; l < 3; ++l) CHECK(tab[size_t(t * 3 + l)] == s.AssigneeFor(t, l, 3));
  CHECK((StationaryLayerStarters(2, 7, 3) == V{2, 1, 0, 2, 1, 0, 2}));
}

static void Pages() {
  PageAllocator a(4, 128);
  const auto p = a.Alloc(3, 1);
  CHECK((p == V{0, 1, 2}) && a.FreePages() == 1 && a.OwnerOf(1) == 1 && a.OwnerOf(3) == -1);
  CHECK(Throws<CapacityError>([&] { a.Alloc(2, 2); }));
  a.Free({0, 1});
  a.Free({0});  // already free: ignored, never handed out twice
  CHECK(a.FreePages() == 3);
  const auto q = a.Alloc(3, 2);
  CHECK(a.FreePages() == 0 && a.OwnerOf(q[0]) == 2);
}

static void Scheduler() {
  BatchSchedulerCore s(2);
  CHECK(Throws<std::invalid_argument>([] { BatchSchedulerCore bad(0); }));
  const int producers = 4, per = 250;
  std::vector<std::thread> ts;
  for (int t = 0; t < producers; ++t)
    ts.emplace_back([&s, t] {
      for (int i = 0; i < per; ++i) s.Enqueue(uint64_t(t * per + i));
    });
  std::vector<uint64_t> seen;
  while (int64_t(seen.size()) < producers * per) {
    auto id = s.PopPending();
    if (!id) {
      s.WaitForWork(0.01);
      continue;
    }
    s.Activate(*id);
    CHECK(s.NumActive() <= 2);
    seen.push_back(*id);
    CHECK(s.Complete(*id) && !s.Complete(*id));
  }
  for (auto& t : ts) t.join();
  std::vector<int> count(size_t(producers * per), 0);
  for (uint64_t id : seen) ++count[size_t(id)];
  for (int c : count) CHECK(c == 1);
  s.Enqueue(7);
  s.Enqueue(8);
  s.Enqueue(9);
  auto a = s.PopPending();
  s.RequeueFront(*a);
  CHECK(s.PopPending().value() == 7 && s.Queued() == 2);
  s.Activate(7);
  s.Activate(8);
  CHECK(!s.HasCapacity() && !s.PopPending().has_value() && s.Queued() == 2);
  CHECK((s.Active() == std::vector<uint64_t>{7, 8}));
  s.Complete(7);
  CHECK(s.PopPending().value() == 8);
}

static Field I(int64_t v) {
  Field f;
  f.i = v;
  return f;
}
static Field Arr(V v) {
  Field f;
  f.a = std::move(v);
  return f;
}

static void Protocol() {
  // Prefill: request_id, prompt, chunks, strategy, horizon, tickets?, keep_kv
  Field strat;
  strat.s = "zigzag";
  Field none;
  none.present = false;
  std::vector<Field> prefill{I(5), Arr({9, 8, 7, 6}), Arr({3, 1}), strat, I(16), none, I(1), I(0)};
  const std::string fr = EncodeFrame(1, prefill);
  uint32_t payload;
  std::memcpy(&payload, fr.data(), 4);
  CHECK(payload == fr.size() - 4 && uint8_t(fr[4]) == kProtocolVersion && uint8_t(fr[5]) == 1);
  int type = 0;
  auto back = DecodeFrame(fr, &type);
  CHECK(type == 1 && back.size() == 8 && back[0].i == 5 && (back[1].a == V{9, 8, 7, 6}));
  CHECK(back[3].s == "zigzag" && !back[5].present && back[6].i == 1 && back[7].i == 0);
  // every truncation and any trailing byte is rejected
  for (size_t n = 0; n < fr.size(); ++n)
    CHECK(Throws<ProtocolError>([&] { DecodeFrame(fr.substr(0, n), &type); }));
  CHECK(Throws<ProtocolError>([&] { DecodeFrame(fr + "x", &type); }));
  std::string bad = fr;
  bad[4] = 2;
  CHECK(Throws<ProtocolError>([&] { DecodeFrame(bad, &type); }));
  bad[4] = char(kProtocolVersion);
  bad[5] = 42;
  CHECK(Throws<ProtocolError>([&] { DecodeFrame(bad, &type); }));
  // a count that points past the frame
  std::string lie = fr;
  const uint64_t huge = 1ull << 40;
  std::memcpy(&lie[6 + 8], &huge, 8);
  CHECK(Throws<ProtocolError>([&] { DecodeFrame(lie, &type); }));
  // pairs, optional token, error string, empty message
  back = DecodeFrame(EncodeFrame(66, {Arr({1, 10, 2, 20})}), &type);
  CHECK(type == 66 && (back[0].a == V{1, 10, 2, 20}));
  back = DecodeFrame(EncodeFrame(67, {I(3), none}), &type);
  CHECK(type == 67 && !back[1].present);
  Field msg;
  msg.s = "rank error";
  back = DecodeFrame(EncodeFrame(69, {I(4), msg}), &type);
  CHECK(back[1].s == "rank error");
  CHECK(DecodeFrame(EncodeFrame(8, {}), &type).empty() && type == 8);
  CHECK(Throws<ProtocolError>([&] { EncodeFrame(2, {I(1)}); }));
  CHECK(Throws<ProtocolError>([&] { EncodeFrame(99, {}); }));
  CHECK(Throws<ProtocolError>([&] { EncodeFrame(3, {Arr({1, 2, 3})}); }));
}

static void Oracle() {
  // the reference's seven uneven chunk / block cases (non-causal MHA) plus causal GQA layouts:
  // ring == full attention in double precision
  struct Case {
    V chunks, blocks;
    int64_t H, Hkv, D;
    bool causal;
    RingStrategy s;
  };
  const std::vector<Case> cases = {
      {{80, 48}, {16, 12}, 4, 4, 16, false, RingStrategy::kVanilla},
      {{64, 40, 56}, {32, 10, 14}, 3, 3, 24, false, RingStrategy::kVanilla},
      {{32, 64, 48, 48}, {7, 16, 11, 13}, 2, 2, 32, false, RingStrategy::kVanilla},
      {{512, 256, 256}, {128, 64, 64}, 8, 8, 64, false, RingStrategy::kVanilla},
      {{64}, {64}, 4, 4, 16, false, RingStrategy::kVanilla},
      {{16, 16}, {1, 1}, 2, 2, 8, false, RingStrategy::kVanilla},
      {{128}, {32}, 4, 4, 16, false, RingStrategy::kVanilla},
      {{250, 250, 50}, {64, 64, 64}, 8, 2, 32, true, RingStrategy::kZigzag},
      {{64, 32, 48, 16}, {16, 8, 16, 4}, 4, 1, 16, true, RingStrategy::kStriped},
  };
  std::mt19937_64 rng(42);
  std::normal_distribution<double> nd(0.0, 1.0);
  for (const auto& c : cases) {
    int64_t L = 0;
    for (int64_t x : c.chunks) L += x;
    std::vector<double> q(size_t(L * c.H * c.D)), k(size_t(L * c.Hkv * c.D)), v(k.size());
    for (auto* t : {&q, &k, &v})
      for (auto& x : *t) x = nd(rng);
    const auto full = FullAttentionF64(q, k, v, L, c.H, c.Hkv, c.D, c.causal);
    const auto pos = BuildDomainPositions(BuildAssignment(c.chunks, c.s), int64_t(c.chunks.size()));
    const auto ring = RingAttentionF64(q, k, v, L, c.H, c.Hkv, c.D, pos, c.blocks, c.causal);
    double err = 0.0;
    for (size_t i = 0; i < full.o.size(); ++i) err = std::max(err, std::fabs(full.o[i] - ring.o[i]));
    for (size_t i = 0; i < full.lse.size(); ++i) err = std::max(err, std::fabs(full.lse[i] - ring.lse[i]));
    CHECK(err < 1e-10);
  }
  CHECK(Throws<RingError>([] { FullAttentionF64({1.0}, {1.0}, {1.0}, 1, 2, 1, 1, false); }));
}

int main() {
  Layouts();
  Capacity();
  Schedule();
  Pages();
  Scheduler();
  Protocol();
  Oracle();
  std::printf("host_test ok (%d checks)\n", g_checks);
  return 0;
}
