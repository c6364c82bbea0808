// Domain runtime implementation (see hcp/core/runtime.h).
#include "hcp/core/runtime.h"

#include <cstdio>
#include <cstring>

#include "../kernels/attn_fwd_sm100.h"
#include "../kernels/decode.h"
#include "../kernels/elementwise.h"
#include "../kernels/gemm_sm100.h"

namespace hcp {

namespace {
size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

Status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return Status::Ok();
  return Status(StatusCode::kCudaError, std::string(what) + ": " + cudaGetErrorString(e));
}
}  // namespace

DomainRuntime::~DomainRuntime() { Shutdown(); }

Status DomainRuntime::Init(const RuntimeConfig& cfg) {
  if (base_ != nullptr) return Status::InvalidArgument("runtime already initialised");
  if (cfg.world < 1 || cfg.world > kMaxRanks) return Status::InvalidArgument("world out of range");
  if (cfg.rank < 0 || cfg.rank >= cfg.world) return Status::InvalidArgument("rank out of range");
  if (cfg.geom.d != 64 && cfg.geom.d != 128) return Status::InvalidArgument("head_dim must be 64 or 128");
  if (cfg.geom.page <= 0 || cfg.geom.page % 128) return Status::InvalidArgument("page size must be a multiple of 128");
  if (cfg.geom.layers <= 0 || cfg.geom.pages <= 0 || cfg.geom.hkv <= 0)
    return Status::InvalidArgument("arena geometry must be positive");
  if (cfg.num_heads <= 0 || cfg.num_heads % cfg.geom.hkv) return Status::InvalidArgument("num_heads % hkv");
  cfg_ = cfg;
  auto st = cuda_status(cudaSetDevice(cfg.device), "cudaSetDevice");
  if (!st.ok()) return st;
  st = cuda_status(cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, cfg.device),
                   "cudaDeviceGetAttribute");
  if (!st.ok()) return st;
  off_flags_ = 0;
  size_t flags_bytes = size_t(kFlagWords) * sizeof(unsigned long long);
  off_tflags_ = align_up(off_flags_ + flags_bytes, 4096);
  const size_t tiles = (size_t(cfg.stage_cap) + kRingTile - 1) / kRingTile;
  tflag_parity_bytes_ = align_up(tiles * cfg.world * sizeof(unsigned long long), 256);
  off_gflags_ = align_up(off_tflags_ + 2 * tflag_parity_bytes_, 256);
  const size_t gflag_bytes = size_t(cfg.world) * cfg.max_batch * cfg.geom.hkv * sizeof(unsigned long long);
  off_aslot_ = align_up(off_gflags_ + gflag_bytes, 256);
  const size_t aslot_bytes = size_t(2) * cfg.world * cfg.max_batch * 2 * sizeof(unsigned long long);
  off_xslot_ = align_up(off_aslot_ + aslot_bytes, 4096);
  xslot_bytes_ = size_t(2) * cfg.world * cfg.max_batch * cfg.num_heads * (cfg.geom.d + 1) * sizeof(float);
  off_stage_ = align_up(off_xslot_ + xslot_bytes_, 4096);
  stage_parity_bytes_ = size_t(2) * cfg.geom.hkv * size_t(cfg.stage_cap) * cfg.geom.d * 2;
  stage_parity_bytes_ = align_up(stage_parity_bytes_, 4096);
  off_arena_ = align_up(off_stage_ + 2 * stage_parity_bytes_, 1 << 16);
  arena_bytes_ = size_t(cfg.geom.layer_stride()) * cfg.geom.layers * 2;
  region_bytes_ = align_up(off_arena_ + arena_bytes_, 1 << 21);
  void* p = nullptr;
  st = cuda_status(cudaMalloc(&p, region_bytes_), "cudaMalloc(shared region)");
  if (!st.ok()) return st;
  base_ = static_cast<uint8_t*>(p);
  st = cuda_status(cudaMemset(base_, 0, off_arena_), "cudaMemset(flags/xslot/stage)");
  if (!st.ok()) return st;
  void* q = nullptr;
  st = cuda_status(cudaMalloc(&q, 4096), "cudaMalloc(status)");
  if (!st.ok()) return st;
  status_ = static_cast<int*>(q);
  counters_ = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(q) + 1024);
  cudaMemset(q, 0, 4096);
  peer_base_.assign(cfg.world, nullptr);
  peer_opened_ipc_.assign(cfg.world, false);
  peer_base_[cfg.rank] = base_;
  if (cfg.world == 1) return BuildTables();
  return Status::Ok();
}

std::vector<uint8_t> DomainRuntime::ExportHandle() const {
  std::vector<uint8_t> out;
  if (base_ == nullptr) return out;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, base_) != cudaSuccess) return out;
  out.resize(sizeof(h));
  std::memcpy(out.data(), &h, sizeof(h));
  return out;
}

Status DomainRuntime::OpenPeers(const std::vector<std::vector<uint8_t>>& handles) {
  if (base_ == nullptr) return Status::InvalidArgument("runtime not initialised");
  if (int(handles.size()) != cfg_.world) return Status::InvalidArgument("need one handle per rank");
  cudaSetDevice(cfg_.device);
  for (int r = 0; r < cfg_.world; ++r) {
    if (r == cfg_.rank) continue;
    if (handles[r].size() != sizeof(cudaIpcMemHandle_t))
      return Status::InvalidArgument("bad IPC handle size for rank " + std::to_string(r));
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles[r].data(), sizeof(h));
    void* p = nullptr;
    auto st = cuda_status(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess),
                          "cudaIpcOpenMemHandle");
    if (!st.ok()) return st;
    peer_base_[r] = static_cast<uint8_t*>(p);
    peer_opened_ipc_[r] = true;
  }
  return BuildTables();
}

Status DomainRuntime::OpenPeersLocal(const std::vector<DomainRuntime*>& peers) {
  if (base_ == nullptr) return Status::InvalidArgument("runtime not initialised");
  if (int(peers.size()) != cfg_.world) return Status::InvalidArgument("need one runtime per rank");
  for (int r = 0; r < cfg_.world; ++r) {
    if (peers[r] == nullptr || !peers[r]->initialized())
      return Status::InvalidArgument("peer runtime not initialised");
    if (peers[r]->region_bytes() != region_bytes_) return Status::InvalidArgument("peer geometry mismatch");
    peer_base_[r] = peers[r]->base();
  }
  return BuildTables();
}

Status DomainRuntime::BuildTables() {
  const int n = cfg_.world;
  std::vector<void*> st0(n), st1(n);
  std::vector<unsigned long long*> ready(n), consumed(n), dready(n), tf0(n), tf1(n), tok(n), gf(n),
      as(n);
  std::vector<float*> xs(n);
  for (int r = 0; r < n; ++r) {
    uint8_t* b = peer_base_[r];
    if (b == nullptr) return Status::Internal("peer " + std::to_string(r) + " not mapped");
    st0[r] = b + off_stage_;
    st1[r] = b + off_stage_ + stage_parity_bytes_;
    auto* fl = reinterpret_cast<unsigned long long*>(b + off_flags_);
    ready[r] = fl + kFlagKvReady + cfg_.rank;
    consumed[r] = fl + kFlagConsumed + cfg_.rank;
    dready[r] = fl + kFlagDecReady + cfg_.rank;
    tok[r] = fl + kFlagToken;
    gf[r] = reinterpret_cast<unsigned long long*>(b + off_gflags_);
    as[r] = reinterpret_cast<unsigned long long*>(b + off_aslot_);
    tf0[r] = reinterpret_cast<unsigned long long*>(b + off_tflags_);
    tf1[r] = reinterpret_cast<unsigned long long*>(b + off_tflags_ + tflag_parity_bytes_);
    xs[r] = reinterpret_cast<float*>(b + off_xslot_);
  }
  auto alloc_copy = [&](void** dst, const void* src, size_t bytes) -> Status {
    if (*dst == nullptr) {
      auto s = cuda_status(cudaMalloc(dst, bytes), "cudaMalloc(table)");
      if (!s.ok()) return s;
    }
    return cuda_status(cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice), "cudaMemcpy(table)");
  };
  const size_t pb = sizeof(void*) * n;
  Status s;
  if (!(s = alloc_copy(reinterpret_cast<void**>(&stage_tab_[0]), st0.data(), pb)).ok()) return s;
  if (!(s = alloc_copy(reinterpret_cast<void**>(&stage_tab_[1]), st1.data(), pb)).ok()) return s;
  if (!(s = alloc_copy(reinterpret_cast<void**>(&kv_ready_tab_), ready.data(), pb)).ok()) return s;
  if (!(s = alloc_copy(reinterpret_cast<void**>(&consumed_tab_), consumed.data(), pb)).ok()) return s;
  if (!(s = alloc_copy(reinterpret_cast<void**>(&dec_ready_tab_), dready.data(), pb)).ok()) return s;
  if (!(s = alloc_copy(reinterpret_cast<void**>(&xslot_tab_), xs.data(), pb)).ok()) return s;
  if (!(s = alloc_copy(reinterpret_cast<void**>(&tflag_tab_[0]), tf0.data(), pb)).ok()) return s;
  if (!(s = alloc_copy(reinterpret_cast<void**>(&tflag_tab_[1]), tf1.data(), pb)).ok()) return s;
  if (!(s = alloc_copy(reinterpret_cast<void**>(&token_tab_), tok.data(), pb)).ok()) return s;
  if (!(s = alloc_copy(reinterpret_cast<void**>(&gflag_tab_), gf.data(), pb)).ok()) return s;
  if (!(s = alloc_copy(reinterpret_cast<void**>(&aslot_tab_), as.data(), pb)).ok()) return s;
  return Status::Ok();
}

Status DomainRuntime::RunRingAttentionLayer(const RingLayerArgs& a, cudaStream_t stream) {
  Status s = PushLayer(a, stream);
  if (!s.ok()) return s;
  return AttendLayer(a, stream);
}

Status DomainRuntime::PushLayer(const RingLayerArgs& a, cudaStream_t stream) {
  if (base_ == nullptr || stage_tab_[0] == nullptr) return Status::InvalidArgument("runtime not ready");
  if (a.L > cfg_.stage_cap) return Status::InvalidArgument("context longer than the staging capacity");
  if (a.H != cfg_.num_heads) return Status::InvalidArgument("head count mismatch");
  const int parity = int(a.epoch & 1ull);
  const int n = cfg_.world;
  unsigned long long* fl = flags();
  const bool overlap = a.tile_src != nullptr && n > 1;
  if (overlap && a.existing_n > 0)
    return Status::InvalidArgument("continuation segments use the serial ring (no tile sources)");
  // overlapped ring: this rank's rows go to its own staging buffer only (the attention kernel
  // pushes them to the peers); nothing to wait for, only this rank reads its own buffer
  void* const* stage_dst = overlap ? stage_tab_[parity] + cfg_.rank : stage_tab_[parity];
  const int n_dst = overlap ? 1 : n;
  // 1. the staging parity we write must have been released by every rank (epoch - 2 consumed)
  if (!overlap && n > 1 && a.epoch > 2) {
    const char* e = ew::wait_consumed(fl + kFlagConsumed, n, a.epoch - 2, cfg_.peer_wait_budget_ns,
                                      status_, stream);
    if (e) return Status::Internal(e);
  }
  // 2a. continuation: re-push this rank's already-stored rows of the session
  if (a.existing_n > 0) {
    ew::StagePushArgs sp{};
    sp.arena = static_cast<const __nv_bfloat16*>(arena());
    sp.geom = cfg_.geom;
    sp.layer = a.layer;
    sp.page_table = a.page_table;
    sp.slot_pos = a.existing_slot_pos;
    sp.n = a.existing_n;
    sp.stage_ptrs = stage_tab_[parity];
    sp.n_stage = n;
    sp.stage_cap = cfg_.stage_cap;
    const char* e = ew::stage_push(sp, stream);
    if (e) return Status::Internal(e);
  }
  // 2. RoPE + Q write + arena write + push K/V to every rank's staging buffer, then kv_ready;
  //    fused into the projection GEMM's epilogue when the layer input is given
  if (a.x != nullptr && a.T > 0) {
    gemm::GemmArgs g{};
    g.A = static_cast<const __nv_bfloat16*>(a.x);
    g.lda = a.ldx;
    g.B = static_cast<const __nv_bfloat16*>(a.w_qkv);
    g.ldb = a.hidden;
    g.M = a.T;
    g.N = (a.H + 2 * cfg_.geom.hkv) * cfg_.geom.d;
    g.K = a.hidden;
    g.bias = static_cast<const __nv_bfloat16*>(a.b_qkv);
    g.status = status_;
    g.num_sms = num_sms_;
    gemm::QkvPushArgs q{};
    q.pos = a.pos;
    q.cos_t = a.cos_t;
    q.sin_t = a.sin_t;
    q.max_pos = a.max_pos;
    q.H = a.H;
    q.Hkv = cfg_.geom.hkv;
    q.D = cfg_.geom.d;
    q.q_out = static_cast<__nv_bfloat16*>(a.q_out);
    q.arena = a.page_table ? static_cast<__nv_bfloat16*>(arena()) : nullptr;
    q.geom = cfg_.geom;
    q.layer = a.layer;
    q.page_table = a.page_table;
    q.slot_base = a.slot_base;
    q.slot_cap = a.slot_cap;
    q.stage_ptrs = stage_dst;
    q.n_stage = n_dst;
    q.stage_cap = cfg_.stage_cap;
    q.done_counter = (n > 1 && !overlap) ? counters_ : nullptr;
    q.ready_ptrs = kv_ready_tab_;
    q.epoch = a.epoch;
    const char* e = gemm::gemm_qkv_push(g, q, stream);
    if (e) return Status::Internal(e);
    return Status::Ok();
  }
  ew::QkvPrefillArgs q{};
  q.qkv = static_cast<const __nv_bfloat16*>(a.qkv);
  q.ld_qkv = a.ld_qkv;
  q.pos = a.pos;
  q.cos_t = a.cos_t;
  q.sin_t = a.sin_t;
  q.max_pos = a.max_pos;
  q.T = a.T;
  q.H = a.H;
  q.Hkv = cfg_.geom.hkv;
  q.D = cfg_.geom.d;
  q.q_out = static_cast<__nv_bfloat16*>(a.q_out);
  q.arena = a.page_table ? static_cast<__nv_bfloat16*>(arena()) : nullptr;
  q.geom = cfg_.geom;
  q.layer = a.layer;
  q.page_table = a.page_table;
  q.slot_base = a.slot_base;
  q.slot_cap = a.slot_cap;
  q.stage_ptrs = stage_dst;
  q.n_stage = n_dst;
  q.stage_cap = cfg_.stage_cap;
  q.done_counter = (n > 1 && !overlap) ? counters_ : nullptr;
  q.ready_ptrs = kv_ready_tab_;
  q.epoch = a.epoch;
  q.status = status_;
  if (a.T > 0) {
    const char* e = ew::qkv_prefill(q, stream);
    if (e) return Status::Internal(e);
  } else if (n > 1 && !overlap) {
    // a rank without tokens still has to publish its (empty) contribution
    const char* e = ew::signal_peers(kv_ready_tab_, n, a.epoch, stream);
    if (e) return Status::Internal(e);
  }
  return Status::Ok();
}

Status DomainRuntime::AttendLayer(const RingLayerArgs& a, cudaStream_t stream) {
  if (base_ == nullptr || stage_tab_[0] == nullptr) return Status::InvalidArgument("runtime not ready");
  const int parity = int(a.epoch & 1ull);
  const int n = cfg_.world;
  unsigned long long* fl = flags();
  // 3. ring attention over the position-ordered staging buffer; remote tiles wait for kv_ready
  if (a.T > 0) {
    attn::AttnArgs at{};
    at.Q = static_cast<const __nv_bfloat16*>(a.q_out);
    auto* sk = static_cast<const __nv_bfloat16*>(stage(parity));
    at.K = sk;
    at.V = sk + size_t(cfg_.geom.hkv) * cfg_.stage_cap * cfg_.geom.d;
    at.O = static_cast<__nv_bfloat16*>(a.o_out);
    at.lse = a.lse_out;
    at.q_pos = a.pos;
    at.T = a.T;
    at.H = a.H;
    at.Hkv = cfg_.geom.hkv;
    at.D = cfg_.geom.d;
    at.L = a.L;
    at.kv_head_stride = long(cfg_.stage_cap) * cfg_.geom.d;
    at.scale = a.scale;
    at.causal = a.causal;
    at.wait_budget_ns = cfg_.peer_wait_budget_ns;
    at.status = status_;
    if (a.tile_src != nullptr && n > 1) {
      // overlapped ring: the kernel pushes this rank's rows, waits per remote tile and releases
      // the parity itself (no barrier or signal launches)
      attn::RingArgs& rg = at.ring;
      rg.world = n;
      rg.my_rank = cfg_.rank;
      rg.epoch = a.epoch;
      rg.tile_src = a.tile_src;
      rg.tile_flags = tile_flags(parity);
      rg.push_tiles = a.push_tiles;
      rg.n_push = a.n_push;
      rg.own_stage = sk;
      rg.stage_ptrs = stage_tab_[parity];
      rg.tflag_ptrs = tflag_tab_[parity];
      rg.consumed = fl + kFlagConsumed;
      rg.consumed_ptrs = consumed_tab_;
      rg.counters = counters_ + 16;
      rg.stage_cap = cfg_.stage_cap;
      const char* e = attn::attn_fwd(at, stream);
      if (e) return Status::Internal(e);
      return Status::Ok();
    }
    if (n > 1) {
      // all ranks' pushes must have landed before the kernel reads remote rows
      const char* e = ew::wait_consumed(fl + kFlagKvReady, n, a.epoch, cfg_.peer_wait_budget_ns,
                                        status_, stream);
      if (e) return Status::Internal(e);
    }
    const char* e = attn::attn_fwd(at, stream);
    if (e) return Status::Internal(e);
  }
  // 4. tell every rank we are done reading this parity
  if (n > 1) {
    const char* e = ew::signal_peers(consumed_tab_, n, a.epoch, stream);
    if (e) return Status::Internal(e);
  }
  return Status::Ok();
}

Status DomainRuntime::PublishTiles(const int* push_tiles, int n_push, uint64_t epoch,
                                   cudaStream_t stream) {
  if (base_ == nullptr || stage_tab_[0] == nullptr) return Status::InvalidArgument("runtime not ready");
  if (n_push == 0) return Status::Ok();
  const char* e = ew::publish_tiles(push_tiles, n_push, tflag_tab_[int(epoch & 1ull)], cfg_.world,
                                    cfg_.rank, epoch, stream);
  return e ? Status::Internal(e) : Status::Ok();
}

Status DomainRuntime::BroadcastToken(long long* tok, int src, uint64_t epoch, cudaStream_t stream) {
  if (base_ == nullptr || token_tab_ == nullptr) return Status::InvalidArgument("runtime not ready");
  if (src < 0 || src >= cfg_.world) return Status::InvalidArgument("token source rank out of range");
  if (cfg_.world == 1) return Status::Ok();
  const char* e = ew::token_bcast(tok, token_tab_, flags() + kFlagToken, cfg_.world,
                                  src == cfg_.rank, epoch, cfg_.peer_wait_budget_ns, status_, stream);
  return e ? Status::Internal(e) : Status::Ok();
}

Status DomainRuntime::ArgmaxExchange(const unsigned long long* local, int B, int* tok32,
                                     long long* tok64, const unsigned long long* epoch_src,
                                     cudaStream_t stream) {
  if (base_ == nullptr || aslot_tab_ == nullptr) return Status::InvalidArgument("runtime not ready");
  if (B < 1 || B > cfg_.max_batch) return Status::InvalidArgument("argmax exchange: rows out of range");
  dec::ArgmaxXchgArgs a{};
  a.local = local;
  a.B = B;
  a.slot_ptrs = aslot_tab_;
  a.own_slots = argmax_slots();
  a.world = cfg_.world;
  a.my_rank = cfg_.rank;
  a.max_batch = cfg_.max_batch;
  a.epoch_src = epoch_src;
  a.tok32 = tok32;
  a.tok64 = tok64;
  a.budget_ns = cfg_.peer_wait_budget_ns;
  a.status = status_;
  const char* e = dec::argmax_exchange(a, stream);
  return e ? Status::Internal(e) : Status::Ok();
}

Status DomainRuntime::CheckDevice(cudaStream_t stream) {
  if (status_ == nullptr) return Status::Ok();
  auto st = cuda_status(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
  if (!st.ok()) return st;
  int h[kStatusWords];
  st = cuda_status(cudaMemcpy(h, status_, sizeof(h), cudaMemcpyDeviceToHost), "status read");
  if (!st.ok()) return st;
  if (h[0] == 0) return Status::Ok();
  cudaMemset(status_, 0, sizeof(h));
  return Status(static_cast<StatusCode>(h[0]), "device error at site " + std::to_string(h[1]) +
                                                   " (info " + std::to_string(h[2]) + ", " +
                                                   std::to_string(h[3]) + ")");
}

Status DomainRuntime::Shutdown() {
  if (base_ == nullptr) return Status::Ok();
  cudaSetDevice(cfg_.device);
  cudaDeviceSynchronize();
  for (int r = 0; r < int(peer_base_.size()); ++r) {
    if (peer_opened_ipc_[r] && peer_base_[r]) cudaIpcCloseMemHandle(peer_base_[r]);
  }
  peer_base_.clear();
  peer_opened_ipc_.clear();
  for (void* t : {static_cast<void*>(stage_tab_[0]), static_cast<void*>(stage_tab_[1]),
                  static_cast<void*>(kv_ready_tab_), static_cast<void*>(consumed_tab_),
                  static_cast<void*>(dec_ready_tab_), static_cast<void*>(xslot_tab_),
                  static_cast<void*>(tflag_tab_[0]), static_cast<void*>(tflag_tab_[1]),
                  static_cast<void*>(token_tab_), static_cast<void*>(gflag_tab_),
                  static_cast<void*>(aslot_tab_)})
    if (t) cudaFree(t);
  stage_tab_[0] = stage_tab_[1] = nullptr;
  tflag_tab_[0] = tflag_tab_[1] = nullptr;
  token_tab_ = nullptr;
  gflag_tab_ = nullptr;
  aslot_tab_ = nullptr;
  kv_ready_tab_ = consumed_tab_ = dec_ready_tab_ = nullptr;
  xslot_tab_ = nullptr;
  if (status_) cudaFree(status_);
  status_ = nullptr;
  counters_ = nullptr;
  cudaFree(base_);
  base_ = nullptr;
  return Status::Ok();
}

}  // namespace hcp
