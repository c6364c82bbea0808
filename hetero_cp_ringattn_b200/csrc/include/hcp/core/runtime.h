// Domain runtime: owns one rank's device memory for context-parallel inference and its NVLink
// peer mappings.
//
// Parity: the reference's RingAttnRuntime interface (include/hcp_ringattn/core/
// ringattn_runtime.h:13-28: Init / RunRingAttentionLayer / Shutdown) whose only implementation
// is a no-op validator (src/ringattn_runtime.cc:10-70). Here Init binds the GPU and allocates
// the shared region, OpenPeers maps every peer's region through CUDA IPC, and
// RunRingAttentionLayer launches the fused KV push + ring attention kernels for one layer.
//
// Shared region (one cudaMalloc, exported with one IPC handle; identical offsets on every rank):
//   flags     uint64[kFlagWords]                           (kv_ready / consumed / dec_ready / ...)
//   tflags    uint64[2][ceil(stage_cap / 128)][world]      per-(KV tile, source rank) ready epochs
//   gflags    uint64[world][max_batch][Hkv]                decode (O, LSE) per-(source, row, KV head)
//   aslot     uint64[2][world][max_batch][2]               greedy argmax exchange (value, epoch)
//   xslot     fp32 [2][world][max_batch][H][D+1]          decode (O, LSE) exchange slots
//   stage     bf16 [2 parity][2 K/V][Hkv][stage_cap][D]   position-ordered prefill KV
//   arena     bf16 [layers][pages][2][Hkv][page][D]       paged KV cache shard
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "hcp/core/status.h"
#include "hcp/core/types.h"
#include "../../../kernels/kv_layout.h"

namespace hcp {

struct RuntimeConfig {
  int rank = 0;
  int world = 1;
  int device = 0;
  ArenaGeom geom{};       // layers, pages, page, hkv, d
  int num_heads = 0;      // H (decode exchange slot width)
  int stage_cap = 0;      // staging capacity in positions (max prompt / context length)
  int max_batch = 8;      // decode rows
  int num_sms = 148;
  uint64_t peer_wait_budget_ns = 5000000000ull;
};

struct RingLayerArgs {
  // projection output [T, (H + 2 Hkv) D] (q | k | v, bias already added)
  const void* qkv = nullptr;
  long ld_qkv = 0;
  const int* pos = nullptr;         // [T] global positions of this rank's tokens
  const float* cos_t = nullptr;     // [max_pos, D/2]
  const float* sin_t = nullptr;
  int max_pos = 0;
  int T = 0;
  int H = 0;
  int layer = 0;
  const int* page_table = nullptr;  // this request's pages (same ids for all layers)
  int slot_base = 0;
  int slot_cap = 0;
  int L = 0;                        // total context length (positions 0..L-1)
  float scale = 0.f;
  int causal = 1;
  void* q_out = nullptr;            // [T, H, D] scratch
  void* o_out = nullptr;            // [T, H, D]
  float* lse_out = nullptr;         // [H, T] (optional)
  uint64_t epoch = 0;               // strictly increasing per layer step (same on all ranks)
  // session continuation: already-stored slots [0, existing_n) of this layer to re-push
  const int* existing_slot_pos = nullptr;
  int existing_n = 0;
  // fused projection (optional): with x set, PushLayer computes the projection x w_qkv^T
  // (+ b_qkv) with the tcgen05 GEMM whose epilogue rotates, writes Q and pushes K/V, and `qkv`
  // is not read
  const void* x = nullptr;          // [T, hidden] bf16, the normalised layer input
  long ldx = 0;
  const void* w_qkv = nullptr;      // [(H + 2 Hkv) D, hidden] bf16
  const void* b_qkv = nullptr;      // optional [(H + 2 Hkv) D] bias
  int hidden = 0;
  // overlapped ring (context-parallel prefill, tile_src set): PushLayer writes only this rank's
  // own staging buffer, and AttendLayer's attention kernel pushes the rows to the peers itself
  // and waits per KV tile. Unset: serial ring (every row pushed and waited for before the
  // attention launch), which continuation segments (existing_n > 0) always use.
  const unsigned long long* tile_src = nullptr;  // [ceil(L / 128)] bitmask of ranks per tile
  const int* push_tiles = nullptr;  // [n_push][3] (tile, first, end) rows of `pos` per own tile
  int n_push = 0;
};

class DomainRuntime {
 public:
  DomainRuntime() = default;
  ~DomainRuntime();
  DomainRuntime(const DomainRuntime&) = delete;
  DomainRuntime& operator=(const DomainRuntime&) = delete;

  Status Init(const RuntimeConfig& cfg);
  // CUDA IPC handle of the shared region (64 bytes).
  std::vector<uint8_t> ExportHandle() const;
  // handles[r] for every rank r (own entry ignored).
  Status OpenPeers(const std::vector<std::vector<uint8_t>>& handles);
  // Emulated peers inside one process (tests): peers[r] are other runtimes on the same GPU.
  Status OpenPeersLocal(const std::vector<DomainRuntime*>& peers);
  // PushLayer: RoPE + KV write + P2P push of this rank's K/V into every rank's staging buffer.
  // AttendLayer: wait (bounded) for every rank's push, run ring attention, release the buffer.
  // RunRingAttentionLayer = PushLayer + AttendLayer. Emulated multi-rank runs on one GPU call
  // PushLayer for every rank before any AttendLayer, so no launch ever waits on a later one.
  Status RunRingAttentionLayer(const RingLayerArgs& a, cudaStream_t stream);
  Status PushLayer(const RingLayerArgs& a, cudaStream_t stream);
  Status AttendLayer(const RingLayerArgs& a, cudaStream_t stream);
  // Marks this rank's own tiles `push_tiles[k][0]` of the layer step `epoch` as present on every
  // rank (tile flags), for rows already stored everywhere by a serial push (tests emulating
  // several ranks on one GPU, where no kernel may wait on another launch).
  Status PublishTiles(const int* push_tiles, int n_push, uint64_t epoch, cudaStream_t stream);
  // First token of a prefill: rank `src` stores the int64 at `tok` into every rank's token slot
  // (value, then a release of `epoch`); every other rank waits (bounded) for `epoch` in its own
  // slot and copies the value into `tok`. All on the device, no host round trip.
  Status BroadcastToken(long long* tok, int src, uint64_t epoch, cudaStream_t stream);
  // Greedy decode with the LM head split over the vocabulary: `local` [B] holds this rank's packed
  // (value, index) maxima; the tokens of the whole vocabulary's argmax go to tok32 / tok64 [B]
  // (either may be null) on every rank. epoch = *epoch_src, the decode step counter (>= 1, the
  // same on every rank); the slots are double-buffered on its parity.
  Status ArgmaxExchange(const unsigned long long* local, int B, int* tok32, long long* tok64,
                        const unsigned long long* epoch_src, cudaStream_t stream);
  Status Shutdown();

  // Reads and clears the device status words (synchronises the given stream first).
  Status CheckDevice(cudaStream_t stream);

  const RuntimeConfig& config() const { return cfg_; }
  bool initialized() const { return base_ != nullptr; }
  uint8_t* base() const { return base_; }
  size_t region_bytes() const { return region_bytes_; }
  unsigned long long* flags() const { return reinterpret_cast<unsigned long long*>(base_ + off_flags_); }
  unsigned long long* group_flags() const {
    return reinterpret_cast<unsigned long long*>(base_ + off_gflags_);
  }
  unsigned long long* const* group_flag_table() const { return gflag_tab_; }
  unsigned long long* argmax_slots() const {
    return reinterpret_cast<unsigned long long*>(base_ + off_aslot_);
  }
  unsigned long long* tile_flags(int parity) const {
    return reinterpret_cast<unsigned long long*>(base_ + off_tflags_ + size_t(parity) * tflag_parity_bytes_);
  }
  float* xslot() const { return reinterpret_cast<float*>(base_ + off_xslot_); }
  void* stage(int parity) const { return base_ + off_stage_ + size_t(parity) * stage_parity_bytes_; }
  void* arena() const { return base_ + off_arena_; }
  size_t arena_bytes() const { return arena_bytes_; }
  size_t stage_parity_bytes() const { return stage_parity_bytes_; }
  size_t xslot_bytes() const { return xslot_bytes_; }
  int* status() const { return status_; }
  unsigned int* counters() const { return counters_; }
  // device pointer tables (arrays in device memory, indexed by rank)
  void* const* stage_table(int parity) const { return stage_tab_[parity]; }
  unsigned long long* const* kv_ready_table() const { return kv_ready_tab_; }
  unsigned long long* const* consumed_table() const { return consumed_tab_; }
  unsigned long long* const* dec_ready_table() const { return dec_ready_tab_; }
  float* const* xslot_table() const { return xslot_tab_; }
  // host copies of peer region bases (index = rank)
  const std::vector<uint8_t*>& peer_bases() const { return peer_base_; }

 private:
  Status BuildTables();

  RuntimeConfig cfg_{};
  uint8_t* base_ = nullptr;
  size_t region_bytes_ = 0;
  size_t off_flags_ = 0, off_tflags_ = 0, off_gflags_ = 0, off_aslot_ = 0, off_xslot_ = 0,
         off_stage_ = 0, off_arena_ = 0;
  size_t tflag_parity_bytes_ = 0;
  size_t xslot_bytes_ = 0, stage_parity_bytes_ = 0, arena_bytes_ = 0;
  int* status_ = nullptr;            // kStatusWords int32
  unsigned int* counters_ = nullptr; // 64 uint32 (last-CTA-done counters)
  int num_sms_ = 0;
  void** stage_tab_[2] = {nullptr, nullptr};
  unsigned long long** kv_ready_tab_ = nullptr;
  unsigned long long** consumed_tab_ = nullptr;
  unsigned long long** dec_ready_tab_ = nullptr;
  unsigned long long** tflag_tab_[2] = {nullptr, nullptr};
  unsigned long long** token_tab_ = nullptr;
  unsigned long long** gflag_tab_ = nullptr;
  unsigned long long** aslot_tab_ = nullptr;
  float** xslot_tab_ = nullptr;
  std::vector<uint8_t*> peer_base_;
  std::vector<bool> peer_opened_ipc_;
};

}  // namespace hcp
