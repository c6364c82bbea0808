// Memory layouts shared by the host runtime and the kernels.
//
// Paged, position-tagged KV arena (one per rank, allocated once by the domain runtime and
// exported to peers through CUDA IPC):
//     bf16 arena[layers][pages][2 (K, V)][Hkv][page][D]
// A request owns a list of pages (the same page ids for every layer) and a slot count; slot s of
// a request lives at page_table[s / page], row s % page. Each slot also carries the global
// position of its token (int32), so peers can place it in position order.
//
// Position-ordered staging buffer (per rank, double-buffered by layer parity, written by every
// rank's push and read by the attention kernel):
//     bf16 stage[2 (parity)][2 (K, V)][Hkv][Lcap][D]
//
// Flag region (per rank, uint64 words, exported through CUDA IPC):
//     [0, 64)    prefill kv_ready[src]     epoch when `src` finished pushing a layer
//     [64, 128)  prefill consumed[dst]     epoch when `dst` finished reading a layer
//     [128, 192) decode dec_ready[src]     epoch when `src` stored its (O, LSE) partial
//     [192]      decode step epoch counter (advanced on device once per decode step)
//     [200, 204) first-token broadcast: value / epoch pairs of two parities
//     [256, ...) counters for last-CTA-done signalling (uint32 pairs)
//
// Tile flags (per rank, after the flag region, exported with it): uint64
//     tflags[2 (parity)][tiles = ceil(Lcap / 128)][world]
// tflags[p][t][src] = epoch once `src` has stored all of its rows of KV tile t (positions
// [128 t, 128 t + 128)) of the layer step `epoch` into this rank's staging parity p. The
// overlapped ring attention waits on exactly the (tile, src) pairs it reads.
#pragma once

#include <stdint.h>

namespace hcp {

constexpr int kMaxRanks = 64;
constexpr int kFlagKvReady = 0;
constexpr int kFlagConsumed = 64;
constexpr int kFlagDecReady = 128;
constexpr int kFlagDecEpoch = 192;
constexpr int kFlagToken = 200;      // [value, epoch] x 2 parities
constexpr int kRingTile = 128;       // KV tile (positions) of the tile flags and the attention
constexpr int kFlagCounters = 256;   // uint32 counters start here (as uint64 index)
constexpr int kFlagWords = 1024;     // total uint64 words in the flag region

struct ArenaGeom {
  int layers;
  int pages;
  int page;   // tokens per page
  int hkv;
  int d;
  __host__ __device__ long head_stride() const { return long(page) * d; }
  __host__ __device__ long kv_stride() const { return long(hkv) * page * d; }
  __host__ __device__ long page_stride() const { return 2L * hkv * page * d; }
  __host__ __device__ long layer_stride() const { return long(pages) * page_stride(); }
  // element offset of (layer, page, kv, head, row)
  __host__ __device__ long offset(int layer, int pg, int kv, int h, int row) const {
    return long(layer) * layer_stride() + long(pg) * page_stride() + long(kv) * kv_stride() +
           long(h) * head_stride() + long(row) * d;
  }
};

}  // namespace hcp
