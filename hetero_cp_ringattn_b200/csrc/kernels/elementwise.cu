// Memory-bound kernels of the model: token embedding, RMSNorm, the prefill QKV post-processing
// (RoPE at absolute positions, Q write, KV write into the local paged arena and P2P push into
// every rank's position-ordered staging buffer), the decode QKV post-processing (RoPE, Q write,
// KV append on the owner rank), and the decode argmax reset.
//
// Parity:
//   * RMSNorm: rust/src/model/layers/norm.rs:31-34 (fp32 statistics, HF rounding order).
//   * RoPE: rust/src/model/layers/rotary.rs:57-159 (rotate-half, absolute position ids,
//     cos/sin table indexed by position).
//   * KV cache update: rust/src/model/cache.rs:83-97 and self_driving.rs:180-228 (slab copy at
//     a reserved offset); the reference's per-step `cat` and GQA `repeat_kv` (ring.rs:1962-1984)
//     are gone: the arena is paged and kernels index KV heads directly.
//   * KV ring send (ring.rs:1085-1092, 1200-1204; wire format quic.rs:924-1010): replaced by
//     bf16 P2P stores from this kernel into the peers' staging buffers over NVLink, followed by a
//     release flag per peer (last-CTA-done), instead of host-staged f32 QUIC frames.
#include "common.cuh"
#include "elementwise.h"
#include "launch.h"
#include "kv_layout.h"

namespace hcp {
namespace ew {

using namespace hcp::dev;

// ----------------------------------------------------------------------------- embedding
__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ W,
                                 __nv_bfloat16* __restrict__ out, int T, int hidden, int vocab,
                                 int* status) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  if (t >= T) return;
  int id = ids[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) report_error(status, int(StatusCode::kOutOfBounds), 301, id, t);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(W + (long)id * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out + (long)t * hidden);
  for (int i = threadIdx.x; i < hidden / 8; i += blockDim.x) dst[i] = src[i];
}

// ----------------------------------------------------------------------------- rmsnorm
// one warp per row; hidden % 256 == 0 (8 bf16 per lane per step)
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                               __nv_bfloat16* __restrict__ y, int T, int hidden, long ldx,
                               long ldy, float eps) {
  const int warps = blockDim.x / 32;
  const int row = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= T) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (long)row * ldx);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + (long)row * ldy);
  const int nvec = hidden / 8;
  float ss = 0.f;
  for (int i = lane; i < nvec; i += 32) {
    uint4 v = xr[i];
    uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a = bf16_lo(vv[j]), b = bf16_hi(vv[j]);
      ss += a * a + b * b;
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / float(hidden) + eps);
  for (int i = lane; i < nvec; i += 32) {
    uint4 v = xr[i];
    uint4 ww = wr[i];
    uint32_t vv[4] = {v.x, v.y, v.z, v.w};
    uint32_t wv[4] = {ww.x, ww.y, ww.z, ww.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // HF order: normalise in fp32, round to bf16, then scale by the bf16 weight
      float a = __bfloat162float(__float2bfloat16(bf16_lo(vv[j]) * r)) * bf16_lo(wv[j]);
      float b = __bfloat162float(__float2bfloat16(bf16_hi(vv[j]) * r)) * bf16_hi(wv[j]);
      o[j] = pack_bf16x2(a, b);
    }
    yr[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ----------------------------------------------------------------------------- prefill QKV post
// One CTA per token: RoPE(q), RoPE(k) at the token's global position; q -> Qout[T,H,D];
// k, v -> local arena slot (slot_base + t) and -> every rank's staging buffer row `pos`.
__global__ void qkv_prefill_kernel(QkvPrefillArgs a) {
  extern __shared__ float sm[];  // [(H + Hkv) * D] rotated q/k (fp32)
  const int t = blockIdx.x;
  if (t >= a.T) return;
  const int D = a.D, H = a.H, Hkv = a.Hkv, half = D / 2;
  const int pos = a.pos[t];
  const __nv_bfloat16* row = a.qkv + (long)t * a.ld_qkv;
  const bool pos_ok = pos >= 0 && pos < a.max_pos;
  if (!pos_ok && threadIdx.x == 0) report_error(a.status, int(StatusCode::kOutOfBounds), 311, pos, t);
  // rotate q and k heads (pairs i, i + D/2)
  const int n_pairs = (H + Hkv) * half;
  for (int i = threadIdx.x; i < n_pairs; i += blockDim.x) {
    const int hh = i / half, j = i % half;
    const int col = hh * D + j;  // q heads then k heads are contiguous in the qkv row
    const float x1 = __bfloat162float(row[col]);
    const float x2 = __bfloat162float(row[col + half]);
    const float c = pos_ok ? a.cos_t[(long)pos * half + j] : 1.f;
    const float s = pos_ok ? a.sin_t[(long)pos * half + j] : 0.f;
    sm[hh * D + j] = x1 * c - x2 * s;
    sm[hh * D + j + half] = x2 * c + x1 * s;
  }
  __syncthreads();
  // q out: [T, H, D] bf16 (vectorised by 8)
  const int qvec = H * D / 8;
  uint4* qdst = reinterpret_cast<uint4*>(a.q_out + (long)t * H * D);
  for (int i = threadIdx.x; i < qvec; i += blockDim.x) {
    const float* s = sm + i * 8;
    qdst[i] = make_uint4(pack_bf16x2(s[0], s[1]), pack_bf16x2(s[2], s[3]),
                         pack_bf16x2(s[4], s[5]), pack_bf16x2(s[6], s[7]));
  }
  // k / v rows, 8 elements per vector: kvvec = 2 * Hkv * D / 8
  const int dvec = D / 8;
  const int kvvec = 2 * Hkv * dvec;
  const int slot = a.slot_base + t;
  const bool arena_ok = a.arena != nullptr && slot >= 0 && slot < a.slot_cap;
  int page = -1;
  if (a.arena != nullptr) {
    if (arena_ok) page = a.page_table[slot / a.geom.page];
    else if (threadIdx.x == 0) report_error(a.status, int(StatusCode::kOutOfBounds), 312, slot, t);
  }
  for (int i = threadIdx.x; i < kvvec; i += blockDim.x) {
    const int kv = i / (Hkv * dvec);
    const int rem = i % (Hkv * dvec);
    const int h = rem / dvec, e = rem % dvec;
    uint4 val;
    if (kv == 0) {
      const float* s = sm + (H + h) * D + e * 8;
      val = make_uint4(pack_bf16x2(s[0], s[1]), pack_bf16x2(s[2], s[3]),
                       pack_bf16x2(s[4], s[5]), pack_bf16x2(s[6], s[7]));
    } else {
      val = *reinterpret_cast<const uint4*>(row + (H + Hkv) * D + h * D + e * 8);
    }
    if (page >= 0) {
      __nv_bfloat16* dst = a.arena + a.geom.offset(a.layer, page, kv, h, slot % a.geom.page) + e * 8;
      *reinterpret_cast<uint4*>(dst) = val;
    }
    if (pos_ok && pos < a.stage_cap) {
      const long soff = ((long)(kv * Hkv + h) * a.stage_cap + pos) * D + e * 8;
      for (int r = 0; r < a.n_stage; ++r) {
        __nv_bfloat16* sb = reinterpret_cast<__nv_bfloat16*>(a.stage_ptrs[r]);
        *reinterpret_cast<uint4*>(sb + soff) = val;
      }
    }
  }
  // last-CTA-done: once every CTA's stores are visible system-wide, publish the epoch to every
  // rank's kv_ready[my_rank] (P2P release store).
  if (a.done_counter != nullptr) {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      const unsigned prev = atomicAdd(a.done_counter, 1u);
      if (prev == gridDim.x - 1) {
        __threadfence_system();
        for (int r = 0; r < a.n_stage; ++r) st_release_sys(a.ready_ptrs[r], a.epoch);
        *a.done_counter = 0;
      }
    }
  }
}

// Re-push rows already stored in the local arena (slots [0, n) of `layer`, global positions
// slot_pos[0..n)) into every rank's staging buffer: used when a continuation segment attends to a
// session's existing KV (prompt + decoded tokens spread over the ranks).
__global__ void stage_push_kernel(StagePushArgs a) {
  const int slot = blockIdx.x;
  if (slot >= a.n) return;
  const int pos = a.slot_pos[slot];
  if (pos < 0 || pos >= a.stage_cap) return;
  const int page = a.page_table[slot / a.geom.page];
  const int row = slot % a.geom.page;
  const int Hkv = a.geom.hkv, D = a.geom.d, dvec = D / 8;
  for (int i = threadIdx.x; i < 2 * Hkv * dvec; i += blockDim.x) {
    const int kv = i / (Hkv * dvec), rem = i % (Hkv * dvec);
    const int h = rem / dvec, e = rem % dvec;
    const uint4 val = *reinterpret_cast<const uint4*>(a.arena + a.geom.offset(a.layer, page, kv, h, row) + e * 8);
    const long soff = ((long)(kv * Hkv + h) * a.stage_cap + pos) * D + e * 8;
    for (int r = 0; r < a.n_stage; ++r)
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.stage_ptrs[r]) + soff) = val;
  }
}

// Wait (bounded) until every peer has released the staging buffer parity we are about to write:
// consumed[r] >= epoch - 2 for all ranks r. One CTA, one warp.
__global__ void wait_consumed_kernel(const unsigned long long* consumed, int n,
                                     unsigned long long need, unsigned long long budget_ns,
                                     int* status) {
  const int r = threadIdx.x;
  if (r < n) wait_flag_geq_sys(consumed + r, need, budget_ns, status, 321, r);
}

// Publish `epoch` into each rank's slot (P2P release stores), e.g. consumed[my_rank].
__global__ void signal_kernel(unsigned long long* const* ptrs, int n, unsigned long long epoch) {
  __threadfence_system();
  const int r = threadIdx.x;
  if (r < n) st_release_sys(ptrs[r], epoch);
}

// Tile flags of rows already present on every rank (see DomainRuntime::PublishTiles).
__global__ void publish_tiles_kernel(const int* push_tiles, int n_push,
                                     unsigned long long* const* tflag_ptrs, int world, int my_rank,
                                     unsigned long long epoch) {
  __threadfence_system();
  for (int i = threadIdx.x; i < n_push * world; i += blockDim.x) {
    const int k = i / world, r = i % world;
    st_release_sys(tflag_ptrs[r] + (long)push_tiles[3 * k] * world + my_rank, epoch);
  }
}

__global__ void publish_range_kernel(unsigned long long* const* ptrs, int world, long base, int n,
                                     unsigned long long epoch) {
  __threadfence_system();
  for (int i = threadIdx.x; i < n * world; i += blockDim.x)
    st_release_sys(ptrs[i % world] + base + i / world, epoch);
}

// First-token broadcast from the rank that holds the last prompt position (one thread).
__global__ void token_bcast_kernel(long long* tok, unsigned long long* const* slots,
                                   const unsigned long long* own_slot, int world, int is_src,
                                   unsigned long long epoch, unsigned long long budget_ns,
                                   int* status) {
  if (threadIdx.x != 0) return;
  const int par = int(epoch & 1ull);
  if (is_src) {
    const unsigned long long v = static_cast<unsigned long long>(*tok);
    for (int r = 0; r < world; ++r) {
      unsigned long long* sl = slots[r] + 2 * par;
      *reinterpret_cast<volatile unsigned long long*>(sl) = v;
      st_release_sys(sl + 1, epoch);   // orders the value store before the epoch
    }
  } else if (wait_flag_geq_sys(own_slot + 2 * par + 1, epoch, budget_ns, status, 323, 0)) {
    *tok = static_cast<long long>(*reinterpret_cast<const volatile unsigned long long*>(own_slot + 2 * par));
  }
}

// ----------------------------------------------------------------------------- decode QKV post
// One CTA per request row b. qkv [B, (H+2Hkv)D] fp32 (GEMV output incl. bias). RoPE at pos[b],
// q -> q_out [B,H,D] bf16, and on the owner rank k/v -> arena slot `slot[b]` (owner[b] != 0).
__global__ void qkv_decode_kernel(QkvDecodeArgs a) {
  const int b = blockIdx.x;
  if (b >= a.B) return;
  const int D = a.D, H = a.H, Hkv = a.Hkv, half = D / 2;
  const int pos = a.pos[b];
  const bool pos_ok = pos >= 0 && pos < a.max_pos;
  const float* row = a.qkv + (long)b * (H + 2 * Hkv) * D;
  const int layer = a.layer;
  const int own = a.owner[b * a.owner_stride + layer];
  const int slot = a.slot[b * a.owner_stride + layer];
  int page = -1;
  if (own) {
    if (slot >= 0 && slot < a.slot_cap) page = a.page_tables[(long)b * a.pt_stride + slot / a.geom.page];
    else if (threadIdx.x == 0) report_error(a.status, int(StatusCode::kOutOfBounds), 331, slot, b);
#if HCP_DEBUG_BOUNDS
    if (page >= a.geom.pages) {   // skip the KV writes below
      if (threadIdx.x == 0) report_error(a.status, int(StatusCode::kOutOfBounds), 335, page, b);
      page = -1;
    }
#endif
  }
  const int n_pairs = (H + Hkv) * half;
  for (int i = threadIdx.x; i < n_pairs; i += blockDim.x) {
    const int hh = i / half, j = i % half;
    const int col = hh * D + j;
    const float x1 = row[col], x2 = row[col + half];
    const float c = pos_ok ? a.cos_t[(long)pos * half + j] : 1.f;
    const float s = pos_ok ? a.sin_t[(long)pos * half + j] : 0.f;
    // round the projection to bf16 first (the reference's bf16 linear output)
    const float y1 = __bfloat162float(__float2bfloat16(x1)), y2 = __bfloat162float(__float2bfloat16(x2));
    const __nv_bfloat16 o1 = __float2bfloat16(y1 * c - y2 * s);
    const __nv_bfloat16 o2 = __float2bfloat16(y2 * c + y1 * s);
    if (hh < H) {
      a.q_out[((long)b * H + hh) * D + j] = o1;
      a.q_out[((long)b * H + hh) * D + j + half] = o2;
    } else if (page >= 0) {
      __nv_bfloat16* dst = a.arena + a.geom.offset(layer, page, 0, hh - H, slot % a.geom.page);
      dst[j] = o1;
      dst[j + half] = o2;
    }
  }
  if (page >= 0) {
    for (int i = threadIdx.x; i < Hkv * D; i += blockDim.x) {
      const int h = i / D, e = i % D;
      __nv_bfloat16* dst = a.arena + a.geom.offset(layer, page, 1, h, slot % a.geom.page);
      dst[e] = __float2bfloat16(row[(H + Hkv) * D + i]);
    }
  }
}

// ----------------------------------------------------------------------------- host launchers
const char* embedding(const int* ids, const __nv_bfloat16* W, __nv_bfloat16* out, int T, int hidden,
                      int vocab, int* status, cudaStream_t s) {
  if (hidden % 8) return "embedding: hidden must be a multiple of 8";
  if (T == 0) return nullptr;
  return launch_pdl(embedding_kernel, dim3(T), dim3(128), 0, s, ids, W, out, T, hidden, vocab, status) == cudaSuccess ? nullptr : "embedding: launch failed";
}

const char* rmsnorm(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, int T,
                    int hidden, long ldx, long ldy, float eps, cudaStream_t s) {
  if (hidden % 8 || ldx % 8 || ldy % 8) return "rmsnorm: hidden/ld must be multiples of 8";
  if (T == 0) return nullptr;
  const int warps = 8;
  rmsnorm_kernel<<<(T + warps - 1) / warps, warps * 32, 0, s>>>(x, w, y, T, hidden, ldx, ldy, eps);
  return cudaGetLastError() == cudaSuccess ? nullptr : "rmsnorm: launch failed";
}

const char* qkv_prefill(const QkvPrefillArgs& a, cudaStream_t s) {
  if (a.D % 16 || a.ld_qkv % 8) return "qkv_prefill: D % 16 and ld % 8 required";
  if (a.T == 0) return nullptr;
  const size_t smem = size_t(a.H + a.Hkv) * a.D * sizeof(float);
  if (smem > 48 * 1024) {
    static std::atomic<unsigned long long> attr{0};
    if (once_per_device(attr, [] {
          return cudaFuncSetAttribute(qkv_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      200 * 1024);
        }) != cudaSuccess)
      return "qkv_prefill: shared-memory opt-in failed";
  }
  qkv_prefill_kernel<<<a.T, 256, smem, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? nullptr : "qkv_prefill: launch failed";
}

const char* stage_push(const StagePushArgs& a, cudaStream_t s) {
  if (a.n == 0) return nullptr;
  stage_push_kernel<<<a.n, 128, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? nullptr : "stage_push: launch failed";
}

const char* wait_consumed(const unsigned long long* consumed, int n, unsigned long long need,
                          unsigned long long budget_ns, int* status, cudaStream_t s) {
  if (n > 32) return "wait_consumed: at most 32 ranks per launch";
  wait_consumed_kernel<<<1, 32, 0, s>>>(consumed, n, need, budget_ns, status);
  return cudaGetLastError() == cudaSuccess ? nullptr : "wait_consumed: launch failed";
}

const char* signal_peers(unsigned long long* const* ptrs, int n, unsigned long long epoch,
                         cudaStream_t s) {
  if (n > 64) return "signal: too many ranks";
  signal_kernel<<<1, 64, 0, s>>>(ptrs, n, epoch);
  return cudaGetLastError() == cudaSuccess ? nullptr : "signal: launch failed";
}

const char* publish_tiles(const int* push_tiles, int n_push, unsigned long long* const* tflag_ptrs,
                          int world, int my_rank, unsigned long long epoch, cudaStream_t s) {
  if (n_push == 0) return nullptr;
  publish_tiles_kernel<<<1, 256, 0, s>>>(push_tiles, n_push, tflag_ptrs, world, my_rank, epoch);
  return cudaGetLastError() == cudaSuccess ? nullptr : "publish_tiles: launch failed";
}

const char* publish_range(unsigned long long* const* ptrs, int world, long base, int n,
                          unsigned long long epoch, cudaStream_t s) {
  if (n <= 0) return nullptr;
  publish_range_kernel<<<1, 256, 0, s>>>(ptrs, world, base, n, epoch);
  return cudaGetLastError() == cudaSuccess ? nullptr : "publish_range: launch failed";
}

const char* token_bcast(long long* tok, unsigned long long* const* slots,
                        const unsigned long long* own_slot, int world, bool is_src,
                        unsigned long long epoch, unsigned long long budget_ns, int* status,
                        cudaStream_t s) {
  token_bcast_kernel<<<1, 32, 0, s>>>(tok, slots, own_slot, world, is_src ? 1 : 0, epoch,
                                       budget_ns, status);
  return cudaGetLastError() == cudaSuccess ? nullptr : "token_bcast: launch failed";
}

const char* qkv_decode(const QkvDecodeArgs& a, cudaStream_t s) {
  if (a.B == 0) return nullptr;
  qkv_decode_kernel<<<a.B, 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? nullptr : "qkv_decode: launch failed";
}

}  // namespace ew
}  // namespace hcp
