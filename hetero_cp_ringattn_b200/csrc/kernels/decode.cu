// Decode-path kernels (B <= 8 rows per step):
//
//  * gemv_*: weight-streaming GEMV y[B,N] = x[B,K] W[N,K]^T with fused epilogues (fp32 out + bias
//    for QKV, in-place residual add for O/down projections, SwiGLU on 128-row interleaved
//    gate||up weights, fp32 logits + packed argmax for the LM head). Decode is bound by reading
//    the weights once per step, so these run on the CUDA cores at HBM bandwidth instead of
//    padding M=1..8 up to a 128-row tensor-core tile.
//  * K2 cp decode: split-KV flash-decoding over this rank's paged KV shard (GQA group packed in
//    one CTA), the split combine in the last CTA of each (row, kv-head), then the rank's partial
//    (O, LSE) is stored straight into every rank's exchange slots through NVLink peer mappings,
//    followed by a release flag; `decode_combine` waits (bounded) for all ranks' flags and does
//    the log-sum-exp combine in rank order, so every rank computes bit-identical outputs.
//
// Parity: replaces the reference's decode routes: the Q-ring partial/merge
// (rust/src/model/attention/ring.rs:625-663, 682-818: local (O, LSE), N-1 serial hops, merge
// with durable KV) and the self-driving packet walk (rust/src/model/self_driving.rs:333-675,
// rust/src/worker_sdk/tch_backend.rs:634-904). All ranks compute their partial concurrently and
// exchange O(B*H*D) bytes once per layer instead of N-1 serial network hops.
#include "common.cuh"
#include "decode.h"
#include "gemm_sm100.h"
#include "kv_layout.h"
#include "launch.h"

namespace hcp {
namespace dec {

using namespace hcp::dev;

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxDecodeSplits = 128;

__device__ __forceinline__ void dot8_acc(const uint4 w, const uint4 x, float& acc) {
  const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
  const uint32_t xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    acc = fmaf(bf16_lo(wv[j]), bf16_lo(xv[j]), acc);
    acc = fmaf(bf16_hi(wv[j]), bf16_hi(xv[j]), acc);
  }
}

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// This CTA's slice of each range into L2: one async bulk prefetch by thread 0, or (pf.lines) a
// 128-byte line prefetch per thread and line, which leaves the CTA's TMA unit to its own loads.
__device__ __forceinline__ void prefetch_l2_slices(const L2Prefetch& pf) {
  if (!pf.lines && threadIdx.x != 0) return;
  const unsigned long long nblk = (unsigned long long)gridDim.x * gridDim.y * gridDim.z;
  const unsigned long long blk =
      blockIdx.x + (unsigned long long)gridDim.x * (blockIdx.y + (unsigned long long)gridDim.y * blockIdx.z);
  const int nthr = blockDim.x * blockDim.y * blockDim.z;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const unsigned long long total = pf.bytes[i];
    if (pf.ptr[i] == nullptr || total == 0) continue;
    const unsigned long long per = ((total + nblk - 1) / nblk + 127) & ~127ull;
    const unsigned long long off = blk * per;
    if (off >= total) continue;
    const unsigned long long n = total - off < per ? total - off : per;
    const char* base = static_cast<const char*>(pf.ptr[i]) + off;
    if (!pf.lines) {
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base), "r"(uint32_t(n)) : "memory");
    } else {
      for (unsigned long long o = (unsigned long long)threadIdx.x * 128; o < n; o += (unsigned long long)nthr * 128)
        asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(base + o) : "memory");
    }
  }
}

__device__ __forceinline__ unsigned long long pack_argmax(float v, int idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // order-preserving float -> uint
  return (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - uint32_t(idx));
}

// Persistent decode GEMV, y[b, o] = epi(sum_k W[o, k] x[b, k]). The grid is one wave of CTAs
// (8 warps each); every warp owns whole output rows (a gate/up row pair for SwiGLU) and walks
// its (row, K-chunk) items with two register buffers: the loads of item i + 1 are issued before
// item i is consumed, so each warp always has KC 16-byte streaming loads per lane in flight, and
// the first item's loads are issued before the x prologue, hiding its latency. Lane l reads the
// 16-byte columns l, l + 32, ... of a chunk; a row ends with one 5-step shuffle reduction and no
// block barrier. x is staged once per CTA in shared memory; with NORM it is RMS-normalised
// there first (the statistics of the 1-8 input rows cost far less than a separate launch).
// D (+)= A B for one m16n8k16 bf16 tile (fp32 accumulate).
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Epilogue of output item o (a weight row, or a gate / rotation pair of rows for the paired
// epilogues, whose second row's sum is v2) for input row b, shared by both GEMV kernels. The
// argmax epilogue only stores the logit here; the packed maxima are kept by the caller.
template <int EPI>
__device__ __forceinline__ void gemv_epilogue_one(const GemvArgs& a, int o, int b, float v, float v2,
                                                  int half) {
  if (EPI == kGemvF32) {
    a.y_f32[(long)b * a.ldy + o] = a.bias ? v + __bfloat162float(a.bias[o]) : v;
  } else if (EPI == kGemvResidual) {
    __nv_bfloat16* y = a.y_bf16 + (long)b * a.ldy + o;
    *y = __float2bfloat16(__bfloat162float(__float2bfloat16(v)) + __bfloat162float(__ldcg(y)));
  } else if (EPI == kGemvSwiGLU) {
    const float g = __bfloat162float(__float2bfloat16(v));
    const float uu = __bfloat162float(__float2bfloat16(v2));
    const float sg = g / (1.f + fast_exp2(-g * kLog2e));
    a.y_bf16[(long)b * a.ldy + o] = __float2bfloat16(sg * uu);
  } else if (EPI == kGemvArgmax) {
    if (a.y_f32) a.y_f32[(long)b * a.ldy + o] = v;
  } else if (EPI == kGemvQkvRope) {
    const GemvRopeArgs& rp = a.rope;
    const int r0 = (o / half) * 2 * half + (o % half);  // row j of head hh; its pair is j + half
    const int hh = r0 / rp.D, j = r0 % rp.D;
    float y1 = v, y2 = v2;
    if (a.bias) {
      y1 += __bfloat162float(a.bias[r0]);
      y2 += __bfloat162float(a.bias[r0 + half]);
    }
    // the bf16 linear output, then the rotation
    y1 = __bfloat162float(__float2bfloat16(y1));
    y2 = __bfloat162float(__float2bfloat16(y2));
    const int pos = rp.pos[b];
    float o1 = y1, o2 = y2;
    if (hh < rp.H + rp.Hkv) {
      if (pos >= 0 && pos < rp.max_pos) {
        const float c = rp.cos_t[(long)pos * half + j], sn = rp.sin_t[(long)pos * half + j];
        o1 = y1 * c - y2 * sn;
        o2 = y2 * c + y1 * sn;
      } else if (j == 0 && hh == 0) {
        report_error(rp.status, int(StatusCode::kOutOfBounds), 332, pos, b);
      }
    }
    if (hh < rp.H) {
      __nv_bfloat16* dst = rp.q_out + ((long)b * rp.H + hh) * rp.D;
      dst[j] = __float2bfloat16(o1);
      dst[j + half] = __float2bfloat16(o2);
    } else if (rp.owner[b * rp.owner_stride + rp.layer]) {
      const int slot = rp.slot[b * rp.owner_stride + rp.layer];
      if (slot >= 0 && slot < rp.slot_cap) {
        const int page = rp.page_tables[(long)b * rp.pt_stride + slot / rp.geom.page];
        const int kv = hh < rp.H + rp.Hkv ? 0 : 1;
        const int kh = hh - rp.H - kv * rp.Hkv;
#if HCP_DEBUG_BOUNDS
        if (page < 0 || page >= rp.geom.pages) {
          if (j == 0) report_error(rp.status, int(StatusCode::kOutOfBounds), 333, page, b);
        } else {
#endif
        __nv_bfloat16* dst = rp.arena + rp.geom.offset(rp.layer, page, kv, kh, slot % rp.geom.page);
        dst[j] = __float2bfloat16(o1);
        dst[j + half] = __float2bfloat16(o2);
#if HCP_DEBUG_BOUNDS
        }
#endif
      } else if (j == 0) {
        report_error(rp.status, int(StatusCode::kOutOfBounds), 331, slot, b);
      }
    }
  }
}

constexpr int GEMV_THREADS = 256;
constexpr int kBulkMaxStages = 12;  // ring stages of the streaming GEMV at most

// x rows into shared memory (xs [B][K/8]), RMS-normalised there with NORM (the statistics of the
// 1-8 input rows cost far less than a separate launch); the caller synchronises afterwards. x is
// read through L2 (ld.global.cg): in a GEMV chain it was written by other SMs earlier in the same
// launch, so no SM may serve it from its own L1.
template <int B, bool NORM>
__device__ __forceinline__ void gemv_stage_x(const GemvArgs& a, uint4* xs, float (*red)[B],
                                             float* rstd) {
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const int kvec = a.K / 8;
  if (NORM) {
    float ss[B];
#pragma unroll
    for (int b = 0; b < B; ++b) ss[b] = 0.f;
    for (int k = tid; k < kvec; k += GEMV_THREADS) {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(a.x + (long)b * a.ldx) + k);
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) ss[b] += bf16_lo(vv[j]) * bf16_lo(vv[j]) + bf16_hi(vv[j]) * bf16_hi(vv[j]);
      }
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const float v = warp_sum(ss[b]);
      if (lane == 0) red[warp][b] = v;
    }
    __syncthreads();
    if (tid < B) {
      float t = 0.f;
      for (int w = 0; w < GEMV_THREADS / 32; ++w) t += red[w][tid];
      rstd[tid] = rsqrtf(t / float(a.K) + a.eps);
    }
    __syncthreads();
    for (int k = tid; k < kvec; k += GEMV_THREADS) {
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(a.norm_w) + k);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(a.x + (long)b * a.ldx) + k);
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float lo = __bfloat162float(__float2bfloat16(bf16_lo(vv[j]) * rstd[b])) * bf16_lo(ww[j]);
          const float hi = __bfloat162float(__float2bfloat16(bf16_hi(vv[j]) * rstd[b])) * bf16_hi(ww[j]);
          o[j] = pack_bf16x2(lo, hi);
        }
        xs[b * kvec + k] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  } else {
    for (int k = tid; k < kvec; k += GEMV_THREADS)
#pragma unroll
      for (int b = 0; b < B; ++b) xs[b * kvec + k] = __ldcg(reinterpret_cast<const uint4*>(a.x + (long)b * a.ldx) + k);
  }
}

// x = the rank-order log-sum-exp combine of every rank's (O, LSE) partial (see GemvCombineArgs);
// thread k builds the 8 columns [8k, 8k + 8) of head 8k / D of every row. If a flag wait runs out
// (bounded, reported into the status word), x is staged as zeros.
template <int B>
__device__ __forceinline__ void gemv_stage_combined(const GemvArgs& a, uint4* xs) {
  const int tid = threadIdx.x;
  const int kvec = a.K / 8;
  const GemvCombineArgs& c = a.cmb;
  const unsigned long long e = *c.epoch_src * c.epoch_mul + c.epoch_add;
  __shared__ int ok;
  if (tid == 0) ok = 1;
  __syncthreads();
  if (tid < c.ranks && !wait_flag_geq_sys(c.ready + tid, e, c.budget_ns, c.status, 402, tid)) ok = 0;
  __syncthreads();
  const long rank_stride = (long)c.slot_B * c.H * (c.D + 1);
  const float* xsl = c.xslot + (long)(e & 1ull) * c.ranks * rank_stride;
  for (int k = tid; k < kvec; k += GEMV_THREADS) {
    const int hh = (k * 8) / c.D, d0 = (k * 8) % c.D;
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float out[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j] = 0.f;
      const float* row = xsl + ((long)(c.row0 + b) * c.H + hh) * (c.D + 1);
      if (ok) {
        float mx = -INFINITY;
        for (int r = 0; r < c.ranks; ++r) mx = fmaxf(mx, __ldcg(row + r * rank_stride + c.D));
        if (mx > -INFINITY) {
          float ws = 0.f, acc[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = 0.f;
          for (int r = 0; r < c.ranks; ++r) {
            const float* src = row + r * rank_stride;
            const float w = fast_exp2(__ldcg(src + c.D) - mx);
            ws += w;
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] += w * __ldcg(src + d0 + j);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) out[j] = acc[j] / ws;
        }
      }
      xs[b * kvec + k] = make_uint4(pack_bf16x2(out[0], out[1]), pack_bf16x2(out[2], out[3]),
                                    pack_bf16x2(out[4], out[5]), pack_bf16x2(out[6], out[7]));
    }
  }
}

// Output item o complete (acc holds each lane's partial sums over k = lane + 32 m): every lane
// gets every warp sum, lane b runs the epilogue of input row b, and the argmax epilogue folds the
// logit into the warp's running maxima.
template <int EPI, int B, int NWR>
__device__ __forceinline__ void gemv_item_done(const GemvArgs& a, int o, int lane, int half,
                                               float (&acc)[NWR][B], unsigned long long (&best)[B]) {
#pragma unroll
  for (int q = 0; q < NWR; ++q)
#pragma unroll
    for (int b = 0; b < B; ++b) acc[q][b] = warp_sum(acc[q][b]);
#pragma unroll
  for (int b = 0; b < B; ++b) {
    const float v = acc[0][b];
    if (EPI == kGemvArgmax) {
      const unsigned long long cnd = pack_argmax(v, o + a.index_base);
      best[b] = cnd > best[b] ? cnd : best[b];
    }
    if (lane != b) continue;
    gemv_epilogue_one<EPI>(a, o, b, v, NWR > 1 ? acc[NWR - 1][b] : 0.f, half);
  }
}

// The register-load GEMV over the whole grid (warp gw takes items gw, gw + warps, ...): each warp
// loads its first weight chunk, then `before_x()` (the dependency wait of a launch of its own, or
// the grid barrier between the phases of a GEMV chain; false: skip the phase), then x is staged
// and the items run with the next chunk's loads in flight. xs [B][K/8] is the x stage.
template <int EPI, int B, bool NORM, class BeforeX>
__device__ __forceinline__ void gemv_body(const GemvArgs& a, uint4* xs, float (*red)[B], float* rstd,
                                          BeforeX&& before_x) {
  constexpr bool PAIRED = (EPI == kGemvSwiGLU) || (EPI == kGemvQkvRope);
  constexpr int NWR = PAIRED ? 2 : 1;  // weight rows per output item (gate/up, rotation pair)
  constexpr int KC = 8 / NWR;          // 16-byte columns per lane per chunk and row
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const int kvec = a.K / 8;
  const int out_rows = PAIRED ? a.N / 2 : a.N;
  const int half = (EPI == kGemvQkvRope) ? a.rope.D / 2 : 128;  // offset of the item's second row
  const int nchunk = (kvec + 32 * KC - 1) / (32 * KC);
  const int gw = blockIdx.x * (GEMV_THREADS / 32) + warp;
  const int nwarps = gridDim.x * (GEMV_THREADS / 32);
  const int my_rows = gw < out_rows ? (out_rows - 1 - gw) / nwarps + 1 : 0;
  const int items = my_rows * nchunk;
  auto load = [&](int item, uint4 (&buf)[NWR][KC]) {
    const int o = gw + (item / nchunk) * nwarps;
    const int c = item % nchunk;
    const int w0 = PAIRED ? (o / half) * 2 * half + (o % half) : o;
#pragma unroll
    for (int q = 0; q < NWR; ++q) {
      const uint4* wp = reinterpret_cast<const uint4*>(a.W + (long)(w0 + q * half) * a.K);
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        const int k = c * 32 * KC + j * 32 + lane;
        buf[q][j] = k < kvec ? ld_stream(wp + k) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
  };
  uint4 bufA[NWR][KC], bufB[NWR][KC];
  if (items > 0) load(0, bufA);  // weights: nothing in flight writes them
  if (!before_x()) return;       // x, residual rows, positions, ... come from predecessors
  if (EPI == kGemvResidual && !NORM && a.cmb.xslot != nullptr) {
    gemv_stage_combined<B>(a, xs);
  } else {
    gemv_stage_x<B, NORM>(a, xs, red, rstd);
  }
  __syncthreads();

  float acc[NWR][B];
  unsigned long long best[B];
#pragma unroll
  for (int b = 0; b < B; ++b) best[b] = 0ull;
  auto consume = [&](int item, const uint4 (&buf)[NWR][KC]) {
    const int o = gw + (item / nchunk) * nwarps;
    const int c = item % nchunk;
    if (c == 0) {
#pragma unroll
      for (int q = 0; q < NWR; ++q)
#pragma unroll
        for (int b = 0; b < B; ++b) acc[q][b] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < KC; ++j) {
      const int k = c * 32 * KC + j * 32 + lane;
      if (k < kvec) {
#pragma unroll
        for (int b = 0; b < B; ++b) {
          const uint4 xv = xs[b * kvec + k];
#pragma unroll
          for (int q = 0; q < NWR; ++q) dot8_acc(buf[q][j], xv, acc[q][b]);
        }
      }
    }
    if (c == nchunk - 1) gemv_item_done<EPI, B, NWR>(a, o, lane, half, acc, best);
  };
  for (int i = 0; i < items; i += 2) {
    if (i + 1 < items) load(i + 1, bufB);
    consume(i, bufA);
    if (i + 1 < items) {
      if (i + 2 < items) load(i + 2, bufA);
      consume(i + 1, bufB);
    }
  }
  if (EPI == kGemvArgmax && lane == 0) {
#pragma unroll
    for (int b = 0; b < B; ++b)
      if (best[b]) atomicMax(a.argmax + b, best[b]);
  }
}

template <int EPI, int B, bool NORM>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(GemvArgs a) {
  extern __shared__ uint4 xs[];                     // [B][K/8] (normalised when NORM)
  __shared__ float red[GEMV_THREADS / 32][B];
  __shared__ float rstd[B];
  pdl_trigger();
  prefetch_l2_slices(a.pf);
  gemv_body<EPI, B, NORM>(a, xs, red, rstd, [] {
    pdl_wait();
    return true;
  });
}

// Streaming decode GEMV for 1-4 input rows: the products, the per-lane summation order and the
// epilogues of gemv_kernel (so the results are the same bits), with the weights brought in by the
// copy engine instead of by register loads. Each CTA owns a contiguous run of 8-item groups (8
// consecutive output items; their weight rows - both rows of each gate / rotation pair for the
// paired epilogues - are one or two contiguous runs of 8 full rows) and streams them through a
// ring of stages in shared memory: a stage is one group, brought in by one untiled bulk copy
// (cp.async.bulk) per run, issued by one thread, completing on the stage's mbarrier. Measured on
// B200, bulk copies stream DRAM at up to 0.97 of the measured HBM copy rate when each copy moves
// 32-64 KB and 3-4 of them are in flight per SM, while copies of 1-8 KB stay at 0.4-0.6 (a cost
// per copy), hence whole 8-row runs (32 KB at K = 2048) and no K chunking. Weights are written by
// nothing in flight, so the whole ring is requested before the dependency wait: every CTA's
// first stages stream while the previous kernel of the decode chain finishes. Warp w computes
// item w of each stage against x in shared memory and releases the stage on its "empty"
// mbarrier; thread 0 refills a slot once all 8 warps have released it. Every wait is bounded and
// reports into the status word. Parity: the decode-token projections of the reference's layers
// (x.matmul(W^T) in rust/src/model/layers/mlp.rs:42-67 and the attention projections), with
// their norms, activation and residuals fused as epilogues.
template <int EPI, int B, bool NORM>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_bulk_kernel(GemvArgs a) {
  extern __shared__ __align__(128) unsigned char gsm[];  // [x rows][ring of stages]
  __shared__ float red[GEMV_THREADS / 32][B];
  __shared__ float rstd[B];
  __shared__ __align__(8) uint64_t full_bar[kBulkMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kBulkMaxStages];
  constexpr bool PAIRED = (EPI == kGemvSwiGLU) || (EPI == kGemvQkvRope);
  constexpr int NWR = PAIRED ? 2 : 1;          // weight rows per output item
  constexpr int IPS = GEMV_THREADS / 32;       // items per stage: one per warp
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const int kvec = a.K / 8;
  const int half = (EPI == kGemvQkvRope) ? a.rope.D / 2 : 128;
  const int nst = a.bulk_nst;
  const size_t stage_elems = size_t(IPS) * NWR * a.K;
  uint4* xs = reinterpret_cast<uint4*>(gsm);
  __nv_bfloat16* ring =
      reinterpret_cast<__nv_bfloat16*>(gsm + ((size_t(B) * a.K * 2 + 127) & ~size_t(127)));
  const int ngroups = (PAIRED ? a.N / 2 : a.N) / IPS;
  const int g0 = int((long)blockIdx.x * ngroups / gridDim.x);
  const int nstage = int((long)(blockIdx.x + 1) * ngroups / gridDim.x) - g0;
  int* st = a.status ? a.status : (EPI == kGemvQkvRope ? a.rope.status : a.cmb.status);

  // stage s: items [8 g, 8 g + 8) of group g = g0 + s, into slot s % nst
  auto issue = [&](int s) {
    const int slot = s % nst;
    const int o = (g0 + s) * IPS;
    const int w0 = PAIRED ? (o / half) * 2 * half + (o % half) : o;
    const uint32_t run_bytes = uint32_t(IPS) * uint32_t(a.K) * 2u;
    __nv_bfloat16* dst = ring + slot * stage_elems;
    mbar_arrive_expect_tx(&full_bar[slot], NWR * run_bytes);
#pragma unroll
    for (int q = 0; q < NWR; ++q)
      bulk_load(dst + size_t(q) * IPS * a.K, a.W + (long)(w0 + q * half) * a.K, run_bytes, &full_bar[slot]);
  };

  pdl_trigger();
  prefetch_l2_slices(a.pf);
  int issued = 0;
  if (tid == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], IPS);
    }
    fence_barrier_init();
    for (; issued < nst && issued < nstage; ++issued) issue(issued);
  }
  pdl_wait();                    // x, residual rows, positions, ... come from predecessors
  if (EPI == kGemvResidual && !NORM && a.cmb.xslot != nullptr) {
    gemv_stage_combined<B>(a, xs);
  } else {
    gemv_stage_x<B, NORM>(a, xs, red, rstd);
  }
  __syncthreads();               // x staged; the barriers initialised

  float acc[NWR][B];
  unsigned long long best[B];
#pragma unroll
  for (int b = 0; b < B; ++b) best[b] = 0ull;
  bool ok = true;
  int s = 0;
  for (; s < nstage; ++s) {
    const int slot = s % nst;
    const uint32_t par = uint32_t(s / nst) & 1u;
    if (!mbar_wait(&full_bar[slot], par, st, 350)) {
      ok = false;
      break;
    }
#pragma unroll
    for (int q = 0; q < NWR; ++q)
#pragma unroll
      for (int b = 0; b < B; ++b) acc[q][b] = 0.f;
    const uint4* wr[NWR];
#pragma unroll
    for (int q = 0; q < NWR; ++q)
      wr[q] = reinterpret_cast<const uint4*>(ring + slot * stage_elems + size_t(q * IPS + warp) * a.K);
    // lane l visits k = l + 32 m in increasing m, the order of gemv_kernel
#pragma unroll 8
    for (int k = lane; k < kvec; k += 32) {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const uint4 xv = xs[b * kvec + k];
#pragma unroll
        for (int q = 0; q < NWR; ++q) dot8_acc(wr[q][k], xv, acc[q][b]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[slot]);
    if (tid == 0 && issued < nstage) {   // refill this slot with stage s + nst
      if (mbar_wait(&empty_bar[slot], par, st, 351)) {
        issue(issued++);
      } else {
        ok = false;
      }
    }
    gemv_item_done<EPI, B, NWR>(a, (g0 + s) * IPS + warp, lane, half, acc, best);
    if (!ok) break;
  }
  if (!ok && tid == 0) {
    // a wait ran out: let the copies still in flight land before the CTA exits (bounded)
    for (int t = s + 1; t < issued; ++t)
      if (!mbar_wait(&full_bar[t % nst], uint32_t(t / nst) & 1u, st, 352)) break;
  }
  if (EPI == kGemvArgmax && lane == 0) {
#pragma unroll
    for (int b = 0; b < B; ++b)
      if (best[b]) atomicMax(a.argmax + b, best[b]);
  }
}

// Tensor-core decode GEMV for several input rows: the same products and epilogues as gemv_kernel,
// computed with warp-level m16n8k16 bf16 MMAs (fp32 accumulate). A tile of 16 output items (16
// weight rows, or 16 gate / rotation pairs) is the MMA's M side and the input rows (up to 8)
// its N side, so every 16-byte weight load feeds all B rows with a handful of instructions,
// where the CUDA-core kernel spends 8 FMAs per weight pair and row and turns compute-bound at
// B = 8. The 8 warps of a CTA split the tile's K into contiguous ranges of 64-element chunks and
// meet in shared memory: partial sums in a fixed warp order, then threads (row, input row) run
// the epilogue. K is permuted identically for W and x: lane t of a row group reads the 16-byte
// pieces t and 4 + t of every 64-element chunk of its two rows (full 32-byte sectors per
// instruction) and uses their elements 4 ks .. 4 ks + 3 as the k-step ks columns {2t, 2t + 1}
// and {2t + 8, 2t + 9}; the x fragment of input row g takes the same pieces of x.
template <int EPI, int B, bool NORM>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_tc_kernel(GemvArgs a) {
  extern __shared__ uint4 xs[];                     // [B][K/8] (normalised when NORM)
  __shared__ float red_n[GEMV_THREADS / 32][B];
  __shared__ float rstd[B];
  constexpr bool PAIRED = (EPI == kGemvSwiGLU) || (EPI == kGemvQkvRope);
  constexpr int NWR = PAIRED ? 2 : 1;
  constexpr int NWARP = GEMV_THREADS / 32;
  __shared__ float part[2][NWARP][NWR][16][8];      // [tile parity][warp][row group][row][input row]
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const int g = lane / 4, t = lane % 4;
  const int kvec = a.K / 8;
  const int out_rows = PAIRED ? a.N / 2 : a.N;
  const int half = (EPI == kGemvQkvRope) ? a.rope.D / 2 : 128;
  const int tiles = out_rows / 16;
  const int nch = a.K / 64;
  const int c_lo = warp * nch / NWARP, c_hi = (warp + 1) * nch / NWARP;  // >= 1 chunk (nch >= 8)
  const int my_chunks = c_hi - c_lo;
  const int my_tiles = tiles > int(blockIdx.x) ? (tiles - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;
  const int items = my_tiles * my_chunks;
  // item i: chunk c_lo + i % my_chunks of the CTA's (i / my_chunks)-th tile
  auto load = [&](int item, uint4 (&buf)[NWR][2][2]) {
    const int tile = int(blockIdx.x) + (item / my_chunks) * int(gridDim.x);
    const int c = c_lo + item % my_chunks;
    const int o0 = tile * 16;
    const int w0 = PAIRED ? (o0 / half) * 2 * half + (o0 % half) : o0;
#pragma unroll
    for (int q = 0; q < NWR; ++q)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint4* wp = reinterpret_cast<const uint4*>(a.W + (long)(w0 + q * half + g + 8 * r) * a.K) + c * 8;
        buf[q][r][0] = ld_stream(wp + t);
        buf[q][r][1] = ld_stream(wp + 4 + t);
      }
  };
  uint4 bufA[NWR][2][2], bufB[NWR][2][2];
  pdl_trigger();
  prefetch_l2_slices(a.pf);
  if (items > 0) load(0, bufA);  // weights: nothing in flight writes them
  pdl_wait();
  gemv_stage_x<B, NORM>(a, xs, red_n, rstd);
  __syncthreads();
  float d[NWR][4];
#pragma unroll
  for (int q = 0; q < NWR; ++q) d[q][0] = d[q][1] = d[q][2] = d[q][3] = 0.f;
  unsigned long long best = 0ull;                   // argmax: this thread's input row's maximum
  const int er = tid % 16, eb = tid / 16;            // epilogue: output row er of the tile, input row eb
  auto consume = [&](int item, const uint4 (&buf)[NWR][2][2]) {
    const int c = c_lo + item % my_chunks;
    uint32_t xb[8];
    if (g < B) {
      const uint4 x0 = xs[g * kvec + c * 8 + t], x1 = xs[g * kvec + c * 8 + 4 + t];
      xb[0] = x0.x; xb[1] = x0.y; xb[2] = x0.z; xb[3] = x0.w;
      xb[4] = x1.x; xb[5] = x1.y; xb[6] = x1.z; xb[7] = x1.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) xb[j] = 0u;
    }
#pragma unroll
    for (int q = 0; q < NWR; ++q) {
      const uint32_t lo[8] = {buf[q][0][0].x, buf[q][0][0].y, buf[q][0][0].z, buf[q][0][0].w,
                              buf[q][0][1].x, buf[q][0][1].y, buf[q][0][1].z, buf[q][0][1].w};
      const uint32_t hi[8] = {buf[q][1][0].x, buf[q][1][0].y, buf[q][1][0].z, buf[q][1][0].w,
                              buf[q][1][1].x, buf[q][1][1].y, buf[q][1][1].z, buf[q][1][1].w};
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint32_t af[4] = {lo[2 * ks], hi[2 * ks], lo[2 * ks + 1], hi[2 * ks + 1]};
        mma16816(d[q], af, xb[2 * ks], xb[2 * ks + 1]);
      }
    }
    if (item % my_chunks != my_chunks - 1) return;
    // the warp's K range of this tile is done: partial sums to shared memory, every warp meets
    // here once per tile (named barrier), then the epilogue threads add the 8 warps in order
    const int k_tile = item / my_chunks;
    const int par = k_tile & 1;
#pragma unroll
    for (int q = 0; q < NWR; ++q) {
      part[par][warp][q][g][2 * t] = d[q][0];
      part[par][warp][q][g][2 * t + 1] = d[q][1];
      part[par][warp][q][g + 8][2 * t] = d[q][2];
      part[par][warp][q][g + 8][2 * t + 1] = d[q][3];
      d[q][0] = d[q][1] = d[q][2] = d[q][3] = 0.f;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(GEMV_THREADS) : "memory");
    if (eb < B) {
      float v = 0.f, v2 = 0.f;
#pragma unroll
      for (int w = 0; w < NWARP; ++w) {
        v += part[par][w][0][er][eb];
        if (PAIRED) v2 += part[par][w][NWR - 1][er][eb];
      }
      const int o = (int(blockIdx.x) + k_tile * int(gridDim.x)) * 16 + er;
      if (EPI == kGemvArgmax) {
        const unsigned long long cnd = pack_argmax(v, o + a.index_base);
        best = cnd > best ? cnd : best;
      }
      gemv_epilogue_one<EPI>(a, o, eb, v, v2, half);
    }
  };
  for (int i = 0; i < items; i += 2) {
    if (i + 1 < items) load(i + 1, bufB);
    consume(i, bufA);
    if (i + 1 < items) {
      if (i + 2 < items) load(i + 2, bufA);
      consume(i + 1, bufB);
    }
  }
  if (EPI == kGemvArgmax && eb < B && best) atomicMax(a.argmax + eb, best);
}

// Tensor-core kernel for B >= HCP_GEMV_TC input rows (default 8; 0: never), when the shape fits
// it: 16-item output tiles, K a multiple of 64 and at least 8 chunks (one per warp), gate /
// rotation pairs aligned to the tiles, and no combine prologue (CUDA-core kernel only). Measured
// in the Llama-3.2-1B decode step at 32k (ms per step, CUDA-core / tensor-core GEMVs): B = 2
// 1.41 / 2.16, B = 4 2.03 / 2.27, B = 8 3.99 / 2.74; at B <= 4 the CUDA-core kernel is not yet
// compute-bound and the tensor-core kernel's per-tile barrier costs more than it saves.
static bool gemv_use_tc_shape(const GemvArgs& a) {
  const bool paired = a.epi == kGemvSwiGLU || a.epi == kGemvQkvRope;
  const int out_rows = paired ? a.N / 2 : a.N;
  const int half = a.epi == kGemvQkvRope ? a.rope.D / 2 : 128;
  return a.cmb.xslot == nullptr && out_rows % 16 == 0 && a.K % 64 == 0 && a.K >= 512 &&
         !(paired && half % 16);
}

static bool gemv_use_tc(const GemvArgs& a) {
  static int min_b = -2;
  if (min_b == -2) {
    const char* e = getenv("HCP_GEMV_TC");
    min_b = (e && *e) ? atoi(e) : 8;
  }
  return min_b > 0 && a.B >= min_b && gemv_use_tc_shape(a);
}

static int env_int(const char* name, int dflt) {
  const char* e = getenv(name);
  return (e && *e) ? atoi(e) : dflt;
}

// Stage plan of the streaming kernel: a stage is 8 items x NWR full weight rows (at most 64 KB;
// larger rows stay on the CUDA-core kernel), the ring as many stages as fit in
// HCP_GEMV_BULK_RING_KB (default 64 KB; at least 2, at most kBulkMaxStages).
struct GemvBulkPlan {
  int nst = 0;
  size_t smem = 0;
};

static bool gemv_bulk_plan(const GemvArgs& a, GemvBulkPlan& p) {
  static const int ring_kb = env_int("HCP_GEMV_BULK_RING_KB", 64);
  const bool paired = a.epi == kGemvSwiGLU || a.epi == kGemvQkvRope;
  const int nwr = paired ? 2 : 1;
  const int out_rows = paired ? a.N / 2 : a.N;
  const int half = a.epi == kGemvQkvRope ? a.rope.D / 2 : 128;
  if (a.B > 4 || out_rows % 8 || (paired && half % 8)) return false;
  const size_t stage = size_t(8) * nwr * a.K * 2;
  if (stage > 64 * 1024) return false;
  size_t nst = size_t(ring_kb) * 1024 / stage;
  if (nst < 2) nst = 2;
  if (nst > size_t(kBulkMaxStages)) nst = kBulkMaxStages;
  p.nst = int(nst);
  p.smem = ((size_t(a.B) * a.K * 2 + 127) & ~size_t(127)) + nst * stage;
  return p.smem <= 200 * 1024;
}

static bool gemv_use_bulk(const GemvArgs& a) {
  static const int mode = env_int("HCP_GEMV_BULK", 1);
  return a.bulk >= 0 ? a.bulk != 0 : mode != 0;
}

template <int EPI, bool NORM>
static cudaError_t gemv_launch(const GemvArgs& a0, cudaStream_t s) {
  const bool tc = a0.tc >= 0 ? (a0.tc != 0 && gemv_use_tc_shape(a0)) : gemv_use_tc(a0);
  GemvBulkPlan bp;
  const bool bulk = !tc && gemv_use_bulk(a0) && gemv_bulk_plan(a0, bp);
  GemvArgs a = a0;
  a.bulk_nst = bp.nst;
  const size_t smem = bulk ? bp.smem : size_t(a.B) * a.K * 2;
  auto go = [&](auto kernel) -> cudaError_t {
    // the whole decode chain runs with the maximum shared-memory carveout, so consecutive
    // (overlapping) kernels never need the SM's L1 / shared split reconfigured; the same
    // once-per-kernel step opens dynamic shared memory up to the opt-in limit less the kernel's
    // static shared memory, so no launch needs it again (every batch size and all three
    // kernels go through this one helper)
    cudaError_t ce = once_per_device_kernel(reinterpret_cast<const void*>(kernel), [&] {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                           cudaSharedmemCarveoutMaxShared);
      if (e != cudaSuccess) return e;
      cudaFuncAttributes fa;
      int dev = 0, optin = 0;
      if ((e = cudaFuncGetAttributes(&fa, kernel)) != cudaSuccess) return e;
      if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
      if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
        return e;
      return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  optin - int(fa.sharedSizeBytes));
    });
    if (ce != cudaSuccess) return ce;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, GEMV_THREADS, smem) != cudaSuccess || occ < 1)
      occ = 1;
    const int out_rows = (EPI == kGemvSwiGLU || EPI == kGemvQkvRope) ? a.N / 2 : a.N;
    int need, cap = occ * a.num_sms;
    if (bulk) {
      // up to HCP_GEMV_BULK_CTAS CTAs per SM (default 2, as many as fit)
      static const int per_sm = env_int("HCP_GEMV_BULK_CTAS", 2);
      need = out_rows / 8;
      cap = (per_sm < occ ? (per_sm > 0 ? per_sm : 1) : occ) * a.num_sms;
    } else if (tc) {
      need = out_rows / 16;    // one CTA per 16-item tile
    } else {
      need = (out_rows + GEMV_THREADS / 32 - 1) / (GEMV_THREADS / 32);  // one warp per item
    }
    const int grid = need < cap ? need : cap;
    return launch_pdl(kernel, dim3(grid), dim3(GEMV_THREADS), smem, s, a);
  };
  if (bulk) {
    switch (a.B) {
      case 1: return go(gemv_bulk_kernel<EPI, 1, NORM>);
      case 2: return go(gemv_bulk_kernel<EPI, 2, NORM>);
      case 4: return go(gemv_bulk_kernel<EPI, 4, NORM>);
      default: return cudaErrorInvalidValue;
    }
  }
  if (tc) {
    switch (a.B) {
      case 1: return go(gemv_tc_kernel<EPI, 1, NORM>);
      case 2: return go(gemv_tc_kernel<EPI, 2, NORM>);
      case 4: return go(gemv_tc_kernel<EPI, 4, NORM>);
      case 8: return go(gemv_tc_kernel<EPI, 8, NORM>);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (a.B) {
    case 1: return go(gemv_kernel<EPI, 1, NORM>);
    case 2: return go(gemv_kernel<EPI, 2, NORM>);
    case 4: return go(gemv_kernel<EPI, 4, NORM>);
    case 8: return go(gemv_kernel<EPI, 8, NORM>);
    default: return cudaErrorInvalidValue;
  }
}

template <int EPI>
static cudaError_t gemv_dispatch(const GemvArgs& a, cudaStream_t s) {
  return a.norm_w ? gemv_launch<EPI, true>(a, s) : gemv_launch<EPI, false>(a, s);
}

const char* gemv_check(const GemvArgs& a) {
  if (a.K % 8 || a.ldx % 8) return "gemv: K and ldx must be multiples of 8";
  if (a.B != 1 && a.B != 2 && a.B != 4 && a.B != 8) return "gemv: B must be 1, 2, 4 or 8";
  if (a.epi == kGemvSwiGLU && a.N % 256) return "gemv: SwiGLU needs N % 256 == 0";
  if (a.epi == kGemvQkvRope &&
      (a.rope.q_out == nullptr || a.rope.D % 2 || a.N != (a.rope.H + 2 * a.rope.Hkv) * a.rope.D))
    return "gemv: QKV rope epilogue needs q_out and N = (H + 2 Hkv) D";
  if ((reinterpret_cast<uintptr_t>(a.W) | reinterpret_cast<uintptr_t>(a.x)) & 15)
    return "gemv: W/x must be 16-byte aligned";
  for (int i = 0; i < 2; ++i)
    if (a.pf.ptr[i] && ((reinterpret_cast<uintptr_t>(a.pf.ptr[i]) | a.pf.bytes[i]) & 15))
      return "gemv: L2 prefetch ranges must be 16-byte aligned multiples of 16 bytes";
  if (a.cmb.xslot != nullptr &&
      (a.epi != kGemvResidual || a.norm_w != nullptr || a.cmb.D % 8 || a.K != a.cmb.H * a.cmb.D ||
       a.cmb.ranks < 1 || a.cmb.ranks > GEMV_THREADS || a.cmb.row0 + a.B > a.cmb.slot_B ||
       !a.cmb.ready || !a.cmb.epoch_src))
    return "gemv: the combine prologue needs the residual epilogue, no norm, K = H * D, D % 8 == 0";
  if (size_t(a.K) * 2 > 200 * 1024) return "gemv: needs K*2 <= 200 KB (x is staged in shared memory)";
  return nullptr;
}

const char* gemv(const GemvArgs& a, cudaStream_t s) {
  if (const char* err = gemv_check(a)) return err;
  if (size_t(a.B) * a.K * 2 > 200 * 1024) {
    // x rows are staged in shared memory: run the batch in halves (their rows are independent)
    GemvArgs lo = a, hi = a;
    lo.B = hi.B = a.B / 2;
    const int o = a.B / 2;
    hi.x = a.x + (long)o * a.ldx;
    if (a.y_f32) hi.y_f32 = a.y_f32 + (long)o * a.ldy;
    if (a.y_bf16) hi.y_bf16 = a.y_bf16 + (long)o * a.ldy;
    if (a.argmax) hi.argmax = a.argmax + o;
    hi.cmb.row0 = a.cmb.row0 + o;
    if (a.epi == kGemvQkvRope) {
      hi.rope.pos = a.rope.pos + o;
      hi.rope.q_out = a.rope.q_out + (long)o * a.rope.H * a.rope.D;
      hi.rope.page_tables = a.rope.page_tables + (long)o * a.rope.pt_stride;
      hi.rope.owner = a.rope.owner + (long)o * a.rope.owner_stride;
      hi.rope.slot = a.rope.slot + (long)o * a.rope.owner_stride;
    }
    const char* err = gemv(lo, s);
    return err ? err : gemv(hi, s);
  }
  cudaError_t e;
  switch (a.epi) {
    case kGemvF32: e = gemv_dispatch<kGemvF32>(a, s); break;
    case kGemvResidual: e = gemv_dispatch<kGemvResidual>(a, s); break;
    case kGemvSwiGLU: e = gemv_dispatch<kGemvSwiGLU>(a, s); break;
    case kGemvArgmax: e = gemv_dispatch<kGemvArgmax>(a, s); break;
    case kGemvQkvRope: e = gemv_dispatch<kGemvQkvRope>(a, s); break;
    default: return "gemv: unknown epilogue";
  }
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

// ----------------------------------------------------------------------------- GEMV chain
// Grid barrier of the chain kernel: every CTA arrives on ctr[0] (release), then waits (bounded)
// until the grid's CTAs have arrived `target` times in all (acquire). CTA-uniform result.
__device__ __forceinline__ bool chain_barrier(unsigned int* ctr, unsigned int target, int* status,
                                              int site) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(ctr, 1u);
    int ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int it = 0;; ++it) {
      unsigned int v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
      if (v >= target) break;
      if (it >= 8) __nanosleep(32);   // back off: every CTA of the grid polls this one word
      if ((it & 255) == 255) {
        if (error_raised(status)) {
          ok = 0;
          break;
        }
        if (globaltimer_ns() - t0 > kPipeTimeoutNs) {
          report_error(status, int(StatusCode::kMbarTimeout), site, int(target), int(v));
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// The decode GEMVs between two attention launches as one cooperative launch: the output
// projection (+ residual; with the cross-rank combine in its prologue when its arguments carry
// one), RMSNorm + gate/up + SwiGLU, the down projection (+ residual), then RMSNorm + either the
// next layer's QKV projection with RoPE and the KV append (LAST = kGemvQkvRope) or the LM head
// with the argmax (LAST = kGemvArgmax). The phases run the register-load GEMV body over the whole
// grid, separated by grid barriers, and every warp requests its first weight chunk of a phase
// before it waits at the barrier. One launch replaces four, whose boundaries (the drain of one
// grid, the ramp of the next, the dependency wait) cost several microseconds each in the decode
// step. The phase sequence is fixed at compile time, so every phase reads its arguments at a
// constant offset. Measured on B200 it is slower than the four launches it replaces (Llama-3.2-1B
// decode at 32k: 1.18-1.27 against 1.09-1.12 ms per token at batch 1, 2.50-2.61 against
// 1.96-2.09 at batch 4, also with a back-off in the barrier poll and with the launch allowed to
// start early), so the engine runs it only with HCP_DECODE_CHAIN=1. Parity: the decoder layer's
// attention residual, post-attention RMSNorm, MLP and MLP residual (rust/src/model/layers/mod.rs:
// 59-77; the MLP rust/src/model/layers/mlp.rs:42-67), then the next layer's input RMSNorm and
// projection or the final norm and LM head, for one decode token per row. The dependent launch (the next attention) is released once the last barrier
// is passed. ctr[0] counts barrier arrivals and ctr[1] CTAs done; the last CTA out sets both back
// to zero, so one counter pair serves every replay of a captured graph.
template <int B, int LAST>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_chain_kernel(const __grid_constant__ GemvChainArgs c) {
  extern __shared__ uint4 xs[];
  __shared__ float red[GEMV_THREADS / 32][B];
  __shared__ float rstd[B];
  bool ok = true;
  auto barrier = [&](int phase) {
    if (!chain_barrier(c.ctr, unsigned(phase) * gridDim.x, c.status, 360 + phase)) {
      ok = false;
      return false;
    }
    if (phase == 3) pdl_trigger();
    return true;
  };
  gemv_body<kGemvResidual, B, false>(c.ph[0], xs, red, rstd, [] {
    pdl_wait();
    return true;
  });
  gemv_body<kGemvSwiGLU, B, true>(c.ph[1], xs, red, rstd, [&] { return barrier(1); });
  if (ok) gemv_body<kGemvResidual, B, false>(c.ph[2], xs, red, rstd, [&] { return barrier(2); });
  if (ok) gemv_body<LAST, B, true>(c.ph[3], xs, red, rstd, [&] { return barrier(3); });
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(c.ctr + 1, 1u) == gridDim.x - 1) {   // every CTA is past every barrier wait
      atomicExch(c.ctr, 0u);
      atomicExch(c.ctr + 1, 0u);
    }
  }
}

template <int B, int LAST>
static cudaError_t launch_chain(const GemvChainArgs& c, size_t smem, cudaStream_t s) {
  auto kernel = gemv_chain_kernel<B, LAST>;
  cudaError_t ce = once_per_device_kernel(reinterpret_cast<const void*>(kernel), [&] {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  if (ce != cudaSuccess) return ce;
  int occ = 0;
  if ((ce = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, GEMV_THREADS, smem)) != cudaSuccess)
    return ce;
  if (occ < 1) return cudaErrorInvalidConfiguration;
  // a cooperative launch: all CTAs are resident together (they wait for one another)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(occ * c.ph[0].num_sms);
  cfg.blockDim = dim3(GEMV_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, c);
}

bool gemv_chain_supported(const GemvArgs* ph, int n) {
  if (n != kGemvChainPhases) return false;
  const int epi[3] = {kGemvResidual, kGemvSwiGLU, kGemvResidual};
  for (int i = 0; i < n; ++i) {
    const GemvArgs& a = ph[i];
    if (a.B != ph[0].B || a.B > 4 || size_t(a.B) * a.K * 2 > 200 * 1024 || a.num_sms != ph[0].num_sms)
      return false;
    if (i < 3 && (a.epi != epi[i] || (a.norm_w != nullptr) != (i == 1))) return false;
    if (i == 3 && ((a.epi != kGemvQkvRope && a.epi != kGemvArgmax) || a.norm_w == nullptr)) return false;
  }
  return true;
}

const char* gemv_chain(const GemvArgs* ph, int n, unsigned int* ctr, int* status, cudaStream_t s) {
  if (!gemv_chain_supported(ph, n))
    return "gemv_chain: residual, norm + SwiGLU, residual, norm + (QKV rope | argmax); 1, 2 or 4 rows";
  if (ctr == nullptr) return "gemv_chain: needs a zeroed counter pair";
  GemvChainArgs c;
  size_t smem = 0;
  for (int i = 0; i < n; ++i) {
    if (const char* err = gemv_check(ph[i])) return err;
    c.ph[i] = ph[i];
    const size_t need = size_t(ph[i].B) * ph[i].K * 2;
    smem = need > smem ? need : smem;
  }
  c.ctr = ctr;
  c.status = status;
  const bool qkv = ph[3].epi == kGemvQkvRope;
  cudaError_t e;
  switch (ph[0].B) {
    case 1: e = qkv ? launch_chain<1, kGemvQkvRope>(c, smem, s) : launch_chain<1, kGemvArgmax>(c, smem, s); break;
    case 2: e = qkv ? launch_chain<2, kGemvQkvRope>(c, smem, s) : launch_chain<2, kGemvArgmax>(c, smem, s); break;
    default: e = qkv ? launch_chain<4, kGemvQkvRope>(c, smem, s) : launch_chain<4, kGemvArgmax>(c, smem, s); break;
  }
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

// ----------------------------------------------------------------------------- K2 decode attention
// grid (splits, Hkv, B), 128 threads (4 warps). A CTA streams its split's token range through a
// STAGES-deep shared-memory ring of 64-token chunks: one thread issues TMA tile loads (128-byte
// swizzle, 64 rows x 64 head dims per box, so each box moves 8 KB) of the chunk's K and V rows
// straight from the paged arena (a chunk never straddles a 256-row page); every warp waits on the
// chunk's mbarrier (bounded), works on its own 16 rows of the chunk and arrives on the stage's
// "empty" barrier, which gates the reuse of that stage.
//
// The math runs on the tensor cores with warp-level m16n8k16 bf16 MMAs (the GQA group has at most
// 8 query rows, below the 64-row minimum of tcgen05, and the loop is memory-bound, so the MMAs are
// only there to cut the instruction count per token):
//   S = Q K^T   A = the group's q rows (16 rows, G used), B = K^T of 8 tokens. The head-dim
//               order inside the dot product is permuted so lane t's B operand is one contiguous
//               run of D/4 dims of a K row (two or four conflict-free 16-byte shared loads); the
//               q fragments use the same permutation.
//   O += P V    A = P straight from S's accumulator fragments (packed to bf16), B = V through
//               ldmatrix.trans (the swizzle makes the 8 row addresses conflict-free).
// One running-max update per head and 16-row slice; the row sums are per-lane partials reduced at
// the end; the 4 warps are merged through shared memory and the split's (O, LSE) partial written.
constexpr int kDecCC = 64;   // tokens per chunk (one TMA box of rows)
constexpr int kDecWR = 16;   // rows of a chunk per warp (two 8-token MMA n-tiles)
constexpr int kDecMinChunks = 4;  // chunks a split streams at least (fewer active splits)

template <int D>
struct DecCfg {
  static constexpr int NH = D / 64;                      // 64-dim swizzled sub-tiles per row
  static constexpr int SUB = kDecCC * 128;               // bytes of one sub-tile (64 rows x 128 B)
  static constexpr int STAGE = 2 * NH * SUB;             // K then V sub-tiles
  static constexpr int STAGES = (D == 64) ? 3 : 2;      // 4 / 3 CTAs per SM
  static constexpr int SMEM = 1024 + STAGES * STAGE;     // + alignment slack
};


__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// byte offset of 16-byte chunk c of row r inside a 128-byte-swizzled tile (TMA SWIZZLE_128B)
__device__ __forceinline__ uint32_t swz(int r, int c) { return uint32_t(r * 128 + ((c ^ (r & 7)) << 4)); }

template <int D, int G>
__global__ void __launch_bounds__(128) decode_attn_kernel(const __grid_constant__ CUtensorMap tm_kv,
                                                          DecodeAttnArgs a) {
  using C = DecCfg<D>;
  // Programmatic dependent launch: this kernel starts while the QKV projection (which writes q and
  // the new token's K/V row n - 1 on its owner rank) is still running. Everything before
  // pdl_wait() below reads only data no kernel in flight writes: the row lengths and page tables
  // (copied from the host before the step) and the KV rows of earlier tokens, so the first
  // pipeline stages stream while the projection finishes.
  pdl_trigger();
  prefetch_l2_slices(a.pf);               // later kernels' weights (before any early return)
  constexpr int NW = 4;                    // warps per CTA
  constexpr int CC = kDecCC;
  constexpr int DQ = D / 4;                // contiguous dims of a K row per lane in S = Q K^T
  constexpr int KS = D / 16;               // MMA k-steps over the head dim
  constexpr int NT = D / 8;                // 8-dim n-tiles of O
  static_assert(G >= 1 && G <= 16, "GQA group of at most 16 query heads");
  // heads g and g + 8 of the group are rows g and g + 8 of the 16-row MMA tiles: groups of up to
  // 8 heads use rows 0..7 only, larger groups the second row group too (R2)
  constexpr bool R2 = G > 8;
  static_assert(NW * kDecWR == CC, "warps x rows per warp = chunk");
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[C::STAGES];
  __shared__ __align__(8) uint64_t empty[C::STAGES];
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int g = lane / 4, t = lane % 4;    // MMA fragment row group / column pair
  // a row's KV length is bounded by its page-table row (pt_stride pages); a longer one is
  // reported and clamped, so the page-table reads below stay inside the caller's row
  int n = a.n_tokens[b];
  const int n_cap = a.pt_stride * a.geom.page;
  if (n > n_cap || n < 0) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0)
      report_error(a.status, int(StatusCode::kOutOfBounds), 304, n, b);
    n = n < 0 ? 0 : n_cap;
  }
  // active splits: as many as the launch has, but each streams at least kDecMinChunks chunks
  // (a short local shard, e.g. a rank's part at high CP, would otherwise give every split a
  // single chunk and pay the pipeline latency and the split combine for nothing); the CTAs of
  // the other splits exit here
  const int eff = max(1, min(a.splits, (n + kDecMinChunks * CC - 1) / (kDecMinChunks * CC)));
  if (split >= eff) return;
  // chunk-aligned split ranges
  int per = (n + eff - 1) / eff;
  per = (per + CC - 1) / CC * CC;
  const int s0 = min(n, split * per);
  const int s1 = min(n, s0 + per);
  const int nc = (s1 - s0 + CC - 1) / CC;
  const int H = a.Hkv * G;

  if (threadIdx.x == 0) {
    for (int st = 0; st < C::STAGES; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], NW);
    }
    fence_barrier_init();
  }
  __syncthreads();

  const int* pt = a.page_tables + (long)b * a.pt_stride;
  const long rows_per_layer = (long)a.geom.pages * 2 * a.geom.hkv * a.geom.page;
  auto issue = [&](int c) {
    const int t0 = s0 + c * CC;
#if HCP_DEBUG_BOUNDS
    int page = pt[t0 / a.geom.page];
    if (page < 0 || page >= a.geom.pages) {   // read page 0 instead; the result is flagged
      report_error(a.status, int(StatusCode::kOutOfBounds), 334, page, b);
      page = 0;
    }
#else
    const int page = pt[t0 / a.geom.page];
#endif
    const long krow = (long)a.layer * rows_per_layer +
                      ((long)(page * 2 + 0) * a.geom.hkv + h) * a.geom.page + (t0 % a.geom.page);
    const long vrow = krow + (long)a.geom.hkv * a.geom.page;
    uint8_t* dst = dsm + (c % C::STAGES) * C::STAGE;
    uint64_t* bar = &full[c % C::STAGES];
    mbar_arrive_expect_tx(bar, C::STAGE);
#pragma unroll
    for (int j = 0; j < C::NH; ++j) {
      tma_load_2d(dst + j * C::SUB, &tm_kv, bar, j * 64, int(krow));
      tma_load_2d(dst + (C::NH + j) * C::SUB, &tm_kv, bar, j * 64, int(vrow));
    }
  };
  const bool producer = threadIdx.x == 0;
  int pre = 0;   // chunks issued before the dependency wait: those that end before row n - 1
  if (producer) {
    tma_prefetch_desc(&tm_kv);
    while (pre < C::STAGES - 1 && pre < nc && s0 + (pre + 1) * CC <= n - 1) issue(pre++);
  }
  pdl_wait();
  if (producer)
    for (int c = pre; c < C::STAGES - 1 && c < nc; ++c) issue(c);

  // q fragments (A of S = Q K^T): row g = head g of the group, pre-scaled into the log2 domain;
  // k-step ks, lane t covers dims t * DQ + 4 ks + {0, 1} (a0) and + {2, 3} (a2)
  uint32_t qa[KS][2];
  uint32_t qb[KS][2];                      // R2: head g + 8 (zero otherwise)
  {
    const float qs = a.scale * kLog2e;
    auto load_q = [&](int gg, uint32_t (&dst)[KS][2]) {
      float qf[DQ];
      if (gg < G) {
        const __nv_bfloat16* qp = a.q + ((long)b * H + h * G + gg) * D + t * DQ;
#pragma unroll
        for (int v = 0; v < DQ / 8; ++v) {
          const uint4 w = *reinterpret_cast<const uint4*>(qp + v * 8);
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            qf[v * 8 + 2 * j] = bf16_lo(ww[j]) * qs;
            qf[v * 8 + 2 * j + 1] = bf16_hi(ww[j]) * qs;
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < DQ; ++i) qf[i] = 0.f;
      }
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        dst[ks][0] = pack_bf16x2(qf[4 * ks], qf[4 * ks + 1]);
        dst[ks][1] = pack_bf16x2(qf[4 * ks + 2], qf[4 * ks + 3]);
      }
    };
    load_q(g, qa);
    if (R2) {
      load_q(g + 8, qb);
    } else {
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) qb[ks][0] = qb[ks][1] = 0u;
    }
  }
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m = -INFINITY, l = 0.f;  // head g's running max (log2 domain) and this lane's row-sum part
  float m2 = -INFINITY, l2 = 0.f;  // R2: the same for head g + 8
  int issued = min(nc, C::STAGES - 1);
  bool ok = true;
  const int wr0 = warp * kDecWR;           // this warp's rows inside a chunk
  for (int c = 0; c < nc; ++c) {
    if (producer && c + C::STAGES - 1 < nc) {
      // stage (c - 1) % STAGES is reused once every warp has released chunk c - 1
      const int k = c + C::STAGES - 1;
      if (k >= C::STAGES && !mbar_wait(&empty[k % C::STAGES], ((k / C::STAGES) - 1) & 1, a.status, 303)) {
        ok = false;
      } else {
        fence_proxy_async_smem();
        issue(k);
        issued = k + 1;
      }
    }
    ok = __all_sync(0xffffffffu, ok && mbar_wait(&full[c % C::STAGES], (c / C::STAGES) & 1, a.status, 301));
    if (!ok) break;
    uint8_t* sk = dsm + (c % C::STAGES) * C::STAGE;
    uint8_t* sv = sk + C::NH * C::SUB;
    const int t0 = s0 + c * CC + wr0;      // first token of this warp's 16 rows
    const int valid = max(0, min(kDecWR, s1 - t0));
    if (valid < kDecWR) {
      // rows past the range hold whatever the page had: zero V there (p is 0 for them, and
      // 0 * a non-finite value would not be)
      for (int i = lane; i < (kDecWR - valid) * C::NH * 8; i += 32) {
        const int r = wr0 + valid + i / (C::NH * 8), rem = i % (C::NH * 8);
        *reinterpret_cast<uint4*>(sv + (rem / 8) * C::SUB + r * 128 + (rem % 8) * 16) = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }
    if (valid > 0) {
      // S = Q K^T for the two 8-token n-tiles
      float s[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
        const int r = wr0 + nt * 8 + g;
        uint32_t kw[DQ / 2];
#pragma unroll
        for (int v = 0; v < DQ / 8; ++v) {
          const int dim = t * DQ + v * 8;
          const uint4 w = *reinterpret_cast<const uint4*>(sk + (dim / 64) * C::SUB + swz(r, (dim % 64) / 8));
          kw[4 * v] = w.x;
          kw[4 * v + 1] = w.y;
          kw[4 * v + 2] = w.z;
          kw[4 * v + 3] = w.w;
        }
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          const uint32_t af[4] = {qa[ks][0], qb[ks][0], qa[ks][1], qb[ks][1]};
          mma16816(s[nt], af, kw[2 * ks], kw[2 * ks + 1]);
        }
      }
      // head g's scores: tokens 2t, 2t + 1 (n-tile 0) and 8 + 2t, 9 + 2t (n-tile 1); head g + 8's
      // (R2) are the accumulators' second row pair
      float sc[4] = {s[0][0], s[0][1], s[1][0], s[1][1]};
      float sc2[4] = {s[0][2], s[0][3], s[1][2], s[1][3]};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = (e >> 1) * 8 + 2 * t + (e & 1);
        if (tok >= valid) sc[e] = sc2[e] = -INFINITY;
      }
      // online softmax of one row: running max mm / row-sum part ll, O columns acc[][c0, c0 + 1]
      auto row_softmax = [&](const float (&x)[4], float& mm, float& ll, int c0, float (&pe)[4]) {
        float cm = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
        cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 1));
        cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 2));
        if (cm > mm) {
          const float al = fast_exp2(mm - cm);  // 0 while nothing has been accumulated
          mm = cm;
          ll *= al;
#pragma unroll
          for (int i = 0; i < NT; ++i) {
            acc[i][c0] *= al;
            acc[i][c0 + 1] *= al;
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) pe[e] = (mm == -INFINITY) ? 0.f : fast_exp2(x[e] - mm);
        ll += (pe[0] + pe[1]) + (pe[2] + pe[3]);
      };
      float pe[4], pe2[4];
      row_softmax(sc, m, l, 0, pe);
      uint32_t pa[4] = {pack_bf16x2(pe[0], pe[1]), 0u, pack_bf16x2(pe[2], pe[3]), 0u};
      if (R2) {
        row_softmax(sc2, m2, l2, 2, pe2);
        pa[1] = pack_bf16x2(pe2[0], pe2[1]);
        pa[3] = pack_bf16x2(pe2[2], pe2[3]);
      }
      // O += P V: ldmatrix.trans gives the V fragments of two 8-dim n-tiles per call
      const int lr = wr0 + (lane & 7) + ((lane >> 3) & 1) * 8;  // token row this lane addresses
      const int lc = lane >> 4;                                  // +0 / +1 chunk (second n-tile)
#pragma unroll
      for (int j = 0; j < NT / 2; ++j) {
        const int dim = j * 16;
        uint32_t vb[4];
        ldsm_x4_trans(vb, smem_u32(sv + (dim / 64) * C::SUB + swz(lr, (dim % 64) / 8 + lc)));
        mma16816(acc[2 * j], pa, vb[0], vb[1]);
        mma16816(acc[2 * j + 1], pa, vb[2], vb[3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[c % C::STAGES]);
  }
  if (!ok && producer) {
    // a wait gave up: let the copies still in flight land (bounded) before the CTA exits
    for (int c = 0; c < issued; ++c)
      mbar_wait(&full[c % C::STAGES], (c / C::STAGES) & 1, a.status, 302);
  }
  // the 4 lanes of a row group hold parts of head g's (and g + 8's) row sum
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  l2 += __shfl_xor_sync(0xffffffffu, l2, 1);
  l2 += __shfl_xor_sync(0xffffffffu, l2, 2);
  // merge the 4 warps through shared memory, reusing the ring (every warp is past its last read
  // of it and every issued copy has landed: each was waited on)
  constexpr int GR = R2 ? 16 : 8;          // heads per warp's accumulators
  static_assert(NW * GR * (D + 2) * 4 <= C::STAGES * C::STAGE, "merge buffers fit in the ring");
  __syncthreads();
  float (*sm_acc)[GR][D] = reinterpret_cast<float (*)[GR][D]>(dsm);
  float (*sm_m)[GR] = reinterpret_cast<float (*)[GR]>(dsm + NW * GR * D * 4);
  float (*sm_l)[GR] = reinterpret_cast<float (*)[GR]>(dsm + NW * GR * D * 4 + NW * GR * 4);
  if (t == 0) {
    sm_m[warp][g] = m;
    sm_l[warp][g] = l;
    if (R2) {
      sm_m[warp][(g + 8) % GR] = m2;
      sm_l[warp][(g + 8) % GR] = l2;
    }
  }
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    sm_acc[warp][g][i * 8 + 2 * t] = acc[i][0];
    sm_acc[warp][g][i * 8 + 2 * t + 1] = acc[i][1];
    if (R2) {
      sm_acc[warp][(g + 8) % GR][i * 8 + 2 * t] = acc[i][2];
      sm_acc[warp][(g + 8) % GR][i * 8 + 2 * t + 1] = acc[i][3];
    }
  }
  __syncthreads();
  // each thread finalises (g, d) entries: G * D outputs over 128 threads
  float* po = a.part_o + ((long)(b * H + h * G) * a.splits + split) * D;   // [B,H,splits,D]
  float* pml = a.part_lse + (long)(b * H + h * G) * a.splits + split;      // [B,H,splits]
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int gg = i / D, d = i % D;
    float mx = -INFINITY;
#pragma unroll
    for (int r = 0; r < NW; ++r) mx = fmaxf(mx, sm_m[r][gg]);
    float ls = 0.f, o = 0.f;
    if (mx > -INFINITY) {
#pragma unroll
      for (int r = 0; r < NW; ++r) {
        const float w = fast_exp2(sm_m[r][gg] - mx);
        ls += sm_l[r][gg] * w;
        o += sm_acc[r][gg][d] * w;
      }
    }
    po[(long)gg * a.splits * D + d] = ls > 0.f ? o / ls : 0.f;
    if (d == 0) pml[(long)gg * a.splits] = ls > 0.f ? mx + __log2f(ls) : -INFINITY;
  }
  // last CTA of this (b, h) combines the splits and publishes the rank partial
  __shared__ bool is_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(a.split_counter + b * a.Hkv + h, 1u);
    is_last = (prev == unsigned(eff) - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const unsigned long long epoch =
      a.epoch_parity_src ? (*a.epoch_parity_src * a.epoch_mul + a.epoch_add) : a.epoch_add;
  const int parity = int(epoch & 1ull);
  // split weights: all LSEs into shared memory at once (L2 reads, the other CTAs' writes are
  // visible after the fence + counter), then one warp per head reduces max and weight sum
  __shared__ float s_w[G][kMaxDecodeSplits];
  __shared__ float s_mx[G], s_ws[G];
  {
    // every load issued before any store (G * eff <= 16 * 128: at most 16 per thread)
    constexpr int LW = (G * kMaxDecodeSplits + 127) / 128;
    float lw[LW];
#pragma unroll
    for (int k = 0; k < LW; ++k) {
      const int i = threadIdx.x + k * 128;
      lw[k] = i < G * eff ? __ldcg(a.part_lse + (long)(b * H + h * G + i / eff) * a.splits + i % eff) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < LW; ++k) {
      const int i = threadIdx.x + k * 128;
      if (i < G * eff) s_w[i / eff][i % eff] = lw[k];
    }
  }
  __syncthreads();
  for (int g = warp; g < G; g += 4) {
    float mx = -INFINITY;
    for (int s = lane; s < eff; s += 32) mx = fmaxf(mx, s_w[g][s]);
    mx = warp_max(mx);
    float ws = 0.f;
    for (int s = lane; s < eff; s += 32) {
      const float w = mx == -INFINITY ? 0.f : fast_exp2(s_w[g][s] - mx);
      s_w[g][s] = w;
      ws += w;
    }
    ws = warp_sum(ws);
    if (lane == 0) {
      s_mx[g] = mx;
      s_ws[g] = ws;
    }
  }
  __syncthreads();
  // work item = 4 consecutive dims of one head (G * D / 4 items); with fewer items than threads
  // the splits of an item are dealt to `parts` threads (split s to thread s % parts) whose
  // partial sums meet in shared memory, so each thread has ceil(eff / parts) instead of eff
  // splits to load: 16-byte L2 loads, 16 in flight per round. This tail runs after every split
  // of the group is done, so its latency adds to the kernel's.
  constexpr int ITEMS = G * (D / 4);
  constexpr int PARTS = ITEMS >= 128 ? 1 : 128 / ITEMS;
  __shared__ float4 s_part[PARTS > 1 ? (PARTS - 1) * ITEMS : 1];
  auto accum = [&](int g, int d4, int first) {
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    if (s_mx[g] == -INFINITY) return o;
    const float4* pof = reinterpret_cast<const float4*>(a.part_o + (long)(b * H + h * G + g) * a.splits * D) + d4;
    for (int s0 = first; s0 < eff; s0 += 16 * PARTS) {
      float4 v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int sp = s0 + j * PARTS;
        v[j] = sp < eff ? __ldcg(pof + (long)sp * (D / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int sp = s0 + j * PARTS;
        if (sp < eff) {
          const float w = s_w[g][sp];
          o.x = fmaf(w, v[j].x, o.x);
          o.y = fmaf(w, v[j].y, o.y);
          o.z = fmaf(w, v[j].z, o.z);
          o.w = fmaf(w, v[j].w, o.w);
        }
      }
    }
    return o;
  };
  float4 o_part = make_float4(0.f, 0.f, 0.f, 0.f);
  if (PARTS > 1) {
    const int item = threadIdx.x % ITEMS, part = threadIdx.x / ITEMS;
    if (part < PARTS) {
      o_part = accum(item / (D / 4), item % (D / 4), part);
      if (part > 0) s_part[(part - 1) * ITEMS + item] = o_part;
    }
    __syncthreads();
  }
  for (int c = threadIdx.x; c < ITEMS; c += blockDim.x) {
    const int g = c / (D / 4), d4 = c % (D / 4);
    float4 o;
    if (PARTS > 1) {
      o = o_part;
#pragma unroll
      for (int q = 1; q < PARTS; ++q) {
        const float4 u = s_part[(q - 1) * ITEMS + c];
        o = make_float4(o.x + u.x, o.y + u.y, o.z + u.z, o.w + u.w);
      }
    } else {
      o = accum(g, d4, 0);
    }
    if (s_mx[g] != -INFINITY) {
      const float inv = 1.f / s_ws[g];
      o = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
    }
    if (a.final_out != nullptr) {
      // single rank: this is the layer's attention output
      __nv_bfloat16* dst = a.final_out + ((long)b * H + h * G + g) * D + d4 * 4;
      *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(o.x, o.y), pack_bf16x2(o.z, o.w));
      continue;
    }
    // exchange slot layout: [2 parity][N src][B][H][D+1] fp32
    const long off = (((long)parity * a.n_ranks + a.my_rank) * a.B * H + (long)b * H + h * G + g) * (D + 1) + d4 * 4;
    for (int r = 0; r < a.n_ranks; ++r) {
      float* x = a.xslot_ptrs[r] + off;
      x[0] = o.x;
      x[1] = o.y;
      x[2] = o.z;
      x[3] = o.w;
    }
  }
  if (a.final_out == nullptr && threadIdx.x < G) {
    const int g = threadIdx.x;
    const float lse = s_mx[g] == -INFINITY ? -INFINITY : s_mx[g] + __log2f(s_ws[g]);
    const long off = (((long)parity * a.n_ranks + a.my_rank) * a.B * H + (long)b * H + h * G + g) * (D + 1) + D;
    for (int r = 0; r < a.n_ranks; ++r) a.xslot_ptrs[r][off] = lse;
  }
  if (threadIdx.x == 0) a.split_counter[b * a.Hkv + h] = 0;
  if (a.final_out != nullptr) return;  // single rank: nothing to signal
  if (a.combine_out != nullptr) {
    // in-kernel exchange of this (row, KV head) group: publish, wait for the other ranks' partial
    // of the same group, combine in rank order (every rank computes identical bits)
    __shared__ int all_arrived;
    const long gslot = (long)b * a.Hkv + h;
    __syncthreads();
    if (threadIdx.x == 0) {
      all_arrived = 1;
      __threadfence_system();
      for (int r = 0; r < a.n_ranks; ++r)
        st_release_sys(a.group_flag_ptrs[r] + (long)a.my_rank * a.group_stride + gslot, epoch);
    }
    __syncthreads();
    if (threadIdx.x < a.n_ranks && threadIdx.x != a.my_rank &&
        !wait_flag_geq_sys(a.group_flags + (long)threadIdx.x * a.group_stride + gslot, epoch,
                           a.budget_ns, a.status, 305, threadIdx.x))
      all_arrived = 0;
    __syncthreads();
    const float* xs = a.xslot_ptrs[a.my_rank] + (long)parity * a.n_ranks * a.B * H * (D + 1);
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
      const int g = i / D, d = i % D;
      const int hh = h * G + g;
      float out = 0.f;
      if (all_arrived) {
        float mx = -INFINITY;
        for (int r = 0; r < a.n_ranks; ++r)
          mx = fmaxf(mx, __ldcg(xs + (((long)r * a.B + b) * H + hh) * (D + 1) + D));
        if (mx > -INFINITY) {
          float ws = 0.f, o = 0.f;
          for (int r = 0; r < a.n_ranks; ++r) {
            const long base = (((long)r * a.B + b) * H + hh) * (D + 1);
            const float w = fast_exp2(__ldcg(xs + base + D) - mx);
            ws += w;
            o += w * __ldcg(xs + base + d);
          }
          out = o / ws;
        }
      }
      a.combine_out[((long)b * H + hh) * D + d] = __float2bfloat16(out);
    }
    return;
  }
  // grid-wide last CTA signals every rank that this rank's partial has landed
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned prev = atomicAdd(a.grid_counter, 1u);
    if (prev == unsigned(a.B * a.Hkv) - 1) {
      __threadfence_system();
      for (int r = 0; r < a.n_ranks; ++r) st_release_sys(a.ready_ptrs[r], epoch);
      *a.grid_counter = 0;
    }
  }
}

// grid (B, H), block D: wait for every rank's partial (bounded), then LSE-combine in rank
// order (the same order on every rank, so every rank produces bit-identical outputs).
__global__ void decode_combine_kernel(DecodeCombineArgs a) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, hh = blockIdx.y, d = threadIdx.x;
  const unsigned long long e = a.epoch_src ? (*a.epoch_src * a.epoch_mul + a.epoch_add) : a.epoch_add;
  const int parity = int(e & 1ull);
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (a.ready != nullptr && threadIdx.x < a.n_ranks) {
    if (!wait_flag_geq_sys(a.ready + threadIdx.x, e, a.budget_ns, a.status, 401, threadIdx.x)) ok = 0;
  }
  __syncthreads();
  const int H = a.H, D = a.D;
  const float* xs = a.xslot + (long)parity * a.n_ranks * a.B * H * (D + 1);
  float out = 0.f;
  if (ok) {
    float mx = -INFINITY;
    for (int r = 0; r < a.n_ranks; ++r)
      mx = fmaxf(mx, __ldcg(xs + (((long)r * a.B + b) * H + hh) * (D + 1) + D));
    if (mx > -INFINITY) {
      float ws = 0.f, o = 0.f;
      for (int r = 0; r < a.n_ranks; ++r) {
        const long base = (((long)r * a.B + b) * H + hh) * (D + 1);
        const float w = fast_exp2(__ldcg(xs + base + D) - mx);
        ws += w;
        o += w * __ldcg(xs + base + d);
      }
      out = o / ws;
    }
  }
  a.out[((long)b * H + hh) * D + d] = __float2bfloat16(out);
}

template <int D, int G>
static cudaError_t prepare_attn() {
  static std::atomic<unsigned long long> done{0};
  return once_per_device(done, [] {
    cudaError_t e = cudaFuncSetAttribute(decode_attn_kernel<D, G>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, DecCfg<D>::SMEM);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(decode_attn_kernel<D, G>, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
    return e;
  });
}

template <int D, int G>
static cudaError_t launch_attn(const CUtensorMap& tm, const DecodeAttnArgs& a, cudaStream_t s) {
  cudaError_t e = prepare_attn<D, G>();
  if (e != cudaSuccess) return e;
  dim3 grid(a.splits, a.Hkv, a.B);
  if (a.combine_out != nullptr) {
    // the groups' last CTAs wait for the other ranks' CTAs: every CTA must be resident at once
    int occ = 0, dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_attn_kernel<D, G>, 128, DecCfg<D>::SMEM);
    if (long(a.splits) * a.Hkv * a.B > long(occ) * sms) return cudaErrorCooperativeLaunchTooLarge;
  }
  return launch_pdl(decode_attn_kernel<D, G>, grid, dim3(128), size_t(DecCfg<D>::SMEM), s, tm, a);
}

const char* decode_attn(const DecodeAttnArgs& a, cudaStream_t s) {
  const int G = a.H / a.Hkv;
  if (a.H % a.Hkv) return "decode_attn: H % Hkv";
  if (a.n_ranks < 1 || a.n_ranks > kMaxRanks) return "decode_attn: bad n_ranks";
  if (a.final_out != nullptr && a.n_ranks != 1) return "decode_attn: final_out is for a single rank";
  if (a.combine_out != nullptr &&
      (a.n_ranks < 2 || a.n_ranks > 128 || a.group_flag_ptrs == nullptr || a.group_flags == nullptr ||
       a.group_stride < a.B * a.Hkv))
    return "decode_attn: the in-kernel combine needs 2+ ranks and the group flags";
  if (a.splits < 1 || a.splits > kMaxDecodeSplits) return "decode_attn: splits must be in [1, 128]";
  if ((a.D != 64 && a.D != 128) || a.geom.page % kDecCC)
    return "decode_attn: head_dim must be 64 or 128 and the page a multiple of 64 rows";
  if (G > 16) return "decode_attn: at most 16 query heads per KV head";
  for (int i = 0; i < 2; ++i)
    if (a.pf.ptr[i] && ((reinterpret_cast<uintptr_t>(a.pf.ptr[i]) | a.pf.bytes[i]) & 15))
      return "decode_attn: L2 prefetch ranges must be 16-byte aligned multiples of 16 bytes";
  if (a.pt_stride < 1) return "decode_attn: page-table row stride must be at least 1";
  if (reinterpret_cast<uintptr_t>(a.arena) & 15) return "decode_attn: arena must be 16-byte aligned";
  // the whole arena as one [rows, D] bf16 matrix; boxes of 64 rows x 64 dims, 128-byte swizzle
  const unsigned long long rows =
      (unsigned long long)a.geom.layers * a.geom.pages * 2 * a.geom.hkv * a.geom.page;
  if (rows >= (1ull << 31)) return "decode_attn: arena has too many rows for 32-bit TMA coordinates";
  CUtensorMap tm;
  if (!gemm::make_tma_2d_bf16(&tm, a.arena, uint64_t(a.D), rows, uint64_t(a.D) * 2, 64, kDecCC))
    return "decode_attn: TMA descriptor for the arena failed";
  cudaError_t e = cudaErrorInvalidValue;
#define HCP_DEC_CASE(DD, GG) \
  if (a.D == DD && G == GG) e = launch_attn<DD, GG>(tm, a, s);
  // every GQA group size up to 16 query heads per KV head: 1, 2, 4, 8 (Llama 3, Qwen2.5-3B),
  // 3 (Llama-3.2-3B), 5 (Qwen2.5-14B), 6 (Qwen2.5-1.5B), 7 (Qwen2-0.5B, Qwen2.5-7B), 16
  // (Llama-3.1-405B) and the sizes between
  HCP_DEC_CASE(64, 1) HCP_DEC_CASE(64, 2) HCP_DEC_CASE(64, 3) HCP_DEC_CASE(64, 4)
  HCP_DEC_CASE(64, 5) HCP_DEC_CASE(64, 6) HCP_DEC_CASE(64, 7) HCP_DEC_CASE(64, 8)
  HCP_DEC_CASE(64, 9) HCP_DEC_CASE(64, 10) HCP_DEC_CASE(64, 11) HCP_DEC_CASE(64, 12)
  HCP_DEC_CASE(64, 13) HCP_DEC_CASE(64, 14) HCP_DEC_CASE(64, 15) HCP_DEC_CASE(64, 16)
  HCP_DEC_CASE(128, 1) HCP_DEC_CASE(128, 2) HCP_DEC_CASE(128, 3) HCP_DEC_CASE(128, 4)
  HCP_DEC_CASE(128, 5) HCP_DEC_CASE(128, 6) HCP_DEC_CASE(128, 7) HCP_DEC_CASE(128, 8)
  HCP_DEC_CASE(128, 9) HCP_DEC_CASE(128, 10) HCP_DEC_CASE(128, 11) HCP_DEC_CASE(128, 12)
  HCP_DEC_CASE(128, 13) HCP_DEC_CASE(128, 14) HCP_DEC_CASE(128, 15) HCP_DEC_CASE(128, 16)
#undef HCP_DEC_CASE
  if (e == cudaErrorInvalidValue) return "decode_attn: unsupported (D, H/Hkv)";
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

int decode_attn_ctas_per_sm(int D, int G) {
  int n = 0;
#define HCP_DEC_OCC(DD, GG)                                                                      \
  if (D == DD && G == GG && prepare_attn<DD, GG>() == cudaSuccess)                                 \
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_attn_kernel<DD, GG>, 128, DecCfg<DD>::SMEM);
  HCP_DEC_OCC(64, 1) HCP_DEC_OCC(64, 2) HCP_DEC_OCC(64, 3) HCP_DEC_OCC(64, 4)
  HCP_DEC_OCC(64, 5) HCP_DEC_OCC(64, 6) HCP_DEC_OCC(64, 7) HCP_DEC_OCC(64, 8)
  HCP_DEC_OCC(64, 9) HCP_DEC_OCC(64, 10) HCP_DEC_OCC(64, 11) HCP_DEC_OCC(64, 12)
  HCP_DEC_OCC(64, 13) HCP_DEC_OCC(64, 14) HCP_DEC_OCC(64, 15) HCP_DEC_OCC(64, 16)
  HCP_DEC_OCC(128, 1) HCP_DEC_OCC(128, 2) HCP_DEC_OCC(128, 3) HCP_DEC_OCC(128, 4)
  HCP_DEC_OCC(128, 5) HCP_DEC_OCC(128, 6) HCP_DEC_OCC(128, 7) HCP_DEC_OCC(128, 8)
  HCP_DEC_OCC(128, 9) HCP_DEC_OCC(128, 10) HCP_DEC_OCC(128, 11) HCP_DEC_OCC(128, 12)
  HCP_DEC_OCC(128, 13) HCP_DEC_OCC(128, 14) HCP_DEC_OCC(128, 15) HCP_DEC_OCC(128, 16)
#undef HCP_DEC_OCC
  return n;
}

const char* decode_combine(const DecodeCombineArgs& a, cudaStream_t s) {
  if (a.n_ranks > a.D) return "decode_combine: more ranks than head_dim threads";
  return launch_pdl(decode_combine_kernel, dim3(a.B, a.H), dim3(a.D), 0, s, a) == cudaSuccess
             ? nullptr
             : "decode_combine: launch failed";
}

// ----------------------------------------------------------------------------- small helpers
__global__ void fill_u64_kernel(unsigned long long* p, int n, unsigned long long v) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

__global__ void argmax_finalize_kernel(const unsigned long long* packed, int B, int* tokens_out,
                                       long long* tokens_out64) {
  pdl_trigger();
  pdl_wait();
  const int b = threadIdx.x;
  if (b < B) {
    const int idx = int(0xFFFFFFFFu - uint32_t(packed[b] & 0xFFFFFFFFull));
    if (tokens_out) tokens_out[b] = idx;
    if (tokens_out64) tokens_out64[b] = idx;
  }
}

// One CTA: thread t < world * B first stores row b = t % B of this rank's maxima into rank
// t / B's slot [parity][my_rank][b], then reads rank t / B's entry of row b from its own slots.
// For t / B == my_rank the store and the read are the same thread's, in program order.
__global__ void argmax_exchange_kernel(ArgmaxXchgArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ unsigned long long best[8];
  const int t = threadIdx.x;
  const unsigned long long e = *a.epoch_src;
  const int par = int(e & 1ull);
  if (t < a.B) best[t] = 0ull;
  __syncthreads();
  if (t < a.world * a.B) {
    const int r = t / a.B, b = t % a.B;
    unsigned long long* sl = a.slot_ptrs[r] + ((long(par) * a.world + a.my_rank) * a.max_batch + b) * 2;
    *reinterpret_cast<volatile unsigned long long*>(sl) = a.local[b];
    st_release_sys(sl + 1, e);   // orders the value store before the epoch
    const unsigned long long* own = a.own_slots + ((long(par) * a.world + r) * a.max_batch + b) * 2;
    if (wait_flag_geq_sys(own + 1, e, a.budget_ns, a.status, 306, r))
      atomicMax(&best[b], *reinterpret_cast<const volatile unsigned long long*>(own));
  }
  __syncthreads();
  if (t < a.B) {
    const int idx = int(0xFFFFFFFFu - uint32_t(best[t] & 0xFFFFFFFFull));
    if (a.tok32) a.tok32[t] = idx;
    if (a.tok64) a.tok64[t] = idx;
  }
}

__global__ void add_u64_kernel(unsigned long long* p, unsigned long long v) {
  pdl_trigger();
  pdl_wait();
  *p += v;
}

const char* fill_u64(unsigned long long* p, int n, unsigned long long v, cudaStream_t s) {
  if (n == 0) return nullptr;
  return launch_pdl(fill_u64_kernel, dim3((n + 255) / 256), dim3(256), 0, s, p, n, v) == cudaSuccess ? nullptr : "fill_u64: launch failed";
}

const char* argmax_finalize(const unsigned long long* packed, int B, int* tok, long long* tok64,
                            cudaStream_t s) {
  return launch_pdl(argmax_finalize_kernel, dim3(1), dim3(32), 0, s, packed, B, tok, tok64) == cudaSuccess ? nullptr : "argmax_finalize: launch failed";
}

const char* argmax_exchange(const ArgmaxXchgArgs& a, cudaStream_t s) {
  if (a.B < 1 || a.B > 8 || a.B > a.max_batch) return "argmax_exchange: B must be in [1, min(8, max_batch)]";
  if (a.world < 1 || a.world * a.B > 1024 || a.my_rank < 0 || a.my_rank >= a.world)
    return "argmax_exchange: bad world / rank";
  if (!a.local || !a.slot_ptrs || !a.own_slots || !a.epoch_src) return "argmax_exchange: null pointer";
  const int threads = (a.world * a.B + 31) / 32 * 32;
  return launch_pdl(argmax_exchange_kernel, dim3(1), dim3(threads), 0, s, a) == cudaSuccess
             ? nullptr
             : "argmax_exchange: launch failed";
}

const char* add_u64(unsigned long long* p, unsigned long long v, cudaStream_t s) {
  return launch_pdl(add_u64_kernel, dim3(1), dim3(1), 0, s, p, v) == cudaSuccess ? nullptr : "add_u64: launch failed";
}

}  // namespace dec
}  // namespace hcp

// ============================================================================================
// Allocation-free single-rank decode attention (see decode_noalloc.h for the contract).
//
// For callers that cannot allocate device memory: the split-KV scratch (partials, counters, the
// one-rank exchange slot and its pointer tables) and a device status word live in
// `g_decode_noalloc_scratch`, a file-scope array every device holds while the library is
// loaded. Host code never passes the array's name to a kernel (in host code it is only a
// stand-in for the symbol); it passes the device address obtained with cudaGetSymbolAddress once
// per device context.
// ============================================================================================
#include <mutex>
#include <string>

#include "decode_noalloc.h"

namespace {

constexpr unsigned long long kNoAllocBytes = HCP_DECODE_NOALLOC_SCRATCH_BYTES;
constexpr int kNoAllocMaxDevices = 64;
constexpr unsigned long long kNoAllocTooBig = ~0ull;

static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[HCP_DECODE_NOALLOC_SCRATCH_BYTES];

// Status area at the start of the array: the live words the kernels of the current call report
// into (code, site, info, info), then the first error of an earlier call that was not read yet.
constexpr unsigned long long kStatusLive = 0;
constexpr unsigned long long kStatusHeld = 16;
constexpr unsigned long long kStatusBytes = 256;

struct DeviceSlot {
  void* addr = nullptr;            // device address of the scratch array in this context
  unsigned long long ctx_id = 0;   // the context it was looked up in (0: unknown)
};

std::mutex g_noalloc_mu;
DeviceSlot g_noalloc_slot[kNoAllocMaxDevices];
thread_local std::string g_noalloc_err;

// Identifier of the current context (driver API, looked up at run time): a primary context that
// was reset and created again gets a new identifier, so a cached address is looked up again.
unsigned long long current_context_id() {
  typedef int (*CtxGetCurrent)(void**);
  typedef int (*CtxGetId)(void*, unsigned long long*);
  static CtxGetCurrent get_cur = nullptr;
  static CtxGetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<CtxGetCurrent>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetId>(f);
  });
  if (get_cur == nullptr || get_id == nullptr) return 0;
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (get_cur(&ctx) != 0 || ctx == nullptr || get_id(ctx, &id) != 0) return 0;
  return id;
}

// Byte layout inside the scratch array (all offsets 256-byte aligned, sizes in 64-bit
// arithmetic so no product of the caller's sizes can overflow).
struct NoAllocLayout {
  unsigned long long counters, tables, flag, part_o, part_lse, xslot, total;
};

unsigned long long align256(unsigned long long v) { return (v + 255ull) & ~255ull; }

NoAllocLayout noalloc_layout(int B, int H, int Hkv, int D, int splits) {
  const unsigned long long b = (unsigned long long)B, h = (unsigned long long)H,
                           hkv = (unsigned long long)Hkv, d = (unsigned long long)D,
                           sp = (unsigned long long)splits;
  NoAllocLayout l{};
  unsigned long long off = kStatusBytes;
  l.counters = off;
  off = align256(off + sizeof(unsigned int) * (b * hkv + 1ull));
  l.tables = off;  // float* xslot_ptrs[1]; unsigned long long* ready_ptrs[1]
  off = align256(off + 2 * sizeof(void*));
  l.flag = off;
  off = align256(off + sizeof(unsigned long long));
  l.part_o = off;
  off = align256(off + sizeof(float) * b * h * sp * d);
  l.part_lse = off;
  off = align256(off + sizeof(float) * b * h * sp);
  l.xslot = off;
  off = align256(off + sizeof(float) * 2ull * b * h * (d + 1ull));
  l.total = off;
  return l;
}

// Start of a call: the first unread error of the previous calls moves to the held slot, the live
// words restart at zero (so a stale error cannot cut this call's waits short), the completion
// counters are cleared and the one-entry tables point at the scratch.
__global__ void noalloc_setup_kernel(unsigned char* base, NoAllocLayout l, int n_counters) {
  unsigned int* counters = reinterpret_cast<unsigned int*>(base + l.counters);
  for (int i = threadIdx.x; i < n_counters; i += blockDim.x) counters[i] = 0u;
  if (threadIdx.x == 0) {
    int* live = reinterpret_cast<int*>(base + kStatusLive);
    int* held = reinterpret_cast<int*>(base + kStatusHeld);
    if (live[0] != 0 && held[0] == 0)
      for (int i = 0; i < 4; ++i) held[i] = live[i];
    for (int i = 0; i < 4; ++i) live[i] = 0;
    void** tables = reinterpret_cast<void**>(base + l.tables);
    tables[0] = base + l.xslot;
    tables[1] = base + l.flag;
    *reinterpret_cast<unsigned long long*>(base + l.flag) = 0ull;
  }
}

int noalloc_fail(int code, const std::string& msg) {
  g_noalloc_err = msg;
  return code;
}

// Device address of the scratch array for the current device and context (looked up the first
// time a device or a new context is seen).
int noalloc_base(unsigned char** base) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return noalloc_fail(int(e), cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return noalloc_fail(-8, "hcp_decode_attention_noalloc: device index out of range");
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  DeviceSlot& slot = g_noalloc_slot[dev];
  if (slot.addr == nullptr || (ctx != 0 && slot.ctx_id != ctx)) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
    if (e != cudaSuccess)
      return noalloc_fail(int(e), std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    slot.addr = p;
    slot.ctx_id = ctx;
  }
  *base = static_cast<unsigned char*>(slot.addr);
  return 0;
}

}  // namespace

extern "C" unsigned long long hcp_decode_attention_noalloc_scratch_bytes(int batch, int heads,
                                                                         int hkv, int d,
                                                                         int splits) {
  if (batch < 1 || heads < 1 || hkv < 1 || d < 1 || splits < 1) return kNoAllocTooBig;
  return noalloc_layout(batch, heads, hkv, d, splits).total;
}

extern "C" const char* hcp_decode_attention_noalloc_error(void) { return g_noalloc_err.c_str(); }

extern "C" int hcp_decode_attention_noalloc_status(int* words, cudaStream_t stream) {
  g_noalloc_err.clear();
  if (words == nullptr) return noalloc_fail(-1, "hcp_decode_attention_noalloc_status: null words");
  unsigned char* base = nullptr;
  int rc = noalloc_base(&base);
  if (rc != 0) return rc;
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return noalloc_fail(int(e), cudaGetErrorString(e));
  int st[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  e = cudaMemcpy(st, base + kStatusLive, sizeof(st), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return noalloc_fail(int(e), cudaGetErrorString(e));
  const int* first = st[4] != 0 ? st + 4 : st;   // an earlier call's unread error comes first
  for (int i = 0; i < 4; ++i) words[i] = first[i];
  const int zero[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  e = cudaMemcpy(base + kStatusLive, zero, sizeof(zero), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return noalloc_fail(int(e), cudaGetErrorString(e));
  return 0;
}

extern "C" int hcp_decode_attention_noalloc(const void* q, const void* arena, int layers,
                                            int pages, int page, int hkv, int d, int layer,
                                            const int* page_tables, int pt_stride,
                                            const int* n_tokens, int batch, int heads,
                                            float scale, int splits, void* out,
                                            cudaStream_t stream) {
  g_noalloc_err.clear();
  if (!q || !arena || !page_tables || !n_tokens || !out)
    return noalloc_fail(-1, "hcp_decode_attention_noalloc: null pointer argument");
  if (batch < 1 || heads < 1 || hkv < 1 || splits < 1 || layers < 1 || pages < 1 || page < 1 ||
      pt_stride < 1)
    return noalloc_fail(-2, "hcp_decode_attention_noalloc: sizes (and the page-table row stride) must be positive");
  if (layer < 0 || layer >= layers)
    return noalloc_fail(-3, "hcp_decode_attention_noalloc: layer out of range");
  if (d != 64 && d != 128) return noalloc_fail(-4, "hcp_decode_attention_noalloc: head_dim must be 64 or 128");
  if (heads % hkv) return noalloc_fail(-5, "hcp_decode_attention_noalloc: heads % kv_heads != 0");
  const int G = heads / hkv;
  if (G < 1 || G > 16)
    return noalloc_fail(-6, "hcp_decode_attention_noalloc: heads / kv_heads must be 1 to 16");
  if ((long long)pt_stride * page > 0x7fffffffLL)
    return noalloc_fail(-2, "hcp_decode_attention_noalloc: pt_stride * page exceeds 2^31 - 1 tokens");
  const NoAllocLayout lay = noalloc_layout(batch, heads, hkv, d, splits);
  if (lay.total > kNoAllocBytes)
    return noalloc_fail(-7, "hcp_decode_attention_noalloc: problem needs " + std::to_string(lay.total) +
                                " bytes of scratch, more than the static maximum of " +
                                std::to_string(kNoAllocBytes) + " bytes; lower batch or splits");
  unsigned char* base = nullptr;
  int rc = noalloc_base(&base);
  if (rc != 0) return rc;
  int* status = reinterpret_cast<int*>(base + kStatusLive);
  noalloc_setup_kernel<<<1, 256, 0, stream>>>(base, lay, batch * hkv + 1);
  hcp::dec::DecodeAttnArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.arena = static_cast<const __nv_bfloat16*>(arena);
  a.geom = hcp::ArenaGeom{layers, pages, page, hkv, d};
  a.layer = layer;
  a.page_tables = page_tables;
  a.pt_stride = pt_stride;
  a.n_tokens = n_tokens;
  a.B = batch;
  a.H = heads;
  a.Hkv = hkv;
  a.D = d;
  a.scale = scale;
  a.splits = splits;
  a.part_o = reinterpret_cast<float*>(base + lay.part_o);
  a.part_lse = reinterpret_cast<float*>(base + lay.part_lse);
  a.split_counter = reinterpret_cast<unsigned int*>(base + lay.counters);
  a.grid_counter = a.split_counter + batch * hkv;
  a.xslot_ptrs = reinterpret_cast<float* const*>(base + lay.tables);
  a.n_ranks = 1;
  a.my_rank = 0;
  a.ready_ptrs = reinterpret_cast<unsigned long long* const*>(base + lay.tables + sizeof(void*));
  a.epoch_parity_src = nullptr;
  a.epoch_mul = 0;
  a.epoch_add = 1;
  a.status = status;
  const char* err = hcp::dec::decode_attn(a, stream);
  if (err) return noalloc_fail(-9, err);
  hcp::dec::DecodeCombineArgs c{};
  c.xslot = reinterpret_cast<const float*>(base + lay.xslot);
  c.ready = nullptr;
  c.epoch_src = nullptr;
  c.epoch_mul = 0;
  c.epoch_add = 1;
  c.n_ranks = 1;
  c.B = batch;
  c.H = heads;
  c.D = d;
  c.out = static_cast<__nv_bfloat16*>(out);
  c.budget_ns = 0;
  c.status = status;
  err = hcp::dec::decode_combine(c, stream);
  if (err) return noalloc_fail(-10, err);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : noalloc_fail(int(e), cudaGetErrorString(e));
}
