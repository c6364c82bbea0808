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
#include "kv_layout.h"

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
constexpr int GEMV_THREADS = 256;

template <int EPI, int B, bool NORM>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(GemvArgs a) {
  extern __shared__ uint4 xs[];                     // [B][K/8] (normalised when NORM)
  __shared__ float red[GEMV_THREADS / 32][B];
  __shared__ float rstd[B];
  constexpr int NWR = (EPI == kGemvSwiGLU) ? 2 : 1;  // weight rows per output row
  constexpr int KC = 8 / NWR;                        // 16-byte columns per lane per chunk and row
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const int kvec = a.K / 8;
  const int out_rows = (EPI == kGemvSwiGLU) ? a.N / 2 : a.N;
  const int nchunk = (kvec + 32 * KC - 1) / (32 * KC);
  const int gw = blockIdx.x * (GEMV_THREADS / 32) + warp;
  const int nwarps = gridDim.x * (GEMV_THREADS / 32);
  const int my_rows = gw < out_rows ? (out_rows - 1 - gw) / nwarps + 1 : 0;
  const int items = my_rows * nchunk;
  auto load = [&](int item, uint4 (&buf)[NWR][KC]) {
    const int o = gw + (item / nchunk) * nwarps;
    const int c = item % nchunk;
    const int w0 = (EPI == kGemvSwiGLU) ? (o / 128) * 256 + (o % 128) : o;
#pragma unroll
    for (int q = 0; q < NWR; ++q) {
      const uint4* wp = reinterpret_cast<const uint4*>(a.W + (long)(w0 + q * 128) * a.K);
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        const int k = c * 32 * KC + j * 32 + lane;
        buf[q][j] = k < kvec ? ld_stream(wp + k) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
  };
  uint4 bufA[NWR][KC], bufB[NWR][KC];
  if (items > 0) load(0, bufA);
  if (NORM) {
    float ss[B];
#pragma unroll
    for (int b = 0; b < B; ++b) ss[b] = 0.f;
    for (int k = tid; k < kvec; k += GEMV_THREADS) {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(a.x + (long)b * a.ldx) + k);
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
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(a.x + (long)b * a.ldx) + k);
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
      for (int b = 0; b < B; ++b) xs[b * kvec + k] = __ldg(reinterpret_cast<const uint4*>(a.x + (long)b * a.ldx) + k);
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
    if (c != nchunk - 1) return;
    // row complete: every lane gets every sum; lane b finishes input row b
#pragma unroll
    for (int q = 0; q < NWR; ++q)
#pragma unroll
      for (int b = 0; b < B; ++b) acc[q][b] = warp_sum(acc[q][b]);
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const float v = acc[0][b];
      if (EPI == kGemvArgmax) {
        const unsigned long long cnd = pack_argmax(v, o);
        best[b] = cnd > best[b] ? cnd : best[b];
      }
      if (lane != b) continue;
      if (EPI == kGemvF32) {
        a.y_f32[(long)b * a.ldy + o] = a.bias ? v + __bfloat162float(a.bias[o]) : v;
      } else if (EPI == kGemvResidual) {
        __nv_bfloat16* y = a.y_bf16 + (long)b * a.ldy + o;
        *y = __float2bfloat16(__bfloat162float(__float2bfloat16(v)) + __bfloat162float(*y));
      } else if (EPI == kGemvSwiGLU) {
        const float g = __bfloat162float(__float2bfloat16(v));
        const float uu = __bfloat162float(__float2bfloat16(acc[NWR - 1][b]));
        const float sg = g / (1.f + fast_exp2(-g * kLog2e));
        a.y_bf16[(long)b * a.ldy + o] = __float2bfloat16(sg * uu);
      } else if (EPI == kGemvArgmax) {
        if (a.y_f32) a.y_f32[(long)b * a.ldy + o] = v;
      }
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
  if (EPI == kGemvArgmax && lane == 0) {
#pragma unroll
    for (int b = 0; b < B; ++b)
      if (best[b]) atomicMax(a.argmax + b, best[b]);
  }
}

template <int EPI, bool NORM>
static cudaError_t gemv_launch(const GemvArgs& a, cudaStream_t s) {
  const size_t smem = size_t(a.B) * a.K * 2;
  auto go = [&](auto kernel) -> cudaError_t {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      if (e != cudaSuccess) return e;
    }
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, GEMV_THREADS, smem) != cudaSuccess || occ < 1)
      occ = 1;
    const int out_rows = (EPI == kGemvSwiGLU) ? a.N / 2 : a.N;
    const int need = (out_rows + GEMV_THREADS / 32 - 1) / (GEMV_THREADS / 32);
    const int grid = need < occ * a.num_sms ? need : occ * a.num_sms;
    kernel<<<grid, GEMV_THREADS, smem, s>>>(a);
    return cudaGetLastError();
  };
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

const char* gemv(const GemvArgs& a, cudaStream_t s) {
  if (a.K % 8 || a.ldx % 8) return "gemv: K and ldx must be multiples of 8";
  if (a.B != 1 && a.B != 2 && a.B != 4 && a.B != 8) return "gemv: B must be 1, 2, 4 or 8";
  if (a.epi == kGemvSwiGLU && a.N % 256) return "gemv: SwiGLU needs N % 256 == 0";
  if ((reinterpret_cast<uintptr_t>(a.W) | reinterpret_cast<uintptr_t>(a.x)) & 15)
    return "gemv: W/x must be 16-byte aligned";
  if (size_t(a.B) * a.K * 2 > 200 * 1024) return "gemv: needs B*K*2 <= 200 KB (x is staged in shared memory)";
  cudaError_t e;
  switch (a.epi) {
    case kGemvF32: e = gemv_dispatch<kGemvF32>(a, s); break;
    case kGemvResidual: e = gemv_dispatch<kGemvResidual>(a, s); break;
    case kGemvSwiGLU: e = gemv_dispatch<kGemvSwiGLU>(a, s); break;
    case kGemvArgmax: e = gemv_dispatch<kGemvArgmax>(a, s); break;
    default: return "gemv: unknown epilogue";
  }
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

// ----------------------------------------------------------------------------- K2 decode attention
// grid (splits, Hkv, B), 128 threads (4 warps). Each warp owns a contiguous, chunk-aligned token
// range of its split and streams it through a private STAGES-deep shared-memory ring: lane 0
// issues one bulk copy for the K rows and one for the V rows of a chunk (CT tokens, 2 KB each;
// chunks never straddle a 256-row page) and the warp waits on the chunk's mbarrier (bounded).
// A token's rows are spread over LPT lanes that each own DPL consecutive head dims (16, or 8
// for 8-head GQA groups so q and the accumulators of all G heads fit in registers). Per chunk:
// scores with packed f32x2 FMAs and an LPT-lane shuffle reduction, one warp-wide running-max
// update per head (the accumulator rescale happens once per chunk, not per token), then
// p = 2^(s - m) and O += p V with packed FMAs. The warp's token groups and the 4 warps are
// merged at the end and the split's (O, LSE) partial is written.
constexpr int kDecStages = 4;

template <int D>
struct DecChunk {
  static constexpr int CT = 1024 / D;                  // tokens per chunk (2 KB of K rows)
  static constexpr int BYTES = CT * D * 2;             // K (or V) bytes per chunk
  static constexpr int WARP_SMEM = kDecStages * 2 * BYTES;
  static constexpr int SMEM = 4 * WARP_SMEM;           // dynamic shared memory per CTA
};

template <int D, int G>
__global__ void __launch_bounds__(128) decode_attn_kernel(DecodeAttnArgs a) {
  constexpr int DPL = (G >= 8) ? 8 : 16;   // head dims per lane
  constexpr int NV = DPL / 8;              // 16-byte vectors per lane per K (or V) row
  constexpr int LPT = D / DPL;             // lanes per token
  constexpr int TPW = 32 / LPT;            // tokens per warp step
  constexpr int NW = 4;                    // warps per CTA
  constexpr int CT = DecChunk<D>::CT;
  constexpr int STEPS = CT / TPW;          // warp steps per chunk
  constexpr int BYTES = DecChunk<D>::BYTES;
  static_assert(LPT >= 1 && LPT <= 32 && 32 % LPT == 0 && CT % TPW == 0 && 256 % CT == 0, "tiling");
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ __align__(8) uint64_t bars[NW][kDecStages];
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int gl = lane % LPT;               // lane within the token group
  const int n = a.n_tokens[b];
  // chunk-aligned ranges: split -> 4 warp ranges -> CT-token chunks
  int per = (n + a.splits - 1) / a.splits;
  per = (per + NW * CT - 1) / (NW * CT) * (NW * CT);
  const int s0 = split * per;
  const int s1 = min(n, s0 + per);
  const int w0 = min(s1, s0 + warp * (per / NW));
  const int w1 = min(s1, w0 + per / NW);
  const int nc = (w1 - w0 + CT - 1) / CT;
  const int H = a.Hkv * G;
  uint8_t* wsm = dsm + warp * DecChunk<D>::WARP_SMEM;  // [stage][K | V][CT][D] bf16

  // zero the ring once (rows past the end of a range are then finite and get p = 0), init the
  // barriers, make both visible to the async proxy
  for (int i = threadIdx.x; i < DecChunk<D>::SMEM / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(dsm)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (lane == 0)
    for (int st = 0; st < kDecStages; ++st) mbar_init(&bars[warp][st], 1);
  fence_barrier_init();
  fence_proxy_async_smem();
  __syncthreads();

  const int* pt = a.page_tables + (long)b * a.pt_stride;
  auto issue = [&](int c) {
    const int t0 = w0 + c * CT;
    const int rows = min(CT, w1 - t0);
    const int page = pt[t0 / a.geom.page];
    const __nv_bfloat16* src = a.arena + a.geom.offset(a.layer, page, 0, h, t0 % a.geom.page);
    uint8_t* dst = wsm + (c % kDecStages) * 2 * BYTES;
    uint64_t* bar = &bars[warp][c % kDecStages];
    const uint32_t bytes = uint32_t(rows) * D * 2;
    mbar_arrive_expect_tx(bar, 2 * bytes);
    bulk_load(dst, src, bytes, bar);
    bulk_load(dst + BYTES, src + a.geom.kv_stride(), bytes, bar);
  };
  if (lane == 0)
    for (int c = 0; c < kDecStages - 1 && c < nc; ++c) issue(c);

  // q slice of every head of the group, pre-scaled into the log2 domain
  float2 q[G][DPL / 2];
  const float qs = a.scale * kLog2e;
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const uint4 w = *reinterpret_cast<const uint4*>(a.q + ((long)b * H + h * G + g) * D + gl * DPL + v * 8);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) q[g][v * 4 + j] = make_float2(bf16_lo(ww[j]) * qs, bf16_hi(ww[j]) * qs);
    }
  float2 acc[G][DPL / 2];
  float m[G], l[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL / 2; ++i) acc[g][i] = make_float2(0.f, 0.f);
  }
  int consumed = 0;
  bool ok = true;
  for (int c = 0; c < nc; ++c) {
    if (lane == 0 && c + kDecStages - 1 < nc) {
      fence_proxy_async_smem();  // the warp's reads of that stage (chunk c - 1) come first
      issue(c + kDecStages - 1);
    }
    ok = __all_sync(0xffffffffu, mbar_wait(&bars[warp][c % kDecStages], (c / kDecStages) & 1, a.status, 301));
    if (!ok) break;
    consumed = c + 1;
    const __nv_bfloat16* sk = reinterpret_cast<const __nv_bfloat16*>(wsm + (c % kDecStages) * 2 * BYTES);
    const __nv_bfloat16* sv = sk + CT * D;
    const int t0 = w0 + c * CT;
    float sc[STEPS][G];
#pragma unroll
    for (int u = 0; u < STEPS; ++u) {
      const int tt = u * TPW + lane / LPT;
      const bool valid = t0 + tt < w1;
      float2 kf[DPL / 2];
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const uint4 kw = *reinterpret_cast<const uint4*>(sk + tt * D + gl * DPL + v * 8);
        const uint32_t ww[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) kf[v * 4 + j] = make_float2(bf16_lo(ww[j]), bf16_hi(ww[j]));
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < DPL / 2; ++i) d2 = __ffma2_rn(q[g][i], kf[i], d2);
        float x = d2.x + d2.y;
#pragma unroll
        for (int o = LPT / 2; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        sc[u][g] = valid ? x : -INFINITY;
      }
    }
    // one running-max update per head and chunk (warp-uniform)
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float cm = sc[0][g];
#pragma unroll
      for (int u = 1; u < STEPS; ++u) cm = fmaxf(cm, sc[u][g]);
#pragma unroll
      for (int o = LPT; o < 32; o <<= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
      if (cm > m[g]) {
        const float al = fast_exp2(m[g] - cm);  // 0 while nothing has been accumulated
        m[g] = cm;
        l[g] *= al;
        const float2 al2 = make_float2(al, al);
#pragma unroll
        for (int i = 0; i < DPL / 2; ++i) acc[g][i] = __fmul2_rn(acc[g][i], al2);
      }
    }
#pragma unroll
    for (int u = 0; u < STEPS; ++u) {
      const int tt = u * TPW + lane / LPT;
      float2 vf[DPL / 2];
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const uint4 vw = *reinterpret_cast<const uint4*>(sv + tt * D + gl * DPL + v * 8);
        const uint32_t ww[4] = {vw.x, vw.y, vw.z, vw.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) vf[v * 4 + j] = make_float2(bf16_lo(ww[j]), bf16_hi(ww[j]));
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        // m[g] is -inf only while every score so far was -inf; p is 0 then
        const float pp = m[g] == -INFINITY ? 0.f : fast_exp2(sc[u][g] - m[g]);
        l[g] += pp;
        const float2 p2 = make_float2(pp, pp);
#pragma unroll
        for (int i = 0; i < DPL / 2; ++i) acc[g][i] = __ffma2_rn(p2, vf[i], acc[g][i]);
      }
    }
    __syncwarp();
  }
  if (!ok && lane == 0) {
    // a wait gave up: let the copies still in flight land (bounded) before the CTA exits
    for (int c = consumed; c < nc && c < consumed + kDecStages; ++c)
      mbar_wait(&bars[warp][c % kDecStages], (c / kDecStages) & 1, a.status, 302);
  }
  // merge the warp's token groups (same m in every lane of the warp): sum l and O over the lanes
  // that own the same head dims
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int o = LPT; o < 32; o <<= 1) {
      l[g] += __shfl_xor_sync(0xffffffffu, l[g], o);
#pragma unroll
      for (int i = 0; i < DPL / 2; ++i) {
        acc[g][i].x += __shfl_xor_sync(0xffffffffu, acc[g][i].x, o);
        acc[g][i].y += __shfl_xor_sync(0xffffffffu, acc[g][i].y, o);
      }
    }
  }
  // then the 4 warps through shared memory
  __shared__ float sm_m[NW][G];
  __shared__ float sm_l[NW][G];
  __shared__ float sm_acc[NW][G][D];
  if (lane < LPT) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (lane == 0) {
        sm_m[warp][g] = m[g];
        sm_l[warp][g] = l[g];
      }
#pragma unroll
      for (int i = 0; i < DPL / 2; ++i) {
        sm_acc[warp][g][gl * DPL + 2 * i] = acc[g][i].x;
        sm_acc[warp][g][gl * DPL + 2 * i + 1] = acc[g][i].y;
      }
    }
  }
  __syncthreads();
  // each thread finalises (g, d) entries: G * D outputs over 128 threads
  float* po = a.part_o + ((long)(b * H + h * G) * a.splits + split) * D;   // [B,H,splits,D]
  float* pml = a.part_lse + (long)(b * H + h * G) * a.splits + split;      // [B,H,splits]
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float mx = -INFINITY;
#pragma unroll
    for (int r = 0; r < NW; ++r) mx = fmaxf(mx, sm_m[r][g]);
    float ls = 0.f, o = 0.f;
    if (mx > -INFINITY) {
#pragma unroll
      for (int r = 0; r < NW; ++r) {
        const float w = fast_exp2(sm_m[r][g] - mx);
        ls += sm_l[r][g] * w;
        o += sm_acc[r][g][d] * w;
      }
    }
    po[(long)g * a.splits * D + d] = ls > 0.f ? o / ls : 0.f;
    if (d == 0) pml[(long)g * a.splits] = ls > 0.f ? mx + __log2f(ls) : -INFINITY;
  }
  // last CTA of this (b, h) combines the splits and publishes the rank partial
  __shared__ bool is_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(a.split_counter + b * a.Hkv + h, 1u);
    is_last = (prev == unsigned(a.splits) - 1);
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
  for (int i = threadIdx.x; i < G * a.splits; i += blockDim.x) {
    const int g = i / a.splits, s = i % a.splits;
    s_w[g][s] = __ldcg(a.part_lse + (long)(b * H + h * G + g) * a.splits + s);
  }
  __syncthreads();
  for (int g = warp; g < G; g += 4) {
    float mx = -INFINITY;
    for (int s = lane; s < a.splits; s += 32) mx = fmaxf(mx, s_w[g][s]);
    mx = warp_max(mx);
    float ws = 0.f;
    for (int s = lane; s < a.splits; s += 32) {
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
  for (int i = threadIdx.x; i < G * (D + 1); i += blockDim.x) {
    const int g = i / (D + 1), d = i % (D + 1);
    float val;
    if (s_mx[g] == -INFINITY) {
      val = (d < D) ? 0.f : -INFINITY;
    } else if (d == D) {
      val = s_mx[g] + __log2f(s_ws[g]);
    } else {
      const float* pof = a.part_o + (long)(b * H + h * G + g) * a.splits * D + d;
      float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
      int s = 0;
      for (; s + 4 <= a.splits; s += 4) {
        o0 = fmaf(s_w[g][s], __ldcg(pof + (long)s * D), o0);
        o1 = fmaf(s_w[g][s + 1], __ldcg(pof + (long)(s + 1) * D), o1);
        o2 = fmaf(s_w[g][s + 2], __ldcg(pof + (long)(s + 2) * D), o2);
        o3 = fmaf(s_w[g][s + 3], __ldcg(pof + (long)(s + 3) * D), o3);
      }
      for (; s < a.splits; ++s) o0 = fmaf(s_w[g][s], __ldcg(pof + (long)s * D), o0);
      val = ((o0 + o1) + (o2 + o3)) / s_ws[g];
    }
    // exchange slot layout: [2 parity][N src][B][H][D+1] fp32
    const long off = (((long)parity * a.n_ranks + a.my_rank) * a.B * H + (long)b * H + h * G + g) * (D + 1) + d;
    for (int r = 0; r < a.n_ranks; ++r) a.xslot_ptrs[r][off] = val;
  }
  if (threadIdx.x == 0) a.split_counter[b * a.Hkv + h] = 0;
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
  static bool done = false;
  if (done) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(decode_attn_kernel<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       DecChunk<D>::SMEM);
  done = (e == cudaSuccess);
  return e;
}

template <int D, int G>
static cudaError_t launch_attn(const DecodeAttnArgs& a, cudaStream_t s) {
  cudaError_t e = prepare_attn<D, G>();
  if (e != cudaSuccess) return e;
  dim3 grid(a.splits, a.Hkv, a.B);
  decode_attn_kernel<D, G><<<grid, 128, DecChunk<D>::SMEM, s>>>(a);
  return cudaGetLastError();
}

const char* decode_attn(const DecodeAttnArgs& a, cudaStream_t s) {
  const int G = a.H / a.Hkv;
  if (a.H % a.Hkv) return "decode_attn: H % Hkv";
  if (a.n_ranks < 1 || a.n_ranks > kMaxRanks) return "decode_attn: bad n_ranks";
  if (a.splits < 1 || a.splits > kMaxDecodeSplits) return "decode_attn: splits must be in [1, 128]";
  if ((a.D != 64 && a.D != 128) || a.geom.page % (1024 / a.D))
    return "decode_attn: head_dim must be 64 or 128 and the page a multiple of 1024 / head_dim rows";
  if (reinterpret_cast<uintptr_t>(a.arena) & 15) return "decode_attn: arena must be 16-byte aligned";
  cudaError_t e = cudaErrorInvalidValue;
#define HCP_DEC_CASE(DD, GG) \
  if (a.D == DD && G == GG) e = launch_attn<DD, GG>(a, s);
  HCP_DEC_CASE(64, 1) HCP_DEC_CASE(64, 2) HCP_DEC_CASE(64, 4) HCP_DEC_CASE(64, 8)
  HCP_DEC_CASE(128, 1) HCP_DEC_CASE(128, 2) HCP_DEC_CASE(128, 4) HCP_DEC_CASE(128, 8)
#undef HCP_DEC_CASE
  if (e == cudaErrorInvalidValue) return "decode_attn: unsupported (D, H/Hkv)";
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

int decode_attn_ctas_per_sm(int D, int G) {
  int n = 0;
#define HCP_DEC_OCC(DD, GG)                                                                      \
  if (D == DD && G == GG && prepare_attn<DD, GG>() == cudaSuccess)                                 \
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_attn_kernel<DD, GG>, 128, DecChunk<DD>::SMEM);
  HCP_DEC_OCC(64, 1) HCP_DEC_OCC(64, 2) HCP_DEC_OCC(64, 4) HCP_DEC_OCC(64, 8)
  HCP_DEC_OCC(128, 1) HCP_DEC_OCC(128, 2) HCP_DEC_OCC(128, 4) HCP_DEC_OCC(128, 8)
#undef HCP_DEC_OCC
  return n;
}

const char* decode_combine(const DecodeCombineArgs& a, cudaStream_t s) {
  if (a.n_ranks > a.D) return "decode_combine: more ranks than head_dim threads";
  decode_combine_kernel<<<dim3(a.B, a.H), a.D, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? nullptr : "decode_combine: launch failed";
}

// ----------------------------------------------------------------------------- small helpers
__global__ void fill_u64_kernel(unsigned long long* p, int n, unsigned long long v) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

__global__ void argmax_finalize_kernel(const unsigned long long* packed, int B, int* tokens_out,
                                       long long* tokens_out64) {
  const int b = threadIdx.x;
  if (b < B) {
    const int idx = int(0xFFFFFFFFu - uint32_t(packed[b] & 0xFFFFFFFFull));
    if (tokens_out) tokens_out[b] = idx;
    if (tokens_out64) tokens_out64[b] = idx;
  }
}

__global__ void add_u64_kernel(unsigned long long* p, unsigned long long v) { *p += v; }

const char* fill_u64(unsigned long long* p, int n, unsigned long long v, cudaStream_t s) {
  if (n == 0) return nullptr;
  fill_u64_kernel<<<(n + 255) / 256, 256, 0, s>>>(p, n, v);
  return cudaGetLastError() == cudaSuccess ? nullptr : "fill_u64: launch failed";
}

const char* argmax_finalize(const unsigned long long* packed, int B, int* tok, long long* tok64,
                            cudaStream_t s) {
  argmax_finalize_kernel<<<1, 32, 0, s>>>(packed, B, tok, tok64);
  return cudaGetLastError() == cudaSuccess ? nullptr : "argmax_finalize: launch failed";
}

const char* add_u64(unsigned long long* p, unsigned long long v, cudaStream_t s) {
  add_u64_kernel<<<1, 1, 0, s>>>(p, v);
  return cudaGetLastError() == cudaSuccess ? nullptr : "add_u64: launch failed";
}

}  // namespace dec
}  // namespace hcp

// ============================================================================================
// Allocation-free single-rank decode attention (see decode_noalloc.h for the contract).
//
// For callers that cannot allocate device memory: the split-KV scratch (partials, counters, the
// one-rank exchange slot and its pointer tables) lives in `g_decode_noalloc_scratch`, a
// file-scope array every device holds while the library is loaded. Host code never passes the
// array's name to a kernel (in host code it is only a stand-in for the symbol); it passes the
// device address obtained once per device with cudaGetSymbolAddress.
// ============================================================================================
#include <mutex>
#include <string>

#include "decode_noalloc.h"

namespace {

constexpr unsigned long long kNoAllocBytes = HCP_DECODE_NOALLOC_SCRATCH_BYTES;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[HCP_DECODE_NOALLOC_SCRATCH_BYTES];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoAllocMaxDevices] = {nullptr};
thread_local std::string g_noalloc_err;

// Byte layout inside the scratch array (all offsets 256-byte aligned).
struct NoAllocLayout {
  unsigned long long counters, tables, flag, part_o, part_lse, xslot, total;
};

unsigned long long align256(unsigned long long v) { return (v + 255ull) & ~255ull; }

NoAllocLayout noalloc_layout(int B, int H, int Hkv, int D, int splits) {
  NoAllocLayout l{};
  unsigned long long off = 0;
  l.counters = off;
  off = align256(off + sizeof(unsigned int) * (unsigned long long)(B * Hkv + 1));
  l.tables = off;  // float* xslot_ptrs[1]; unsigned long long* ready_ptrs[1]
  off = align256(off + 2 * sizeof(void*));
  l.flag = off;
  off = align256(off + sizeof(unsigned long long));
  l.part_o = off;
  off = align256(off + sizeof(float) * (unsigned long long)B * H * splits * D);
  l.part_lse = off;
  off = align256(off + sizeof(float) * (unsigned long long)B * H * splits);
  l.xslot = off;
  off = align256(off + sizeof(float) * 2ull * B * H * (D + 1));
  l.total = off;
  return l;
}

// Resets the state that must start at zero and points the one-entry tables at the scratch.
__global__ void noalloc_setup_kernel(unsigned char* base, NoAllocLayout l, int n_counters) {
  unsigned int* counters = reinterpret_cast<unsigned int*>(base + l.counters);
  for (int i = threadIdx.x; i < n_counters; i += blockDim.x) counters[i] = 0u;
  if (threadIdx.x == 0) {
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

}  // namespace

extern "C" unsigned long long hcp_decode_attention_noalloc_scratch_bytes(int batch, int heads,
                                                                         int hkv, int d,
                                                                         int splits) {
  return noalloc_layout(batch, heads, hkv, d, splits).total;
}

extern "C" const char* hcp_decode_attention_noalloc_error(void) { return g_noalloc_err.c_str(); }

extern "C" int hcp_decode_attention_noalloc(const void* q, const void* arena, int layers,
                                            int pages, int page, int hkv, int d, int layer,
                                            const int* page_tables, int pt_stride,
                                            const int* n_tokens, int batch, int heads,
                                            float scale, int splits, void* out,
                                            cudaStream_t stream) {
  g_noalloc_err.clear();
  if (!q || !arena || !page_tables || !n_tokens || !out)
    return noalloc_fail(-1, "hcp_decode_attention_noalloc: null pointer argument");
  if (batch < 1 || heads < 1 || hkv < 1 || splits < 1 || layers < 1 || pages < 1 || page < 1)
    return noalloc_fail(-2, "hcp_decode_attention_noalloc: sizes must be positive");
  if (layer < 0 || layer >= layers)
    return noalloc_fail(-3, "hcp_decode_attention_noalloc: layer out of range");
  if (d != 64 && d != 128) return noalloc_fail(-4, "hcp_decode_attention_noalloc: head_dim must be 64 or 128");
  if (heads % hkv) return noalloc_fail(-5, "hcp_decode_attention_noalloc: heads % kv_heads != 0");
  const int G = heads / hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return noalloc_fail(-6, "hcp_decode_attention_noalloc: heads / kv_heads must be 1, 2, 4 or 8");
  const NoAllocLayout lay = noalloc_layout(batch, heads, hkv, d, splits);
  if (lay.total > kNoAllocBytes)
    return noalloc_fail(-7, "hcp_decode_attention_noalloc: problem needs " + std::to_string(lay.total) +
                                " bytes of scratch, more than the static maximum of " +
                                std::to_string(kNoAllocBytes) + " bytes; lower batch or splits");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return noalloc_fail(int(e), cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return noalloc_fail(-8, "hcp_decode_attention_noalloc: device index out of range");
  unsigned char* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (g_noalloc_addr[dev] == nullptr) {
      // one-time set-up for this device (device `dev` is current): device address of the array
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
      if (e != cudaSuccess) return noalloc_fail(int(e), std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      g_noalloc_addr[dev] = p;
    }
    base = static_cast<unsigned char*>(g_noalloc_addr[dev]);
  }
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
  a.status = nullptr;
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
  c.status = nullptr;
  err = hcp::dec::decode_combine(c, stream);
  if (err) return noalloc_fail(-10, err);
  e = cudaGetLastError();
  return e == cudaSuccess ? 0 : noalloc_fail(int(e), cudaGetErrorString(e));
}
