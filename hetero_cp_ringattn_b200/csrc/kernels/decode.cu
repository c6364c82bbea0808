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

// One CTA (8 warps) computes R output rows (R gate/up pairs for SwiGLU) for all B inputs. The
// whole CTA splits K: thread t reads uint4 columns t, t + 256, ... of each row, so every thread
// issues its R row loads for several k steps back to back (no dependent-load chains), and the
// partial dot products are reduced across the 8 warps through shared memory.
// NORM: the input rows are RMS-normalised on the fly (statistics recomputed per CTA from the
// 2-8 input rows, which is cheaper than a separate normalisation launch for decode).
constexpr int GEMV_THREADS = 256;

template <int EPI, int B, int R, bool NORM>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(GemvArgs a) {
  extern __shared__ uint4 xs[];                     // NORM: normalised x, [B][K/8]
  __shared__ float red[GEMV_THREADS / 32][2 * R * B];
  __shared__ float rstd[B];
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32;
  const int kvec = a.K / 8;
  const int out_rows = (EPI == kGemvSwiGLU) ? a.N / 2 : a.N;
  const int base = blockIdx.x * R;
  if (NORM) {
    // sum of squares per input row, then the normalised bf16 row into shared memory
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
    __syncthreads();
  }
  int wrow[R], urow[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    int o = base + r;
    if (o >= out_rows) o = out_rows - 1;
    if (EPI == kGemvSwiGLU) {
      wrow[r] = (o / 128) * 256 + (o % 128);
      urow[r] = wrow[r] + 128;
    } else {
      wrow[r] = o;
      urow[r] = o;
    }
  }
  float acc[R][B], accu[R][B];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) acc[r][b] = accu[r][b] = 0.f;
#pragma unroll 4
  for (int k = tid; k < kvec; k += GEMV_THREADS) {
    uint4 w[R], u[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      w[r] = ld_stream(reinterpret_cast<const uint4*>(a.W + (long)wrow[r] * a.K) + k);
      if (EPI == kGemvSwiGLU) u[r] = ld_stream(reinterpret_cast<const uint4*>(a.W + (long)urow[r] * a.K) + k);
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const uint4 xv = NORM ? xs[b * kvec + k] : __ldg(reinterpret_cast<const uint4*>(a.x + (long)b * a.ldx) + k);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        dot8_acc(w[r], xv, acc[r][b]);
        if (EPI == kGemvSwiGLU) dot8_acc(u[r], xv, accu[r][b]);
      }
    }
  }
  if (NORM) __syncthreads();  // `red` is reused below
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const float v = warp_sum(acc[r][b]);
      if (lane == 0) red[warp][r * B + b] = v;
      if (EPI == kGemvSwiGLU) {
        const float vu = warp_sum(accu[r][b]);
        if (lane == 0) red[warp][R * B + r * B + b] = vu;
      }
    }
  __syncthreads();
  if (tid < R * B) {
    const int r = tid / B, b = tid % B;
    const int o = base + r;
    float v = 0.f, vu = 0.f;
#pragma unroll
    for (int w = 0; w < GEMV_THREADS / 32; ++w) {
      v += red[w][r * B + b];
      if (EPI == kGemvSwiGLU) vu += red[w][R * B + r * B + b];
    }
    if (o < out_rows) {
      if (EPI == kGemvF32) {
        if (a.bias) v += __bfloat162float(a.bias[o]);
        a.y_f32[(long)b * a.ldy + o] = v;
      } else if (EPI == kGemvResidual) {
        __nv_bfloat16* y = a.y_bf16 + (long)b * a.ldy + o;
        *y = __float2bfloat16(__bfloat162float(__float2bfloat16(v)) + __bfloat162float(*y));
      } else if (EPI == kGemvSwiGLU) {
        const float g = __bfloat162float(__float2bfloat16(v));
        const float uu = __bfloat162float(__float2bfloat16(vu));
        const float sg = g / (1.f + fast_exp2(-g * kLog2e));
        a.y_bf16[(long)b * a.ldy + o] = __float2bfloat16(sg * uu);
      } else if (EPI == kGemvArgmax) {
        if (a.y_f32) a.y_f32[(long)b * a.ldy + o] = v;
        red[0][2 * R * B - 1 - tid] = v;  // keep for the per-CTA argmax below (disjoint slots)
      }
    }
  }
  if (EPI == kGemvArgmax) {
    __syncthreads();
    if (tid < B) {
      unsigned long long best = 0;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int o = base + r;
        if (o < out_rows) {
          const unsigned long long c = pack_argmax(red[0][2 * R * B - 1 - (r * B + tid)], o);
          best = c > best ? c : best;
        }
      }
      atomicMax(a.argmax + tid, best);
    }
  }
}

template <int EPI, bool NORM>
static cudaError_t gemv_launch(const GemvArgs& a, cudaStream_t s) {
  constexpr int R = 4;  // output rows (gate/up pairs for SwiGLU) per CTA
  const int out_rows = (EPI == kGemvSwiGLU) ? a.N / 2 : a.N;
  const int grid = (out_rows + R - 1) / R;
  const size_t smem = NORM ? size_t(a.B) * a.K * 2 : 0;
  auto go = [&](auto kernel) -> cudaError_t {
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      if (e != cudaSuccess) return e;
    }
    kernel<<<grid, GEMV_THREADS, smem, s>>>(a);
    return cudaGetLastError();
  };
  switch (a.B) {
    case 1: return go(gemv_kernel<EPI, 1, R, NORM>);
    case 2: return go(gemv_kernel<EPI, 2, R, NORM>);
    case 4: return go(gemv_kernel<EPI, 4, R, NORM>);
    case 8: return go(gemv_kernel<EPI, 8, R, NORM>);
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
  if (a.norm_w && (size_t(a.B) * a.K * 2 > 200 * 1024)) return "gemv: fused norm needs B*K*2 <= 200 KB";
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
// grid (splits, Hkv, B), 128 threads. Each group of D/8 lanes handles one token at a time.
template <int D, int G>
__global__ void __launch_bounds__(128) decode_attn_kernel(DecodeAttnArgs a) {
  constexpr int LPG = D / 8;        // lanes per token
  constexpr int TPW = 32 / LPG;     // tokens per warp step
  constexpr int GROUPS = 4 * TPW;   // token groups per CTA
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  const int gl = lane % LPG;                  // lane within group
  const int grp = warp * TPW + lane / LPG;    // group id within CTA
  const int n = a.n_tokens[b];
  const int per = (n + a.splits - 1) / a.splits;
  const int s0 = split * per;
  const int s1 = min(n, s0 + per);
  const int H = a.Hkv * G;

  // q slice (pre-scaled into the log2 domain)
  float q[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint4 v = *reinterpret_cast<const uint4*>(a.q + ((long)b * H + h * G + g) * D + gl * 8);
    const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      q[g][2 * j] = bf16_lo(vv[j]) * a.scale * kLog2e;
      q[g][2 * j + 1] = bf16_hi(vv[j]) * a.scale * kLog2e;
    }
  }
  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[g][j] = 0.f;
  }
  const int* pt = a.page_tables + (long)b * a.pt_stride;
  // The loop bound is warp-uniform (it depends on the warp, not the lane group) because the
  // body reduces scores with full-warp shuffles; a lane group past the end of the split runs
  // the step with `valid == false` and leaves its state untouched. UNR token steps are loaded
  // before any is consumed, so each lane keeps 2 * UNR 16-byte loads in flight.
  constexpr int UNR = 4;
  for (int base = s0 + warp * TPW; base < s1; base += GROUPS * UNR) {
    uint4 kvs[UNR], vvs[UNR];
    bool valid[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int t = base + u * GROUPS + lane / LPG;
      valid[u] = t < s1;
      kvs[u] = make_uint4(0u, 0u, 0u, 0u);
      vvs[u] = make_uint4(0u, 0u, 0u, 0u);
      if (valid[u]) {
        const int page = pt[t / a.geom.page];
        const int row = t % a.geom.page;
        const __nv_bfloat16* kp = a.arena + a.geom.offset(a.layer, page, 0, h, row) + gl * 8;
        kvs[u] = *reinterpret_cast<const uint4*>(kp);
        vvs[u] = *reinterpret_cast<const uint4*>(kp + a.geom.kv_stride());
      }
    }
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const uint32_t kw[4] = {kvs[u].x, kvs[u].y, kvs[u].z, kvs[u].w};
      const uint32_t vw[4] = {vvs[u].x, vvs[u].y, vvs[u].z, vvs[u].w};
      float vf[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        vf[2 * j] = bf16_lo(vw[j]);
        vf[2 * j + 1] = bf16_hi(vw[j]);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float sc = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sc = fmaf(q[g][2 * j], bf16_lo(kw[j]), sc);
          sc = fmaf(q[g][2 * j + 1], bf16_hi(kw[j]), sc);
        }
#pragma unroll
        for (int o = LPG / 2; o > 0; o >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
        if (!valid[u]) continue;
        const float mn = fmaxf(m[g], sc);
        const float al = fast_exp2(m[g] - mn);
        const float pp = fast_exp2(sc - mn);
        l[g] = l[g] * al + pp;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[g][j] = fmaf(acc[g][j], al, pp * vf[j]);
        m[g] = mn;
      }
    }
  }
  // CTA reduction over the GROUPS token groups through shared memory
  __shared__ float sm_m[GROUPS][G];
  __shared__ float sm_l[GROUPS][G];
  __shared__ float sm_acc[GROUPS][G][D];
  if (gl == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      sm_m[grp][g] = m[g];
      sm_l[grp][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < 8; ++j) sm_acc[grp][g][gl * 8 + j] = acc[g][j];
  __syncthreads();
  // each thread finalises (g, d) entries: G * D outputs over 128 threads
  float* po = a.part_o + ((long)(b * H + h * G) * a.splits + split) * D;   // [B,H,splits,D]
  float* pml = a.part_lse + (long)(b * H + h * G) * a.splits + split;      // [B,H,splits]
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float mx = -INFINITY;
    for (int r = 0; r < GROUPS; ++r) mx = fmaxf(mx, sm_m[r][g]);
    float ls = 0.f, o = 0.f;
    if (mx > -INFINITY) {
      for (int r = 0; r < GROUPS; ++r) {
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
static cudaError_t launch_attn(const DecodeAttnArgs& a, cudaStream_t s) {
  dim3 grid(a.splits, a.Hkv, a.B);
  decode_attn_kernel<D, G><<<grid, 128, 0, s>>>(a);
  return cudaGetLastError();
}

const char* decode_attn(const DecodeAttnArgs& a, cudaStream_t s) {
  const int G = a.H / a.Hkv;
  if (a.H % a.Hkv) return "decode_attn: H % Hkv";
  if (a.n_ranks < 1 || a.n_ranks > kMaxRanks) return "decode_attn: bad n_ranks";
  if (a.splits < 1 || a.splits > kMaxDecodeSplits) return "decode_attn: splits must be in [1, 128]";
  cudaError_t e = cudaErrorInvalidValue;
#define HCP_DEC_CASE(DD, GG) \
  if (a.D == DD && G == GG) e = launch_attn<DD, GG>(a, s);
  HCP_DEC_CASE(64, 1) HCP_DEC_CASE(64, 2) HCP_DEC_CASE(64, 4) HCP_DEC_CASE(64, 8)
  HCP_DEC_CASE(128, 1) HCP_DEC_CASE(128, 2) HCP_DEC_CASE(128, 4) HCP_DEC_CASE(128, 8)
#undef HCP_DEC_CASE
  if (e == cudaErrorInvalidValue) return "decode_attn: unsupported (D, H/Hkv)";
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
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
