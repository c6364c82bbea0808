// K1: blockwise online-softmax attention on tcgen05 / TMEM, with log-sum-exp output and a
// causal skip driven by global token positions (vanilla, striped and zigzag layouts, uneven
// chunks).
//
// Replaces the reference's ring block step `process_kv_block` (rust/src/model/attention/
// ring.rs:201-370: S = Q K^T * s, global-position causal mask, row max, exp, row sum, P V,
// online rescale of (m, l, O), fully-future block skip) and its q-chunk / micro-block loops
// (ring.rs:861-1399). Instead of materialising a [qc, kc] score tensor per block and ~10 ATen
// launches, one CTA streams KV tiles through shared memory and keeps S and O in TMEM.
//
// KV operand: a position-ordered K/V staging buffer [Hkv, L, D] (row p holds the key of global
// position p). In context-parallel runs the ring module fills it with this rank's own shard and
// the peers' shards over NVLink; the kernel's kv-tile order starts at `kv_start_tile` (this
// rank's own chunk) so local tiles are consumed while remote ones are still arriving, and an
// optional per-tile ready flag array lets the producer wait (bounded) for a tile to land.
//
// CTA layout (256 threads): warp 0 TMA producer, warp 1 MMA issuer, warp 2 TMEM allocator,
// warp 3 idle, warps 4-7 softmax/correction/epilogue (thread i <-> q row i <-> TMEM lane i).
// TMEM: S double buffer (2 x 128 fp32 columns) + O (D columns).
#include "attn_fwd_sm100.h"
#include "common.cuh"
#include "gemm_sm100.h"

namespace hcp {
namespace attn {

using namespace hcp::dev;

constexpr int BQ = 128;      // q rows per CTA
constexpr int BKV = 128;     // kv rows per tile
constexpr float kRescaleThreshold = 8.0f;  // log2 units: lazy O rescale (values bounded by 2^8)

template <int D>
struct Cfg {
  static constexpr int ATOMS = D / 64;                 // 128-byte swizzle atoms along D
  static constexpr int Q_BYTES = BQ * D * 2;
  static constexpr int KV_BYTES = BKV * D * 2;
  static constexpr int STAGES = (D == 64) ? 3 : 2;
  static constexpr int P_BYTES = BQ * BKV * 2;
  static constexpr int SMEM = 1024 + Q_BYTES + 2 * STAGES * KV_BYTES + P_BYTES + 512;
  static constexpr int TMEM_COLS = 512;
  static constexpr int O_COL = 256;
};

struct KParams {
  int T, H, Hkv, L;
  const int* q_pos;
  __nv_bfloat16* O;
  float* lse;
  float scale_log2;
  int causal;
  int num_q_tiles;
  int kv_start_tile;
  const unsigned long long* kv_ready;  // optional [Hkv][num_kv_tiles] ready epochs
  unsigned long long kv_epoch;
  int num_kv_tiles_total;
  unsigned long long wait_budget_ns;
  int* status;
};

// processing order: kv_start_tile .. n-1 ascending, then kv_start_tile-1 .. 0 descending
__device__ __forceinline__ int kv_tile_at(int j, int n, int start) {
  if (start >= n) start = 0;
  const int up = n - start;
  return j < up ? start + j : start - 1 - (j - up);
}

template <int D>
__global__ void __launch_bounds__(256, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, KParams p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::Q_BYTES;
  uint8_t* sV = sK + C::STAGES * C::KV_BYTES;
  uint8_t* sP = sV + C::STAGES * C::KV_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + C::P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + C::STAGES;
  uint64_t* v_full = k_empty + C::STAGES;
  uint64_t* v_empty = v_full + C::STAGES;
  uint64_t* s_full = v_empty + C::STAGES;  // [2]
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = p_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 1);
  int* s_qmin = reinterpret_cast<int*>(tmem_slot + 1);
  int* s_qmax = s_qmin + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  // heaviest q tiles first (largest positions last in local order): LPT-like balance
  const int q_tile = p.num_q_tiles - 1 - int(blockIdx.x) / p.H;
  const int head = int(blockIdx.x) % p.H;
  const int kv_head = head / (p.H / p.Hkv);
  const int row0 = q_tile * BQ;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    *s_qmin = 0x7fffffff;
    *s_qmax = -1;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // q position range of this tile; softmax warps 4-7 own rows 0..127 (thread 128 + i <-> row i)
  int my_pos = -1;
  if (threadIdx.x >= 128) {
    const int r = row0 + int(threadIdx.x) - 128;
    if (r < p.T) my_pos = p.q_pos[r];
    if (my_pos >= 0) {
      atomicMin(s_qmin, my_pos);
      atomicMax(s_qmax, my_pos);
    }
  }
  __syncthreads();
  const uint32_t tmem_base = *tmem_slot;
  const int qmin = *s_qmin;
  const int qmax = *s_qmax;
  const int kv_tiles_L = (p.L + BKV - 1) / BKV;
  int n_tiles = p.causal ? (qmax >= 0 ? qmax / BKV + 1 : 0) : kv_tiles_L;
  if (n_tiles > kv_tiles_L) n_tiles = kv_tiles_L;
  const int start = p.kv_start_tile < n_tiles ? p.kv_start_tile : 0;

  if (warp == 0) {
    if (elect_one() && n_tiles > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int a = 0; a < C::ATOMS; ++a)
        tma_load_3d(sQ + a * (BQ * 128), &tmQ, q_full, a * 64, head, row0);
      for (int j = 0; j < n_tiles; ++j) {
        const int t = kv_tile_at(j, n_tiles, start);
        const int s = j % C::STAGES;
        const uint32_t ph = (j / C::STAGES) & 1;
        if (p.kv_ready != nullptr) {
          const unsigned long long* f = p.kv_ready + (long)kv_head * p.num_kv_tiles_total + t;
          if (!wait_flag_geq_gpu(f, p.kv_epoch, p.wait_budget_ns, p.status, 210, t)) break;
        }
        if (!mbar_wait(&k_empty[s], ph ^ 1, p.status, 201)) break;
        mbar_arrive_expect_tx(&k_full[s], C::KV_BYTES);
#pragma unroll
        for (int a = 0; a < C::ATOMS; ++a)
          tma_load_3d(sK + s * C::KV_BYTES + a * (BKV * 128), &tmK, &k_full[s], a * 64, t * BKV,
                      kv_head);
        if (!mbar_wait(&v_empty[s], ph ^ 1, p.status, 202)) break;
        mbar_arrive_expect_tx(&v_full[s], C::KV_BYTES);
#pragma unroll
        for (int a = 0; a < C::ATOMS; ++a)
          tma_load_3d(sV + s * C::KV_BYTES + a * (BKV * 128), &tmV, &v_full[s], a * 64, t * BKV,
                      kv_head);
      }
    }
  } else if (warp == 1) {
    if (elect_one() && n_tiles > 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(BQ, BKV, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(BQ, D, false, true);
      const uint32_t sq = smem_u32(sQ);
      const uint32_t sp = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, p.status, 203);
      tc_fence_after();
      auto issue_pv = [&](int jj) -> bool {
        const int s = jj % C::STAGES;
        const uint32_t ph = (jj / C::STAGES) & 1;
        if (!mbar_wait(p_full, jj & 1, p.status, 204)) return false;
        if (!mbar_wait(&v_full[s], ph, p.status, 205)) return false;
        tc_fence_after();
        const uint32_t sv = smem_u32(sV + s * C::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          // A = P (K-major, 2 atoms of 64 kv), B = V tile (MN-major: D contiguous)
          const uint64_t ad = sdesc_sw128(sp + (kk / 4) * (BQ * 128) + (kk % 4) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(sv + kk * 2048, BKV * 128, 1024);
          umma_bf16_ss(tmem_base + C::O_COL, ad, bd, idesc_o, (jj > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(pv_done);
        umma_commit(&v_empty[s]);
        return true;
      };
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int s = j % C::STAGES;
        const uint32_t ph = (j / C::STAGES) & 1;
        if (!mbar_wait(&k_full[s], ph, p.status, 206)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sk = smem_u32(sK + s * C::KV_BYTES);
        const uint32_t d_s = tmem_base + uint32_t((j & 1) * BKV);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk / 4) * (BQ * 128) + (kk % 4) * 32;
          const uint32_t offk = (kk / 4) * (BKV * 128) + (kk % 4) * 32;
          umma_bf16_ss(d_s, sdesc_sw128(sq + off, 16, 1024), sdesc_sw128(sk + offk, 16, 1024),
                       idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[j & 1]);
        umma_commit(&k_empty[s]);
        if (j >= 1 && !issue_pv(j - 1)) ok = false;
      }
      if (ok) issue_pv(n_tiles - 1);
    }
  } else if (warp >= 4) {
    const int q = warp - 4;
    const int row = q * 32 + lane;
    const int grow = row0 + row;
    const uint32_t lane_base = tmem_base + (uint32_t(q * 32) << 16);
    float m_ref = -INFINITY;  // max used for exponentiation (log2 domain)
    float l_sum = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int t = kv_tile_at(j, n_tiles, start);
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, p.status, 207)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(lane_base + uint32_t((j & 1) * BKV + c * 32), sr + 32 * c);
      tmem_wait_ld();
      const int kv0 = t * BKV;
      const bool need_mask = (p.causal && kv0 + BKV - 1 > qmin) || (kv0 + BKV > p.L) || my_pos < 0;
      float s[128];
      float tmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        float x = __uint_as_float(sr[c]) * p.scale_log2;
        if (need_mask) {
          const int kp = kv0 + c;
          const bool masked = (kp >= p.L) || my_pos < 0 || (p.causal && kp > my_pos);
          x = masked ? -INFINITY : x;
        }
        s[c] = x;
        tmax = fmaxf(tmax, x);
      }
      // lazy rescale: only move the reference max when it grows by more than the threshold
      float alpha = 1.f;
      bool resc = false;
      if (tmax > m_ref + kRescaleThreshold || (m_ref == -INFINITY && tmax > -INFINITY)) {
        alpha = (m_ref == -INFINITY) ? 0.f : fast_exp2(m_ref - tmax);
        m_ref = tmax;
        resc = true;
      }
      const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
      float rs = 0.f;
      uint32_t pk[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float p0 = fast_exp2(s[2 * c] - m_use);
        const float p1 = fast_exp2(s[2 * c + 1] - m_use);
        rs += p0 + p1;
        pk[c] = pack_bf16x2(p0, p1);
      }
      l_sum = l_sum * alpha + rs;
      // PV of the previous tile must be complete before P is overwritten / O is rescaled
      if (j >= 1) {
        if (!mbar_wait(pv_done, (j - 1) & 1, p.status, 208)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, resc)) {
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(lane_base + uint32_t(C::O_COL + c * 32), o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(lane_base + uint32_t(C::O_COL + c * 32), o);
          }
          tmem_wait_st();
        }
      }
      // write P (bf16) into the K-major 128B-swizzled operand tile: row `row`, 2 atoms of 64 kv
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        uint8_t* base = sP + a * (BQ * 128) + row * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const int pos = (ch ^ (row & 7)) * 16;
          const int w = a * 32 + ch * 4;
          *reinterpret_cast<uint4*>(base + pos) = make_uint4(pk[w], pk[w + 1], pk[w + 2], pk[w + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // epilogue: O / l, LSE
    if (ok && n_tiles > 0 && mbar_wait(pv_done, (n_tiles - 1) & 1, p.status, 209)) {
      tc_fence_after();
      const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
      __nv_bfloat16* dst = p.O + ((long)grow * p.H + head) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(lane_base + uint32_t(C::O_COL + c * 32), o);
        tmem_wait_ld();
        if (grow < p.T) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            d4[i] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * i]) * inv, __uint_as_float(o[8 * i + 1]) * inv),
                               pack_bf16x2(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv),
                               pack_bf16x2(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv),
                               pack_bf16x2(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv));
        }
      }
      if (grow < p.T && p.lse != nullptr) {
        p.lse[(long)head * p.T + grow] =
            l_sum > 0.f ? (m_ref + __log2f(l_sum)) * 0.6931471805599453f : -INFINITY;
      }
    } else if (n_tiles == 0 && grow < p.T) {
      // no visible key (only possible for padding rows / empty KV): O = 0, LSE = -inf
      __nv_bfloat16* dst = p.O + ((long)grow * p.H + head) * D;
      for (int i = 0; i < D; ++i) dst[i] = __float2bfloat16(0.f);
      if (p.lse != nullptr) p.lse[(long)head * p.T + grow] = -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <int D>
static cudaError_t launch(const AttnArgs& a, const CUtensorMap& tq, const CUtensorMap& tk,
                          const CUtensorMap& tv, const KParams& p, cudaStream_t stream) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel<D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D>::SMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int grid = p.num_q_tiles * p.H;
  attn_fwd_kernel<D><<<grid, 256, Cfg<D>::SMEM, stream>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

const char* attn_fwd(const AttnArgs& a, cudaStream_t stream) {
  if (a.D != 64 && a.D != 128) return "attn: head_dim must be 64 or 128";
  if (a.H % a.Hkv) return "attn: H must be a multiple of Hkv";
  if (a.T <= 0) return nullptr;
  if (a.L <= 0) return "attn: empty KV";
  if ((reinterpret_cast<uintptr_t>(a.Q) | reinterpret_cast<uintptr_t>(a.K) |
       reinterpret_cast<uintptr_t>(a.V) | reinterpret_cast<uintptr_t>(a.O)) & 15)
    return "attn: Q/K/V/O must be 16-byte aligned";
  CUtensorMap tq, tk, tv;
  // Q [T, H, D]: dims (D, H, T)
  if (!gemm::make_tma_3d_bf16(&tq, a.Q, a.D, a.H, a.T, uint64_t(a.D) * 2, uint64_t(a.H) * a.D * 2,
                              64, 1, BQ))
    return "attn: TMA descriptor for Q failed";
  // K/V [Hkv, Lstride, D]: dims (D, L, Hkv)
  if (!gemm::make_tma_3d_bf16(&tk, a.K, a.D, a.L, a.Hkv, uint64_t(a.D) * 2,
                              uint64_t(a.kv_head_stride) * 2, 64, BKV, 1))
    return "attn: TMA descriptor for K failed";
  if (!gemm::make_tma_3d_bf16(&tv, a.V, a.D, a.L, a.Hkv, uint64_t(a.D) * 2,
                              uint64_t(a.kv_head_stride) * 2, 64, BKV, 1))
    return "attn: TMA descriptor for V failed";
  KParams p;
  p.T = a.T;
  p.H = a.H;
  p.Hkv = a.Hkv;
  p.L = a.L;
  p.q_pos = a.q_pos;
  p.O = a.O;
  p.lse = a.lse;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.causal = a.causal;
  p.num_q_tiles = (a.T + BQ - 1) / BQ;
  p.kv_start_tile = a.kv_start_tile;
  p.kv_ready = a.kv_ready;
  p.kv_epoch = a.kv_epoch;
  p.num_kv_tiles_total = (a.L + BKV - 1) / BKV;
  p.wait_budget_ns = a.wait_budget_ns;
  p.status = a.status;
  cudaError_t e = a.D == 64 ? launch<64>(a, tq, tk, tv, p, stream)
                            : launch<128>(a, tq, tk, tv, p, stream);
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

}  // namespace attn
}  // namespace hcp
