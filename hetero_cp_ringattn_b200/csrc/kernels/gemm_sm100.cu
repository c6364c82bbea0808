// K3/K6: persistent tcgen05 GEMM  C[M,N] = A[M,K] * B[N,K]^T  (bf16 in, fp32 accumulate in TMEM)
// with fused epilogues: plain store, +bias (Qwen2 QKV), +residual (O-proj / down-proj, may run
// in place on the residual stream), and SwiGLU (gate||up weight interleaved in 128-row blocks,
// writes silu(gate) * up).
//
// Replaces the reference's cuBLAS GEMM call sites (rust/src/model/attention/ring.rs:1865-1876
// QKV, :2022-2027 O-proj; rust/src/model/layers/mlp.rs:42-67 SwiGLU MLP; model.rs:310-333 LM
// head), which the reference dispatches through libtorch.
//
// Design (sm_100a):
//   * one CTA per SM (persistent), 128x256 output tile, BK = 64 (one 128-byte swizzle atom),
//     4-stage TMA ring for A/B tiles (each CTA loads its own tiles from local memory);
//   * warp 0: TMA producer; warp 1: single-thread tcgen05.mma issuer (M=128, N=256, K=16);
//     warp 2: TMEM allocator; warps 4-7: epilogue (thread i owns accumulator row i);
//   * two 256-column TMEM accumulators so the epilogue of tile i overlaps the mainloop of i+1;
//   * every mbarrier wait is bounded and reports through the status word.
//
// Pair variant (gemm2_kernel, the default): clusters of two CTAs on two SMs compute 256x256
// tiles with tcgen05.mma.cta_group::2 (M = 256): each CTA loads its own 128 rows of A and its own
// 128 rows of B (the N half) into its own shared memory with plain per-CTA TMA loads,
// both signalling the leader CTA's full barrier; the leader's single MMA thread reads both CTAs'
// tiles, each CTA's TMEM receives its 128 rows of the 256-column accumulator, and the commits
// arrive on the barriers of both CTAs. Per SM that moves 32 KB instead of 48 KB of operands
// from L2 per 64-deep k step for the same MMA work.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemm_sm100.h"
#include "launch.h"

namespace hcp {
namespace gemm {

using namespace hcp::dev;

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_STAGE = BM * BK * 2;  // 16 KB
constexpr int B_STAGE = BN * BK * 2;  // 32 KB
constexpr int TMEM_COLS = 512;
constexpr int SMEM_BYTES = 1024 + STAGES * (A_STAGE + B_STAGE) + 256;
// pair variant: per CTA 128 rows of A and 128 rows of B per stage
constexpr int STAGES2 = 6;
constexpr int HALF_STAGE = 128 * BK * 2;                 // 16 KB
constexpr int SMEM_BYTES2 = 1024 + STAGES2 * 2 * HALF_STAGE + 256;

struct Params {
  int M, N, K;
  int num_m_tiles, num_n_tiles;
  int group_m;      // tile order: bands of group_m m-blocks, m fastest inside a band (0: n fastest)
  __nv_bfloat16* C;
  long ldc;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* R;
  long ldr;
  int* status;
  QkvPushArgs qkv;  // kEpiQkvPush only
};

__device__ __forceinline__ void tile_coords(int tile, const Params& p, int& mb, int& nb) {
  if (p.group_m <= 0) {
    // n fastest: concurrently running CTAs share A tiles through L2 and sweep all of B
    mb = tile / p.num_n_tiles;
    nb = tile % p.num_n_tiles;
    return;
  }
  // bands of group_m m-blocks, m fastest within a band: the band's A tiles stay in L2 while B is
  // swept once per band (n fastest sweeps all of B once per m-block, which for a weight larger
  // than L2, e.g. a 28672 x 4096 gate/up projection, re-reads it from DRAM every time)
  const int per_band = p.group_m * p.num_n_tiles;
  const int band = tile / per_band;
  const int first = band * p.group_m;
  const int rows = min(p.group_m, p.num_m_tiles - first);
  const int r = tile - band * per_band;
  mb = first + r % rows;
  nb = r / rows;
}

template <int EPI>
__device__ __forceinline__ void epilogue_tile(const Params& p, uint32_t tacc, int mb, int nb,
                                              int row_in_tile) {
  const int m = mb * BM + row_in_tile;
  const bool row_ok = m < p.M;
  uint32_t r[32];
  if constexpr (EPI == kEpiQkvPush) {
    // heads never straddle a 32-column chunk (D is 64 or 128); a head's rotation pairs column j
    // with j + D/2, both in this thread's accumulator row
    const QkvPushArgs& q = p.qkv;
    const int D = q.D, half = D / 2;
    const int pos = row_ok ? q.pos[m] : -1;
    const bool pos_ok = pos >= 0 && pos < q.max_pos;
    if (row_ok && !pos_ok) report_error(p.status, int(StatusCode::kOutOfBounds), 111, pos, m);
    const int slot = q.slot_base + m;
    int page = -1;
    if (row_ok && q.arena != nullptr) {
      if (slot >= 0 && slot < q.slot_cap) page = q.page_table[slot / q.geom.page];
      else report_error(p.status, int(StatusCode::kOutOfBounds), 112, slot, m);
    }
    const bool stage_ok = pos_ok && pos < q.stage_cap;
#pragma unroll 1
    for (int hb = 0; hb < BN; hb += D) {
      const int col0 = nb * BN + hb;
      if (col0 >= p.N) break;
      const int gh = col0 / D;                           // head index in the q | k | v row
      const int kind = gh < q.H ? 0 : (gh < q.H + q.Hkv ? 1 : 2);
#pragma unroll 1
      for (int jc = 0; jc < half; jc += 32) {
        uint32_t u[32];
        tmem_ld32(tacc + hb + jc, r);
        tmem_ld32(tacc + hb + half + jc, u);
        tmem_wait_ld();
        if (!row_ok) continue;
        float lo[32], hi[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          lo[i] = __uint_as_float(r[i]);
          hi[i] = __uint_as_float(u[i]);
        }
        if (p.bias != nullptr) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            lo[i] += __bfloat162float(p.bias[col0 + jc + i]);
            hi[i] += __bfloat162float(p.bias[col0 + half + jc + i]);
          }
        }
        if (kind < 2 && pos_ok) {
          const float4* c4 = reinterpret_cast<const float4*>(q.cos_t + (long)pos * half + jc);
          const float4* s4 = reinterpret_cast<const float4*>(q.sin_t + (long)pos * half + jc);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 c = c4[i], sn = s4[i];
            const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float x1 = lo[4 * i + e], x2 = hi[4 * i + e];
              lo[4 * i + e] = x1 * cc[e] - x2 * ss[e];
              hi[4 * i + e] = x2 * cc[e] + x1 * ss[e];
            }
          }
        }
        uint4 vlo[4], vhi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          vlo[i] = make_uint4(pack_bf16x2(lo[8 * i], lo[8 * i + 1]), pack_bf16x2(lo[8 * i + 2], lo[8 * i + 3]),
                              pack_bf16x2(lo[8 * i + 4], lo[8 * i + 5]), pack_bf16x2(lo[8 * i + 6], lo[8 * i + 7]));
          vhi[i] = make_uint4(pack_bf16x2(hi[8 * i], hi[8 * i + 1]), pack_bf16x2(hi[8 * i + 2], hi[8 * i + 3]),
                              pack_bf16x2(hi[8 * i + 4], hi[8 * i + 5]), pack_bf16x2(hi[8 * i + 6], hi[8 * i + 7]));
        }
        auto put = [&](__nv_bfloat16* base) {
          uint4* d0 = reinterpret_cast<uint4*>(base + jc);
          uint4* d1 = reinterpret_cast<uint4*>(base + half + jc);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            d0[i] = vlo[i];
            d1[i] = vhi[i];
          }
        };
        if (kind == 0) {
          put(q.q_out + ((long)m * q.H + gh) * D);
        } else {
          const int kv = kind - 1;
          const int h = gh - q.H - kv * q.Hkv;
          if (page >= 0) put(q.arena + q.geom.offset(q.layer, page, kv, h, slot % q.geom.page));
          if (stage_ok) {
            const long soff = ((long)(kv * q.Hkv + h) * q.stage_cap + pos) * D;
            for (int rk = 0; rk < q.n_stage; ++rk)
              put(reinterpret_cast<__nv_bfloat16*>(q.stage_ptrs[rk]) + soff);
          }
        }
      }
    }
  } else if constexpr (EPI == kEpiSwiGLU) {
    // tile columns [0,128) are gate rows, [128,256) the matching up rows
    const int out_n0 = nb * (BN / 2);
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t u[32];
      tmem_ld32(tacc + c * 32, r);
      tmem_ld32(tacc + 128 + c * 32, u);
      tmem_wait_ld();
      const int n0 = out_n0 + c * 32;
      if (row_ok) {
        __nv_bfloat16* dst = p.C + (long)m * p.ldc + n0;
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float g0 = __uint_as_float(r[2 * i]), g1 = __uint_as_float(r[2 * i + 1]);
          float u0 = __uint_as_float(u[2 * i]), u1 = __uint_as_float(u[2 * i + 1]);
          // silu(g) = g / (1 + 2^(-g * log2 e)); the gate is rounded to bf16 first, as the
          // reference's bf16 GEMM output would be
          g0 = __bfloat162float(__float2bfloat16(g0));
          g1 = __bfloat162float(__float2bfloat16(g1));
          u0 = __bfloat162float(__float2bfloat16(u0));
          u1 = __bfloat162float(__float2bfloat16(u1));
          float s0 = g0 / (1.0f + fast_exp2(-g0 * 1.4426950408889634f));
          float s1 = g1 / (1.0f + fast_exp2(-g1 * 1.4426950408889634f));
          packed[i] = pack_bf16x2(s0 * u0, s1 * u1);
        }
        const int nout = (p.N / 2);
        if (n0 + 32 <= nout) {
          uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            d4[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2],
                               packed[4 * i + 3]);
        } else {
          for (int i = 0; i < 32; ++i) {
            if (n0 + i < nout) {
              uint32_t w = packed[i / 2];
              uint16_t h = (i & 1) ? uint16_t(w >> 16) : uint16_t(w & 0xffff);
              reinterpret_cast<uint16_t*>(dst)[i] = h;
            }
          }
        }
      }
    }
  } else {
    const int n_base = nb * BN;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      tmem_ld32(tacc + c * 32, r);
      tmem_wait_ld();
      const int n0 = n_base + c * 32;
      if (!row_ok || n0 >= p.N) continue;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
      const bool full = (n0 + 32 <= p.N);
      if constexpr (EPI == kEpiBias) {
        if (full) {
          const uint4* b4 = reinterpret_cast<const uint4*>(p.bias + n0);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 w = b4[i];
            uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              v[8 * i + 2 * j] += bf16_lo(ww[j]);
              v[8 * i + 2 * j + 1] += bf16_hi(ww[j]);
            }
          }
        } else {
          for (int i = 0; i < 32; ++i)
            if (n0 + i < p.N) v[i] += __bfloat162float(p.bias[n0 + i]);
        }
      }
      if constexpr (EPI == kEpiResidual) {
        const __nv_bfloat16* rsrc = p.R + (long)m * p.ldr + n0;
        if (full) {
          const uint4* r4 = reinterpret_cast<const uint4*>(rsrc);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 w = r4[i];
            uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              // round the GEMM result to bf16 before the add, like a bf16 GEMM + bf16 add
              v[8 * i + 2 * j] = __bfloat162float(__float2bfloat16(v[8 * i + 2 * j])) +
                                 bf16_lo(ww[j]);
              v[8 * i + 2 * j + 1] =
                  __bfloat162float(__float2bfloat16(v[8 * i + 2 * j + 1])) + bf16_hi(ww[j]);
            }
          }
        } else {
          for (int i = 0; i < 32; ++i)
            if (n0 + i < p.N)
              v[i] = __bfloat162float(__float2bfloat16(v[i])) + __bfloat162float(rsrc[i]);
        }
      }
      __nv_bfloat16* dst = p.C + (long)m * p.ldc + n0;
      if (full) {
        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          d4[i] = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]),
                             pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                             pack_bf16x2(v[8 * i + 4], v[8 * i + 5]),
                             pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
      } else {
        for (int i = 0; i < 32; ++i)
          if (n0 + i < p.N) dst[i] = __float2bfloat16(v[i]);
      }
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(256, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * B_STAGE);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = bars + 2 * STAGES + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_tiles = p.num_m_tiles * p.num_n_tiles;
  const int k_iters = (p.K + BK - 1) / BK;

  if (warp == 0) {
    if (elect_one()) {
      int it = 0;
      for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        bool ok = true;
        for (int k = 0; k < k_iters; ++k, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.status, 101)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], A_STAGE + B_STAGE);
          tma_load_2d(sA + s * A_STAGE, &tmA, &full[s], k * BK, mb * BM);
          tma_load_2d(sB + s * B_STAGE, &tmB, &full[s], k * BK, nb * BN);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, false, false);
      int it = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++local) {
        const int b = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[b], aph ^ 1, p.status, 102)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(b * BN);
        bool ok = true;
        for (int k = 0; k < k_iters; ++k, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, p.status, 103)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * A_STAGE);
          const uint32_t b0 = smem_u32(sB + s * B_STAGE);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = sdesc_sw128(a0 + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(b0 + kk * 32, 16, 1024);
            umma_bf16_ss(d_tmem, ad, bd, idesc, (k | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[b]);
      }
    }
  } else if (warp >= 4) {
    const int q = warp - 4;
    const int row_in_tile = q * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++local) {
      const int b = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[b], aph, p.status, 104)) break;
      tc_fence_after();
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      const uint32_t tacc = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(b * BN);
      epilogue_tile<EPI>(p, tacc, mb, nb, row_in_tile);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }

  if constexpr (EPI == kEpiQkvPush) {
    // this thread's peer stores are ordered before the CTA's completion count below
    if (warp >= 4) __threadfence_system();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if constexpr (EPI == kEpiQkvPush) {
    // last CTA done: every CTA's K/V rows are visible system-wide, publish the epoch to every
    // rank's kv_ready slot for this rank
    if (threadIdx.x == 0 && p.qkv.done_counter != nullptr) {
      __threadfence_system();
      const unsigned prev = atomicAdd(p.qkv.done_counter, 1u);
      if (prev == gridDim.x - 1) {
        __threadfence_system();
        for (int rk = 0; rk < p.qkv.n_stage; ++rk) st_release_sys(p.qkv.ready_ptrs[rk], p.qkv.epoch);
        *p.qkv.done_counter = 0;
      }
    }
  }
}

// ----------------------------------------------------------------------------- CTA-pair kernel
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on a barrier of the pair's
// leader CTA (cluster address)
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* map, uint32_t bar_cluster,
                                                 int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void umma_pair_bf16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                                  uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// commit of the pair's MMAs: one arrival on the barrier at this offset in both CTAs
__device__ __forceinline__ void umma_pair_commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
      ::"r"(smem_u32(bar)), "h"(uint16_t(3))
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Tiles of 256 x 256 (num_m_tiles counts 256-row blocks), persistent over the grid's CTA pairs.
// Warp roles as in gemm_kernel; the MMA warp of the follower CTA (cluster rank 1) idles.
// Barriers: full[s] of the leader counts both CTAs' TMA bytes (the leader arrives with the
// expected 64 KB); empty[s] and acc_full[b] of both CTAs receive the leader's commits;
// acc_empty[b] of the leader collects the 4 epilogue warps of each CTA (the follower's arrive
// remotely). The kernel has no early exit: every thread reaches the final cluster barrier, after
// which both CTAs free their TMEM.
template <int EPI>
__global__ void __launch_bounds__(256, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES2 * HALF_STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES2 * HALF_STAGE);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES2;
  uint64_t* acc_full = bars + 2 * STAGES2;
  uint64_t* acc_empty = bars + 2 * STAGES2 + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES2 + 4);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();   // both CTAs' barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_tiles = p.num_m_tiles * p.num_n_tiles;
  const int k_iters = (p.K + BK - 1) / BK;
  const int pair = int(blockIdx.x) / 2, npairs = int(gridDim.x) / 2;

  if (warp == 0) {
    if (elect_one()) {
      int it = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < total_tiles; tile += npairs) {
        int mb, nb;
        tile_coords(tile, p, mb, nb);
        for (int k = 0; k < k_iters; ++k, ++it) {
          const int s = it % STAGES2;
          const uint32_t ph = (it / STAGES2) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, p.status, 121)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[s], 4 * HALF_STAGE);
          const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
          tma_load_2d_pair(sA + s * HALF_STAGE, &tmA, fb, k * BK, mb * 256 + int(rank) * 128);
          tma_load_2d_pair(sB + s * HALF_STAGE, &tmB, fb, k * BK, nb * BN + int(rank) * 128);
        }
      }
      // drain: the last commits on this CTA's empty barriers have landed before the CTA exits
      for (int d = 0; ok && d < STAGES2 && d < it; ++d) {
        const int j = it - 1 - d;
        if (!mbar_wait(&empty[j % STAGES2], (j / STAGES2) & 1, p.status, 125)) ok = false;
      }
    }
  } else if (warp == 1) {
    if (leader && elect_one()) {
      constexpr uint32_t idesc = idesc_bf16_f32(256, BN, false, false);
      int it = 0;
      int local = 0;
      for (int tile = pair; tile < total_tiles; tile += npairs, ++local) {
        const int b = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[b], aph ^ 1, p.status, 122)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(b * BN);
        bool ok = true;
        for (int k = 0; k < k_iters; ++k, ++it) {
          const int s = it % STAGES2;
          const uint32_t ph = (it / STAGES2) & 1;
          if (!mbar_wait(&full[s], ph, p.status, 123)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * HALF_STAGE);
          const uint32_t b0 = smem_u32(sB + s * HALF_STAGE);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = sdesc_sw128(a0 + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(b0 + kk * 32, 16, 1024);
            umma_pair_bf16_ss(d_tmem, ad, bd, idesc, (k | kk) != 0 ? 1u : 0u);
          }
          umma_pair_commit_both(&empty[s]);
        }
        if (!ok) break;
        umma_pair_commit_both(&acc_full[b]);
      }
    }
  } else if (warp >= 4) {
    const int q = warp - 4;
    const int row_in_tile = q * 32 + lane;
    const uint32_t acc_empty_leader[2] = {mapa_shared(smem_u32(&acc_empty[0]), 0),
                                          mapa_shared(smem_u32(&acc_empty[1]), 0)};
    int local = 0;
    for (int tile = pair; tile < total_tiles; tile += npairs, ++local) {
      const int b = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[b], aph, p.status, 124)) break;
      tc_fence_after();
      int mb, nb;
      tile_coords(tile, p, mb, nb);
      const uint32_t tacc = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(b * BN);
      // this CTA's 128 rows of the 256-row tile, as the 128-row block 2 mb + rank
      epilogue_tile<EPI>(p, tacc, 2 * mb + int(rank), nb, row_in_tile);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acc_empty_leader[b]);
    }
  }

  if constexpr (EPI == kEpiQkvPush) {
    if (warp >= 4) __threadfence_system();
  }
  tc_fence_before();
  cluster_sync_all();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
  if constexpr (EPI == kEpiQkvPush) {
    if (threadIdx.x == 0 && p.qkv.done_counter != nullptr) {
      __threadfence_system();
      const unsigned prev = atomicAdd(p.qkv.done_counter, 1u);
      if (prev == gridDim.x - 1) {
        __threadfence_system();
        for (int rk = 0; rk < p.qkv.n_stage; ++rk) st_release_sys(p.qkv.ready_ptrs[rk], p.qkv.epoch);
        *p.qkv.done_counter = 0;
      }
    }
  }
}

// ----------------------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

bool make_tma_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tma_3d_bf16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                      uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1,
                      uint32_t b2) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int EPI>
static cudaError_t launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                          int grid, cudaStream_t stream) {
  static std::atomic<unsigned long long> attr{0};
  cudaError_t e = once_per_device(attr, [] {
    return cudaFuncSetAttribute(gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                SMEM_BYTES);
  });
  if (e != cudaSuccess) return e;
  gemm_kernel<EPI><<<grid, 256, SMEM_BYTES, stream>>>(ta, tb, p);
  return cudaGetLastError();
}

// Pair kernel launch: clusters of 2 CTAs, as many pairs as can be resident at once (at most one
// per tile).
template <int EPI>
static cudaError_t launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                               int tiles, cudaStream_t stream) {
  static std::atomic<unsigned long long> attr{0};
  cudaError_t e = once_per_device(attr, [] {
    return cudaFuncSetAttribute(gemm2_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                SMEM_BYTES2);
  });
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = SMEM_BYTES2;
  cfg.stream = stream;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  static int max_pairs[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (max_pairs[dev] == 0) {
    cfg.gridDim = dim3(2);
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, gemm2_kernel<EPI>, &cfg);
    if (e != cudaSuccess) return e;
    max_pairs[dev] = n > 0 ? n : 1;
  }
  const int pairs = tiles < max_pairs[dev] ? tiles : max_pairs[dev];
  cfg.gridDim = dim3(2 * pairs);
  return cudaLaunchKernelEx(&cfg, gemm2_kernel<EPI>, ta, tb, p);
}

// Tile-order band height in m-blocks: bands of 16 when the weight B (N x K) is larger than
// 64 MB, which does not stay in L2 while n-fastest order sweeps it once per m-block; n fastest
// otherwise. Measured on B200 with the pair kernel (ms, n fastest -> bands of 16): 28672 x 4096
// gate/up at M = 32768 7.55 -> 5.56, 16384 x 2048 gate/up 1.75 -> 1.37; the 2048 x 8192 down
// projection (33 MB) 0.74 -> 0.82 and 6144 x 4096 QKV 1.06 -> 1.22 prefer n fastest.
// HCP_GEMM_GROUP=n forces bands of n (0: n fastest).
static int group_for(long N, long K) {
  static int env = -2;
  if (env == -2) {
    const char* e = getenv("HCP_GEMM_GROUP");
    env = (e && *e) ? atoi(e) : -1;
  }
  if (env >= 0) return env;
  return double(N) * double(K) * 2.0 > 64.0 * (1 << 20) ? 16 : 0;
}

// 1: CTA-pair kernel (default), 0: one CTA per tile (HCP_GEMM_PAIR=0)
static int pair_default() {
  static int env = -2;
  if (env == -2) {
    const char* e = getenv("HCP_GEMM_PAIR");
    env = (e && *e) ? atoi(e) : 1;
  }
  return env != 0 ? 1 : 0;
}

const char* gemm_bf16(const GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return "gemm: empty problem";
  if ((a.lda * 2) % 16 || (a.ldb * 2) % 16) return "gemm: lda/ldb must be multiples of 8 elements";
  if ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.B)) & 15)
    return "gemm: A/B base must be 16-byte aligned";
  if (a.epi == kEpiSwiGLU && (a.N % BN) != 0) return "gemm: SwiGLU needs N % 256 == 0";
  if (a.epi != kEpiSwiGLU && ((a.ldc * 2) % 16 || (reinterpret_cast<uintptr_t>(a.C) & 15)))
    return "gemm: C must be 16-byte aligned with ldc % 8 == 0";
  if (a.epi == kEpiResidual && (a.R == nullptr || (a.ldr * 2) % 16 ||
                                (reinterpret_cast<uintptr_t>(a.R) & 15)))
    return "gemm: residual must be 16-byte aligned with ldr % 8 == 0";
  if (a.epi == kEpiBias && a.bias == nullptr) return "gemm: bias missing";
  const bool pair = a.variant == 2 || (a.variant == 0 && pair_default());
  CUtensorMap ta, tb;
  if (!make_tma_2d_bf16(&ta, a.A, a.K, a.M, uint64_t(a.lda) * 2, BK, BM))
    return "gemm: TMA descriptor for A failed";
  if (!make_tma_2d_bf16(&tb, a.B, a.K, a.N, uint64_t(a.ldb) * 2, BK, pair ? 128 : BN))
    return "gemm: TMA descriptor for B failed";
  Params p;
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.num_m_tiles = (a.M + BM - 1) / BM;
  p.num_n_tiles = (a.N + BN - 1) / BN;
  p.C = a.C;
  p.ldc = a.ldc;
  p.bias = a.bias;
  p.R = a.R;
  p.ldr = a.ldr;
  p.status = a.status;
  p.group_m = a.group >= 0 ? a.group : group_for(a.N, a.K);
  if (pair) {
    p.num_m_tiles = (a.M + 255) / 256;
    const int tiles2 = p.num_m_tiles * p.num_n_tiles;
    cudaError_t e2;
    switch (a.epi) {
      case kEpiStore: e2 = launch_pair<kEpiStore>(ta, tb, p, tiles2, stream); break;
      case kEpiBias: e2 = launch_pair<kEpiBias>(ta, tb, p, tiles2, stream); break;
      case kEpiResidual: e2 = launch_pair<kEpiResidual>(ta, tb, p, tiles2, stream); break;
      case kEpiSwiGLU: e2 = launch_pair<kEpiSwiGLU>(ta, tb, p, tiles2, stream); break;
      default: return "gemm: unknown epilogue";
    }
    return e2 == cudaSuccess ? nullptr : cudaGetErrorString(e2);
  }
  const int tiles = p.num_m_tiles * p.num_n_tiles;
  const int grid = tiles < a.num_sms ? tiles : a.num_sms;
  cudaError_t e;
  switch (a.epi) {
    case kEpiStore: e = launch<kEpiStore>(ta, tb, p, grid, stream); break;
    case kEpiBias: e = launch<kEpiBias>(ta, tb, p, grid, stream); break;
    case kEpiResidual: e = launch<kEpiResidual>(ta, tb, p, grid, stream); break;
    case kEpiSwiGLU: e = launch<kEpiSwiGLU>(ta, tb, p, grid, stream); break;
    default: return "gemm: unknown epilogue";
  }
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

const char* gemm_qkv_push(const GemmArgs& a, const QkvPushArgs& q, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return "gemm_qkv_push: empty problem";
  if ((a.lda * 2) % 16 || (a.ldb * 2) % 16) return "gemm_qkv_push: lda/ldb must be multiples of 8";
  if ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.B)) & 15)
    return "gemm_qkv_push: A/B base must be 16-byte aligned";
  if ((q.D != 64 && q.D != 128) || BN % q.D) return "gemm_qkv_push: head_dim must be 64 or 128";
  if (a.N != (q.H + 2 * q.Hkv) * q.D) return "gemm_qkv_push: N must be (H + 2 Hkv) * D";
  if (q.pos == nullptr || q.cos_t == nullptr || q.sin_t == nullptr || q.q_out == nullptr)
    return "gemm_qkv_push: positions, RoPE tables and q_out are required";
  if ((reinterpret_cast<uintptr_t>(q.q_out) | reinterpret_cast<uintptr_t>(q.cos_t) |
       reinterpret_cast<uintptr_t>(q.sin_t)) & 15)
    return "gemm_qkv_push: q_out and the RoPE tables must be 16-byte aligned";
  if (q.n_stage > 0 && q.stage_ptrs == nullptr) return "gemm_qkv_push: staging pointers missing";
  const bool pair = a.variant == 2 || (a.variant == 0 && pair_default());
  CUtensorMap ta, tb;
  if (!make_tma_2d_bf16(&ta, a.A, a.K, a.M, uint64_t(a.lda) * 2, BK, BM))
    return "gemm_qkv_push: TMA descriptor for A failed";
  if (!make_tma_2d_bf16(&tb, a.B, a.K, a.N, uint64_t(a.ldb) * 2, BK, pair ? 128 : BN))
    return "gemm_qkv_push: TMA descriptor for B failed";
  Params p{};
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.num_m_tiles = (a.M + BM - 1) / BM;
  p.num_n_tiles = (a.N + BN - 1) / BN;
  p.bias = a.bias;
  p.status = a.status;
  p.qkv = q;
  p.group_m = a.group >= 0 ? a.group : group_for(a.N, a.K);
  if (pair) {
    p.num_m_tiles = (a.M + 255) / 256;
    cudaError_t e2 = launch_pair<kEpiQkvPush>(ta, tb, p, p.num_m_tiles * p.num_n_tiles, stream);
    return e2 == cudaSuccess ? nullptr : cudaGetErrorString(e2);
  }
  const int tiles = p.num_m_tiles * p.num_n_tiles;
  const int grid = tiles < a.num_sms ? tiles : a.num_sms;
  cudaError_t e = launch<kEpiQkvPush>(ta, tb, p, grid, stream);
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

}  // namespace gemm
}  // namespace hcp
