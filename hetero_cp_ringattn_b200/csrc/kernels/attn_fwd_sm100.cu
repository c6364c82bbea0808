// K1: blockwise online-softmax attention on tcgen05 / TMEM, with log-sum-exp output and a
// causal skip driven by global token positions (vanilla, striped and zigzag layouts, uneven
// chunks).
//
// Replaces the reference's ring block step `process_kv_block` (rust/src/model/attention/
// ring.rs:201-370: S = Q K^T * s, global-position causal mask, row max, exp, row sum, P V,
// online rescale of (m, l, O), fully-future block skip) and its q-chunk / micro-block loops
// (ring.rs:861-1399). Instead of materialising a [qc, kc] score tensor per block with ~10 ATen
// launches, one CTA streams KV tiles through shared memory and keeps S, P and O in TMEM.
//
// KV operand: a position-ordered K/V staging buffer [Hkv, L, D] (row p holds the key of global
// position p). In context-parallel runs every rank's rows have to reach every rank's staging
// buffer. Overlapped mode (the default; the reference's pipelined ring, ring.rs:1195-1339): the
// projection writes only the local buffer and this kernel does the ring itself: warps 2 and 3
// store this rank's rows into every peer's buffer over NVLink tile by tile and publish a flag
// per (tile, source rank), while the q tiles start on the rank's own rows (each CTA walks its
// KV tiles down from its diagonal, which is always local) and the TMA producer waits (bounded)
// for the flags of each remote tile just before loading it. The last CTA releases the staging parity to every rank. Serial mode
// (the reference's HCP_DISABLE_OVERLAP=1, ring.rs:164-166): every row was pushed and waited for
// before the launch, and the kernel only computes.
//
// CTA layout (one CTA per SM): two q tiles of 128 rows of one head share every K/V tile.
//   warp 0      TMA producer (Q0, Q1 once; K/V tiles through a STAGES-deep ring)
//   warp 1      MMA issuer: S_i = Q_i K^T (SS) and O += P V (TS: P read from TMEM)
//   warp 2      TMEM allocator; with warp 3 the KV ring push (overlapped mode)
//   warpgroups 1..  softmax streams (thread <-> row <-> TMEM lane): head_dim 128 has one stream
//               per q tile (384 threads); head_dim 64 splits each tile's 128 keys into two
//               64-column streams with their own running max, row sum and O (640 threads), so
//               four warpgroups share the exponentials, merged per row in the epilogue.
// The MMA warp alternates between the tiles, so the tensor core works on one tile's products
// while the other tile's streams run their softmax. TMEM: S_i at column 128 i (each stream's P,
// packed bf16, overwrites the first half of its own S columns), O of stream st at 256 + D st.
// Softmax: one TMEM read of S per row (row max, then exponentials from registers), lazy O rescale
// (only when the running max grows by more than 2^8), a share of the exponentials (POLY of every
// 8 pairs) on the FMA pipe, a mask-free variant for tiles below every row's causal bound.
// Registers: warpgroup 0 hands registers to the softmax warpgroups with setmaxnreg.
//
// Pipelined variant (PIPE, head_dim 64, one stream per q tile): P goes to TMEM columns of its own
// (S_i at 128 i, O_i at 256 + 64 i, P_i at 384 + 64 i), so the scores' columns are free as soon
// as the softmax has loaded them. The softmax threads signal that (s_free) right after their
// TMEM load, and the MMA warp issues S_i(j+1) = Q_i K_{j+1}^T at once, while the same q tile's
// exponentials of step j are still being computed; the softmax of step j + 1 in turn computes
// its exponentials while P V of step j runs and only waits for that product (p_free) before it
// stores P and rescales O. Per q tile the serial chain per KV tile is the softmax alone instead
// of softmax + P V + Q K^T.
#include <cstdlib>

#include "attn_fwd_sm100.h"
#include "common.cuh"
#include "gemm_sm100.h"
#include "launch.h"

namespace hcp {
namespace attn {

using namespace hcp::dev;

constexpr int BQ = 128;      // q rows per tile
constexpr int BKV = 128;     // kv rows per tile
constexpr int QT = 2;        // q tiles per CTA
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int D, bool PIPE = false>
struct Cfg {
  static constexpr int ATOMS = D / 64;           // 128-byte swizzle atoms along D
  static constexpr int Q_BYTES = BQ * D * 2;     // one q tile
  static constexpr int KV_BYTES = BKV * D * 2;
  static constexpr int STAGES = (D == 64) ? 3 : 2;
  static constexpr int SMEM = 1024 + QT * Q_BYTES + 2 * STAGES * KV_BYTES + 4096;
  static constexpr int TMEM_COLS = 512;
  static constexpr int O_COL = 256;
  static constexpr int P_COL = 384;              // PIPE: P_i at P_COL + 64 i (head_dim 64)
  // threads: warpgroup 0 (TMA, MMA, TMEM allocator, idle) + one warpgroup per softmax stream
  __host__ __device__ static constexpr int threads(int hv) { return 128 + QT * hv * 128; }
  // register split (setmaxnreg): 128 x wg0 + (threads - 128) x sm must not exceed the launch's
  // threads x registers (168 at 384 threads: 11264 + 53248 <= 64512; 96 at 640: 11264 + 49152
  // <= 61440)
  __host__ __device__ static constexpr int wg0_regs(int hv) { return 88; }
  __host__ __device__ static constexpr int sm_regs(int hv) { return hv == 1 ? 208 : 96; }
  static_assert(!PIPE || D == 64, "the pipelined variant needs head_dim 64 (TMEM columns)");
};

struct KParams {
  int T, H, Hkv, L;
  const int* q_pos;
  __nv_bfloat16* O;
  float* lse;
  float scale_log2;
  int causal;
  int num_pairs;        // ceil(num_q_tiles / 2)
  int pair_major;       // CTA order: 1 = heaviest q-tile pairs first across all heads
  RingArgs ring;        // in-kernel KV ring (ring.tile_src == nullptr: off)
  unsigned long long wait_budget_ns;
  int* status;
};

// Push of this rank's K/V rows to the peers (one warp; the calling warps take turns through the
// work counter, so whichever CTAs are resident finish every item). An item is (own tile k, peer
// d): wait (bounded) until d has released this staging parity (consumed[d] >= epoch - 2), copy
// the rows of tile k from the local staging buffer to d's with 16-byte loads / peer stores (eight
// in flight per lane), then publish tflags[d][tile][my_rank] = epoch with a system-scope release.
// Items run tile-major from this rank's last tile down, each tile to every peer in rank order
// starting after this rank, so all peers receive the tiles in the same order.
template <int D>
__device__ __forceinline__ void ring_push(const KParams& p, int lane) {
  const RingArgs& g = p.ring;
  const int peers = g.world - 1;
  const int n_items = g.n_push * peers;
  constexpr int dvec = D / 8;                 // 16-byte units of one head row
  const int units = 2 * p.Hkv * dvec;         // units of one position (K and V, every KV head)
  while (true) {
    int item = 0;
    if (lane == 0) item = int(atomicAdd(g.counters, 1u));
    item = __shfl_sync(0xffffffffu, item, 0);
    if (item >= n_items) break;
    const int k = item / peers;
    const int dst = (g.my_rank + 1 + item % peers) % g.world;
    const int tile = g.push_tiles[3 * k], lo = g.push_tiles[3 * k + 1], hi = g.push_tiles[3 * k + 2];
    int ok = 1;
    if (lane == 0 && g.epoch > 2)
      ok = wait_flag_geq_sys(g.consumed + dst, g.epoch - 2, p.wait_budget_ns, p.status, 214, dst);
    if (!__shfl_sync(0xffffffffu, ok, 0)) break;
    __nv_bfloat16* dstb = static_cast<__nv_bfloat16*>(g.stage_ptrs[dst]);
    const int total = (hi - lo) * units;
    for (int u0 = lane; u0 < total; u0 += 32 * 8) {
      uint4 v[8];
      long off[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int u = u0 + 32 * i;
        off[i] = -1;
        if (u < total) {
          const int row = lo + u / units, rem = u % units;
          off[i] = ((long)(rem / dvec) * g.stage_cap + p.q_pos[row]) * D + (rem % dvec) * 8;
          v[i] = ld_nc_v4(g.own_stage + off[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (off[i] >= 0) *reinterpret_cast<uint4*>(dstb + off[i]) = v[i];
    }
    __threadfence_system();
    __syncwarp();
    if (lane == 0) st_release_sys(g.tflag_ptrs[dst] + (long)tile * g.world + g.my_rank, g.epoch);
  }
}

// Processing order of the KV tiles: from the CTA's last visible tile (its diagonal) down to
// tile 0. Every row therefore folds its visible tiles in the same order (its own diagonal tile
// first, then descending) whatever q rows share its CTA: tiles above a row's diagonal are fully
// masked for it and leave no trace (the first visible tile resets the running state with
// alpha = 0). The result is the same bits for a row on one GPU and under any context-parallel
// layout, and in a ring the rows of the rank's own contiguous run come first.
__device__ __forceinline__ int kv_tile_at(int j, int n) { return n - 1 - j; }

// One softmax step of one stream (a q-tile row over CW key columns) held in TMEM: one batch of
// TMEM loads brings the stream's scores into registers, row max with 3-input maxima, lazy
// rescale of the running max and of the stream's O (only when the max grows by more than 2^8),
// then P = 2^(s * scale - m) packed to bf16 into the first CW/2 columns of the stream's S range
// and the row sum. MASK = true applies the causal / length bound (kv position > lim gives
// -inf); tiles below every row's bound use MASK = false and carry no per-element compare.
template <int D, int POLY, int CW, bool MASK>
__device__ __forceinline__ void softmax_step(uint32_t s_addr, uint32_t o_addr, int kv0, int lim,
                                             float scale_log2, bool o_live, float& m_ref,
                                             float& l_sum) {
  uint32_t r[CW];
#pragma unroll
  for (int c = 0; c < CW / 32; ++c) tmem_ld32(s_addr + c * 32, r + c * 32);
  tmem_wait_ld();
  if (MASK) {
#pragma unroll
    for (int e = 0; e < CW; ++e)
      if (kv0 + e > lim) r[e] = __float_as_uint(-INFINITY);
  }
  float tmax;
  {
    float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int e = 0; e < CW; e += 8)
#pragma unroll
      for (int k = 0; k < 4; ++k)
        m4[k] = max3f(m4[k], __uint_as_float(r[e + 2 * k]), __uint_as_float(r[e + 2 * k + 1]));
    tmax = max3f(m4[0], m4[1], fmaxf(m4[2], m4[3])) * scale_log2;
  }
  float alpha = 1.f;
  bool resc = false;
  if (tmax > m_ref + kRescaleThreshold || (m_ref == -INFINITY && tmax > -INFINITY)) {
    alpha = (m_ref == -INFINITY) ? 0.f : fast_exp2(m_ref - tmax);
    m_ref = tmax;
    resc = true;
  }
  const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
  // P in chunks of 32 columns (16 packed TMEM columns each), written over scores already in
  // registers; packed f32x2 arithmetic; POLY of every 8 pairs take the FMA-pipe polynomial
  float2 rs0 = make_float2(0.f, 0.f), rs1 = make_float2(0.f, 0.f);
  const float2 negm = make_float2(-m_use, -m_use);
  const float2 sc2 = make_float2(scale_log2, scale_log2);
#pragma unroll
  for (int hh = 0; hh < CW / 32; ++hh) {
    uint32_t pk[16];
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
      const float2 x = __ffma2_rn(make_float2(__uint_as_float(r[hh * 32 + e]), __uint_as_float(r[hh * 32 + e + 1])),
                                  sc2, negm);
      float2 pp;
      if (POLY > 0 && ((e >> 1) & 7) >= 8 - POLY) {
        pp = poly_exp2_x2(x);
      } else {
        pp.x = fast_exp2(x.x);
        pp.y = fast_exp2(x.y);
      }
      if ((e >> 1) & 1) rs1 = __fadd2_rn(rs1, pp);
      else rs0 = __fadd2_rn(rs0, pp);
      pk[e >> 1] = pack_bf16x2(pp.x, pp.y);
    }
    tmem_st16(s_addr + hh * 16, pk);
  }
  // O rescale after the scores are dead (lower register peak). PV(j-1) of this stream completed
  // before S(j) did (same issuing thread, in-order commits), so O is stable, and PV(j) is only
  // issued after this step arrives on p_full.
  if (o_live && __any_sync(0xffffffffu, resc)) {
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t o[32];
      tmem_ld32(o_addr + c * 32, o);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
      tmem_st32(o_addr + c * 32, o);
    }
  }
  tmem_wait_st();
  l_sum = l_sum * alpha + ((rs0.x + rs0.y) + (rs1.x + rs1.y));
}

// One step of a pipelined stream (PIPE: 128 key columns per q-tile row, P in its own TMEM
// columns). After the TMEM load of S the thread arrives on s_free (the MMA warp may write
// S(j+1) into the same columns); the exponentials are computed into registers, then the thread
// waits until P V of the previous step has completed (p_free: P's columns and O are free) before
// it rescales O (lazy, as above) and stores P. Returns false if a bounded wait ran out.
template <int D, int POLY, bool MASK>
__device__ __forceinline__ bool softmax_step_pipe(uint32_t s_addr, uint32_t o_addr, uint32_t p_addr,
                                                  int kv0, int lim, float scale_log2, int j,
                                                  uint64_t* s_free, uint64_t* p_free, int* status,
                                                  float& m_ref, float& l_sum) {
  constexpr int CW = BKV;
  uint32_t r[CW];
#pragma unroll
  for (int c = 0; c < CW / 32; ++c) tmem_ld32(s_addr + c * 32, r + c * 32);
  tmem_wait_ld();
  tc_fence_before();
  mbar_arrive(s_free);
  if (MASK) {
#pragma unroll
    for (int e = 0; e < CW; ++e)
      if (kv0 + e > lim) r[e] = __float_as_uint(-INFINITY);
  }
  float tmax;
  {
    float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int e = 0; e < CW; e += 8)
#pragma unroll
      for (int k = 0; k < 4; ++k)
        m4[k] = max3f(m4[k], __uint_as_float(r[e + 2 * k]), __uint_as_float(r[e + 2 * k + 1]));
    tmax = max3f(m4[0], m4[1], fmaxf(m4[2], m4[3])) * scale_log2;
  }
  float alpha = 1.f;
  bool resc = false;
  if (tmax > m_ref + kRescaleThreshold || (m_ref == -INFINITY && tmax > -INFINITY)) {
    alpha = (m_ref == -INFINITY) ? 0.f : fast_exp2(m_ref - tmax);
    m_ref = tmax;
    resc = true;
  }
  const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
  float2 rs0 = make_float2(0.f, 0.f), rs1 = make_float2(0.f, 0.f);
  const float2 negm = make_float2(-m_use, -m_use);
  const float2 sc2 = make_float2(scale_log2, scale_log2);
  uint32_t pk[CW / 2];
#pragma unroll
  for (int e = 0; e < CW; e += 2) {
    const float2 x = __ffma2_rn(make_float2(__uint_as_float(r[e]), __uint_as_float(r[e + 1])), sc2, negm);
    float2 pp;
    if (POLY > 0 && ((e >> 1) & 7) >= 8 - POLY) {
      pp = poly_exp2_x2(x);
    } else {
      pp.x = fast_exp2(x.x);
      pp.y = fast_exp2(x.y);
    }
    if ((e >> 1) & 1) rs1 = __fadd2_rn(rs1, pp);
    else rs0 = __fadd2_rn(rs0, pp);
    pk[e >> 1] = pack_bf16x2(pp.x, pp.y);
  }
  if (j > 0) {
    if (!mbar_wait(p_free, uint32_t(j - 1) & 1u, status, 215)) return false;
    tc_fence_after();
    if (__any_sync(0xffffffffu, resc)) {
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(o_addr + c * 32, o);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
        tmem_st32(o_addr + c * 32, o);
      }
    }
  }
#pragma unroll
  for (int hh = 0; hh < CW / 32; ++hh) tmem_st16(p_addr + hh * 16, pk + hh * 16);
  tmem_wait_st();
  l_sum = l_sum * alpha + ((rs0.x + rs0.y) + (rs1.x + rs1.y));
  return true;
}

// POLY: how many of every 8 exponential pairs use the FMA-pipe polynomial instead of the MUFU.
// HV: softmax warpgroups per q tile. HV = 2 (head_dim 64) splits each 128-key tile into two
// 64-column streams with their own running max, row sum and O accumulator (TMEM: S 2 x 128
// columns, O 4 x 64), so four warpgroups share the softmax work, and merges the two streams of a
// row in the epilogue. HV = 1 (head_dim 128) keeps one stream per q tile.
template <int D, int POLY, int HV, bool RING, bool PIPE>
__global__ void __launch_bounds__(Cfg<D>::threads(HV), 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, KParams p) {
  using C = Cfg<D, PIPE>;
  static_assert(!PIPE || HV == 1, "the pipelined variant has one stream per q tile");
  constexpr int CW = BKV / HV;               // key columns per stream
  constexpr int NS = QT * HV;                // softmax streams per CTA
  static_assert(C::O_COL + NS * D <= C::TMEM_COLS, "TMEM columns");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                               // [QT][ATOMS][128 rows x 128 B]
  uint8_t* sK = sQ + QT * C::Q_BYTES;
  uint8_t* sV = sK + C::STAGES * C::KV_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + C::STAGES * C::KV_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + C::STAGES;
  uint64_t* v_full = k_empty + C::STAGES;
  uint64_t* v_empty = v_full + C::STAGES;
  uint64_t* s_full = v_empty + C::STAGES;  // [QT]
  uint64_t* p_full = s_full + QT;          // [NS]
  uint64_t* o_done = p_full + NS;          // [QT]
  uint64_t* merged = o_done + QT;          // [QT] HV = 2: both streams posted (m, l)
  uint64_t* s_free = merged + QT;          // [QT] PIPE: the stream has loaded S (128 arrivals)
  uint64_t* p_free = s_free + QT;          // [QT] PIPE: P V of the stream's last step completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(p_free + QT);
  int* s_qmin = reinterpret_cast<int*>(tmem_slot + 1);  // [QT]
  int* s_qmax = s_qmin + QT;                            // [QT]
  float* s_ml = reinterpret_cast<float*>(s_qmax + QT);  // [QT][2][BQ] m, l of stream h = 1

  const int warp = threadIdx.x / 32;

  // CTA order. KV-head major (long contexts): the CTAs resident at any time (one per SM) are the
  // q heads of one GQA group over a run of q-tile pairs and stream the same K/V tiles in the same
  // order (one KV head's K and V stay in L2 instead of every group's); within a group, heaviest
  // tile pairs first (largest positions are last in local order). Pair major (grids of a few
  // waves): the heaviest pairs of all heads first, a global longest-first order that keeps the
  // last wave short when there are few CTAs per SM (a context-parallel rank's share of the
  // rows, whose zigzag halves differ widely in length).
  const int group = p.H / p.Hkv;
  int pair, head;
  if (p.pair_major) {
    pair = p.num_pairs - 1 - int(blockIdx.x) / p.H;
    head = int(blockIdx.x) % p.H;
  } else {
    const int per_kv = p.num_pairs * group;
    const int kv_head = int(blockIdx.x) / per_kv;
    const int rem = int(blockIdx.x) % per_kv;
    pair = p.num_pairs - 1 - rem / group;
    head = kv_head * group + rem % group;
  }
  const int kv_head = head / group;
  const int row0 = pair * QT * BQ;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < QT; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&o_done[i], 1);
      mbar_init(&merged[i], BQ);
      mbar_init(&s_free[i], BQ);
      mbar_init(&p_free[i], 1);
      s_qmin[i] = 0x7fffffff;
      s_qmax[i] = -1;
    }
    for (int i = 0; i < NS; ++i) mbar_init(&p_full[i], 128);
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // softmax warps: warpgroup 1 + st handles stream st = tile * HV + half; thread <-> row <-> lane
  const int st = (warp >= 4) ? (warp - 4) / 4 : 0;
  const int tile = st / HV;
  const int half = st % HV;
  const int row = (warp >= 4) ? (int(threadIdx.x) - 128 - st * 128) : 0;
  int my_pos = -1;
  if (warp >= 4) {
    const int r = row0 + tile * BQ + row;
    if (r < p.T) my_pos = p.q_pos[r];
    if (my_pos >= 0 && half == 0) {
      atomicMin(&s_qmin[tile], my_pos);
      atomicMax(&s_qmax[tile], my_pos);
    }
  }
  __syncthreads();
  const uint32_t tmem_base = *tmem_slot;
  const int qmax_all = max(s_qmax[0], s_qmax[1]);
  const int kv_tiles_L = (p.L + BKV - 1) / BKV;
  int n_tiles = p.causal ? (qmax_all >= 0 ? qmax_all / BKV + 1 : 0) : kv_tiles_L;
  if (n_tiles > kv_tiles_L) n_tiles = kv_tiles_L;
  const bool tile1_live = (row0 + BQ) < p.T;

  // register split: warpgroup 0 (TMA, MMA, TMEM allocator, idle warp) hands registers to the
  // softmax warpgroups; each warpgroup executes its setmaxnreg at one point, before its warps
  // take their roles
  if (warp < 4) {
  reg_dealloc<C::wg0_regs(HV)>();
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (elect_one() && n_tiles > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, QT * C::Q_BYTES);
#pragma unroll
      for (int i = 0; i < QT; ++i)
#pragma unroll
        for (int a = 0; a < C::ATOMS; ++a)
          tma_load_3d(sQ + i * C::Q_BYTES + a * (BQ * 128), &tmQ, q_full, a * 64, head,
                      row0 + i * BQ);
      for (int j = 0; j < n_tiles; ++j) {
        const int t = kv_tile_at(j, n_tiles);
        const int s = j % C::STAGES;
        const uint32_t ph = (j / C::STAGES) & 1;
        if (RING) {
          // remote rows of this tile: wait (bounded) for every other source rank's flag, then
          // order what the flags made visible before the TMA (async proxy) reads it
          unsigned long long m = p.ring.tile_src[t] & ~(1ull << p.ring.my_rank);
          bool arrived = true;
          while (m != 0ull) {
            const int src = __ffsll((long long)m) - 1;
            m &= m - 1ull;
            if (!wait_flag_geq_sys(p.ring.tile_flags + (long)t * p.ring.world + src, p.ring.epoch,
                                   p.wait_budget_ns, p.status, 210, t)) {
              arrived = false;
              break;
            }
          }
          if (!arrived) break;
          fence_proxy_async_global();
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
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one() && n_tiles > 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(BQ, BKV, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(BQ, D, false, true);
      const uint32_t sq = smem_u32(sQ);
      auto issue_qk = [&](int i, int s) {
        const uint32_t sk = smem_u32(sK + s * C::KV_BYTES);
        const uint32_t qb = sq + i * C::Q_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk / 4) * (BQ * 128) + (kk % 4) * 32;
          const uint32_t offk = (kk / 4) * (BKV * 128) + (kk % 4) * 32;
          umma_bf16_ss(tmem_base + i * BKV, sdesc_sw128(qb + off, 16, 1024),
                       sdesc_sw128(sk + offk, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
      };
      // stream (i, h): O_ih += P_ih V[h * CW, (h + 1) * CW) with P from TMEM (16 keys = 8
      // columns per step) and V rows from the MN-major smem tile (16 rows = 2048 bytes)
      auto issue_pv = [&](int i, int h, int s, bool acc) {
        const uint32_t sv = smem_u32(sV + s * C::KV_BYTES) + h * CW * 128;
#pragma unroll
        for (int kk = 0; kk < CW / 16; ++kk) {
          umma_bf16_ts(tmem_base + C::O_COL + (i * HV + h) * D, tmem_base + i * BKV + h * CW + kk * 8,
                       sdesc_sw128(sv + kk * 2048, BKV * 128, 1024), idesc_o,
                       (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, p.status, 203) && mbar_wait(&k_full[0], 0, p.status, 206);
      if (ok) {
        tc_fence_after();
        issue_qk(0, 0);
        umma_commit(&s_full[0]);
        issue_qk(1, 0);
        umma_commit(&s_full[1]);
        umma_commit(&k_empty[0]);
      }
      if (PIPE) {
        // S_i(j+1) as soon as stream i has loaded S_i(j); P_i(j) V_j as soon as it stored P_i(j)
        for (int j = 0; ok && j < n_tiles; ++j) {
          const int s = j % C::STAGES;
          const int s1 = (j + 1) % C::STAGES;
          const bool more = j + 1 < n_tiles;
          if (more) {
            if (!mbar_wait(&k_full[s1], ((j + 1) / C::STAGES) & 1, p.status, 206)) {
              ok = false;
              break;
            }
#pragma unroll
            for (int i = 0; i < QT; ++i) {
              if (!mbar_wait(&s_free[i], j & 1, p.status, 216)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_qk(i, s1);
              umma_commit(&s_full[i]);
            }
            if (!ok) break;
            umma_commit(&k_empty[s1]);
          }
          if (!mbar_wait(&v_full[s], (j / C::STAGES) & 1, p.status, 205)) {
            ok = false;
            break;
          }
          const uint32_t sv = smem_u32(sV + s * C::KV_BYTES);
#pragma unroll
          for (int i = 0; i < QT; ++i) {
            if (!mbar_wait(&p_full[i], j & 1, p.status, 204 + 3 * i)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < BKV / 16; ++kk)
              umma_bf16_ts(tmem_base + C::O_COL + i * D, tmem_base + C::P_COL + i * (BKV / 2) + kk * 8,
                           sdesc_sw128(sv + kk * 2048, BKV * 128, 1024), idesc_o,
                           (j > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&p_free[i]);
            if (!more) umma_commit(&o_done[i]);
          }
          if (!ok) break;
          umma_commit(&v_empty[s]);
        }
      }
      for (int j = 0; !PIPE && ok && j < n_tiles; ++j) {
        const int s = j % C::STAGES;
        const int s1 = (j + 1) % C::STAGES;
        const bool more = j + 1 < n_tiles;
        if (!mbar_wait(&v_full[s], (j / C::STAGES) & 1, p.status, 205)) {
          ok = false;
          break;
        }
        if (more && !mbar_wait(&k_full[s1], ((j + 1) / C::STAGES) & 1, p.status, 206)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int i = 0; i < QT; ++i) {
          // tile i: O_ih += P_ih V_j for every stream, then S_i = Q_i K_{j+1}^T over the same
          // TMEM columns (in-order issue: the PV reads of P come first)
#pragma unroll
          for (int h = 0; h < HV; ++h) {
            if (!mbar_wait(&p_full[i * HV + h], j & 1, p.status, 204 + 3 * i)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(i, h, s, j > 0);
          }
          if (!ok) break;
          if (i == QT - 1) umma_commit(&v_empty[s]);
          if (more) {
            issue_qk(i, s1);
            umma_commit(&s_full[i]);
            if (i == QT - 1) umma_commit(&k_empty[s1]);
          } else {
            umma_commit(&o_done[i]);
          }
        }
      }
    }
  } else if (RING && p.ring.n_push > 0) {
    // ------------------------------------------------------------------ KV ring push (warps 2, 3)
    ring_push<D>(p, int(threadIdx.x % 32));
  }
  } else {
    reg_alloc<C::sm_regs(HV)>();
    // ------------------------------------------------------------------ softmax streams
    const uint32_t lane_off = uint32_t((warp % 4) * 32) << 16;
    const uint32_t s_addr = tmem_base + lane_off + uint32_t(tile * BKV + half * CW);
    const uint32_t o_addr = tmem_base + lane_off + uint32_t(C::O_COL + st * D);
    const int grow = row0 + tile * BQ + row;
    const bool live = (tile == 0) || tile1_live;
    float m_ref = -INFINITY;  // max used for exponentiation (log2 domain)
    float l_sum = 0.f;
    bool ok = true;
    const uint32_t p_addr = tmem_base + lane_off + uint32_t(C::P_COL + tile * (BKV / 2));
    for (int j = 0; j < n_tiles; ++j) {
      const int t = kv_tile_at(j, n_tiles);
      if (!mbar_wait(&s_full[tile], j & 1, p.status, 208)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int kv0 = t * BKV + half * CW;
      const int lim = p.causal ? min(my_pos, p.L - 1) : p.L - 1;  // last visible kv position
      // the masked variant only for tiles that cross some row's bound (diagonal / tail tiles)
      const bool masked = __any_sync(0xffffffffu, kv0 + CW - 1 > lim);
      if (PIPE) {
        ok = masked ? softmax_step_pipe<D, POLY, true>(s_addr, o_addr, p_addr, kv0, lim, p.scale_log2, j,
                                                       &s_free[tile], &p_free[tile], p.status, m_ref, l_sum)
                    : softmax_step_pipe<D, POLY, false>(s_addr, o_addr, p_addr, kv0, lim, p.scale_log2, j,
                                                        &s_free[tile], &p_free[tile], p.status, m_ref, l_sum);
        if (!ok) break;
      } else if (masked) {
        softmax_step<D, POLY, CW, true>(s_addr, o_addr, kv0, lim, p.scale_log2, j > 0, m_ref, l_sum);
      } else {
        softmax_step<D, POLY, CW, false>(s_addr, o_addr, kv0, lim, p.scale_log2, j > 0, m_ref, l_sum);
      }
      tc_fence_before();
      mbar_arrive(&p_full[st]);
    }
    // epilogue: merge the HV streams of each row (half 1 posts its (m, l), half 0 combines and
    // writes the row: both O accumulators sit in the same TMEM lanes), O / l and LSE
    float m_tot = m_ref, l_tot = l_sum, a_own = 1.f, a_oth = 0.f;
    if (HV == 2) {
      float* ml = s_ml + tile * 2 * BQ;
      if (half == 1) {
        ml[row] = m_ref;
        ml[BQ + row] = l_sum;
        mbar_arrive(&merged[tile]);
      } else if (ok) {
        ok = mbar_wait(&merged[tile], 0, p.status, 213);
        if (ok) {
          const float m1 = ml[row], l1 = ml[BQ + row];
          m_tot = fmaxf(m_ref, m1);
          a_own = m_tot == -INFINITY ? 0.f : fast_exp2(m_ref - m_tot);
          a_oth = m_tot == -INFINITY ? 0.f : fast_exp2(m1 - m_tot);
          l_tot = l_sum * a_own + l1 * a_oth;
        }
      }
    }
    // HV = 2: half 0 finishes the row (both O accumulators are in the same TMEM lanes)
    const bool writer = (HV == 1) || (half == 0);
    if (ok && n_tiles > 0 && mbar_wait(&o_done[tile], 0, p.status, 209)) {
      tc_fence_after();
      if (writer) {
        const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
        __nv_bfloat16* dst = p.O + ((long)grow * p.H + head) * D;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + c * 32, o);
          if (HV == 2) {
            uint32_t o2[32];
            tmem_ld32(o_addr + D + c * 32, o2);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e)
              o[e] = __float_as_uint(__uint_as_float(o[e]) * a_own + __uint_as_float(o2[e]) * a_oth);
          } else {
            tmem_wait_ld();
          }
          if (live && grow < p.T) {
            uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              d4[i] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * i]) * inv, __uint_as_float(o[8 * i + 1]) * inv),
                                 pack_bf16x2(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv),
                                 pack_bf16x2(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv),
                                 pack_bf16x2(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv));
          }
        }
        if (live && grow < p.T && p.lse != nullptr) {
          p.lse[(long)head * p.T + grow] =
              l_tot > 0.f ? (m_tot + __log2f(l_tot)) * 0.6931471805599453f : -INFINITY;
        }
      }
    } else if (n_tiles == 0 && writer && live && grow < p.T) {
      // no visible key (padding rows / empty KV): O = 0, LSE = -inf
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
  if (RING && threadIdx.x == 0) {
    // last CTA: every CTA's reads of this staging parity and pushes are done; tell every rank
    // it may overwrite the parity (layer step epoch + 2) and reset the counters for the next step
    __threadfence_system();
    const unsigned prev = atomicAdd(p.ring.counters + 1, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int r = 0; r < p.ring.world; ++r) st_release_sys(p.ring.consumed_ptrs[r], p.ring.epoch);
      p.ring.counters[0] = 0u;
      p.ring.counters[1] = 0u;
    }
  }
}

template <int D, int POLY, int HV, bool RING, bool PIPE = false>
static cudaError_t launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                          const KParams& p, cudaStream_t stream) {
  static_assert(Cfg<D>::threads(HV) <= 1024, "threads");
  static_assert(128 * Cfg<D>::wg0_regs(HV) + (Cfg<D>::threads(HV) - 128) * Cfg<D>::sm_regs(HV) <=
                    Cfg<D>::threads(HV) * ((65536 / Cfg<D>::threads(HV)) / 8 * 8),
                "register split exceeds the launch's registers");
  static std::atomic<unsigned long long> attr{0};
  cudaError_t e = once_per_device(attr, [] {
    return cudaFuncSetAttribute(attn_fwd_kernel<D, POLY, HV, RING, PIPE>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D>::SMEM);
  });
  if (e != cudaSuccess) return e;
  const int grid = p.num_pairs * p.H;
  attn_fwd_kernel<D, POLY, HV, RING, PIPE><<<grid, Cfg<D>::threads(HV), Cfg<D>::SMEM, stream>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

// Head_dim 64 kernel variant: HCP_ATTN_HV=2 two softmax streams per q tile, =1 one stream,
// =3 one stream with P in its own TMEM columns (the pipelined variant, PIPE).
static int hv64() {
  static int env = -2;
  if (env == -2) {
    const char* s = getenv("HCP_ATTN_HV");
    env = (s && *s) ? atoi(s) : 2;
  }
  return (env == 1 || env == 3) ? env : 2;
}

// Polynomial share (out of 8 exponential pairs), the same for head_dim 64 and 128; HCP_ATTN_POLY
// overrides it (0, 2, 3 or 4).
static int poly_share() {
  static int env = -2;
  if (env == -2) {
    const char* s = getenv("HCP_ATTN_POLY");
    env = (s && *s) ? atoi(s) : -1;
  }
  if (env == 0 || (env >= 2 && env <= 4)) return env;
  // measured on B200 (32k causal, 32/8 heads, one TMEM read of S per step): 3 of 8 pairs is the
  // best split for D=64 and 128 (748 / 1263 TFLOP/s; 4 of 8 gives 703 / 1152)
  return 3;
}

template <int D, int HV, bool PIPE = false>
static cudaError_t launch_hv(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                             const KParams& p, cudaStream_t stream) {
  switch (poly_share()) {
    case 2: return launch<D, 2, HV, false, PIPE>(tq, tk, tv, p, stream);
    case 3: return launch<D, 3, HV, false, PIPE>(tq, tk, tv, p, stream);
    case 4: return launch<D, 4, HV, false, PIPE>(tq, tk, tv, p, stream);
    default: return launch<D, 0, HV, false, PIPE>(tq, tk, tv, p, stream);
  }
}

template <int D>
static cudaError_t launch_d(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                            const KParams& p, int variant, cudaStream_t stream) {
  const int v = D == 64 ? (variant >= 1 && variant <= 3 ? variant : hv64()) : 1;
  if (p.ring.tile_src != nullptr) {
    // the in-kernel ring (push warps, per-tile waits, consumed release) is compiled into its own
    // variants, with the default exponential split, so the single-rank kernels carry none of it
    if (v == 3) return launch<64, 3, 1, true, true>(tq, tk, tv, p, stream);
    return v == 2 ? launch<64, 3, 2, true>(tq, tk, tv, p, stream) : launch<D, 3, 1, true>(tq, tk, tv, p, stream);
  }
  if (v == 3) return launch_hv<64, 1, true>(tq, tk, tv, p, stream);
  if (v == 2) return launch_hv<64, 2>(tq, tk, tv, p, stream);
  return launch_hv<D, 1>(tq, tk, tv, p, stream);
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
  const int num_q_tiles = (a.T + BQ - 1) / BQ;
  p.num_pairs = (num_q_tiles + QT - 1) / QT;
  // pair-major order when the grid is at most 8 waves of one CTA per SM (a context-parallel
  // rank's share of the rows: measured on B200 at CP=8, 32k, head_dim 64, the slowest rank's
  // attention 0.876 -> 0.804 ms); KV-head major for longer grids, where its L2 reuse wins (one
  // rank at 32k: 5.52 vs 5.72 ms at head_dim 64, 7.31 vs 7.81 at 128). HCP_ATTN_ORDER=0 / 1
  // forces one order, AttnArgs::order overrides both
  {
    static int env = -2;
    if (env == -2) {
      const char* e = getenv("HCP_ATTN_ORDER");
      env = (e && *e) ? atoi(e) : -1;
    }
    static int sm_cache[64] = {0};
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
      if (sm_cache[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        sm_cache[dev] = n > 0 ? n : 148;
      }
      sms = sm_cache[dev];
    }
    const long grid = long(p.num_pairs) * a.H;
    p.pair_major = env >= 0 ? (env != 0) : (grid <= 8L * sms ? 1 : 0);
    if (a.order >= 0) p.pair_major = a.order;
  }
  p.ring = a.ring;
  if (p.ring.tile_src != nullptr) {
    if (p.ring.world < 2 || p.ring.world > 64 || p.ring.my_rank < 0 || p.ring.my_rank >= p.ring.world)
      return "attn: ring needs 2 to 64 ranks";
    if (p.ring.tile_flags == nullptr || p.ring.consumed_ptrs == nullptr || p.ring.counters == nullptr)
      return "attn: ring flags / counters missing";
    if (p.ring.n_push > 0 &&
        (p.ring.push_tiles == nullptr || p.ring.own_stage == nullptr || p.ring.stage_ptrs == nullptr ||
         p.ring.tflag_ptrs == nullptr || p.ring.consumed == nullptr || p.ring.stage_cap < a.L))
      return "attn: ring push arguments missing";
  } else if (p.ring.n_push > 0 || p.ring.consumed_ptrs != nullptr) {
    return "attn: ring push / consumed signal need the tile sources";
  }
  p.wait_budget_ns = a.wait_budget_ns;
  p.status = a.status;
  if (a.variant < 0 || a.variant > 3) return "attn: variant must be 0 to 3";
  cudaError_t e = a.D == 64 ? launch_d<64>(tq, tk, tv, p, a.variant, stream)
                            : launch_d<128>(tq, tk, tv, p, a.variant, stream);
  return e == cudaSuccess ? nullptr : cudaGetErrorString(e);
}

}  // namespace attn
}  // namespace hcp
