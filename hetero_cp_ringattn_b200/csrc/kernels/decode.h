// Host interface of the decode-path kernels (GEMV, K2 cp decode attention + combine).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "kv_layout.h"

namespace hcp {
namespace dec {

enum GemvEpilogue : int {
  kGemvF32 = 0,       // y_f32 = x W^T (+ bias)
  kGemvResidual = 1,  // y_bf16 += bf16(x W^T)     (in place)
  kGemvSwiGLU = 2,    // y_bf16[:, j] = silu(g_j) * u_j, W rows interleaved [128 gate | 128 up]
  kGemvArgmax = 3,    // optional y_f32 logits + packed argmax per row into `argmax`
  kGemvQkvRope = 4,   // QKV projection + bias + RoPE, q -> rope.q_out, k/v appended (GemvRopeArgs)
};

// Weights of later kernels of the decode step to pull into L2 while this kernel runs: CTA i of
// n issues one bulk L2 prefetch of the i-th 1/n slice of each range when it starts (before its
// dependency wait: weights are never written in flight). A decode step reads ~120 MB of weights
// per layer in small latency-bound kernels; prefetched, the next kernel finds them in L2.
// Ranges must start 16-byte aligned and be a multiple of 16 bytes long (null / 0: none).
struct L2Prefetch {
  const void* ptr[2];
  unsigned long long bytes[2];
  int lines;   // 0: one bulk prefetch per CTA and range; 1: every thread prefetches 128-byte lines
};

// kGemvQkvRope epilogue: the projection rows of a head are computed in rotation pairs (j, j + D/2),
// rounded to bf16 (the bf16 linear output), rotated at pos[b] (q and k heads); q goes to q_out
// [B, H, D], k and v to the arena slot slot[b, layer] when this rank stores the row
// (owner[b, layer] != 0).
struct GemvRopeArgs {
  const int* pos;
  const float* cos_t;
  const float* sin_t;
  int max_pos;
  int H, Hkv, D;
  __nv_bfloat16* q_out;
  __nv_bfloat16* arena;
  ArenaGeom geom;
  int layer;
  const int* page_tables;  // [B, pt_stride]
  int pt_stride;
  int slot_cap;
  const int* owner;        // [B, owner_stride]
  const int* slot;
  int owner_stride;
  int* status;
};

// kGemvResidual with `xslot` set: x is not read. Each CTA waits (bounded) until every rank's
// dec_ready flag reaches the epoch, then builds x in shared memory as the log-sum-exp combine in
// rank order of the ranks' (O, LSE) partials in the exchange slots [2][ranks][slot_B][H][D+1]
// (rows row0 .. row0 + B - 1), the same arithmetic as decode_combine, so the decode step needs
// no combine launch between the attention and the output projection.
struct GemvCombineArgs {
  const float* xslot;                  // local exchange slots (null: x is read)
  const unsigned long long* ready;     // local dec_ready[ranks]
  const unsigned long long* epoch_src; // epoch = (*epoch_src) * epoch_mul + epoch_add
  unsigned long long epoch_mul;
  unsigned long long epoch_add;
  int ranks, H, D, slot_B, row0;
  unsigned long long budget_ns;
  int* status;
};

struct GemvArgs {
  const __nv_bfloat16* x;  // [B, K]
  long ldx;
  const __nv_bfloat16* W;  // [N, K]
  int B, N, K;
  int epi;
  const __nv_bfloat16* bias;
  float* y_f32;
  __nv_bfloat16* y_bf16;
  long ldy;
  unsigned long long* argmax;  // [B] packed (value, index); caller zeroes it
  int index_base;              // kGemvArgmax: added to the row index (W is a vocabulary slice)
  int num_sms;
  const __nv_bfloat16* norm_w; // optional fused input RMSNorm weight [K]
  float eps;
  GemvRopeArgs rope;           // kGemvQkvRope only
  GemvCombineArgs cmb;         // kGemvResidual only (optional)
  L2Prefetch pf;               // optional
  int tc = -1;                 // tensor-core kernel: -1 by batch size (HCP_GEMV_TC, default B = 8), 0 never,
                               // 1 whenever the shape allows it
  int bulk = -1;               // bulk-copy streaming kernel where the tensor-core one is not used:
                               // -1 by HCP_GEMV_BULK, 0 never, 1 whenever the shape allows it
  int bulk_nst = 0;            // set by the launcher: ring stages of the streaming kernel
  int* status = nullptr;       // optional status word for the pipeline waits
};

struct DecodeAttnArgs {
  const __nv_bfloat16* q;      // [B, H, D]
  const __nv_bfloat16* arena;  // local paged KV arena
  ArenaGeom geom;
  int layer;
  const int* page_tables;      // [B, pt_stride]
  int pt_stride;
  const int* n_tokens;         // [B] local KV rows per request (incl. the appended token)
  int B, H, Hkv, D;
  float scale;
  int splits;
  float* part_o;               // [B, H, splits, D] scratch
  float* part_lse;             // [B, H, splits] scratch (log2 domain)
  unsigned int* split_counter; // [B * Hkv] zero-initialised
  unsigned int* grid_counter;  // [1] zero-initialised
  // exchange: every rank's slot array (P2P mapped), own rank index, flags
  float* const* xslot_ptrs;    // device array [n_ranks]
  int n_ranks;
  int my_rank;
  unsigned long long* const* ready_ptrs;  // device array [n_ranks]: &dec_ready[my_rank] on rank r
  __nv_bfloat16* final_out;    // single rank: the last CTA writes O [B, H*D] here (no exchange)
  // several ranks, in-kernel combine (combine_out set): the last CTA of each (row b, KV head h)
  // stores the rank's partial into every rank's slots, publishes group_flag[my_rank][b][h] =
  // epoch on every rank, waits (bounded) for every other rank's flag of the same group and
  // writes the log-sum-exp combine in rank order into combine_out [B, H*D] (no combine launch)
  __nv_bfloat16* combine_out;
  unsigned long long* const* group_flag_ptrs;  // [n_ranks]: rank r's group-flag base
  const unsigned long long* group_flags;       // local base [n_ranks][group_stride]
  int group_stride;                            // max_batch * Hkv
  unsigned long long budget_ns;
  const unsigned long long* epoch_parity_src;  // device step counter (may be null)
  unsigned long long epoch_mul;  // epoch = (*src) * mul + add
  unsigned long long epoch_add;
  int* status;
  L2Prefetch pf;               // optional
};

struct DecodeCombineArgs {
  const float* xslot;          // local exchange slots [2][N][B][H][D+1]
  const unsigned long long* ready;  // local dec_ready[N] (null: no wait, single rank)
  const unsigned long long* epoch_src;
  unsigned long long epoch_mul;
  unsigned long long epoch_add;
  int n_ranks, B, H, D;
  __nv_bfloat16* out;          // [B, H*D]
  unsigned long long budget_ns;
  int* status;
};

// Greedy argmax across the ranks of a vocabulary-split LM head: every rank holds the packed
// (value, index) maximum of its own vocabulary rows per decode row in `local` [B]. Each rank
// stores its entries into every rank's slots (value, then a release of the epoch), waits
// (bounded) for every rank's entries in its own slots and writes the largest one's index to
// tok32 / tok64 [B]. Ties between ranks go to the smaller index, as inside one GEMV, so the token
// is the full head's argmax.
struct ArgmaxXchgArgs {
  const unsigned long long* local;        // [B] this rank's packed maxima
  int B;                                  // <= 8
  unsigned long long* const* slot_ptrs;   // device array [world]: rank r's slot base
  const unsigned long long* own_slots;    // this rank's slot base: [2][world][max_batch][2]
  int world, my_rank, max_batch;
  const unsigned long long* epoch_src;    // device step counter; epoch = *epoch_src (>= 1)
  int* tok32;                             // optional [B]
  long long* tok64;                       // optional [B]
  unsigned long long budget_ns;
  int* status;
};

const char* gemv(const GemvArgs& a, cudaStream_t s);
// The argument checks of gemv() alone (nullptr when the launch would be accepted).
const char* gemv_check(const GemvArgs& a);

// The four decode GEMVs between two attention launches as one cooperative launch with grid
// barriers between them, in this order: residual (output projection, optionally with the
// cross-rank combine prologue), RMSNorm + SwiGLU (gate/up), residual (down projection), RMSNorm +
// QKV rope (the next layer) or RMSNorm + argmax (LM head). Same batch size (1, 2 or 4 rows) in
// every phase. `ctr` is a zeroed pair of 32-bit counters owned by this launch site (the launch
// leaves it zeroed again); `status` receives barrier timeouts.
constexpr int kGemvChainPhases = 4;
struct GemvChainArgs {
  GemvArgs ph[kGemvChainPhases];
  unsigned int* ctr = nullptr;
  int* status = nullptr;
};
bool gemv_chain_supported(const GemvArgs* ph, int n);
const char* gemv_chain(const GemvArgs* ph, int n, unsigned int* ctr, int* status, cudaStream_t s);
const char* argmax_exchange(const ArgmaxXchgArgs& a, cudaStream_t s);
const char* decode_attn(const DecodeAttnArgs& a, cudaStream_t s);
// Resident decode_attn CTAs per SM for (head_dim, GQA group size); 0 when unsupported. Callers
// size the split count so the grid fills the GPU in one wave.
int decode_attn_ctas_per_sm(int D, int G);
const char* decode_combine(const DecodeCombineArgs& a, cudaStream_t s);
const char* fill_u64(unsigned long long* p, int n, unsigned long long v, cudaStream_t s);
const char* argmax_finalize(const unsigned long long* packed, int B, int* tok, long long* tok64,
                            cudaStream_t s);
const char* add_u64(unsigned long long* p, unsigned long long v, cudaStream_t s);

}  // namespace dec
}  // namespace hcp
