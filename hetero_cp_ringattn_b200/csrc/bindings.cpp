// Python bindings of the sm_100a kernels and the domain runtime (torch extension `_C`).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "hcp/core/runtime.h"
#include "kernels/attn_fwd_sm100.h"
#include "kernels/decode.h"
#include "kernels/elementwise.h"
#include "kernels/gemm_sm100.h"

namespace {

using hcp::ArenaGeom;

#define HCP_CHECK_OK(err) TORCH_CHECK((err) == nullptr, "hcp kernel: ", (err))

// Decode page tables: int32 [B, pages per row] with contiguous rows (the kernels read row b at
// b * stride(0) and bound each row's KV length by stride(0) * page).
static void check_page_tables(const torch::Tensor& pt) {
  TORCH_CHECK(pt.is_cuda() && pt.scalar_type() == torch::kInt32, "page_tables must be a CUDA int32 tensor");
  TORCH_CHECK(pt.dim() == 2 && pt.stride(1) == 1 && pt.size(1) >= 1, "page_tables must be [B, pages] with contiguous rows");
}

void check_cuda_bf16(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, name, " must be bfloat16");
}

template <typename T>
T* ptr_or_null(const c10::optional<torch::Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

int sm_count(int dev) {
  static int cached[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// Up to two weight tensors a decode kernel prefetches into L2 for the kernels after it.
hcp::dec::L2Prefetch make_prefetch(const std::vector<torch::Tensor>& ts) {
  TORCH_CHECK(ts.size() <= 2, "at most two L2 prefetch ranges");
  hcp::dec::L2Prefetch pf{};
  static const int lines = [] {
    const char* e = getenv("HCP_DECODE_PREFETCH");
    return (e && atoi(e) >= 2) ? 1 : 0;
  }();
  pf.lines = lines;
  for (size_t i = 0; i < ts.size(); ++i) {
    TORCH_CHECK(ts[i].is_cuda() && ts[i].is_contiguous(), "prefetch ranges must be contiguous CUDA tensors");
    pf.ptr[i] = ts[i].data_ptr();
    pf.bytes[i] = uint64_t(ts[i].numel()) * ts[i].element_size();
  }
  return pf;
}

// ----------------------------------------------------------------------------- kernels
void gemm(torch::Tensor A, torch::Tensor B, torch::Tensor C, int64_t epi,
          c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> R,
          c10::optional<torch::Tensor> status, int64_t variant, int64_t group) {
  check_cuda_bf16(A, "A");
  check_cuda_bf16(B, "B");
  check_cuda_bf16(C, "C");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm expects 2-D tensors");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "inner dim must be contiguous");
  TORCH_CHECK(A.size(1) == B.size(1), "K mismatch");
  const c10::cuda::CUDAGuard g(A.device());
  hcp::gemm::GemmArgs a{};
  a.A = reinterpret_cast<const __nv_bfloat16*>(A.data_ptr());
  a.lda = A.stride(0);
  a.B = reinterpret_cast<const __nv_bfloat16*>(B.data_ptr());
  a.ldb = B.stride(0);
  a.C = reinterpret_cast<__nv_bfloat16*>(C.data_ptr());
  a.ldc = C.stride(0);
  a.M = int(A.size(0));
  a.N = int(B.size(0));
  a.K = int(A.size(1));
  a.epi = int(epi);
  a.bias = ptr_or_null<const __nv_bfloat16>(bias);
  if (R.has_value() && R->defined()) {
    check_cuda_bf16(*R, "R");
    a.R = reinterpret_cast<const __nv_bfloat16*>(R->data_ptr());
    a.ldr = R->stride(0);
  }
  const int64_t n_out = (epi == hcp::gemm::kEpiSwiGLU) ? a.N / 2 : a.N;
  TORCH_CHECK(C.size(0) == a.M && C.size(1) == n_out, "C has the wrong shape");
  a.status = ptr_or_null<int>(status);
  a.num_sms = sm_count(A.get_device());
  a.variant = int(variant);
  a.group = int(group);
  HCP_CHECK_OK(hcp::gemm::gemm_bf16(a, cur_stream()));
}

void attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o,
              c10::optional<torch::Tensor> lse, torch::Tensor q_pos, int64_t L,
              int64_t kv_head_stride, double scale, bool causal,
              c10::optional<torch::Tensor> status, int64_t variant, int64_t order) {
  check_cuda_bf16(q, "q");
  check_cuda_bf16(k, "k");
  check_cuda_bf16(v, "v");
  check_cuda_bf16(o, "o");
  TORCH_CHECK(q.dim() == 3 && q.is_contiguous(), "q must be [T, H, D] contiguous");
  TORCH_CHECK(o.sizes() == q.sizes() && o.is_contiguous(), "o must match q");
  TORCH_CHECK(q_pos.scalar_type() == torch::kInt32 && q_pos.is_cuda(), "q_pos must be int32 cuda");
  TORCH_CHECK(q_pos.numel() == q.size(0), "q_pos length");
  const int Hkv = int(k.size(0));
  TORCH_CHECK(k.size(k.dim() - 1) == q.size(2), "head dim mismatch");
  const c10::cuda::CUDAGuard g(q.device());
  hcp::attn::AttnArgs a{};
  a.Q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.K = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.V = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.O = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.lse = ptr_or_null<float>(lse);
  if (lse.has_value() && lse->defined()) {
    TORCH_CHECK(lse->scalar_type() == torch::kFloat32 && lse->numel() == q.size(0) * q.size(1),
                "lse must be fp32 [H, T]");
  }
  a.q_pos = q_pos.data_ptr<int>();
  a.T = int(q.size(0));
  a.H = int(q.size(1));
  a.Hkv = Hkv;
  a.D = int(q.size(2));
  a.L = int(L);
  a.kv_head_stride = kv_head_stride;
  TORCH_CHECK(kv_head_stride >= L * a.D, "kv_head_stride too small");
  a.scale = float(scale);
  a.causal = causal ? 1 : 0;
  a.status = ptr_or_null<int>(status);
  a.variant = int(variant);
  a.order = int(order);
  HCP_CHECK_OK(hcp::attn::attn_fwd(a, cur_stream()));
}

void embedding(torch::Tensor ids, torch::Tensor W, torch::Tensor out,
               c10::optional<torch::Tensor> status) {
  check_cuda_bf16(W, "W");
  check_cuda_bf16(out, "out");
  TORCH_CHECK(ids.scalar_type() == torch::kInt32 && ids.is_cuda(), "ids must be int32 cuda");
  const c10::cuda::CUDAGuard g(W.device());
  HCP_CHECK_OK(hcp::ew::embedding(ids.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(W.data_ptr()),
                                  reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), int(ids.numel()),
                                  int(W.size(1)), int(W.size(0)), ptr_or_null<int>(status), cur_stream()));
}

void rmsnorm(torch::Tensor x, torch::Tensor w, torch::Tensor y, double eps) {
  check_cuda_bf16(x, "x");
  check_cuda_bf16(w, "w");
  check_cuda_bf16(y, "y");
  TORCH_CHECK(x.stride(-1) == 1 && y.stride(-1) == 1, "rows must be contiguous");
  const c10::cuda::CUDAGuard g(x.device());
  const int hidden = int(x.size(-1));
  const int T = int(x.numel() / hidden);
  HCP_CHECK_OK(hcp::ew::rmsnorm(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                                reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                                reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), T, hidden,
                                x.dim() > 1 ? x.stride(-2) : hidden, y.dim() > 1 ? y.stride(-2) : hidden,
                                float(eps), cur_stream()));
}

// GEMV chain recording: between gemv_chain_begin() and gemv_chain_end() the decode GEMV entry
// points (gemv, qkv_gemv_rope, o_proj_combine) check their arguments and record them instead of
// launching; gemv_chain_end launches the recorded GEMVs as one chain kernel when they form its
// phase sequence, else one after the other. Per host thread (the thread that captures a decode
// graph records its own GEMVs).
thread_local bool g_chain_recording = false;
thread_local std::vector<hcp::dec::GemvArgs> g_chain_phases;

static void launch_gemv(const hcp::dec::GemvArgs& a) {
  if (g_chain_recording) {
    HCP_CHECK_OK(hcp::dec::gemv_check(a));
    g_chain_phases.push_back(a);
    return;
  }
  HCP_CHECK_OK(hcp::dec::gemv(a, cur_stream()));
}

// Starts a recording; one left open by an exception in the middle of a recorded region is
// discarded.
void gemv_chain_begin() {
  g_chain_phases.clear();
  g_chain_recording = true;
}

// Returns true when the recorded GEMVs ran as one chain launch. `ctr`: a zeroed int32 pair on
// the GEMVs' device, owned by this launch site.
bool gemv_chain_end(torch::Tensor ctr, c10::optional<torch::Tensor> status, bool chain) {
  TORCH_CHECK(g_chain_recording, "gemv_chain_end without gemv_chain_begin");
  g_chain_recording = false;
  std::vector<hcp::dec::GemvArgs> ph;
  ph.swap(g_chain_phases);
  const int n = int(ph.size());
  if (chain && hcp::dec::gemv_chain_supported(ph.data(), n)) {
    TORCH_CHECK(ctr.is_cuda() && ctr.scalar_type() == torch::kInt32 && ctr.numel() >= 2 && ctr.is_contiguous(),
                "gemv_chain_end: ctr must be a contiguous CUDA int32 tensor of 2 elements");
    const c10::cuda::CUDAGuard g(ctr.device());
    HCP_CHECK_OK(hcp::dec::gemv_chain(ph.data(), n, reinterpret_cast<unsigned int*>(ctr.data_ptr()),
                                      ptr_or_null<int>(status), cur_stream()));
    return true;
  }
  for (const auto& a : ph) HCP_CHECK_OK(hcp::dec::gemv(a, cur_stream()));
  return false;
}

void gemv(torch::Tensor x, torch::Tensor W, int64_t epi, c10::optional<torch::Tensor> bias,
          c10::optional<torch::Tensor> y_f32, c10::optional<torch::Tensor> y_bf16,
          c10::optional<torch::Tensor> argmax, c10::optional<torch::Tensor> norm_w, double eps,
          int64_t index_base, std::vector<torch::Tensor> prefetch, int64_t tc, int64_t bulk,
          c10::optional<torch::Tensor> status) {
  check_cuda_bf16(x, "x");
  check_cuda_bf16(W, "W");
  const c10::cuda::CUDAGuard g(x.device());
  hcp::dec::GemvArgs a{};
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.ldx = x.stride(0);
  a.W = reinterpret_cast<const __nv_bfloat16*>(W.data_ptr());
  a.B = int(x.size(0));
  a.N = int(W.size(0));
  a.K = int(W.size(1));
  TORCH_CHECK(x.size(1) == a.K, "gemv K mismatch");
  a.epi = int(epi);
  a.bias = ptr_or_null<const __nv_bfloat16>(bias);
  a.y_f32 = ptr_or_null<float>(y_f32);
  a.y_bf16 = ptr_or_null<__nv_bfloat16>(y_bf16);
  if (y_f32.has_value() && y_f32->defined()) a.ldy = y_f32->stride(0);
  else if (y_bf16.has_value() && y_bf16->defined()) a.ldy = y_bf16->stride(0);
  a.argmax = ptr_or_null<unsigned long long>(argmax);
  a.index_base = int(index_base);
  TORCH_CHECK(index_base >= 0 && index_base + a.N < (int64_t(1) << 31), "index_base out of range");
  a.pf = make_prefetch(prefetch);
  a.tc = int(tc);
  a.bulk = int(bulk);
  a.status = ptr_or_null<int>(status);
  a.num_sms = sm_count(x.get_device());
  a.norm_w = ptr_or_null<const __nv_bfloat16>(norm_w);
  a.eps = float(eps);
  if (a.norm_w) TORCH_CHECK(norm_w->numel() == a.K && norm_w->scalar_type() == torch::kBFloat16, "norm_w [K] bf16");
  if (epi == hcp::dec::kGemvArgmax) TORCH_CHECK(a.argmax != nullptr, "argmax buffer required");
  if (epi == hcp::dec::kGemvF32) TORCH_CHECK(a.y_f32 != nullptr, "y_f32 required");
  if (epi == hcp::dec::kGemvResidual || epi == hcp::dec::kGemvSwiGLU)
    TORCH_CHECK(a.y_bf16 != nullptr, "y_bf16 required");
  launch_gemv(a);
}

void fill_u64(torch::Tensor t, int64_t v) {
  TORCH_CHECK(t.is_cuda() && t.element_size() == 8, "fill_u64 needs a cuda 64-bit tensor");
  const c10::cuda::CUDAGuard g(t.device());
  HCP_CHECK_OK(hcp::dec::fill_u64(reinterpret_cast<unsigned long long*>(t.data_ptr()), int(t.numel()),
                                  static_cast<unsigned long long>(v), cur_stream()));
}

void argmax_finalize(torch::Tensor packed, c10::optional<torch::Tensor> tok32,
                     c10::optional<torch::Tensor> tok64) {
  const c10::cuda::CUDAGuard g(packed.device());
  HCP_CHECK_OK(hcp::dec::argmax_finalize(reinterpret_cast<const unsigned long long*>(packed.data_ptr()),
                                         int(packed.numel()), ptr_or_null<int>(tok32),
                                         ptr_or_null<long long>(tok64), cur_stream()));
}

void add_u64(torch::Tensor t, int64_t v) {
  const c10::cuda::CUDAGuard g(t.device());
  HCP_CHECK_OK(hcp::dec::add_u64(reinterpret_cast<unsigned long long*>(t.data_ptr()),
                                 static_cast<unsigned long long>(v), cur_stream()));
}

int64_t num_sms(int64_t dev) { return sm_count(int(dev)); }

int64_t decode_attn_ctas_per_sm(int64_t D, int64_t G) {
  return hcp::dec::decode_attn_ctas_per_sm(int(D), int(G));
}

// ----------------------------------------------------------------------------- runtime
// The overlapped ring's per-request plan (built on the host once per request): tile_src int64
// [ceil(L / 128)] bitmask of the ranks with rows in each KV tile, push_tiles int32 [n, 3] this
// rank's own tiles as (tile, first, end) row ranges of `pos`. No tile_src: the serial ring.
struct RingPlan {
  c10::optional<torch::Tensor> tile_src, push_tiles;
  RingPlan(c10::optional<torch::Tensor> t, c10::optional<torch::Tensor> p)
      : tile_src(std::move(t)), push_tiles(std::move(p)) {}
  void apply(hcp::RingLayerArgs& a, int world) const {
    if (!tile_src.has_value() || !tile_src->defined()) return;
    TORCH_CHECK(tile_src->is_cuda() && tile_src->scalar_type() == torch::kInt64 && tile_src->is_contiguous(),
                "tile_src must be a contiguous CUDA int64 tensor");
    TORCH_CHECK(tile_src->numel() >= (a.L + 127) / 128, "tile_src needs one word per KV tile");
    a.tile_src = reinterpret_cast<const unsigned long long*>(tile_src->data_ptr<int64_t>());
    if (push_tiles.has_value() && push_tiles->defined() && push_tiles->numel() > 0) {
      TORCH_CHECK(push_tiles->is_cuda() && push_tiles->scalar_type() == torch::kInt32 &&
                      push_tiles->is_contiguous() && push_tiles->dim() == 2 && push_tiles->size(1) == 3,
                  "push_tiles must be a contiguous CUDA int32 [n, 3] tensor");
      a.push_tiles = push_tiles->data_ptr<int>();
      a.n_push = int(push_tiles->size(0));
    }
    (void)world;
  }
};

class PyRuntime {
 public:
  PyRuntime(int64_t rank, int64_t world, int64_t device, int64_t layers, int64_t pages,
            int64_t page, int64_t hkv, int64_t d, int64_t num_heads, int64_t stage_cap,
            int64_t max_batch, int64_t wait_budget_ms) {
    hcp::RuntimeConfig c;
    c.rank = int(rank);
    c.world = int(world);
    c.device = int(device);
    c.geom = ArenaGeom{int(layers), int(pages), int(page), int(hkv), int(d)};
    c.num_heads = int(num_heads);
    c.stage_cap = int(stage_cap);
    c.max_batch = int(max_batch);
    c.num_sms = sm_count(int(device));
    c.peer_wait_budget_ns = uint64_t(wait_budget_ms) * 1000000ull;
    auto st = rt_.Init(c);
    TORCH_CHECK(st.ok(), "runtime init: ", st.ToString());
  }

  py::bytes export_handle() {
    auto h = rt_.ExportHandle();
    TORCH_CHECK(!h.empty(), "cudaIpcGetMemHandle failed");
    return py::bytes(reinterpret_cast<const char*>(h.data()), h.size());
  }

  void open_peers(const std::vector<py::bytes>& handles) {
    std::vector<std::vector<uint8_t>> hs;
    for (const auto& b : handles) {
      std::string s = b;
      hs.emplace_back(s.begin(), s.end());
    }
    auto st = rt_.OpenPeers(hs);
    TORCH_CHECK(st.ok(), "open_peers: ", st.ToString());
  }

  void open_peers_local(const std::vector<PyRuntime*>& peers) {
    std::vector<hcp::DomainRuntime*> ps;
    for (auto* p : peers) ps.push_back(&p->rt_);
    auto st = rt_.OpenPeersLocal(ps);
    TORCH_CHECK(st.ok(), "open_peers_local: ", st.ToString());
  }

  hcp::RingLayerArgs layer_args(torch::Tensor qkv, torch::Tensor pos, torch::Tensor cos_t,
                                torch::Tensor sin_t, int64_t layer,
                                c10::optional<torch::Tensor> page_table, int64_t slot_base,
                                int64_t L, double scale, bool causal,
                                torch::Tensor q_out, torch::Tensor o_out,
                                c10::optional<torch::Tensor> lse_out, int64_t epoch,
                                c10::optional<torch::Tensor> existing_slot_pos, bool has_qkv,
                                const RingPlan& ring) {
    check_cuda_bf16(qkv, "qkv");
    check_cuda_bf16(q_out, "q_out");
    check_cuda_bf16(o_out, "o_out");
    TORCH_CHECK(pos.scalar_type() == torch::kInt32, "pos must be int32");
    TORCH_CHECK(cos_t.scalar_type() == torch::kFloat32 && sin_t.scalar_type() == torch::kFloat32, "cos/sin fp32");
    const auto& c = rt_.config();
    hcp::RingLayerArgs a;
    a.qkv = qkv.data_ptr();
    a.ld_qkv = qkv.stride(0);
    a.pos = pos.data_ptr<int>();
    a.cos_t = cos_t.data_ptr<float>();
    a.sin_t = sin_t.data_ptr<float>();
    a.max_pos = int(cos_t.size(0));
    a.T = int(qkv.size(0));
    a.H = int(q_out.size(1));
    if (has_qkv) {
      TORCH_CHECK(qkv.size(1) >= (a.H + 2 * c.geom.hkv) * c.geom.d, "qkv too narrow");
    } else {
      a.qkv = nullptr;
    }
    a.layer = int(layer);
    if (page_table.has_value() && page_table->defined()) {
      TORCH_CHECK(page_table->scalar_type() == torch::kInt32, "page table int32");
      a.page_table = page_table->data_ptr<int>();
      a.slot_cap = int(page_table->numel()) * c.geom.page;
    }
    a.slot_base = int(slot_base);
    a.L = int(L);
      a.scale = float(scale);
    a.causal = causal ? 1 : 0;
    a.q_out = q_out.data_ptr();
    a.o_out = o_out.data_ptr();
    a.lse_out = ptr_or_null<float>(lse_out);
    a.epoch = uint64_t(epoch);
    if (existing_slot_pos.has_value() && existing_slot_pos->defined() && existing_slot_pos->numel() > 0) {
      TORCH_CHECK(existing_slot_pos->scalar_type() == torch::kInt32, "existing_slot_pos int32");
      TORCH_CHECK(a.page_table != nullptr, "existing rows need the page table");
      a.existing_slot_pos = existing_slot_pos->data_ptr<int>();
      a.existing_n = int(existing_slot_pos->numel());
    }
    ring.apply(a, c.world);
    return a;
  }

  void push_layer(torch::Tensor qkv, torch::Tensor pos, torch::Tensor cos_t, torch::Tensor sin_t,
                  int64_t layer, c10::optional<torch::Tensor> page_table, int64_t slot_base,
                  int64_t L, double scale, bool causal, torch::Tensor q_out,
                  torch::Tensor o_out, c10::optional<torch::Tensor> lse_out, int64_t epoch,
                  c10::optional<torch::Tensor> existing_slot_pos,
                  c10::optional<torch::Tensor> tile_src, c10::optional<torch::Tensor> push_tiles) {
    const c10::cuda::CUDAGuard g(qkv.device());
    auto a = layer_args(qkv, pos, cos_t, sin_t, layer, page_table, slot_base, L,
                        scale, causal, q_out, o_out, lse_out, epoch, existing_slot_pos, true,
                        RingPlan(tile_src, push_tiles));
    auto st = rt_.PushLayer(a, cur_stream());
    TORCH_CHECK(st.ok(), "push_layer: ", st.ToString());
  }

  // Fused projection + push: x [T, hidden] (normalised layer input), w_qkv [(H + 2 Hkv) D, hidden]
  // and optional bias; the projection output is never stored.
  void push_layer_fused(torch::Tensor x, torch::Tensor w_qkv, c10::optional<torch::Tensor> b_qkv,
                        torch::Tensor pos, torch::Tensor cos_t, torch::Tensor sin_t, int64_t layer,
                        c10::optional<torch::Tensor> page_table, int64_t slot_base, int64_t L,
                        double scale, bool causal, torch::Tensor q_out,
                        torch::Tensor o_out, c10::optional<torch::Tensor> lse_out, int64_t epoch,
                        c10::optional<torch::Tensor> existing_slot_pos,
                        c10::optional<torch::Tensor> tile_src, c10::optional<torch::Tensor> push_tiles) {
    check_cuda_bf16(x, "x");
    check_cuda_bf16(w_qkv, "w_qkv");
    TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && w_qkv.is_contiguous() && x.size(1) == w_qkv.size(1),
                "x [T, hidden] row-major and w_qkv [N, hidden] contiguous");
    const c10::cuda::CUDAGuard g(x.device());
    auto a = layer_args(x, pos, cos_t, sin_t, layer, page_table, slot_base, L, scale,
                        causal, q_out, o_out, lse_out, epoch, existing_slot_pos, /*has_qkv=*/false,
                        RingPlan(tile_src, push_tiles));
    a.x = x.data_ptr();
    a.ldx = x.stride(0);
    a.w_qkv = w_qkv.data_ptr();
    a.hidden = int(x.size(1));
    if (b_qkv.has_value() && b_qkv->defined()) {
      check_cuda_bf16(*b_qkv, "b_qkv");
      TORCH_CHECK(b_qkv->numel() == w_qkv.size(0), "b_qkv size");
      a.b_qkv = b_qkv->data_ptr();
    }
    TORCH_CHECK(w_qkv.size(0) == (a.H + 2 * rt_.config().geom.hkv) * rt_.config().geom.d, "w_qkv rows");
    auto st = rt_.PushLayer(a, cur_stream());
    TORCH_CHECK(st.ok(), "push_layer_fused: ", st.ToString());
  }

  void attend_layer(torch::Tensor qkv, torch::Tensor pos, torch::Tensor cos_t, torch::Tensor sin_t,
                    int64_t layer, c10::optional<torch::Tensor> page_table, int64_t slot_base,
                    int64_t L, double scale, bool causal,
                    torch::Tensor q_out, torch::Tensor o_out, c10::optional<torch::Tensor> lse_out,
                    int64_t epoch, c10::optional<torch::Tensor> existing_slot_pos,
                    c10::optional<torch::Tensor> tile_src, c10::optional<torch::Tensor> push_tiles) {
    // `qkv` only gives the row count here (the projection output or the layer input)
    const c10::cuda::CUDAGuard g(qkv.device());
    auto a = layer_args(qkv, pos, cos_t, sin_t, layer, page_table, slot_base, L,
                        scale, causal, q_out, o_out, lse_out, epoch, existing_slot_pos, false,
                        RingPlan(tile_src, push_tiles));
    auto st = rt_.AttendLayer(a, cur_stream());
    TORCH_CHECK(st.ok(), "attend_layer: ", st.ToString());
  }

  void publish_tiles(torch::Tensor push_tiles, int64_t epoch) {
    TORCH_CHECK(push_tiles.is_cuda() && push_tiles.scalar_type() == torch::kInt32 &&
                    push_tiles.is_contiguous() && push_tiles.dim() == 2 && push_tiles.size(1) == 3,
                "push_tiles must be a contiguous CUDA int32 [n, 3] tensor");
    const c10::cuda::CUDAGuard g(push_tiles.device());
    auto st = rt_.PublishTiles(push_tiles.data_ptr<int>(), int(push_tiles.size(0)), uint64_t(epoch),
                               cur_stream());
    TORCH_CHECK(st.ok(), "publish_tiles: ", st.ToString());
  }

  // Marks this rank's decode partials of rows [0, B) as present on every rank (group flags), for
  // partials already stored by a decode_attn launch without the in-kernel combine: tests that
  // emulate several ranks on one GPU, where no kernel may wait on another launch.
  void publish_decode_groups(int64_t B, int64_t epoch) {
    const auto& c = rt_.config();
    TORCH_CHECK(B >= 1 && B <= c.max_batch, "rows out of range");
    const c10::cuda::CUDAGuard g(c10::Device(c10::DeviceType::CUDA, c.device));
    HCP_CHECK_OK(hcp::ew::publish_range(rt_.group_flag_table(), c.world,
                                        long(c.rank) * c.max_batch * c.geom.hkv,
                                        int(B) * c.geom.hkv, uint64_t(epoch), cur_stream()));
  }

  void broadcast_token(torch::Tensor tok, int64_t src, int64_t epoch) {
    TORCH_CHECK(tok.is_cuda() && tok.scalar_type() == torch::kInt64 && tok.numel() >= 1,
                "tok must be a CUDA int64 tensor");
    const c10::cuda::CUDAGuard g(tok.device());
    auto st = rt_.BroadcastToken(reinterpret_cast<long long*>(tok.data_ptr<int64_t>()), int(src),
                                 uint64_t(epoch), cur_stream());
    TORCH_CHECK(st.ok(), "broadcast_token: ", st.ToString());
  }

  void argmax_exchange(torch::Tensor local, torch::Tensor epoch_src, c10::optional<torch::Tensor> tok32,
                       c10::optional<torch::Tensor> tok64) {
    TORCH_CHECK(local.is_cuda() && local.element_size() == 8 && local.is_contiguous(),
                "local must be a contiguous CUDA 64-bit tensor");
    TORCH_CHECK(epoch_src.is_cuda() && epoch_src.element_size() == 8, "epoch_src must be a CUDA 64-bit tensor");
    const int B = int(local.numel());
    if (tok32.has_value() && tok32->defined())
      TORCH_CHECK(tok32->is_cuda() && tok32->scalar_type() == torch::kInt32 && tok32->numel() >= B, "tok32 [B] int32");
    if (tok64.has_value() && tok64->defined())
      TORCH_CHECK(tok64->is_cuda() && tok64->scalar_type() == torch::kInt64 && tok64->numel() >= B, "tok64 [B] int64");
    const c10::cuda::CUDAGuard g(local.device());
    auto st = rt_.ArgmaxExchange(reinterpret_cast<const unsigned long long*>(local.data_ptr()), B,
                                 ptr_or_null<int>(tok32), ptr_or_null<long long>(tok64),
                                 reinterpret_cast<const unsigned long long*>(epoch_src.data_ptr()),
                                 cur_stream());
    TORCH_CHECK(st.ok(), "argmax_exchange: ", st.ToString());
  }

  void qkv_decode(torch::Tensor qkv_f32, torch::Tensor pos, torch::Tensor cos_t, torch::Tensor sin_t,
                  int64_t layer, torch::Tensor page_tables, torch::Tensor owner, torch::Tensor slot,
                  torch::Tensor q_out) {
    TORCH_CHECK(qkv_f32.scalar_type() == torch::kFloat32 && qkv_f32.is_contiguous(), "qkv must be fp32 contiguous");
    check_cuda_bf16(q_out, "q_out");
    TORCH_CHECK(owner.scalar_type() == torch::kInt32 && slot.scalar_type() == torch::kInt32, "owner/slot int32");
    TORCH_CHECK(owner.dim() == 2 && owner.is_contiguous() && slot.sizes() == owner.sizes(), "owner/slot [B, layers]");
    const c10::cuda::CUDAGuard g(qkv_f32.device());
    const auto& c = rt_.config();
    hcp::ew::QkvDecodeArgs a{};
    a.qkv = qkv_f32.data_ptr<float>();
    a.pos = pos.data_ptr<int>();
    a.cos_t = cos_t.data_ptr<float>();
    a.sin_t = sin_t.data_ptr<float>();
    a.max_pos = int(cos_t.size(0));
    a.B = int(qkv_f32.size(0));
    a.H = int(q_out.size(1));
    a.Hkv = c.geom.hkv;
    a.D = c.geom.d;
    TORCH_CHECK(qkv_f32.size(1) == (a.H + 2 * a.Hkv) * a.D, "qkv width");
    a.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
    a.arena = static_cast<__nv_bfloat16*>(rt_.arena());
    a.geom = c.geom;
    a.layer = int(layer);
    a.page_tables = page_tables.data_ptr<int>();
    check_page_tables(page_tables);
    a.pt_stride = int(page_tables.stride(0));
    a.slot_cap = int(page_tables.size(1)) * c.geom.page;
    a.owner = owner.data_ptr<int>();
    a.slot = slot.data_ptr<int>();
    a.owner_stride = int(owner.size(1));
    a.status = rt_.status();
    HCP_CHECK_OK(hcp::ew::qkv_decode(a, cur_stream()));
  }

  void decode_attn(torch::Tensor q, int64_t layer, torch::Tensor page_tables, torch::Tensor n_tokens,
                   double scale, int64_t splits, torch::Tensor part_o, torch::Tensor part_lse,
                   torch::Tensor counters, c10::optional<torch::Tensor> epoch_src,
                   int64_t epoch_mul, int64_t epoch_add, c10::optional<torch::Tensor> final_out,
                   c10::optional<torch::Tensor> combine_out, std::vector<torch::Tensor> prefetch) {
    check_cuda_bf16(q, "q");
    const c10::cuda::CUDAGuard g(q.device());
    const auto& c = rt_.config();
    hcp::dec::DecodeAttnArgs a{};
    a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
    a.arena = static_cast<const __nv_bfloat16*>(rt_.arena());
    a.geom = c.geom;
    a.layer = int(layer);
    a.page_tables = page_tables.data_ptr<int>();
    check_page_tables(page_tables);
    a.pt_stride = int(page_tables.stride(0));
    a.n_tokens = n_tokens.data_ptr<int>();
    a.B = int(q.size(0));
    a.H = int(q.size(1));
    a.Hkv = c.geom.hkv;
    a.D = c.geom.d;
    TORCH_CHECK(a.B <= c.max_batch, "decode batch larger than the runtime's max_batch");
    a.scale = float(scale);
    a.splits = int(splits);
    a.part_o = part_o.data_ptr<float>();
    a.part_lse = part_lse.data_ptr<float>();
    TORCH_CHECK(part_o.numel() >= int64_t(a.B) * a.H * a.splits * a.D, "part_o too small");
    TORCH_CHECK(part_lse.numel() >= int64_t(a.B) * a.H * a.splits, "part_lse too small");
    TORCH_CHECK(counters.numel() >= int64_t(a.B) * a.Hkv + 1 && counters.scalar_type() == torch::kInt32,
                "counters must be int32 [B*Hkv + 1]");
    a.split_counter = reinterpret_cast<unsigned int*>(counters.data_ptr());
    a.grid_counter = a.split_counter + a.B * a.Hkv;
    a.xslot_ptrs = rt_.xslot_table();
    a.n_ranks = c.world;
    a.my_rank = c.rank;
    a.ready_ptrs = rt_.dec_ready_table();
    a.epoch_parity_src = epoch_src.has_value() && epoch_src->defined()
                             ? reinterpret_cast<const unsigned long long*>(epoch_src->data_ptr())
                             : nullptr;
    a.epoch_mul = uint64_t(epoch_mul);
    a.epoch_add = uint64_t(epoch_add);
    a.status = rt_.status();
    if (final_out.has_value() && final_out->defined()) {
      check_cuda_bf16(*final_out, "final_out");
      TORCH_CHECK(c.world == 1, "final_out: the exchange is skipped only on a single rank");
      TORCH_CHECK(final_out->numel() >= int64_t(a.B) * a.H * a.D, "final_out too small");
      a.final_out = reinterpret_cast<__nv_bfloat16*>(final_out->data_ptr());
    }
    if (combine_out.has_value() && combine_out->defined()) {
      // several ranks: the exchange and the rank-order combine happen inside the kernel
      check_cuda_bf16(*combine_out, "combine_out");
      TORCH_CHECK(c.world > 1, "combine_out: the in-kernel combine is for several ranks");
      TORCH_CHECK(combine_out->numel() >= int64_t(a.B) * a.H * a.D, "combine_out too small");
      a.combine_out = reinterpret_cast<__nv_bfloat16*>(combine_out->data_ptr());
      a.group_flag_ptrs = rt_.group_flag_table();
      a.group_flags = rt_.group_flags();
      a.group_stride = c.max_batch * c.geom.hkv;
      a.budget_ns = c.peer_wait_budget_ns;
    }
    a.pf = make_prefetch(prefetch);
    HCP_CHECK_OK(hcp::dec::decode_attn(a, cur_stream()));
  }

  // Decode QKV projection with the RoPE + KV-append epilogue (replaces gemv f32 + qkv_decode).
  void qkv_gemv_rope(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> bias,
                     c10::optional<torch::Tensor> norm_w, double eps, torch::Tensor pos,
                     torch::Tensor cos_t, torch::Tensor sin_t, int64_t layer,
                     torch::Tensor page_tables, torch::Tensor owner, torch::Tensor slot,
                     torch::Tensor q_out, std::vector<torch::Tensor> prefetch, int64_t tc) {
    check_cuda_bf16(x, "x");
    check_cuda_bf16(w, "w");
    check_cuda_bf16(q_out, "q_out");
    TORCH_CHECK(owner.scalar_type() == torch::kInt32 && slot.scalar_type() == torch::kInt32, "owner/slot int32");
    TORCH_CHECK(owner.dim() == 2 && owner.is_contiguous() && slot.sizes() == owner.sizes(), "owner/slot [B, layers]");
    const c10::cuda::CUDAGuard g(x.device());
    const auto& c = rt_.config();
    hcp::dec::GemvArgs a{};
    a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
    a.ldx = x.stride(0);
    a.W = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
    a.B = int(x.size(0));
    a.N = int(w.size(0));
    a.K = int(w.size(1));
    TORCH_CHECK(x.size(1) == a.K, "qkv_gemv_rope K mismatch");
    a.epi = hcp::dec::kGemvQkvRope;
    a.bias = ptr_or_null<const __nv_bfloat16>(bias);
    a.num_sms = sm_count(x.get_device());
    a.norm_w = ptr_or_null<const __nv_bfloat16>(norm_w);
    a.eps = float(eps);
    auto& r = a.rope;
    r.pos = pos.data_ptr<int>();
    r.cos_t = cos_t.data_ptr<float>();
    r.sin_t = sin_t.data_ptr<float>();
    r.max_pos = int(cos_t.size(0));
    r.H = int(q_out.size(1));
    r.Hkv = c.geom.hkv;
    r.D = c.geom.d;
    r.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
    r.arena = static_cast<__nv_bfloat16*>(rt_.arena());
    r.geom = c.geom;
    r.layer = int(layer);
    r.page_tables = page_tables.data_ptr<int>();
    check_page_tables(page_tables);
    r.pt_stride = int(page_tables.stride(0));
    r.slot_cap = int(page_tables.size(1)) * c.geom.page;
    r.owner = owner.data_ptr<int>();
    r.slot = slot.data_ptr<int>();
    r.owner_stride = int(owner.size(1));
    r.status = rt_.status();
    a.pf = make_prefetch(prefetch);
    a.tc = int(tc);
    launch_gemv(a);
  }

  // Output projection of a decode step on several ranks with the cross-rank combine in its
  // prologue: y += bf16(combine(partials) W^T), where the combine waits for every rank's
  // dec_ready flag at epoch = (*epoch_src) * epoch_mul + epoch_add and merges the (O, LSE)
  // partials of the exchange slots in rank order (x only gives the shape [B, H * D]).
  void o_proj_combine(torch::Tensor x, torch::Tensor w, torch::Tensor y, torch::Tensor epoch_src,
                      int64_t epoch_mul, int64_t epoch_add) {
    check_cuda_bf16(x, "x");
    check_cuda_bf16(w, "w");
    check_cuda_bf16(y, "y");
    TORCH_CHECK(epoch_src.is_cuda() && epoch_src.element_size() == 8, "epoch_src must be a CUDA 64-bit tensor");
    const c10::cuda::CUDAGuard g(x.device());
    const auto& c = rt_.config();
    hcp::dec::GemvArgs a{};
    a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
    a.ldx = x.stride(0);
    a.W = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
    a.B = int(x.size(0));
    a.N = int(w.size(0));
    a.K = int(w.size(1));
    TORCH_CHECK(x.size(1) == a.K && y.size(0) == a.B && y.size(1) == a.N, "o_proj_combine shapes");
    TORCH_CHECK(a.B <= c.max_batch, "o_proj_combine: rows exceed max_batch");
    a.epi = hcp::dec::kGemvResidual;
    a.y_bf16 = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
    a.ldy = y.stride(0);
    a.num_sms = sm_count(x.get_device());
    auto& m = a.cmb;
    m.xslot = rt_.xslot();
    m.ready = rt_.flags() + hcp::kFlagDecReady;
    m.epoch_src = reinterpret_cast<const unsigned long long*>(epoch_src.data_ptr());
    m.epoch_mul = uint64_t(epoch_mul);
    m.epoch_add = uint64_t(epoch_add);
    m.ranks = c.world;
    m.H = c.num_heads;
    m.D = c.geom.d;
    m.slot_B = a.B;
    m.row0 = 0;
    m.budget_ns = c.peer_wait_budget_ns;
    m.status = rt_.status();
    launch_gemv(a);
  }

  void decode_combine(torch::Tensor out, int64_t B, int64_t H, c10::optional<torch::Tensor> epoch_src,
                      int64_t epoch_mul, int64_t epoch_add) {
    check_cuda_bf16(out, "out");
    const c10::cuda::CUDAGuard g(out.device());
    const auto& c = rt_.config();
    hcp::dec::DecodeCombineArgs a{};
    a.xslot = rt_.xslot();
    a.ready = c.world > 1 ? rt_.flags() + hcp::kFlagDecReady : nullptr;
    a.epoch_src = epoch_src.has_value() && epoch_src->defined()
                      ? reinterpret_cast<const unsigned long long*>(epoch_src->data_ptr())
                      : nullptr;
    a.epoch_mul = uint64_t(epoch_mul);
    a.epoch_add = uint64_t(epoch_add);
    a.n_ranks = c.world;
    a.B = int(B);
    a.H = int(H);
    a.D = c.geom.d;
    a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
    a.budget_ns = c.peer_wait_budget_ns;
    a.status = rt_.status();
    HCP_CHECK_OK(hcp::dec::decode_combine(a, cur_stream()));
  }

  // Bounded device-side wait until flags[first + r] >= target for r < n (the same kernel the ring
  // uses for peer flags). Used by tests to exercise the timeout path on a flag nothing sets.
  void wait_flags(int64_t first, int64_t n, int64_t target, int64_t budget_ms) {
    const auto& c = rt_.config();
    TORCH_CHECK(first >= 0 && n > 0 && first + n <= hcp::kFlagWords && n <= 32, "flag range");
    const c10::cuda::CUDAGuard g(c10::Device(c10::DeviceType::CUDA, c.device));
    HCP_CHECK_OK(hcp::ew::wait_consumed(rt_.flags() + first, int(n), uint64_t(target),
                                        uint64_t(budget_ms) * 1000000ull, rt_.status(), cur_stream()));
  }

  torch::Tensor arena() {
    const auto& c = rt_.config();
    auto opts = torch::TensorOptions().dtype(torch::kBFloat16).device(torch::kCUDA, c.device);
    return torch::from_blob(rt_.arena(), {c.geom.layers, c.geom.pages, 2, c.geom.hkv, c.geom.page, c.geom.d}, opts);
  }
  torch::Tensor stage(int64_t parity) {
    const auto& c = rt_.config();
    auto opts = torch::TensorOptions().dtype(torch::kBFloat16).device(torch::kCUDA, c.device);
    return torch::from_blob(rt_.stage(int(parity)), {2, c.geom.hkv, c.stage_cap, c.geom.d}, opts);
  }
  torch::Tensor flags() {
    const auto& c = rt_.config();
    auto opts = torch::TensorOptions().dtype(torch::kInt64).device(torch::kCUDA, c.device);
    return torch::from_blob(rt_.flags(), {hcp::kFlagWords}, opts);
  }
  // The greedy-argmax exchange slots [2 parity][world source][max_batch][value, epoch].
  torch::Tensor argmax_slots() {
    const auto& c = rt_.config();
    auto opts = torch::TensorOptions().dtype(torch::kInt64).device(torch::kCUDA, c.device);
    return torch::from_blob(rt_.argmax_slots(), {2, c.world, c.max_batch, 2}, opts);
  }
  torch::Tensor status_words() {
    const auto& c = rt_.config();
    auto opts = torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, c.device);
    return torch::from_blob(rt_.status(), {hcp::kStatusWords}, opts);
  }
  void check() {
    auto st = rt_.CheckDevice(cur_stream());
    TORCH_CHECK(st.ok(), "device status: ", st.ToString());
  }
  void shutdown() { rt_.Shutdown(); }
  int64_t region_bytes() { return int64_t(rt_.region_bytes()); }
  int64_t rank() { return rt_.config().rank; }
  int64_t world() { return rt_.config().world; }

 private:
  hcp::DomainRuntime rt_;
};

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "hetero_cp_ringattn_b200 sm_100a kernels and domain runtime";
  m.def("gemm", &gemm, "tcgen05 GEMM with fused epilogue", py::arg("A"), py::arg("B"), py::arg("C"),
        py::arg("epi") = 0, py::arg("bias") = py::none(), py::arg("R") = py::none(),
        py::arg("status") = py::none(), py::arg("variant") = 0, py::arg("group") = -1);
  m.def("attn_fwd", &attn_fwd, "tcgen05 flash attention with LSE and position-causal skip",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"), py::arg("q_pos"),
        py::arg("L"), py::arg("kv_head_stride"), py::arg("scale"), py::arg("causal"),
        py::arg("status") = py::none(), py::arg("variant") = 0, py::arg("order") = -1);
  m.def("embedding", &embedding, py::arg("ids"), py::arg("W"), py::arg("out"), py::arg("status") = py::none());
  m.def("rmsnorm", &rmsnorm);
  m.def("gemv", &gemv, py::arg("x"), py::arg("W"), py::arg("epi"), py::arg("bias") = py::none(),
        py::arg("y_f32") = py::none(), py::arg("y_bf16") = py::none(), py::arg("argmax") = py::none(),
        py::arg("norm_w") = py::none(), py::arg("eps") = 1e-6, py::arg("index_base") = 0,
        py::arg("prefetch") = std::vector<torch::Tensor>{}, py::arg("tc") = -1, py::arg("bulk") = -1,
        py::arg("status") = py::none());
  m.def("gemv_chain_begin", &gemv_chain_begin);
  m.def("gemv_chain_end", &gemv_chain_end, py::arg("ctr"), py::arg("status") = py::none(),
        py::arg("chain") = true);
  m.def("fill_u64", &fill_u64);
  m.def("argmax_finalize", &argmax_finalize, py::arg("packed"), py::arg("tok32") = py::none(),
        py::arg("tok64") = py::none());
  m.def("add_u64", &add_u64);
  m.def("num_sms", &num_sms);
  m.def("decode_attn_ctas_per_sm", &decode_attn_ctas_per_sm);
  m.attr("EPI_STORE") = int(hcp::gemm::kEpiStore);
  m.attr("EPI_BIAS") = int(hcp::gemm::kEpiBias);
  m.attr("EPI_RESIDUAL") = int(hcp::gemm::kEpiResidual);
  m.attr("EPI_SWIGLU") = int(hcp::gemm::kEpiSwiGLU);
  m.attr("GEMV_F32") = int(hcp::dec::kGemvF32);
  m.attr("GEMV_RESIDUAL") = int(hcp::dec::kGemvResidual);
  m.attr("GEMV_SWIGLU") = int(hcp::dec::kGemvSwiGLU);
  m.attr("GEMV_ARGMAX") = int(hcp::dec::kGemvArgmax);
  m.attr("FLAG_WORDS") = int(hcp::kFlagWords);
  py::class_<PyRuntime>(m, "Runtime")
      .def(py::init<int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                    int64_t, int64_t, int64_t, int64_t>(),
           py::arg("rank"), py::arg("world"), py::arg("device"), py::arg("layers"), py::arg("pages"),
           py::arg("page"), py::arg("hkv"), py::arg("d"), py::arg("num_heads"),
           py::arg("stage_cap"), py::arg("max_batch"), py::arg("wait_budget_ms"))
      .def("export_handle", &PyRuntime::export_handle)
      .def("open_peers", &PyRuntime::open_peers)
      .def("open_peers_local", &PyRuntime::open_peers_local)
      .def("push_layer", &PyRuntime::push_layer, py::arg("qkv"), py::arg("pos"), py::arg("cos_t"),
           py::arg("sin_t"), py::arg("layer"), py::arg("page_table"), py::arg("slot_base"), py::arg("L"),
           py::arg("scale"), py::arg("causal"), py::arg("q_out"),
           py::arg("o_out"), py::arg("lse_out"), py::arg("epoch"),
           py::arg("existing_slot_pos") = py::none(), py::arg("tile_src") = py::none(), py::arg("push_tiles") = py::none())
      .def("push_layer_fused", &PyRuntime::push_layer_fused, py::arg("x"), py::arg("w_qkv"),
           py::arg("b_qkv"), py::arg("pos"), py::arg("cos_t"), py::arg("sin_t"), py::arg("layer"),
           py::arg("page_table"), py::arg("slot_base"), py::arg("L"),
           py::arg("scale"), py::arg("causal"), py::arg("q_out"), py::arg("o_out"),
           py::arg("lse_out"), py::arg("epoch"),
           py::arg("existing_slot_pos") = py::none(), py::arg("tile_src") = py::none(), py::arg("push_tiles") = py::none())
      .def("attend_layer", &PyRuntime::attend_layer, py::arg("qkv"), py::arg("pos"), py::arg("cos_t"),
           py::arg("sin_t"), py::arg("layer"), py::arg("page_table"), py::arg("slot_base"), py::arg("L"),
           py::arg("scale"), py::arg("causal"), py::arg("q_out"),
           py::arg("o_out"), py::arg("lse_out"), py::arg("epoch"),
           py::arg("existing_slot_pos") = py::none(), py::arg("tile_src") = py::none(), py::arg("push_tiles") = py::none())
      .def("publish_tiles", &PyRuntime::publish_tiles, py::arg("push_tiles"), py::arg("epoch"))
      .def("broadcast_token", &PyRuntime::broadcast_token, py::arg("tok"), py::arg("src"), py::arg("epoch"))
      .def("argmax_exchange", &PyRuntime::argmax_exchange, py::arg("local"), py::arg("epoch_src"),
           py::arg("tok32") = py::none(), py::arg("tok64") = py::none())
      .def("publish_decode_groups", &PyRuntime::publish_decode_groups, py::arg("B"), py::arg("epoch"))
      .def("qkv_decode", &PyRuntime::qkv_decode)
      .def("decode_attn", &PyRuntime::decode_attn, py::arg("q"), py::arg("layer"), py::arg("page_tables"),
           py::arg("n_tokens"), py::arg("scale"), py::arg("splits"), py::arg("part_o"),
           py::arg("part_lse"), py::arg("counters"), py::arg("epoch_src"), py::arg("epoch_mul"),
           py::arg("epoch_add"), py::arg("final_out") = py::none(), py::arg("combine_out") = py::none(),
           py::arg("prefetch") = std::vector<torch::Tensor>{})
      .def("qkv_gemv_rope", &PyRuntime::qkv_gemv_rope, py::arg("x"), py::arg("w"), py::arg("bias"),
           py::arg("norm_w"), py::arg("eps"), py::arg("pos"), py::arg("cos_t"), py::arg("sin_t"),
           py::arg("layer"), py::arg("page_tables"), py::arg("owner"), py::arg("slot"),
           py::arg("q_out"), py::arg("prefetch") = std::vector<torch::Tensor>{}, py::arg("tc") = -1)
      .def("decode_combine", &PyRuntime::decode_combine)
      .def("o_proj_combine", &PyRuntime::o_proj_combine, py::arg("x"), py::arg("w"), py::arg("y"),
           py::arg("epoch_src"), py::arg("epoch_mul"), py::arg("epoch_add"))
      .def("wait_flags", &PyRuntime::wait_flags)
      .def("arena", &PyRuntime::arena)
      .def("stage", &PyRuntime::stage)
      .def("flags", &PyRuntime::flags)
      .def("argmax_slots", &PyRuntime::argmax_slots)
      .def("status_words", &PyRuntime::status_words)
      .def("check", &PyRuntime::check)
      .def("shutdown", &PyRuntime::shutdown)
      .def("region_bytes", &PyRuntime::region_bytes)
      .def("rank", &PyRuntime::rank)
      .def("world", &PyRuntime::world);
}
