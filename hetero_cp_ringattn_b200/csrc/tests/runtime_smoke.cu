// Native coordinator smoke: the domain runtime driven from C++ alone (no Python, no torch).
//
// Parity: src/ringattn_coordinator_smoke_main.cc:6-56 of the reference (3-domain config with
// chunks 512/256/256 and blocks 128/64/64; Init -> Run -> Shutdown per domain). Here the three
// domains are emulated on one GPU (every domain's push runs before any domain's attend, so no
// launch waits on a later one), each runs one real ring-attention layer through the runtime, and
// every domain's rotated Q rows and attention output are compared with a double-precision CPU
// oracle (rotate-half RoPE on the bf16 inputs, then causal GQA softmax attention over all 1024
// positions), the check the reference's ATen bridge makes in src/rust_bridge.cc:614-928.
// Without a GPU only the config checks run.
//
//   hcp_runtime_smoke            exit 0 on success
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <algorithm>
#include <cstdio>
#include <vector>

#include "hcp/core/runtime.h"
#include "hcp/core/types.h"

using namespace hcp;

static int fail(const char* what, const Status& s) {
  std::fprintf(stderr, "[smoke] %s: %s\n", what, s.ToString().c_str());
  return 1;
}

int main() {
  RingAttnConfig cfg;
  cfg.global_seq_len = 1024;
  cfg.num_heads = 8;
  cfg.num_kv_heads = 2;
  cfg.head_dim = 64;
  cfg.domains = {{"cuda-domain-0", "127.0.0.1", 26001, 512, 128, "cuda:0"},
                 {"cuda-domain-1", "127.0.0.1", 26002, 256, 64, "cuda:0"},
                 {"cuda-domain-2", "127.0.0.1", 26003, 256, 64, "cuda:0"}};
  Status st = cfg.Validate();
  if (!st.ok()) return fail("config", st);
  RingAttnConfig bad = cfg;
  bad.domains[1].seq_chunk_len = 255;
  if (bad.Validate().ok()) {
    std::fprintf(stderr, "[smoke] chunk-sum mismatch was not rejected\n");
    return 1;
  }
  std::printf("[smoke] config ok: %zu domains, global_seq_len=%lld\n", cfg.domains.size(),
              (long long)cfg.global_seq_len);

  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    std::printf("[smoke] no GPU: config checks only\n");
    return 0;
  }
  const int N = int(cfg.domains.size()), H = int(cfg.num_heads), HKV = int(cfg.num_kv_heads),
            D = int(cfg.head_dim), L = int(cfg.global_seq_len);
  std::vector<DomainRuntime> rts(N);
  std::vector<DomainRuntime*> ptrs;
  for (int r = 0; r < N; ++r) {
    RuntimeConfig rc;
    rc.rank = r;
    rc.world = N;
    rc.device = 0;
    rc.geom = ArenaGeom{1, 8, 256, HKV, D};
    rc.num_heads = H;
    rc.stage_cap = L;
    rc.max_batch = 1;
    rc.peer_wait_budget_ns = 2000000000ull;
    if (!(st = rts[r].Init(rc)).ok()) return fail("Init", st);
    ptrs.push_back(&rts[r]);
  }
  for (int r = 0; r < N; ++r)
    if (!(st = rts[r].OpenPeersLocal(ptrs)).ok()) return fail("OpenPeersLocal", st);

  // per-domain inputs: qkv rows (deterministic values), positions, RoPE tables, page tables
  const int half = D / 2, width = (H + 2 * HKV) * D;
  std::vector<float> hcos(size_t(L) * half), hsin(size_t(L) * half);
  for (int p = 0; p < L; ++p)
    for (int j = 0; j < half; ++j) {
      const double f = p / std::pow(10000.0, 2.0 * j / D);
      hcos[size_t(p) * half + j] = float(std::cos(f));
      hsin[size_t(p) * half + j] = float(std::sin(f));
    }
  float *dcos, *dsin;
  cudaMalloc(&dcos, hcos.size() * 4);
  cudaMalloc(&dsin, hsin.size() * 4);
  cudaMemcpy(dcos, hcos.data(), hcos.size() * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dsin, hsin.data(), hsin.size() * 4, cudaMemcpyHostToDevice);
  std::vector<RingLayerArgs> args(N);
  std::vector<void*> bufs;
  // host copy of every position's rotated q and k (bf16-rounded, as the kernel stores them) and v
  std::vector<float> rq(size_t(L) * H * D), rk(size_t(L) * HKV * D), rv(size_t(L) * HKV * D);
  auto rope_row = [&](const __nv_bfloat16* x, int p, float* out) {
    for (int j = 0; j < half; ++j) {
      const double a = __bfloat162float(x[j]), b = __bfloat162float(x[j + half]);
      const double c = hcos[size_t(p) * half + j], sn = hsin[size_t(p) * half + j];
      out[j] = __bfloat162float(__float2bfloat16(float(a * c - b * sn)));
      out[j + half] = __bfloat162float(__float2bfloat16(float(b * c + a * sn)));
    }
  };
  int offset = 0;
  for (int r = 0; r < N; ++r) {
    const int T = int(cfg.domains[r].seq_chunk_len);
    std::vector<__nv_bfloat16> hq(size_t(T) * width);
    for (size_t i = 0; i < hq.size(); ++i) hq[i] = __float2bfloat16(float(std::sin(0.37 * double(i + offset * width))) * 0.5f);
    for (int t = 0; t < T; ++t) {
      const int p = offset + t;
      const __nv_bfloat16* row = hq.data() + size_t(t) * width;
      for (int h = 0; h < H; ++h) rope_row(row + h * D, p, rq.data() + (size_t(p) * H + h) * D);
      for (int h = 0; h < HKV; ++h) {
        rope_row(row + (H + h) * D, p, rk.data() + (size_t(p) * HKV + h) * D);
        for (int d = 0; d < D; ++d)
          rv[(size_t(p) * HKV + h) * D + d] = __bfloat162float(row[(H + HKV + h) * D + d]);
      }
    }
    std::vector<int> hpos(T), hpt(4);
    for (int t = 0; t < T; ++t) hpos[t] = offset + t;
    for (int i = 0; i < 4; ++i) hpt[i] = r * 2 + (i % 2);  // 2 pages (512 slots) per domain
    void *qkv, *pos, *pt, *qo, *oo;
    cudaMalloc(&qkv, hq.size() * 2);
    cudaMalloc(&pos, T * 4);
    cudaMalloc(&pt, 2 * 4);
    cudaMalloc(&qo, size_t(T) * H * D * 2);
    cudaMalloc(&oo, size_t(T) * H * D * 2);
    cudaMemcpy(qkv, hq.data(), hq.size() * 2, cudaMemcpyHostToDevice);
    cudaMemcpy(pos, hpos.data(), T * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(pt, hpt.data(), 2 * 4, cudaMemcpyHostToDevice);
    bufs.insert(bufs.end(), {qkv, pos, pt, qo, oo});
    RingLayerArgs& a = args[r];
    a.qkv = qkv;
    a.ld_qkv = width;
    a.pos = static_cast<int*>(pos);
    a.cos_t = dcos;
    a.sin_t = dsin;
    a.max_pos = L;
    a.T = T;
    a.H = H;
    a.layer = 0;
    a.page_table = static_cast<int*>(pt);
    a.slot_base = 0;
    a.slot_cap = 2 * 256;
    a.L = L;
    a.scale = 1.f / std::sqrt(float(D));
    a.causal = 1;
    a.q_out = qo;
    a.o_out = oo;
    a.epoch = 1;
    offset += T;
  }
  for (int r = 0; r < N; ++r)
    if (!(st = rts[r].PushLayer(args[r], 0)).ok()) return fail("PushLayer", st);
  for (int r = 0; r < N; ++r)
    if (!(st = rts[r].AttendLayer(args[r], 0)).ok()) return fail("AttendLayer", st);
  for (int r = 0; r < N; ++r)
    if (!(st = rts[r].CheckDevice(0)).ok()) return fail("CheckDevice", st);
  const double scale = 1.0 / std::sqrt(double(D));
  std::vector<double> sc(L), acc(D);
  offset = 0;
  for (int r = 0; r < N; ++r) {
    const int T = args[r].T;
    std::vector<__nv_bfloat16> ho(size_t(T) * H * D), hqo(size_t(T) * H * D);
    cudaMemcpy(ho.data(), args[r].o_out, ho.size() * 2, cudaMemcpyDeviceToHost);
    cudaMemcpy(hqo.data(), args[r].q_out, hqo.size() * 2, cudaMemcpyDeviceToHost);
    double q_err = 0, o_err = 0, s = 0;
    for (int t = 0; t < T; ++t) {
      const int p = offset + t;
      for (int h = 0; h < H; ++h) {
        const float* q = rq.data() + (size_t(p) * H + h) * D;
        const int g = h / (H / HKV);
        double m = -1e300, l = 0;
        for (int j = 0; j <= p; ++j) {
          const float* k = rk.data() + (size_t(j) * HKV + g) * D;
          double dot = 0;
          for (int d = 0; d < D; ++d) dot += double(q[d]) * k[d];
          sc[j] = dot * scale;
          m = std::max(m, sc[j]);
        }
        std::fill(acc.begin(), acc.end(), 0.0);
        for (int j = 0; j <= p; ++j) {
          const double e = std::exp(sc[j] - m);
          l += e;
          const float* v = rv.data() + (size_t(j) * HKV + g) * D;
          for (int d = 0; d < D; ++d) acc[d] += e * v[d];
        }
        for (int d = 0; d < D; ++d) {
          const size_t i = (size_t(t) * H + h) * D + d;
          const float f = __bfloat162float(ho[i]);
          if (!std::isfinite(f)) {
            std::fprintf(stderr, "[smoke] domain %d produced a non-finite output\n", r);
            return 1;
          }
          o_err = std::max(o_err, std::fabs(double(f) - acc[d] / l));
          q_err = std::max(q_err, std::fabs(double(__bfloat162float(hqo[i])) - q[d]));
          s += std::fabs(f);
        }
      }
    }
    std::printf("[smoke] domain %d: %d rows, mean |o| = %.4f, max |q - oracle| = %.2e, "
                "max |o - oracle| = %.2e\n", r, T, s / double(ho.size()), q_err, o_err);
    if (q_err > 1e-2 || o_err > 2e-2) {
      std::fprintf(stderr, "[smoke] domain %d differs from the CPU oracle\n", r);
      return 1;
    }
    offset += T;
  }
  for (void* b : bufs) cudaFree(b);
  cudaFree(dcos);
  cudaFree(dsin);
  for (int r = 0; r < N; ++r)
    if (!(st = rts[r].Shutdown()).ok()) return fail("Shutdown", st);
  std::printf("[smoke] ok\n");
  return 0;
}
