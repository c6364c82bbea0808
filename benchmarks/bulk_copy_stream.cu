// DRAM streaming rate of untiled bulk copies (cp.async.bulk, global -> shared) against plain
// 16-byte register loads: the measurement behind the stage shape of the streaming decode GEMV.
// Each CTA streams its own contiguous slice of a 1 GiB buffer through a ring of `nst` stages of
// `stage` bytes, each stage moved by `copies` equal bulk copies completing on the stage's
// mbarrier; thread 0 issues, warp 0 waits (bounded) and re-issues, nothing is computed. The L2
// is flushed (256 MB write) before each timed launch; the best of 4 timed launches is printed.
// The tiled variant moves the same bytes as 2D tensor-map boxes (128-byte swizzled rows of 64
// bf16, `rows` rows per box, the decode attention's K/V tile shape at 64 rows), `boxes` per
// stage.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 \
//        -o /tmp/bulk_copy_stream benchmarks/bulk_copy_stream.cu && /tmp/bulk_copy_stream
#include <cstdio>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

__device__ __forceinline__ uint32_t sa(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t gt() { uint64_t t; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)); return t; }

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t par, int* err) {
  uint32_t a = sa(bar);
  uint64_t t0 = gt();
  while (true) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0,1,0,p;\n\t}"
                 : "=r"(ok) : "r"(a), "r"(par) : "memory");
    if (ok) return true;
    if (gt() - t0 > 2000000000ull) { atomicExch(err, 1); return false; }
  }
}

__global__ void __launch_bounds__(128) stream_kernel(const uint8_t* src, size_t per_cta, int nst, int stg, int cps,
                                                     int* err, unsigned long long* sink) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ __align__(8) uint64_t full[16];
  const uint8_t* base = src + per_cta * blockIdx.x;
  const int nstage = int(per_cta / stg);
  if (threadIdx.x == 0) {
    for (int i = 0; i < nst; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(&full[i])), "r"(1));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x >= 32) return;
  auto issue = [&](int s) {
    const int slot = s % nst;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(&full[slot])), "r"(stg) : "memory");
    const int part = stg / cps;
    for (int c = 0; c < cps; ++c)
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       sa(sm + (size_t)slot * stg + c * part)),
                   "l"(base + (size_t)s * stg + c * part), "r"(part), "r"(sa(&full[slot]))
                   : "memory");
  };
  if (threadIdx.x == 0)
    for (int s = 0; s < nst && s < nstage; ++s) issue(s);
  unsigned long long acc = 0;
  int s = 0, issued = nst < nstage ? nst : nstage;
  for (; s < nstage; ++s) {
    const int slot = s % nst;
    if (!wait_bar(&full[slot], (s / nst) & 1, err)) break;
    acc += sm[(size_t)slot * stg + threadIdx.x * 4];
    __syncwarp();
    if (threadIdx.x == 0 && s + nst < nstage) { issue(s + nst); issued = s + nst + 1; }
  }
  if (s < nstage && threadIdx.x == 0)   // drain what is still in flight (bounded)
    for (int t = s + 1; t < issued; ++t)
      if (!wait_bar(&full[t % nst], (t / nst) & 1, err)) break;
  if (threadIdx.x == 0) atomicAdd(sink, acc);
}

__global__ void __launch_bounds__(128) stream_tiled_kernel(const __grid_constant__ CUtensorMap map, int rows_per_cta,
                                                           int nst, int rows, int boxes, int* err,
                                                           unsigned long long* sink) {
  extern __shared__ __align__(1024) uint8_t smt[];
  __shared__ __align__(8) uint64_t full[16];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smt) + 1023) & ~uintptr_t(1023));
  const int stage_rows = rows * boxes;
  const int stg = stage_rows * 128;
  const int nstage = rows_per_cta / stage_rows;
  const int row0 = blockIdx.x * rows_per_cta;
  if (threadIdx.x == 0) {
    for (int i = 0; i < nst; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(&full[i])), "r"(1));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x >= 32) return;
  auto issue = [&](int s) {
    const int slot = s % nst;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(&full[slot])), "r"(stg) : "memory");
    for (int b = 0; b < boxes; ++b)
      asm volatile(
          "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
              sa(sm + (size_t)slot * stg + b * rows * 128)),
          "l"(&map), "r"(sa(&full[slot])), "r"(0), "r"(row0 + s * stage_rows + b * rows)
          : "memory");
  };
  if (threadIdx.x == 0)
    for (int s = 0; s < nst && s < nstage; ++s) issue(s);
  unsigned long long acc = 0;
  int s = 0, issued = nst < nstage ? nst : nstage;
  for (; s < nstage; ++s) {
    const int slot = s % nst;
    if (!wait_bar(&full[slot], (s / nst) & 1, err)) break;
    acc += sm[(size_t)slot * stg + threadIdx.x * 4];
    __syncwarp();
    if (threadIdx.x == 0 && s + nst < nstage) { issue(s + nst); issued = s + nst + 1; }
  }
  if (s < nstage && threadIdx.x == 0)   // drain what is still in flight (bounded)
    for (int t = s + 1; t < issued; ++t)
      if (!wait_bar(&full[t % nst], (t / nst) & 1, err)) break;
  if (threadIdx.x == 0) atomicAdd(sink, acc);
}

// plain register loads for comparison: 8 x 16 bytes in flight per thread
__global__ void __launch_bounds__(256) ld_kernel(const uint4* src, size_t n_per_cta, unsigned long long* sink) {
  const uint4* base = src + n_per_cta * blockIdx.x;
  uint32_t acc = 0;
  for (size_t i = threadIdx.x; i < n_per_cta; i += 256 * 8) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      size_t j = i + u * 256;
      if (j < n_per_cta) asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                                      : "=r"(v[u].x), "=r"(v[u].y), "=r"(v[u].z), "=r"(v[u].w) : "l"(base + j));
      else v[u] = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) acc ^= v[u].x ^ v[u].w;
  }
  if (acc == 0x12345678) atomicAdd(sink, 1ull);
}

int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  const size_t total = size_t(1) << 30;  // 1 GiB streamed
  uint8_t* buf;
  cudaMalloc(&buf, total + (64 << 20));
  cudaMemset(buf, 1, total);
  uint8_t* flush;
  cudaMalloc(&flush, 256 << 20);
  int* err;
  unsigned long long* sink;
  cudaMalloc(&err, 4);
  cudaMalloc(&sink, 8);
  cudaMemset(err, 0, 4);
  cudaFuncSetAttribute(stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  struct Cfg { int nst, stg, cps, ctas_per_sm; };
  Cfg cfgs[] = {{2, 16384, 1, 1}, {4, 16384, 1, 1}, {8, 16384, 1, 1}, {12, 16384, 1, 1},
                {4, 32768, 1, 1}, {6, 32768, 1, 1}, {3, 65536, 1, 1}, {6, 16384, 8, 1},
                {12, 8192, 1, 1}, {6, 16384, 1, 2}, {6, 16384, 16, 1}, {1, 16384, 1, 1}};
  for (const Cfg& c : cfgs) {
    const int grid = sms * c.ctas_per_sm;
    size_t per_cta = total / grid / c.stg * c.stg;
    float best = 1e9f;
    for (int r = 0; r < 5; ++r) {
      cudaMemset(flush, r, 256 << 20);
      cudaEventRecord(a);
      stream_kernel<<<grid, 128, size_t(c.nst) * c.stg>>>(buf, per_cta, c.nst, c.stg, c.cps, err, sink);
      cudaEventRecord(b);
      cudaEventSynchronize(b);
      float ms;
      cudaEventElapsedTime(&ms, a, b);
      if (r > 0 && ms < best) best = ms;
    }
    int herr = 0;
    cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost);
    printf("bulk nst=%2d stage=%6d copies/stage=%2d ctas/sm=%d: %8.1f us  %7.1f GB/s  err=%d  (%s)\n", c.nst, c.stg,
           c.cps, c.ctas_per_sm, best * 1e3, double(per_cta) * grid / (best * 1e-3) / 1e9, herr,
           cudaGetErrorString(cudaGetLastError()));
  }
  // tiled: the buffer as [total / 128 rows][64 bf16], 128-byte swizzle
  typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                               const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  void* fnp = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fnp, cudaEnableDefault, &q);
  cudaFuncSetAttribute(stream_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  struct TCfg { int nst, rows, boxes, ctas_per_sm; };
  TCfg tcfgs[] = {{2, 64, 2, 4}, {3, 64, 2, 4}, {2, 64, 2, 2}, {2, 128, 2, 2}, {3, 128, 2, 2},
                  {2, 256, 2, 1}, {3, 256, 1, 2}, {4, 256, 1, 1}, {6, 64, 2, 1}, {2, 256, 1, 3}};
  for (const TCfg& c : tcfgs) {
    if (fnp == nullptr) break;
    CUtensorMap map;
    const uint64_t nrows = total / 128;
    cuuint64_t dims[2] = {64, nrows};
    cuuint64_t strides[1] = {128};
    cuuint32_t box[2] = {64, (cuuint32_t)c.rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = reinterpret_cast<EncodeFn>(fnp)(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, buf, dims, strides, box,
                                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) { printf("tensor map failed (%d)\n", int(r)); break; }
    const int grid = sms * c.ctas_per_sm;
    const int stage_rows = c.rows * c.boxes;
    const int rows_per_cta = int(nrows / grid / stage_rows * stage_rows);
    const size_t smem = 1024 + size_t(c.nst) * stage_rows * 128;
    float best = 1e9f;
    for (int rep = 0; rep < 5; ++rep) {
      cudaMemset(flush, rep, 256 << 20);
      cudaEventRecord(a);
      stream_tiled_kernel<<<grid, 128, smem>>>(map, rows_per_cta, c.nst, c.rows, c.boxes, err, sink);
      cudaEventRecord(b);
      cudaEventSynchronize(b);
      float ms;
      cudaEventElapsedTime(&ms, a, b);
      if (rep > 0 && ms < best) best = ms;
    }
    int herr = 0;
    cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost);
    printf("tiled nst=%d box=%3d rows x 128 B (%5d B) boxes/stage=%d ctas/sm=%d: %8.1f us  %7.1f GB/s  err=%d  (%s)\n",
           c.nst, c.rows, c.rows * 128, c.boxes, c.ctas_per_sm, best * 1e3,
           double(rows_per_cta) * 128 * grid / (best * 1e-3) / 1e9, herr, cudaGetErrorString(cudaGetLastError()));
  }
  for (int cps : {1, 2, 4}) {
    const int grid = sms * cps;
    size_t n = total / 16 / grid;
    float best = 1e9f;
    for (int r = 0; r < 5; ++r) {
      cudaMemset(flush, r, 256 << 20);
      cudaEventRecord(a);
      ld_kernel<<<grid, 256>>>(reinterpret_cast<const uint4*>(buf), n, sink);
      cudaEventRecord(b);
      cudaEventSynchronize(b);
      float ms;
      cudaEventElapsedTime(&ms, a, b);
      if (r > 0 && ms < best) best = ms;
    }
    printf("ld.global 8x16B/lane, %d CTAs/SM x 256 thr: %8.1f us  %7.1f GB/s\n", cps, best * 1e3,
           double(n) * 16 * grid / (best * 1e-3) / 1e9);
  }
  return 0;
}
