// Latency / throughput probe of tcgen05 MMAs (used by the kernel design notes, not by the engine):
// per iteration, thread 0 issues `n_mma` tcgen05.mma (M=128, N=n, A and B from shared memory, A
// alternating between two 16 KB tiles every 4 MMAs) round-robin over `n_acc` accumulators, then
// tcgen05.commit to an mbarrier that all 128 threads wait on.  kind 0: kind::f16 (K=16); 1:
// kind::mxf8f6f4 block-scaled E2M1 x E4M3 (K=32, scale factors in TMEM); 2: kind::f8f6f4 E4M3 x E4M3.
// Returns the average clock64 cycles per iteration.
#include "launchers.h"
#include "common/sm100.cuh"

namespace {
__global__ void __launch_bounds__(128, 1) tc_latency_kernel(int iters, int n_mma, int n, int n_acc, int kind,
                                                            long long* out, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 65536);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x;
  for (int i = tid; i < 65536 / 4; i += 128) reinterpret_cast<uint32_t*>(smem)[i] = 0;
  if (tid < 32) { pm::tmem_alloc(tslot, 512); pm::tmem_relinquish(); }
  if (tid == 0) { pm::mbar_init(bar, 1); pm::fence_mbar_init(); }
  pm::fence_proxy_async_smem();
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t a0 = pm::smem_u32(smem), b0 = pm::smem_u32(smem + 32768);
  const uint32_t idesc = pm::make_idesc_f16(128, n, 1, 0, 0);
  // only the issuing thread waits (other lanes of its warp spinning on the barrier would compete
  // with it for issue slots); out[0] = cycles per iteration, out[1] = cycles spent issuing
  long long t0 = clock64(), t_issue = 0;
  if (kind >= 3 && tid < 32) {
    // warp-collective issue (kinds 3-5 = kinds 0-2 issued by all of warp 0 with an elected lane)
    const uint32_t tm = __shfl_sync(0xffffffffu, tmem, 0);
    for (int it = 0; it < iters; ++it) {
      const long long ti = clock64();
      for (int k = 0; k < n_mma; ++k) {
        const uint64_t ad = pm::make_sdesc(a0 + ((k >> 2) & 1) * 16384 + (k & 3) * 32, 16, 1024);
        const uint64_t bd = pm::make_sdesc(b0 + (k & 3) * 32, 16, 1024);
        const uint32_t d = tm + (k % n_acc) * n;
        if (kind == 3)
          pm::umma_f16_warp(d, ad, bd, idesc, k >= n_acc);
        else if (kind == 4)
          pm::umma_mxf8_warp(d, ad, bd, pm::make_idesc_mxf8(128, n, 5, 0, k & 3, k & 3), tm + 480, tm + 496, k >= n_acc);
        else
          pm::umma_f8_warp(d, ad, bd, pm::make_idesc_f8(128, n, 0, 0), k >= n_acc);
      }
      pm::umma_commit_warp(bar);
      t_issue += clock64() - ti;
      if (!pm::mbar_wait(bar, it & 1, err, 50)) break;
      pm::tc_fence_after();
    }
  } else if (tid == 0 && kind < 3) {
    for (int it = 0; it < iters; ++it) {
      const long long ti = clock64();
      for (int k = 0; k < n_mma; ++k) {
        const uint64_t ad = pm::make_sdesc(a0 + ((k >> 2) & 1) * 16384 + (k & 3) * 32, 16, 1024);
        const uint64_t bd = pm::make_sdesc(b0 + (k & 3) * 32, 16, 1024);
        const uint32_t d = tmem + (k % n_acc) * n;
        if (kind == 0)
          pm::umma_f16(d, ad, bd, idesc, k >= n_acc);
        else if (kind == 1)
          pm::umma_mxf8(d, ad, bd, pm::make_idesc_mxf8(128, n, 5, 0, k & 3, k & 3), tmem + 480, tmem + 496, k >= n_acc);
        else
          pm::umma_f8(d, ad, bd, pm::make_idesc_f8(128, n, 0, 0), k >= n_acc);
      }
      pm::umma_commit(bar);
      t_issue += clock64() - ti;
      if (!pm::mbar_wait(bar, it & 1, err, 50)) break;
      pm::tc_fence_after();
    }
  }
  long long t1 = clock64();
  if (tid == 0) {
    out[0] = (t1 - t0) / (iters > 0 ? iters : 1);
    out[1] = t_issue / (iters > 0 ? iters : 1);
  }
  pm::tc_fence_before();
  __syncthreads();
  if (tid < 32) pm::tmem_dealloc(tmem, 512);
}
}  // namespace

void launch_tc_latency_probe(int iters, int n_mma, int n, int n_acc, int kind, long long* out, int* err,
                             cudaStream_t stream) {
  const int smem = 65536 + 64 + 1024;
  cudaFuncSetAttribute(tc_latency_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  tc_latency_kernel<<<1, 128, smem, stream>>>(iters, n_mma, n, n_acc, kind, out, err);
}
