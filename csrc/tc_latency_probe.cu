// Latency probe of tcgen05 handshakes (used by the kernel design notes, not by the engine):
// per iteration, thread 0 issues `n_mma` tcgen05.mma (M=128, N=n, K=16, A and B from shared memory)
// round-robin over `n_acc` accumulators, then tcgen05.commit to an mbarrier that all 128 threads
// wait on.  Returns the average clock64 cycles per iteration.
#include "launchers.h"
#include "common/sm100.cuh"

namespace {
__global__ void __launch_bounds__(128, 1) tc_latency_kernel(int iters, int n_mma, int n, int n_acc, long long* out,
                                                            int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 65536);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x;
  for (int i = tid; i < 65536 / 4; i += 128) reinterpret_cast<uint32_t*>(smem)[i] = 0;
  if (tid < 32) { pm::tmem_alloc(tslot, 256); pm::tmem_relinquish(); }
  if (tid == 0) { pm::mbar_init(bar, 1); pm::fence_mbar_init(); }
  pm::fence_proxy_async_smem();
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t a0 = pm::smem_u32(smem), b0 = pm::smem_u32(smem + 32768);
  const uint32_t idesc = pm::make_idesc_f16(128, n, 1, 0, 0);
  long long t0 = clock64();
  for (int it = 0; it < iters; ++it) {
    if (tid == 0) {
      for (int k = 0; k < n_mma; ++k)
        pm::umma_f16(tmem + (k % n_acc) * n, pm::make_sdesc(a0 + (k & 3) * 32, 16, 1024), pm::make_sdesc(b0 + (k & 3) * 32, 16, 1024),
                     idesc, k >= n_acc);
      pm::umma_commit(bar);
    }
    if (!pm::mbar_wait(bar, it & 1, err, 50)) break;
    pm::tc_fence_after();
  }
  long long t1 = clock64();
  if (tid == 0) *out = (t1 - t0) / (iters > 0 ? iters : 1);
  pm::tc_fence_before();
  __syncthreads();
  if (tid < 32) pm::tmem_dealloc(tmem, 256);
}
}  // namespace

void launch_tc_latency_probe(int iters, int n_mma, int n, int n_acc, long long* out, int* err, cudaStream_t stream) {
  const int smem = 65536 + 64 + 1024;
  cudaFuncSetAttribute(tc_latency_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  tc_latency_kernel<<<1, 128, smem, stream>>>(iters, n_mma, n, n_acc, out, err);
}
