// Self-test of the tcgen05 operand layouts used by the attention / MoE kernels.
//
// mode 0: D[128 x N] = A[128 x K] * B[N x K]^T   with A, B K-major (SW128), as S^T = K Q^T.
// mode 1: D[128 x N] = A^T * B                    with A given as [K x 128] (MN-major view) and
//                                                 B given as [K x N] (MN-major), as O^T = V^T P^T.
// mode 2: D[128 x N] = A[128 x K] * B[N x K]^T   with A written into TMEM (lane = row, two f16 per
//                                                 column) by tcgen05.st and B K-major in shared memory.
// mode 3: D[128 x N] = A[128 x K] * B[N x K]^T   with E4M3 operands (kind::f8f6f4), K-major SW128;
//                                                 a, b passed as uint8 codes (K <= 128 bytes per row).
// One CTA of 128 threads; K <= 128, N in {16, 32, 64}.  Used only by tests.
#include "launchers.h"
#include "common/sm100.cuh"

namespace {

__global__ void __launch_bounds__(128, 1) umma_probe_kernel(const __nv_bfloat16* __restrict__ a,
                                                            const __nv_bfloat16* __restrict__ b, int K, int N,
                                                            int mode, float* __restrict__ d, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sA = smem;               // 128 x 128 bf16 max = 32 KB
  uint8_t* sB = smem + 32768;       // 128 x 64 bf16 max = 16 KB
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 49152);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (warp == 0) { pm::tmem_alloc(tslot, 128); pm::tmem_relinquish(); }
  if (tid == 0) { pm::mbar_init(bar, 1); pm::fence_mbar_init(); }
  if (mode == 3) {
    // 8-bit operands: a row of K <= 128 codes is at most one 128-byte swizzle atom row
    const uint8_t* a8 = reinterpret_cast<const uint8_t*>(a);
    const uint8_t* b8 = reinterpret_cast<const uint8_t*>(b);
    for (int idx = tid; idx < 128 * (K / 16); idx += 128) {
      const int row = idx / (K / 16), u = idx % (K / 16);
      *reinterpret_cast<uint4*>(sA + pm::sw128_offset(row, 16 * u, 0)) =
          *reinterpret_cast<const uint4*>(a8 + row * K + 16 * u);
    }
    for (int idx = tid; idx < N * (K / 16); idx += 128) {
      const int row = idx / (K / 16), u = idx % (K / 16);
      *reinterpret_cast<uint4*>(sB + pm::sw128_offset(row, 16 * u, 0)) =
          *reinterpret_cast<const uint4*>(b8 + row * K + 16 * u);
    }
  } else if (mode == 0 || mode == 2) {
    // A rows = 128 (M), K contiguous; chunk stride = 128 rows * 128 B
    for (int idx = tid; idx < 128 * (K / 8); idx += 128) {
      const int row = idx / (K / 8), u = idx % (K / 8);
      *reinterpret_cast<uint4*>(sA + pm::sw128_offset(row, 16 * u, 128 * 128)) =
          *reinterpret_cast<const uint4*>(a + row * K + 8 * u);
    }
    for (int idx = tid; idx < N * (K / 8); idx += 128) {
      const int row = idx / (K / 8), u = idx % (K / 8);
      *reinterpret_cast<uint4*>(sB + pm::sw128_offset(row, 16 * u, N * 128)) =
          *reinterpret_cast<const uint4*>(b + row * K + 8 * u);
    }
  } else {
    // A given as [K x 128]: row k holds 128 M-values (contiguous) -> same tile layout as the KV tile
    for (int idx = tid; idx < K * 16; idx += 128) {
      const int row = idx / 16, u = idx % 16;
      *reinterpret_cast<uint4*>(sA + pm::sw128_offset(row, 16 * u, K * 128)) =
          *reinterpret_cast<const uint4*>(a + row * 128 + 8 * u);
    }
    // B given as [K x N] (N <= 64 contiguous), 128-byte rows
    for (int idx = tid; idx < K * (N / 8); idx += 128) {
      const int row = idx / (N / 8), u = idx % (N / 8);
      *reinterpret_cast<uint4*>(sB + pm::sw128_offset(row, 16 * u, 0)) =
          *reinterpret_cast<const uint4*>(b + row * N + 8 * u);
    }
  }
  pm::fence_proxy_async_smem();
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  const uint32_t tmem = *tslot;
  if (mode == 2) {
    // row (32 warp + lane): K bf16 -> K/2 columns starting at column 64
    for (int c0 = 0; c0 < K / 2; c0 += 16) {
      uint32_t v[16];
      for (int i = 0; i < 16; ++i)
        v[i] = *reinterpret_cast<const uint32_t*>(a + (32 * warp + lane) * K + 2 * (c0 + i));
      pm::tmem_st16u(tmem + 64 + c0 + ((uint32_t)(32 * warp) << 16), v);
    }
    pm::tmem_wait_st();
    pm::tc_fence_before();
    __syncthreads();
    pm::tc_fence_after();
  }
  if (tid == 0) {
    const uint32_t a0 = pm::smem_u32(sA), b0 = pm::smem_u32(sB);
    if (mode == 3) {
      const uint32_t idesc = pm::make_idesc_f8(128, N, 0, 0);
      for (int k = 0; k < K / 32; ++k) {
        const uint64_t ad = pm::make_sdesc(a0 + 32 * k, 16, 1024);
        const uint64_t bd = pm::make_sdesc(b0 + 32 * k, 16, 1024);
        pm::umma_f8(tmem, ad, bd, idesc, k > 0);
      }
    } else if (mode == 2) {
      const uint32_t idesc = pm::make_idesc_f16(128, N, 1, 0, 0);
      for (int k = 0; k < K / 16; ++k) {
        const uint32_t koff = (k * 32) & 127;
        const uint64_t bd = pm::make_sdesc(b0 + (k >> 2) * (N * 128) + koff, 16, 1024);
        pm::umma_f16_tmem_a(tmem, tmem + 64 + 8 * k, bd, idesc, k > 0);
      }
    } else if (mode == 0) {
      const uint32_t idesc = pm::make_idesc_f16(128, N, 1, 0, 0);
      for (int k = 0; k < K / 16; ++k) {
        const uint32_t koff = (k * 32) & 127;
        const uint64_t ad = pm::make_sdesc(a0 + (k >> 2) * (128 * 128) + koff, 16, 1024);
        const uint64_t bd = pm::make_sdesc(b0 + (k >> 2) * (N * 128) + koff, 16, 1024);
        pm::umma_f16(tmem, ad, bd, idesc, k > 0);
      }
    } else {
      const uint32_t idesc = pm::make_idesc_f16(128, N, 1, 1, 1);
      for (int k = 0; k < K / 16; ++k) {
        const uint64_t ad = pm::make_sdesc(a0 + k * 2048, K * 128, 1024);
        const uint64_t bd = pm::make_sdesc(b0 + k * 2048, 8192, 1024);
        pm::umma_f16(tmem, ad, bd, idesc, k > 0);
      }
    }
    pm::umma_commit(bar);
  }
  const bool ok = pm::mbar_wait(bar, 0, err, 10);
  pm::tc_fence_after();
  if (ok) {
    for (int c0 = 0; c0 < N; c0 += 16) {
      float v[16];
      pm::tmem_ld16(tmem + c0 + ((uint32_t)(32 * warp) << 16), v);
      pm::tmem_wait_ld();
      for (int i = 0; i < 16; ++i) d[(32 * warp + lane) * N + c0 + i] = v[i];
    }
  }
  pm::tc_fence_before();
  __syncthreads();
  if (warp == 0) pm::tmem_dealloc(tmem, 128);
}

}  // namespace

void launch_umma_probe(const void* a, const void* b, int K, int N, int mode, float* d, int* err,
                       cudaStream_t stream) {
  const int smem = 49152 + 64 + 1024;
  cudaFuncSetAttribute(umma_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  umma_probe_kernel<<<1, 128, smem, stream>>>(reinterpret_cast<const __nv_bfloat16*>(a),
                                              reinterpret_cast<const __nv_bfloat16*>(b), K, N, mode, d, err);
}
