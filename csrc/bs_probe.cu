// Raw tcgen05 MMA probe for the block-scaled 8/6/4-bit kinds.
//
// The host supplies the shared-memory images of A (128 rows x 128 B) and B (N rows x 128 B), both
// K-major with the 128-byte swizzle already applied, 16 TMEM columns of scale-factor words for A
// (at column 256) and for B (at column 384), and the instruction descriptor.  One MMA (K = 32 for
// the 8/6/4-bit kinds, 64 for kind::mxf4) writes D [128 x N] fp32, which is returned.  Used by the
// tests that pin the operand / scale-factor layouts the block-scaled MoE kernel relies on.
//
// kind 0: kind::f8f6f4 (no scales); 1: kind::mxf8f6f4.block_scale; 2: kind::mxf4.block_scale.
#include "launchers.h"
#include "common/sm100.cuh"

namespace {

__global__ void __launch_bounds__(128, 1) bs_probe_kernel(const uint8_t* __restrict__ a_img,
                                                          const uint8_t* __restrict__ b_img,
                                                          const uint32_t* __restrict__ sfa,
                                                          const uint32_t* __restrict__ sfb, uint32_t idesc,
                                                          int kind, int N, uint32_t sfa_extra, uint32_t sfb_extra,
                                                          float* __restrict__ d, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sA = smem;          // 16 KB
  uint8_t* sB = smem + 16384;  // up to 256 rows x 128 B = 32 KB
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 49152);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  if (warp == 0) { pm::tmem_alloc(tslot, 512); pm::tmem_relinquish(); }
  if (tid == 0) { pm::mbar_init(bar, 1); pm::fence_mbar_init(); }
  for (int i = tid; i < 128 * 8; i += 128)
    reinterpret_cast<uint4*>(sA)[i] = reinterpret_cast<const uint4*>(a_img)[i];
  for (int i = tid; i < N * 8; i += 128)
    reinterpret_cast<uint4*>(sB)[i] = reinterpret_cast<const uint4*>(b_img)[i];
  pm::fence_proxy_async_smem();
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
  {
    uint32_t v[16];
    for (int i = 0; i < 16; ++i) v[i] = sfa[tid * 16 + i];
    pm::tmem_st16u(tmem + lane_base + 256, v);
    for (int i = 0; i < 16; ++i) v[i] = sfb[tid * 16 + i];
    pm::tmem_st16u(tmem + lane_base + 384, v);
    pm::tmem_wait_st();
  }
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  if (tid == 0) {
    const uint64_t ad = pm::make_sdesc(pm::smem_u32(sA), 16, 1024);
    const uint64_t bd = pm::make_sdesc(pm::smem_u32(sB), 16, 1024);
    const uint32_t sa = tmem + 256 + sfa_extra, sb = tmem + 384 + sfb_extra;
    if (kind == 0) {
      pm::umma_f8(tmem, ad, bd, idesc, 0);
    } else if (kind == 1) {
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(tmem),
          "l"(ad), "l"(bd), "r"(idesc), "r"(0), "r"(sa), "r"(sb)
          : "memory");
    } else {
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::1.kind::mxf4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(tmem),
          "l"(ad), "l"(bd), "r"(idesc), "r"(0), "r"(sa), "r"(sb)
          : "memory");
    }
    pm::umma_commit(bar);
  }
  __syncwarp();
  const bool ok = pm::mbar_wait(bar, 0, err, 1);
  pm::tc_fence_after();
  if (ok) {
    for (int c0 = 0; c0 < N; c0 += 16) {
      float v[16];
      pm::tmem_ld16(tmem + lane_base + c0, v);
      for (int i = 0; i < 16; ++i)
        if (c0 + i < N) d[tid * N + c0 + i] = v[i];
    }
  }
  pm::tc_fence_before();
  __syncthreads();
  if (warp == 0) pm::tmem_dealloc(tmem, 512);
}

}  // namespace

void launch_bs_probe(const uint8_t* a_img, const uint8_t* b_img, const uint32_t* sfa, const uint32_t* sfb,
                     uint32_t idesc, int kind, int N, uint32_t sfa_extra, uint32_t sfb_extra, float* d, int* err,
                     cudaStream_t stream) {
  const int smem = 49152 + 64 + 1024;
  cudaFuncSetAttribute(bs_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  bs_probe_kernel<<<1, 128, smem, stream>>>(a_img, b_img, sfa, sfb, idesc, kind, N, sfa_extra, sfb_extra, d, err);
}

// ----------------------------------------------------------------------------- pipeline probe
// A: packed FP4 [128 rows x 128 values] loaded by TMA (unpacking map, 128-byte swizzle); B: E4M3 image
// [N x 128 B] (pre-swizzled); scale factors of A and B from 512-byte tcgen05.cp sources (32 rows x 16 B).
// k_steps MMAs of K = 32 with sf_id = step.  Returns D and the shared-memory image of A.
#include <cuda.h>
namespace {
__global__ void __launch_bounds__(128, 1) bs_probe2_kernel(const __grid_constant__ CUtensorMap tmA,
                                                           const uint8_t* __restrict__ b_img,
                                                           const uint8_t* __restrict__ sfa_src,
                                                           const uint8_t* __restrict__ sfb_src, int N, int k_steps,
                                                           uint32_t expect_tx, float* __restrict__ d,
                                                           uint8_t* __restrict__ a_dump, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sA = smem;                 // 16 KB
  uint8_t* sB = smem + 16384;         // up to 32 KB
  uint8_t* sSFA = smem + 49152;       // 512 B
  uint8_t* sSFB = smem + 49152 + 512; // 512 B
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 50176);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 2);
  const int tid = threadIdx.x, warp = tid >> 5;
  if (warp == 0) { pm::tmem_alloc(tslot, 512); pm::tmem_relinquish(); }
  if (tid == 0) { pm::mbar_init(bar, 1); pm::mbar_init(bar + 1, 1); pm::fence_mbar_init(); }
  __syncthreads();
  if (tid == 0) {
    pm::mbar_arrive_expect_tx(bar, expect_tx);
    pm::tma_load_2d(sA, &tmA, 0, 0, bar);
  }
  for (int i = tid; i < N * 8; i += 128)
    reinterpret_cast<uint4*>(sB)[i] = reinterpret_cast<const uint4*>(b_img)[i];
  for (int i = tid; i < 32; i += 128) {
    reinterpret_cast<uint4*>(sSFA)[i] = reinterpret_cast<const uint4*>(sfa_src)[i];
    reinterpret_cast<uint4*>(sSFB)[i] = reinterpret_cast<const uint4*>(sfb_src)[i];
  }
  pm::fence_proxy_async_smem();
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  const uint32_t tmem = *tslot;
  const bool loaded = pm::mbar_wait(bar, 0, err, 11);
  for (int i = tid; i < 1024; i += 128)
    reinterpret_cast<uint4*>(a_dump)[i] = reinterpret_cast<const uint4*>(sA)[i];
  if (tid == 0 && loaded) {
    pm::tmem_cp_32x128_x4(tmem + 256, pm::smem_u32(sSFA));
    pm::tmem_cp_32x128_x4(tmem + 384, pm::smem_u32(sSFB));
    for (int k = 0; k < k_steps; ++k) {
      const uint64_t ad = pm::make_sdesc(pm::smem_u32(sA) + 32 * k, 16, 1024);
      const uint64_t bd = pm::make_sdesc(pm::smem_u32(sB) + 32 * k, 16, 1024);
      pm::umma_mxf8(tmem, ad, bd, pm::make_idesc_mxf8(128, N, 5, 0, k, k), tmem + 256, tmem + 384, k > 0);
    }
    pm::umma_commit(bar + 1);
  }
  __syncwarp();
  const bool ok = loaded && pm::mbar_wait(bar + 1, 0, err, 12);
  pm::tc_fence_after();
  if (ok) {
    const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
    for (int c0 = 0; c0 < N; c0 += 16) {
      float v[16];
      pm::tmem_ld16(tmem + lane_base + c0, v);
      for (int i = 0; i < 16; ++i)
        if (c0 + i < N) d[tid * N + c0 + i] = v[i];
    }
  }
  pm::tc_fence_before();
  __syncthreads();
  if (warp == 0) pm::tmem_dealloc(tmem, 512);
}
}  // namespace

int launch_bs_probe2(const uint8_t* a_packed, const uint8_t* b_img, const uint8_t* sfa_src, const uint8_t* sfb_src,
                     int N, int k_steps, uint32_t expect_tx, float* d, uint8_t* a_dump, int* err,
                     cudaStream_t stream) {
  CUtensorMap map;
  const int rc = make_tmap_fp4_unpacked(&map, a_packed, 128, 128, 64, 128);
  if (rc != 0) return rc;
  const int smem = 50176 + 64 + 1024;
  cudaFuncSetAttribute(bs_probe2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  bs_probe2_kernel<<<1, 128, smem, stream>>>(map, b_img, sfa_src, sfb_src, N, k_steps, expect_tx, d, a_dump, err);
  return 0;
}
