// Fused tensor-parallel collectives over NVLink peer memory (sm_100a).
//
//   gemm_allreduce_kernel  Y[B, N] = sum over ranks r of X_r[B, K] W_r[N, K]^T
//                          (the row-parallel output projection of attention; reference call site:
//                          o_proj followed by the TP all-reduce, SGLang custom AR / NCCL ring)
//   allreduce_kernel       Y[n] = sum over ranks r of (A_r[n] + F_r[n])  (bf16 A, fp32 F, both optional;
//                          the MoE block's routed fp32 sum plus the shared expert's bf16 output)
//
// Both are two-shot all-reduces written into the producing kernel.  Every rank maps every peer's
// symmetric buffer (CUDA IPC), so plain ld/st reach a peer's HBM over NVLink:
//   1. reduce-scatter: output tile t is owned by rank t % world.  The CTA computing tile t stores
//      its bf16 partial straight from registers into the owner's `recv[src]` slot, then publishes
//      flag_rs[src][t] = epoch with a system-scope release;
//   2. the owner's CTA acquires all sources' flags, sums the partials in fp32 in source order (the
//      sum is computed once, so every rank receives bitwise the same result), and stores the bf16
//      result into every rank's `gath` (all-gather), publishing flag_ag[t];
//   3. every rank's CTA acquires flag_ag[t] and copies the tile into the caller's output tensor.
// Transfers overlap the tensor-core work tile by tile: tiles finish at different times.
//
// No buffer needs double-buffering: a rank can only start call n+1 after every tile of call n has
// been reduced and gathered on every owner, so no peer can still be reading what call n+1 writes.
// Flags hold the per-rank call counter `epoch` (device memory, advanced by the last CTA of each
// launch), so the kernels replay inside CUDA graphs.  Every wait has a time limit; on expiry the
// CTA records kPeerTimeout in the error word and goes on.  All CTAs of a launch are co-resident
// (grid <= SM count), so waits between CTAs of one launch cannot deadlock.  No TMA load here reads
// peer memory; X and W are local and loaded with plain (non-multicast) TMA.
#include <cuda.h>

#include "common/sm100.cuh"
#include "launchers.h"

namespace {
constexpr int kThreads = 192;  // warp 0 TMA producer, warp 1 MMA issuer, warps 2-5 epilogue
constexpr int kTileN = 128;    // weight rows per tile (MMA M)
constexpr int kWBytes = kTileN * 128;
constexpr int kEpiBar = 1;     // named barrier of the 128 epilogue threads
constexpr int kMaxStages = 8;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync %0, 128;" ::"n"(kEpiBar) : "memory"); }

// Wait until *f >= s (wrap-safe), bounded by timeout_ns of GPU time.
__device__ bool wait_flag(const uint32_t* f, uint32_t s, int64_t timeout_ns) {
  if ((int32_t)(ld_acquire_sys(f) - s) >= 0) return true;
  const uint64_t t0 = pm::globaltimer_ns();
  while (true) {
    __nanosleep(32);
    if ((int32_t)(ld_acquire_sys(f) - s) >= 0) return true;
    if ((int64_t)(pm::globaltimer_ns() - t0) > timeout_ns) return false;
  }
}

struct Sym {
  const SymmComm& c;
  __device__ explicit Sym(const SymmComm& cc) : c(cc) {}
  __device__ uint8_t* base(int r) const { return reinterpret_cast<uint8_t*>(__ldg(c.peers + r)); }
  __device__ __nv_bfloat16* recv(int r, int src) const {
    return reinterpret_cast<__nv_bfloat16*>(base(r) + c.recv_off) + (int64_t)src * c.recv_elems;
  }
  __device__ __nv_bfloat16* gath(int r) const { return reinterpret_cast<__nv_bfloat16*>(base(r) + c.gath_off); }
  __device__ uint32_t* flag_rs(int r, int src, int t) const {
    return reinterpret_cast<uint32_t*>(base(r) + c.flag_rs_off) + (int64_t)src * c.max_tiles + t;
  }
  __device__ uint32_t* flag_ag(int r, int t) const {
    return reinterpret_cast<uint32_t*>(base(r) + c.flag_ag_off) + t;
  }
};

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void add_bf16x8(float (&acc)[8], uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    acc[2 * j] += __uint_as_float(w[j] << 16);
    acc[2 * j + 1] += __uint_as_float(w[j] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ uint4 pack8(const float (&a)[8]) {
  return make_uint4(pack_bf16(a[0], a[1]), pack_bf16(a[2], a[3]), pack_bf16(a[4], a[5]), pack_bf16(a[6], a[7]));
}

// Last CTA of the launch advances the call counter (the next launch reads it in stream order).
__device__ __forceinline__ void finish_epoch(const SymmComm& c, uint32_t s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(c.epoch + 1, 1u) == gridDim.x - 1) {
      c.epoch[1] = 0;
      c.epoch[0] = s;
      __threadfence();
    }
  }
}

// ----------------------------------------------------------------------------- GEMM + all-reduce
__global__ void __launch_bounds__(kThreads, 1) gemm_ar_kernel(const __grid_constant__ CUtensorMap tmW,
                                                              const __grid_constant__ CUtensorMap tmX,
                                                              const GemmArParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  const int xbox = p.Bpad <= 256 ? p.Bpad : p.Bpad / 2;  // rows per X box = MMA N
  const int nx = p.Bpad / xbox;
  const int stage_bytes = kWBytes + p.Bpad * 128;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.stages * stage_bytes);
  uint64_t* empty = full + p.stages;
  uint64_t* d_full = empty + p.stages;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(d_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const SymmComm& c = p.c;
  const Sym sym(c);
  const int tile = blockIdx.x / p.S, ks = blockIdx.x % p.S;
  const int nk = p.K / 64 / p.S, k0 = ks * nk;
  const int owner = tile % c.world, src = c.rank * p.S + ks, nsrc = c.world * p.S;
  const uint32_t s = *reinterpret_cast<volatile const uint32_t*>(c.epoch) + 1;
  uint32_t tcols = 32;
  while ((int)tcols < p.Bpad) tcols <<= 1;

  if (warp == 0) {
    pm::tmem_alloc(tslot, tcols);
    pm::tmem_relinquish();
  }
  if (tid == 32) {
    for (int i = 0; i < p.stages; ++i) {
      pm::mbar_init(full + i, 1);
      pm::mbar_init(empty + i, 1);
    }
    pm::mbar_init(d_full, 1);
    *abort_flag = 0;
    pm::fence_mbar_init();
  }
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      int st = 0, issued = 0;
      uint32_t ph = 0;
      uint32_t issued_ph[kMaxStages];
      for (int i = 0; i < nk; ++i) {
        if (!pm::mbar_wait(empty + st, ph ^ 1, c.err, 301)) { *abort_flag = 1; break; }
        uint8_t* sb = smem + st * stage_bytes;
        pm::mbar_arrive_expect_tx(full + st, stage_bytes);
        const int kx = (k0 + i) * 64;  // element offset: a multiple of 64 (128 B)
        pm::tma_load_2d(sb, &tmW, kx, tile * kTileN, full + st);
        for (int h = 0; h < nx; ++h) pm::tma_load_2d(sb + kWBytes + h * xbox * 128, &tmX, kx, h * xbox, full + st);
        issued_ph[st] = ph;
        ++issued;
        if (++st == p.stages) { st = 0; ph ^= 1; }
      }
      if (*abort_flag) {  // let issued copies land before the CTA can exit
        for (int j = 1; j <= p.stages && j <= issued; ++j) {
          const int sj = (st - j + p.stages) % p.stages;
          pm::mbar_wait(full + sj, issued_ph[sj], nullptr, 0, 20000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0;
      const uint32_t idesc = pm::make_idesc_f16(128, xbox, 1, 0, 0);
      for (int i = 0; i < nk && !*abort_flag; ++i) {
        if (!pm::mbar_wait(full + st, ph, c.err, 302)) { *abort_flag = 1; break; }
        pm::tc_fence_after();
        const uint32_t sb = pm::smem_u32(smem + st * stage_bytes);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t a = pm::make_sdesc(sb + 32 * k, 16, 1024);
          for (int h = 0; h < nx; ++h)
            pm::umma_f16(tmem + h * xbox, a, pm::make_sdesc(sb + kWBytes + h * xbox * 128 + 32 * k, 16, 1024), idesc,
                         (i | k) ? 1u : 0u);
        }
        pm::umma_commit(empty + st);
        if (++st == p.stages) { st = 0; ph ^= 1; }
      }
      pm::umma_commit(d_full);  // arrives once every MMA issued above has completed
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-5)
    const int q = warp & 3, r = 32 * q + lane, n = tile * kTileN + r;
    const int et = tid - 64;  // 0..127
    const bool ok = pm::mbar_wait(d_full, 0, c.err, 303);
    pm::tc_fence_after();
    // 1. partial -> owner's recv[src][n][b]
    __nv_bfloat16* dst = sym.recv(owner, src) + (int64_t)n * p.Bpad;
    for (int c0 = 0; c0 < p.B; c0 += 16) {
      float v[16];
      pm::tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + c0, v);
      if (!ok || nk == 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = 0.f;
      }
      uint4 lo = make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
      uint4 hi = make_uint4(pack_bf16(v[8], v[9]), pack_bf16(v[10], v[11]), pack_bf16(v[12], v[13]),
                            pack_bf16(v[14], v[15]));
      reinterpret_cast<uint4*>(dst + c0)[0] = lo;
      reinterpret_cast<uint4*>(dst + c0)[1] = hi;
    }
    epi_sync();
    if (et == 0) {
      __threadfence_system();
      st_release_sys(sym.flag_rs(owner, src, tile), s);
    }
    if (ks == 0) {
      // 2. owner: reduce all sources, all-gather the bf16 result
      if (c.rank == owner) {
        if (et < nsrc && !wait_flag(sym.flag_rs(c.rank, et, tile), s, c.timeout_ns))
          pm::report_error(c.err, pm::kPeerTimeout, 310 + et);
        epi_sync();
        for (int c0 = 0; c0 < p.B; c0 += 8) {
          float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int sr = 0; sr < nsrc; ++sr)
            add_bf16x8(acc, __ldcg(reinterpret_cast<const uint4*>(sym.recv(c.rank, sr) + (int64_t)n * p.Bpad + c0)));
          const uint4 o = pack8(acc);
          for (int d = 0; d < c.world; ++d)
            *reinterpret_cast<uint4*>(sym.gath(d) + (int64_t)n * p.Bpad + c0) = o;
        }
        epi_sync();
        if (et == 0) {
          __threadfence_system();
          for (int d = 0; d < c.world; ++d) st_release_sys(sym.flag_ag(d, tile), s);
        }
      }
      // 3. every rank: wait for the gathered tile, copy it out as Y[b][n]
      if (et == 0 && !wait_flag(sym.flag_ag(c.rank, tile), s, c.timeout_ns))
        pm::report_error(c.err, pm::kPeerTimeout, 309);
      epi_sync();
      const __nv_bfloat16* g = sym.gath(c.rank) + (int64_t)n * p.Bpad;
      for (int c0 = 0; c0 < p.B; c0 += 8) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(g + c0));
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (c0 + j < p.B) p.out[(int64_t)(c0 + j) * p.N + n] = e[j];
      }
    }
  }
  pm::tc_fence_before();
  finish_epoch(c, s);  // contains __syncthreads
  pm::tc_fence_after();
  if (warp == 0) pm::tmem_dealloc(tmem, tcols);
}

// ----------------------------------------------------------------------------- all-reduce
__global__ void __launch_bounds__(256) allreduce_kernel(const ArParams p) {
  const SymmComm& c = p.c;
  const Sym sym(c);
  const int t = blockIdx.x, owner = t % c.world;
  const uint32_t s = *reinterpret_cast<volatile const uint32_t*>(c.epoch) + 1;
  const int64_t lo = (int64_t)t * p.chunk, hi = min(p.n, lo + p.chunk);
  // 1. local addends -> owner's recv[rank]
  __nv_bfloat16* dst = sym.recv(owner, c.rank);
  for (int64_t i = lo + 8 * threadIdx.x; i < hi; i += 8 * blockDim.x) {
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (p.a) add_bf16x8(v, *reinterpret_cast<const uint4*>(p.a + i));
    if (p.f) {
      const float4 f0 = *reinterpret_cast<const float4*>(p.f + i), f1 = *reinterpret_cast<const float4*>(p.f + i + 4);
      v[0] += f0.x; v[1] += f0.y; v[2] += f0.z; v[3] += f0.w;
      v[4] += f1.x; v[5] += f1.y; v[6] += f1.z; v[7] += f1.w;
    }
    *reinterpret_cast<uint4*>(dst + i) = pack8(v);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    st_release_sys(sym.flag_rs(owner, c.rank, t), s);
  }
  // 2. owner: reduce + all-gather
  if (c.rank == owner) {
    if (threadIdx.x < c.world && !wait_flag(sym.flag_rs(c.rank, threadIdx.x, t), s, c.timeout_ns)) {
      pm::report_error(c.err, pm::kPeerTimeout, 320 + threadIdx.x);
    }
    __syncthreads();
    for (int64_t i = lo + 8 * threadIdx.x; i < hi; i += 8 * blockDim.x) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int sr = 0; sr < c.world; ++sr) add_bf16x8(acc, __ldcg(reinterpret_cast<const uint4*>(sym.recv(c.rank, sr) + i)));
      const uint4 o = pack8(acc);
      for (int d = 0; d < c.world; ++d) *reinterpret_cast<uint4*>(sym.gath(d) + i) = o;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      for (int d = 0; d < c.world; ++d) st_release_sys(sym.flag_ag(d, t), s);
    }
  }
  // 3. every rank: gathered chunk -> out
  if (threadIdx.x == 0 && !wait_flag(sym.flag_ag(c.rank, t), s, c.timeout_ns))
    pm::report_error(c.err, pm::kPeerTimeout, 319);
  __syncthreads();
  const __nv_bfloat16* g = sym.gath(c.rank);
  for (int64_t i = lo + 8 * threadIdx.x; i < hi; i += 8 * blockDim.x)
    *reinterpret_cast<uint4*>(p.out + i) = __ldcg(reinterpret_cast<const uint4*>(g + i));
  finish_epoch(c, s);
}
}  // namespace

int gemm_ar_smem_bytes(int Bpad, int stages) { return stages * (kWBytes + Bpad * 128) + 1024 + 256; }

int launch_gemm_allreduce(const GemmArParams& p, const void* w, const void* x, int num_sms, cudaStream_t stream) {
  if (p.B < 1 || p.Bpad < p.B || p.Bpad % 16 || p.Bpad > 512 || (p.Bpad > 256 && p.Bpad % 32) || p.N % kTileN ||
      p.S < 1 || p.K % (64 * p.S) || p.stages < 2 || p.stages > kMaxStages)
    return 1;
  const int ntiles = p.N / kTileN;
  if (ntiles * p.S > num_sms || ntiles > p.c.max_tiles || p.c.world * p.S > p.c.max_src ||
      (int64_t)p.N * p.Bpad > p.c.recv_elems)
    return 2;
  alignas(64) CUtensorMap mw, mx;
  const int xbox = p.Bpad <= 256 ? p.Bpad : p.Bpad / 2;
  if (make_tmap_bf16_sw128(&mw, w, p.K, p.N, (uint64_t)p.K * 2, kTileN)) return 3;
  if (make_tmap_bf16_sw128(&mx, x, p.K, p.B, (uint64_t)p.K * 2, xbox)) return 3;
  const int smem = gemm_ar_smem_bytes(p.Bpad, p.stages);
  cudaFuncSetAttribute(gemm_ar_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  gemm_ar_kernel<<<ntiles * p.S, kThreads, smem, stream>>>(mw, mx, p);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

int launch_allreduce(const ArParams& p, int num_sms, cudaStream_t stream) {
  if (p.n % 8 || p.chunk % 8 || p.chunk <= 0) return 1;
  const int64_t ntiles = (p.n + p.chunk - 1) / p.chunk;
  if (ntiles > num_sms || ntiles > p.c.max_tiles || p.c.world > p.c.max_src || p.n > p.c.recv_elems) return 2;
  allreduce_kernel<<<(int)ntiles, 256, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
