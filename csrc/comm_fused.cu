// Fused tensor-parallel collectives over NVLink peer memory (sm_100a).
//
//   gemm_allreduce_kernel  Y[B, N] = sum over ranks r of X_r[B, K] W_r[N, K]^T
//                          (the row-parallel output projection of attention; reference call site:
//                          o_proj followed by the TP all-reduce, SGLang custom AR / NCCL ring)
//   allreduce_kernel       Y[n] = sum over ranks r of (A_r[n] + F_r[n])  (bf16 A, fp32 F, both optional;
//                          the MoE block's routed fp32 sum plus the shared expert's bf16 output)
//
// The all-reduce is written into the producing kernel.  Every rank maps every peer's symmetric buffer
// (CUDA IPC), so plain ld/st reach a peer's HBM over NVLink.  Output tile t (a 256-column x 128-token
// block, or a chunk of the flat all-reduce) is handled by the CTA with the same index on every rank:
//   one-shot (small messages): the CTA stores its bf16 partial straight from registers into every
//     rank's `recv[rank]` slot and publishes flag_rs[rank][t] = epoch with a system-scope release;
//     each rank then acquires all ranks' flags and sums the partials in fp32 in rank order;
//   two-shot (large messages): partials go only to the tile owner (rank t % world), which reduces
//     and stores the bf16 result into every rank's `gath` (flag_ag[t]); every rank copies it out.
// Either way each rank sums the same bf16 partials in the same order, so all ranks hold bitwise the
// same result.  Transfers overlap the tensor-core work tile by tile: tiles finish at different times.
//
// The partial slots alternate by the parity of the call counter: in one-shot mode a rank may push call
// n+1 while a peer still reduces call n, but it cannot reach call n+2 before that peer has sent its
// call n+1 partials, i.e. finished call n.  Flags hold the per-rank call counter `epoch` (device memory, advanced by the last CTA of
// each launch), so the kernels replay inside CUDA graphs.  Every wait has a time limit; on expiry the
// CTA records kPeerTimeout in the error word and goes on.  All CTAs of a launch are co-resident
// (grid <= SM count), so waits between CTAs of one launch cannot deadlock.  No TMA load here reads
// peer memory; X and W are local and loaded with plain (non-multicast) TMA.
#include <cuda.h>

#include "common/sm100.cuh"
#include "launchers.h"

namespace {
constexpr int kThreads = 192;  // warp 0 TMA producer, warp 1 MMA issuer, warps 2-5 epilogue
constexpr int kTileN = 256;    // weight rows per tile (MMA N)
constexpr int kXBytes = 128 * 128;              // 128 token rows x 64 K (bf16)
constexpr int kStageBytes = kXBytes + kTileN * 128;
constexpr int kSRow = kTileN + 4;               // fp32 row stride of the epilogue tile in shared memory
constexpr int kEpiBar = 1;     // named barrier of the 128 epilogue threads
constexpr int kMaxStages = 4;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync %0, 128;" ::"n"(kEpiBar) : "memory"); }

// Wait until *f >= s (wrap-safe), bounded by timeout_ns of GPU time.
__device__ bool wait_flag(const uint32_t* f, uint32_t s, int64_t timeout_ns) {
  if ((int32_t)(ld_acquire_sys(f) - s) >= 0) return true;
  const uint64_t t0 = pm::globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if ((int32_t)(ld_acquire_sys(f) - s) >= 0) return true;
    if ((i & 63) == 0 && (int64_t)(pm::globaltimer_ns() - t0) > timeout_ns) return false;
  }
}

struct Sym {
  const SymmComm& c;
  __device__ explicit Sym(const SymmComm& cc) : c(cc) {}
  __device__ uint8_t* base(int r) const { return reinterpret_cast<uint8_t*>(__ldg(c.peers + r)); }
  // two parity slots: in one-shot mode a peer may push call n+1 while this rank still reduces call n
  __device__ __nv_bfloat16* recv(int r, int src, uint32_t s) const {
    return reinterpret_cast<__nv_bfloat16*>(base(r) + c.recv_off) +
           ((int64_t)(s & 1) * c.max_src + src) * c.recv_elems;
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
// Operand roles: the (padded) tokens are the M = 128 operand and 256 weight rows the N operand, so each
// tcgen05.mma consumes 256 x 16 weights (the issue cost of one instruction barely depends on N).
// CTA (tile, mb, ks): output columns [256 tile, +256), tokens [128 mb, +128), K slice ks of S.
// Split-K partials stay on this GPU: every split CTA stores its fp32 partial in a local `lpart` slot,
// then CTA ks sums the S partials of column slice ks (width 256 / S) and alone moves that slice across
// NVLink, so the sums and the pushes of a tile run on all S CTAs in parallel.
__global__ void __launch_bounds__(kThreads, 1) gemm_ar_kernel(const __grid_constant__ CUtensorMap tmW,
                                                              const __grid_constant__ CUtensorMap tmX,
                                                              const GemmArParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.stages * kStageBytes);
  uint64_t* empty = full + p.stages;
  uint64_t* d_full = empty + p.stages;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(d_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const SymmComm& c = p.c;
  const Sym sym(c);
  const int ks = blockIdx.x % p.S, tm = blockIdx.x / p.S;  // tm = tile * nmb + mb (flag index)
  const int tile = tm / p.nmb, mb = tm % p.nmb;
  const int n0 = tile * kTileN, b0 = mb * 128;
  const int nk = p.K / 64 / p.S, k0 = ks * nk;
  const uint32_t s = *reinterpret_cast<volatile const uint32_t*>(c.epoch) + 1;
  uint64_t t0 = 0;
  if (p.prof && tid == 64) t0 = pm::globaltimer_ns();

  if (warp == 0) {
    pm::tmem_alloc(tslot, kTileN);
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
        uint8_t* sb = smem + st * kStageBytes;
        pm::mbar_arrive_expect_tx(full + st, kStageBytes);
        const int kx = (k0 + i) * 64;  // element offset: a multiple of 64 (128 B)
        pm::tma_load_2d(sb, &tmX, kx, b0, full + st);
        pm::tma_load_2d(sb + kXBytes, &tmW, kx, n0, full + st);
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
      const uint32_t idesc = pm::make_idesc_f16(128, kTileN, 1, 0, 0);
      for (int i = 0; i < nk && !*abort_flag; ++i) {
        if (!pm::mbar_wait(full + st, ph, c.err, 302)) { *abort_flag = 1; break; }
        pm::tc_fence_after();
        const uint32_t sb = pm::smem_u32(smem + st * kStageBytes);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          pm::umma_f16(tmem, pm::make_sdesc(sb + 32 * k, 16, 1024), pm::make_sdesc(sb + kXBytes + 32 * k, 16, 1024),
                       idesc, (i | k) ? 1u : 0u);
        pm::umma_commit(empty + st);
        if (++st == p.stages) { st = 0; ph ^= 1; }
      }
      pm::umma_commit(d_full);  // arrives once every MMA issued above has completed
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-5)
    // The accumulator rows (one token per TMEM lane) go to shared memory first (the drained stage
    // buffers), so every later step works on 8-column chunks spread over all 128 threads: a tile with
    // few tokens must not serialize its split-K sums and pushes on one thread per row.
    const int q = warp & 3, r = 32 * q + lane;
    const int et = tid - 64;  // 0..127
    const bool ok = pm::mbar_wait(d_full, 0, c.err, 303);
    pm::tc_fence_after();
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
    const int rows = min(128, p.B - b0);
    const int nchunks = rows * (kTileN / 8);
    float* stile = reinterpret_cast<float*>(smem);
    uint64_t t1 = 0, t2 = 0, t3 = 0;
    if (32 * q < rows) {  // warp-uniform: tcgen05.ld is a warp-collective instruction
      for (int c0 = 0; c0 < kTileN; c0 += 16) {
        float v[16];
        pm::tmem_ld16(trow + c0, v);
        float* dst = stile + r * kSRow + c0;
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          *reinterpret_cast<float4*>(dst + j) = ok ? make_float4(v[j], v[j + 1], v[j + 2], v[j + 3])
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    epi_sync();
    // 1. this CTA's fp32 partial -> local slot ks; every split CTA of the tile then owns one column
    //    slice of width 256 / S for the rest of the epilogue (split sum, NVLink push, rank reduction)
    float* lpart = reinterpret_cast<float*>(sym.base(c.rank) + c.lpart_off);
    {
      float* lp = lpart + (int64_t)ks * c.recv_elems;
      for (int id = et; id < nchunks; id += 128) {
        const int row = id / (kTileN / 8), col = (id % (kTileN / 8)) * 8;
        const int64_t off = (int64_t)(b0 + row) * p.N + n0 + col;
        const float* src = stile + row * kSRow + col;
        *reinterpret_cast<float4*>(lp + off) = *reinterpret_cast<const float4*>(src);
        *reinterpret_cast<float4*>(lp + off + 4) = *reinterpret_cast<const float4*>(src + 4);
      }
    }
    epi_sync();
    if (et == 0) st_release_gpu(sym.flag_rs(c.rank, c.world + ks, tm), s);
    if (et < p.S && !wait_flag(sym.flag_rs(c.rank, c.world + et, tm), s, c.timeout_ns))
      pm::report_error(c.err, pm::kPeerTimeout, 330 + et);
    epi_sync();
    if (p.prof && et == 0) t1 = pm::globaltimer_ns();
    const int sw = kTileN / p.S;            // slice width (a multiple of 8)
    const int sc = sw / 8;                  // 8-column chunks per slice row
    const int slice = tm * p.S + ks;        // flag index of this slice
    const int owner = slice % c.world;
    const int nsl = rows * sc;
    // 2. split sum (fp32, split order) -> bf16 partial of this rank -> destination(s)
    const int d_lo = p.one_shot ? 0 : owner, d_hi = p.one_shot ? c.world : owner + 1;
    for (int id = et; id < nsl; id += 128) {
      const int row = id / sc, col = ks * sw + (id % sc) * 8;
      const int64_t off = (int64_t)(b0 + row) * p.N + n0 + col;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
      for (int k2 = 0; k2 < p.S; ++k2) {
        const float* lp = lpart + (int64_t)k2 * c.recv_elems + off;
        const float4 x = __ldcg(reinterpret_cast<const float4*>(lp)), y = __ldcg(reinterpret_cast<const float4*>(lp + 4));
        a.x += x.x; a.y += x.y; a.z += x.z; a.w += x.w;
        b.x += y.x; b.y += y.y; b.z += y.z; b.w += y.w;
      }
      const uint4 o = make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w), pack_bf16(b.x, b.y), pack_bf16(b.z, b.w));
      for (int d = d_lo; d < d_hi; ++d) *reinterpret_cast<uint4*>(sym.recv(d, c.rank, s) + off) = o;
    }
    epi_sync();
    if (et < d_hi - d_lo) st_release_sys(sym.flag_rs(d_lo + et, c.rank, slice), s);
    if (p.prof && et == 0) t2 = pm::globaltimer_ns();
    // 3. reduce the slice over ranks in rank order (every rank computes identical bits)
    if (p.one_shot || c.rank == owner) {
      if (et < c.world && !wait_flag(sym.flag_rs(c.rank, et, slice), s, c.timeout_ns))
        pm::report_error(c.err, pm::kPeerTimeout, 310 + et);
      epi_sync();
      for (int id = et; id < nsl; id += 128) {
        const int64_t off = (int64_t)(b0 + id / sc) * p.N + n0 + ks * sw + (id % sc) * 8;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int sr = 0; sr < c.world; ++sr) add_bf16x8(acc, __ldcg(reinterpret_cast<const uint4*>(sym.recv(c.rank, sr, s) + off)));
        const uint4 o = pack8(acc);
        if (p.one_shot) {
          *reinterpret_cast<uint4*>(p.out + off) = o;
        } else {
          for (int d = 0; d < c.world; ++d) *reinterpret_cast<uint4*>(sym.gath(d) + off) = o;
        }
      }
      if (!p.one_shot) {
        epi_sync();
        if (et < c.world) st_release_sys(sym.flag_ag(et, slice), s);
      }
    }
    if (!p.one_shot) {
      // 4. two-shot: every rank copies the gathered slice out
      if (et == 0 && !wait_flag(sym.flag_ag(c.rank, slice), s, c.timeout_ns))
        pm::report_error(c.err, pm::kPeerTimeout, 309);
      epi_sync();
      for (int id = et; id < nsl; id += 128) {
        const int64_t off = (int64_t)(b0 + id / sc) * p.N + n0 + ks * sw + (id % sc) * 8;
        *reinterpret_cast<uint4*>(p.out + off) = __ldcg(reinterpret_cast<const uint4*>(sym.gath(c.rank) + off));
      }
    }
    if (p.prof && et == 0) {
      t3 = pm::globaltimer_ns();
      atomicAdd(p.prof + 0, (unsigned long long)(t1 - t0));
      atomicAdd(p.prof + 1, (unsigned long long)(t2 - t1));
      atomicAdd(p.prof + 2, (unsigned long long)(t3 - t2));
      atomicAdd(p.prof + 3, 1ull);
      atomicMax(p.prof + 4, (unsigned long long)(t3 - t0));
    }
  }
  pm::tc_fence_before();
  finish_epoch(c, s);  // contains __syncthreads
  pm::tc_fence_after();
  if (warp == 0) pm::tmem_dealloc(tmem, kTileN);
}

// ----------------------------------------------------------------------------- all-reduce
__global__ void __launch_bounds__(256) allreduce_kernel(const ArParams p) {
  const SymmComm& c = p.c;
  const Sym sym(c);
  const int t = blockIdx.x, owner = t % c.world;
  const uint32_t s = *reinterpret_cast<volatile const uint32_t*>(c.epoch) + 1;
  const int64_t lo = (int64_t)t * p.chunk, hi = min(p.n, lo + p.chunk);
  const int d_lo = p.one_shot ? 0 : owner, d_hi = p.one_shot ? c.world : owner + 1;
  // 1. local addends -> recv[rank] of the destination(s)
  for (int64_t i = lo + 8 * threadIdx.x; i < hi; i += 8 * blockDim.x) {
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (p.a) add_bf16x8(v, *reinterpret_cast<const uint4*>(p.a + i));
    if (p.f) {
      const float4 f0 = *reinterpret_cast<const float4*>(p.f + i), f1 = *reinterpret_cast<const float4*>(p.f + i + 4);
      v[0] += f0.x; v[1] += f0.y; v[2] += f0.z; v[3] += f0.w;
      v[4] += f1.x; v[5] += f1.y; v[6] += f1.z; v[7] += f1.w;
    }
    const uint4 o = pack8(v);
    for (int d = d_lo; d < d_hi; ++d) *reinterpret_cast<uint4*>(sym.recv(d, c.rank, s) + i) = o;
  }
  __syncthreads();
  if ((int)threadIdx.x < d_hi - d_lo) st_release_sys(sym.flag_rs(d_lo + threadIdx.x, c.rank, t), s);
  // 2. reduce over ranks in rank order: every rank (one-shot) or the owner (two-shot, then all-gather)
  if (p.one_shot || c.rank == owner) {
    if ((int)threadIdx.x < c.world && !wait_flag(sym.flag_rs(c.rank, threadIdx.x, t), s, c.timeout_ns))
      pm::report_error(c.err, pm::kPeerTimeout, 320 + threadIdx.x);
    __syncthreads();
    for (int64_t i = lo + 8 * threadIdx.x; i < hi; i += 8 * blockDim.x) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int sr = 0; sr < c.world; ++sr) add_bf16x8(acc, __ldcg(reinterpret_cast<const uint4*>(sym.recv(c.rank, sr, s) + i)));
      const uint4 o = pack8(acc);
      if (p.one_shot) {
        *reinterpret_cast<uint4*>(p.out + i) = o;
      } else {
        for (int d = 0; d < c.world; ++d) *reinterpret_cast<uint4*>(sym.gath(d) + i) = o;
      }
    }
    if (!p.one_shot) {
      __syncthreads();
      if ((int)threadIdx.x < c.world) st_release_sys(sym.flag_ag(threadIdx.x, t), s);
    }
  }
  if (!p.one_shot) {
    // 3. two-shot: gathered chunk -> out
    if (threadIdx.x == 0 && !wait_flag(sym.flag_ag(c.rank, t), s, c.timeout_ns))
      pm::report_error(c.err, pm::kPeerTimeout, 319);
    __syncthreads();
    const __nv_bfloat16* g = sym.gath(c.rank);
    for (int64_t i = lo + 8 * threadIdx.x; i < hi; i += 8 * blockDim.x)
      *reinterpret_cast<uint4*>(p.out + i) = __ldcg(reinterpret_cast<const uint4*>(g + i));
  }
  finish_epoch(c, s);
}
}  // namespace

int gemm_ar_smem_bytes(int stages) { return stages * kStageBytes + 1024 + 256; }

int launch_gemm_allreduce(const GemmArParams& p, const void* w, const void* x, int num_sms, cudaStream_t stream) {
  if (p.B < 1 || p.B > 128 * p.nmb || p.nmb < 1 || p.nmb > 4 || p.N % kTileN || p.S < 1 || p.K % (64 * p.S) ||
      p.stages < 2 || p.stages > kMaxStages || p.stages * kStageBytes < 128 * kSRow * 4)
    return 1;
  const int ntm = p.N / kTileN * p.nmb;
  if (ntm * p.S > num_sms || ntm * p.S > p.c.max_tiles || p.c.world + p.S > p.c.max_src || kTileN % (8 * p.S) ||
      (int64_t)p.N * p.B > p.c.recv_elems)
    return 2;
  alignas(64) CUtensorMap mw, mx;
  if (make_tmap_bf16_sw128(&mw, w, p.K, p.N, (uint64_t)p.K * 2, kTileN)) return 3;
  if (make_tmap_bf16_sw128(&mx, x, p.K, p.B, (uint64_t)p.K * 2, 128)) return 3;
  const int smem = gemm_ar_smem_bytes(p.stages);
  cudaFuncSetAttribute(gemm_ar_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  gemm_ar_kernel<<<ntm * p.S, kThreads, smem, stream>>>(mw, mx, p);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

int launch_allreduce(const ArParams& p, int num_sms, cudaStream_t stream) {
  if (p.n % 8 || p.chunk % 8 || p.chunk <= 0) return 1;
  const int64_t ntiles = (p.n + p.chunk - 1) / p.chunk;
  if (ntiles > num_sms || ntiles > p.c.max_tiles || p.c.world > p.c.max_src || p.n > p.c.recv_elems) return 2;
  allreduce_kernel<<<(int)ntiles, 256, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
