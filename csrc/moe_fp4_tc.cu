// MXFP4 routed experts on tcgen05 with the weight operand in tensor memory.
//
// Reference behaviour: FlashInfer `Mxfp4FlashinferCutlassMoEMethod`, which also re-lays out
// the MXFP4 experts at load time ("Preparing DSv4 MXFP4 experts" in the serve log).  Weights are
// E2M1 nibbles (low nibble = even k) with one UE8M0 scale per 32 k; activations BF16 (FP16 here).
//
// Kernel weight layout (packmla/ops/moe.py: tile_fp4): per expert, tiles of 128 rows x 256 k:
//   w_t[e][rt][kt][row][128 B]  with the 16-byte units of each row XOR-swizzled by (row % 8)
//   s_t[e][rt][kt][row][8 B]    UE8M0 scales of the tile's 8 k-blocks
// For gate/up, row tile rt holds gate rows [64 rt, 64 rt + 64) followed by the matching up rows.
//
// Token rows use a padded per-expert "slot" layout: expert e's routed tokens occupy padded rows
// [pad[e], pad[e] + n_e) with pad[e] a multiple of 16, stored as groups of 16 rows:
//   xs[row / 16][k / 64][row % 16][64 fp16]  (16-byte units XOR-swizzled by row % 8)
// so the B operand of one (16-token pass, 256-k tile) is a single contiguous 8 KB block.
//
// Persistent CTAs (one per SM), 22 warps:
//   warp 17 (loader):    cp.async.bulk of the 16 KB weight tile, 1 KB scale tile and 8 KB token
//                        tile into an 8-stage shared ring (mbarrier complete_tx).
//   warps 0-15 (convert): thread (warp w, lane l) owns TMEM lane 32 (w % 4) + l (= weight row) and
//                        k-quarter w / 4: E2M1 -> FP16 x 2^(scale - 127 + 8) with cvt.rn.f16x2.e2m1x2,
//                        tcgen05.st into one of 3 TMEM A stages.
//   warp 16 (MMA):       16 x tcgen05.mma kind::f16 (M=128, N=16, K=16, A from TMEM) per tile,
//                        spread over 4 independent accumulators so the chain is 4 deep, into one
//                        of 2 accumulator sets (double-buffered across passes).
//   warps 18-21 (epilogue): sum the 4 accumulators, x 2^-8; gate/up -> silu(gate) * up written as
//                        FP16 token rows of the down pass; down -> routed-weight scatter-add (FP32).
//                        Runs concurrently with the next pass's stream (no pipeline drain).
// Tokens beyond 16 for one expert are processed in further passes over the same weights.
#include "launchers.h"
#include "common/sm100.cuh"

namespace {

constexpr int kConvWarps = 16;
constexpr int kMmaWarp = 16;
constexpr int kLoadWarp = 17;
constexpr int kThreads = 32 * 22;
constexpr int kKT = 256;                   // k per tile
constexpr int kN = 16;                     // tokens per pass (MMA N)
constexpr int kNS = 8;                     // ring stages
constexpr int kAS = 3;                     // TMEM A stages (128 columns each)
constexpr int kAcc = 4;                    // independent accumulators per pass
constexpr int kScaleBias = 8;              // weights staged as value * 2^8 in FP16
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemD = kAS * 128;     // D sets at [384, 448) and [448, 512)

constexpr int kRawB = kN * kKT * 2;        // 8 KB token tile (B operand), first: 1024-aligned
constexpr int kRawW = 128 * 128;           // 16 KB weight tile
constexpr int kRawS = 128 * 8;             // 1 KB scale tile
constexpr int kRawStage = kRawB + kRawW + kRawS;   // 25 KB (multiple of 1024)
constexpr int kOffRaw = 0;
constexpr int kOffUp = kOffRaw + kNS * kRawStage;
constexpr int kOffBar = kOffUp + kN * 64 * 4;      // upbuf [kN][64] floats
constexpr int kNumBars = 2 * kNS + 2 * kAS + 4;    // ring full/empty, A full/empty, D full[2]/free[2]
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmem = kOffMisc + 64 + 1024;

struct TcParams {
  const __half* xs;        // padded token rows (B operand source)
  __half* act_s;           // gate_up output: padded token rows of the down pass
  int K, R, I, mode, H;
  const uint8_t* w;        // tiled weights
  const uint8_t* s;        // tiled scales
  const int32_t* offsets;  // [E + 1] slot offsets
  const int32_t* pad;      // [E + 1] padded row offsets (multiples of 16)
  const int32_t* slot_token;
  const float* slot_weight;
  const int32_t* active;
  float* out;
  int* err;
  int debug;  // diagnostics only: bit0 skips the MMAs, bit1 skips dequantization + tcgen05.st
};

__device__ __forceinline__ void bar_sync_epi() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

__device__ __forceinline__ void dequant8(uint32_t w, __half2 sc2, uint32_t* o) {
  uint32_t r0, r1, r2, r3;
  asm("{\n\t.reg .b8 a, b, c, d;\n\t"
      "mov.b32 {a, b, c, d}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, a;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, c;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, d;\n\t}"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(w));
  const uint32_t rr[4] = {r0, r1, r2, r3};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __hmul2(*reinterpret_cast<const __half2*>(&rr[i]), sc2);
    o[i] = *reinterpret_cast<uint32_t*>(&h);
  }
}

// Byte offset of (padded row, k) in the padded token layout of row length K (fp16).
__device__ __forceinline__ size_t xs_offset(int row, int k, int K) {
  const int g = row >> 4, r16 = row & 15, c = k >> 6, u = (k >> 3) & 7;
  return ((((size_t)g * (K >> 6) + c) * 16 + r16) * 128) + (size_t)((u ^ (r16 & 7)) << 4) + (size_t)((k & 7) << 1);
}

__global__ void __launch_bounds__(kThreads, 1) moe_fp4_tc_kernel(const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* raw_empty = raw_full + kNS;
  uint64_t* a_full = raw_empty + kNS;
  uint64_t* a_empty = a_full + kAS;
  uint64_t* d_full = a_empty + kAS;  // [2]
  uint64_t* d_free = d_full + 2;     // [2]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 8);
  float* upbuf = reinterpret_cast<float*>(smem + kOffUp);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (warp == 0) {
    pm::tmem_alloc(tslot, kTmemCols);
    pm::tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < kNS; ++i) {
      pm::mbar_init(&raw_full[i], 1);
      pm::mbar_init(&raw_empty[i], kConvWarps + 1);  // converter warps + the MMA commit (B tile read)
    }
    for (int i = 0; i < kAS; ++i) {
      pm::mbar_init(&a_full[i], kConvWarps);
      pm::mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      pm::mbar_init(&d_full[i], 1);
      pm::mbar_init(&d_free[i], 4);  // epilogue warps
    }
    pm::fence_mbar_init();
    *abort_flag = 0;
  }
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  const uint32_t tmem = *tslot;

  const int nrt = p.R / 128;
  const int items = p.active[0] * nrt;
  const int ktiles = p.K / kKT;
  uint32_t g_tile = 0, g_pass = 0;
  const uint32_t idesc = pm::make_idesc_f16(128, kN, 0, 0, 0);

  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int e = p.active[1 + it / nrt];
    const int rt = it % nrt;
    const int lo = p.offsets[e], hi = p.offsets[e + 1];
    const int pad0 = p.pad[e];
    const uint8_t* Wt = p.w + ((size_t)e * nrt + rt) * ktiles * kRawW;
    const uint8_t* St = p.s + ((size_t)e * nrt + rt) * ktiles * kRawS;
    for (int s0 = lo; s0 < hi; s0 += kN) {
      const int nt = min(kN, hi - s0);
      const int prow = pad0 + (s0 - lo);  // padded row of this pass's first token (multiple of 16)
      const int dset = g_pass & 1;
      if (warp == kLoadWarp) {
        // ---------------- loader
        if (lane == 0) {
          for (int kt = 0; kt < ktiles; ++kt) {
            const uint32_t g = g_tile + kt;
            const int st = g % kNS;
            if (g >= (uint32_t)kNS && !pm::mbar_wait(&raw_empty[st], ((g / kNS) - 1) & 1, p.err, 30)) {
              *abort_flag = 1;
              break;
            }
            if (*abort_flag) break;
            uint8_t* dst = smem + kOffRaw + st * kRawStage;
            pm::mbar_arrive_expect_tx(&raw_full[st], kRawStage);
            pm::bulk_g2s(dst, reinterpret_cast<const uint8_t*>(p.xs) + xs_offset(prow, kt * kKT, p.K), kRawB,
                         &raw_full[st]);
            pm::bulk_g2s(dst + kRawB, Wt + (size_t)kt * kRawW, kRawW, &raw_full[st]);
            pm::bulk_g2s(dst + kRawB + kRawW, St + (size_t)kt * kRawS, kRawS, &raw_full[st]);
          }
        }
        __syncwarp();
      } else if (warp < kConvWarps) {
        // ---------------- converters: lane quarter q4, k-quarter kq (64 k = 32 TMEM columns)
        const int q4 = warp & 3, kq = warp >> 2;
        const int lrow = 32 * q4 + lane;
        for (int kt = 0; kt < ktiles; ++kt) {
          const uint32_t g = g_tile + kt;
          const int rs = g % kNS, st = g % kAS;
          if (*abort_flag) break;
          if (!pm::mbar_wait(&raw_full[rs], (g / kNS) & 1, p.err, 31)) { *abort_flag = 1; break; }
          if (g >= (uint32_t)kAS && !pm::mbar_wait(&a_empty[st], ((g / kAS) - 1) & 1, p.err, 32)) {
            *abort_flag = 1;
            break;
          }
          const uint8_t* raw = smem + kOffRaw + rs * kRawStage + kRawB;
          const uint32_t sc2w = *reinterpret_cast<const uint16_t*>(raw + kRawW + lrow * 8 + kq * 2);
          uint4 wq[2];
#pragma unroll
          for (int c = 0; c < 2; ++c)
            wq[c] = *reinterpret_cast<const uint4*>(raw + lrow * 128 + (((kq * 2 + c) ^ (lrow & 7)) << 4));
          __syncwarp();
          if (lane == 0) pm::mbar_arrive(&raw_empty[rs]);
          const uint32_t col0 = st * 128 + kq * 32;
#pragma unroll
          for (int c = 0; c < 2 && !(p.debug & 2); ++c) {
            const int sexp = (int)((sc2w >> (8 * c)) & 0xFF) - 127 + kScaleBias;
            const __half2 sc2 = __float2half2_rn(pm::exp2i(sexp));
            uint32_t cols[16];
            dequant8(wq[c].x, sc2, cols + 0);
            dequant8(wq[c].y, sc2, cols + 4);
            dequant8(wq[c].z, sc2, cols + 8);
            dequant8(wq[c].w, sc2, cols + 12);
            pm::tmem_st16u(tmem + col0 + 16 * c + ((uint32_t)(32 * q4) << 16), cols);
          }
          pm::tmem_wait_st();
          pm::tc_fence_before();
          __syncwarp();
          if (lane == 0) pm::mbar_arrive(&a_full[st]);
        }
      } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer
        if (lane == 0) {
          bool ok = !*abort_flag;
          if (ok && g_pass >= 2 && !pm::mbar_wait(&d_free[dset], ((g_pass >> 1) - 1) & 1, p.err, 34)) {
            *abort_flag = 1;
            ok = false;
          }
          pm::tc_fence_after();
          const uint32_t dbase = tmem + kTmemD + dset * (kAcc * kN);
          for (int kt = 0; kt < ktiles && ok; ++kt) {
            const uint32_t g = g_tile + kt;
            const int st = g % kAS, rs = g % kNS;
            if (!pm::mbar_wait(&a_full[st], (g / kAS) & 1, p.err, 35)) { *abort_flag = 1; break; }
            pm::tc_fence_after();
            const uint32_t b0 = pm::smem_u32(smem + kOffRaw + rs * kRawStage);
#pragma unroll
            for (int j = 0; j < kKT / 16 && !(p.debug & 1); ++j) {
              const uint64_t bd = pm::make_sdesc(b0 + (j >> 2) * (kN * 128) + ((j * 32) & 127), 16, 1024);
              pm::umma_f16_tmem_a(dbase + (j % kAcc) * kN, tmem + st * 128 + 8 * j, bd, idesc,
                                  (kt > 0 || j >= kAcc) ? 1u : 0u);
            }
            pm::umma_commit(&a_empty[st]);
            pm::umma_commit(&raw_empty[rs]);
          }
          pm::umma_commit(&d_full[dset]);
        }
        __syncwarp();
      } else {
        // ---------------- epilogue (warps 18-21: lane quarter warp % 4)
        const int q = warp & 3;
        const int lrow = 32 * q + lane;
        bool ok = !*abort_flag && pm::mbar_wait(&d_full[dset], (g_pass >> 1) & 1, p.err, 33);
        if (!ok) *abort_flag = 1;
        pm::tc_fence_after();
        float d[kN];
#pragma unroll
        for (int i = 0; i < kN; ++i) d[i] = 0.f;
        if (ok) {
#pragma unroll
          for (int a = 0; a < kAcc; ++a) {
            float t[16];
            pm::tmem_ld16(tmem + kTmemD + dset * (kAcc * kN) + a * kN + ((uint32_t)(32 * q) << 16), t);
#pragma unroll
            for (int i = 0; i < kN; ++i) d[i] += t[i];
          }
        }
        pm::tc_fence_before();
        __syncwarp();
        if (lane == 0) pm::mbar_arrive(&d_free[dset]);  // accumulators read: the next-but-one pass may write
        const float unscale = pm::exp2i(-kScaleBias);
        if (p.mode == 0) {
          if (lrow >= 64) {
#pragma unroll
            for (int i = 0; i < kN; ++i) upbuf[i * 64 + (lrow - 64)] = d[i] * unscale;
          }
          bar_sync_epi();
          if (ok && lrow < 64) {
            const int k = rt * 64 + lrow;  // activation column
#pragma unroll
            for (int t = 0; t < kN; ++t) {
              if (t < nt) {
                const float gv = d[t] * unscale;
                const float a = gv / (1.f + __expf(-gv)) * upbuf[t * 64 + lrow];
                *reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(p.act_s) + xs_offset(prow + t, k, p.I)) =
                    __float2half_rn(a);
              }
            }
          }
          bar_sync_epi();
        } else if (ok) {
#pragma unroll
          for (int t = 0; t < kN; ++t)
            if (t < nt)
              atomicAdd(p.out + (size_t)p.slot_token[s0 + t] * p.H + rt * 128 + lrow,
                        p.slot_weight[s0 + t] * d[t] * unscale);
        }
      }
      g_tile += ktiles;
      ++g_pass;
    }
  }
  pm::tc_fence_before();
  __syncthreads();
  if (warp == 0) pm::tmem_dealloc(tmem, kTmemCols);
}

// Gather the routed token rows (bf16) into the padded fp16 slot layout.
__global__ void moe_gather_slots_kernel(const __nv_bfloat16* __restrict__ x, int K, const int32_t* __restrict__ offsets,
                                        const int32_t* __restrict__ pad, const int32_t* __restrict__ slot_token, int E,
                                        __half* __restrict__ xs) {
  const int units = K / 8;
  const int n = offsets[E];
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < n * units; idx += gridDim.x * blockDim.x) {
    const int slot = idx / units, u = idx % units;
    int lo = 0, hi = E;  // expert of this slot: offsets[lo] <= slot < offsets[lo + 1]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (offsets[mid] <= slot) lo = mid; else hi = mid;
    }
    const int row = pad[lo] + (slot - offsets[lo]);
    const uint4 v = *reinterpret_cast<const uint4*>(x + (size_t)slot_token[slot] * K + 8 * u);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
    __half2 h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(b[i]);
      h[i] = __floats2half2_rn(f.x, f.y);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(xs) + xs_offset(row, 8 * u, K)) =
        *reinterpret_cast<uint4*>(h);
  }
}

}  // namespace

void launch_moe_gather_slots(const __nv_bfloat16* x, int K, const int32_t* offsets, const int32_t* pad,
                             const int32_t* slot_token, int E, __half* xs, int num_sms, cudaStream_t stream) {
  moe_gather_slots_kernel<<<num_sms * 4, 256, 0, stream>>>(x, K, offsets, pad, slot_token, E, xs);
}

void launch_moe_fp4_tc(const __nv_bfloat16* x, int T, int H, int I, int E, int max_slots, const int32_t* offsets,
                       const int32_t* pad, const int32_t* slot_token, const float* slot_weight, const int32_t* active,
                       const uint8_t* w13t, const uint8_t* s13t, const uint8_t* w2t, const uint8_t* s2t, __half* xs,
                       __half* act_s, float* out, int num_sms, int* err, int debug, cudaStream_t stream) {
  if (T == 0) return;
  launch_moe_gather_slots(x, H, offsets, pad, slot_token, E, xs, num_sms, stream);
  cudaFuncSetAttribute(moe_fp4_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  TcParams gu{xs, act_s, H, 2 * I, I, 0, H, w13t, s13t, offsets, pad, slot_token, slot_weight, active, out, err, debug};
  moe_fp4_tc_kernel<<<num_sms, kThreads, kSmem, stream>>>(gu);
  TcParams dn{act_s, act_s, I, H, I, 1, H, w2t, s2t, offsets, pad, slot_token, slot_weight, active, out, err, debug};
  moe_fp4_tc_kernel<<<num_sms, kThreads, kSmem, stream>>>(dn);
}
