// MXFP4 routed experts on tcgen05 with the weight operand in tensor memory.
//
// Reference behaviour: FlashInfer `Mxfp4FlashinferCutlassMoEMethod` (K18), which also re-lays out
// the MXFP4 experts at load time ("Preparing DSv4 MXFP4 experts" in the serve log).  Weights are
// E2M1 nibbles (low nibble = even k) with one UE8M0 scale per 32 k; activations BF16 (FP16 here).
//
// Kernel weight layout (packmla/ops/moe.py: tile_experts): per expert, tiles of 128 rows x 256 k:
//   w_t[e][rt][kt][row][128 B]  with the 16-byte units of each row XOR-swizzled by (row % 8)
//   s_t[e][rt][kt][row][8 B]    UE8M0 scales of the tile's 8 k-blocks
// For gate/up, row tile rt holds gate rows [64 rt, 64 rt + 64) followed by the matching up rows.
//
// Persistent CTAs (one per SM) of 10 warps walk items = (active local expert, row tile):
//   warp 9  (loader):    cp.async.bulk of each 16 KB weight tile + 1 KB scale tile into a
//                        4-stage shared ring (mbarrier complete_tx), bounded waits on free slots.
//   warps 0-7 (convert): thread (warp w, lane l) owns TMEM lane 32 (w % 4) + l (= weight row) and
//                        k-half w / 4: reads its 64 B from the ring, converts with
//                        cvt.rn.f16x2.e2m1x2 x 2^(scale - 127 + 8) (FP16), writes 64 columns of the
//                        double-buffered TMEM A operand with tcgen05.st, and stages the expert's
//                        token rows as the K-major 128-byte-swizzled B operand in shared memory.
//   warp 8  (MMA):       16 x tcgen05.mma kind::f16 (M=128, N=32, K=16, A from TMEM) per tile into
//                        the FP32 accumulator D, commits free the A/B stage.
//   epilogue (convert):  D * 2^-8; gate/up -> silu(gate) * up as BF16 activation rows; down ->
//                        routed-weight scatter-add into the FP32 output.
// Tokens beyond 32 for one expert are processed in further passes over the same weights.
#include "launchers.h"
#include "common/sm100.cuh"

namespace {

constexpr int kConvWarps = 16;             // converter warps 0-15
constexpr int kConv = 32 * kConvWarps;
constexpr int kThreads = kConv + 64;       // + MMA warp + loader warp
constexpr int kKT = 256;                   // k per tile
constexpr int kN = 16;                     // tokens per pass (MMA N)
constexpr int kNS = 8;                     // ring stages (~100 KB of weights in flight per SM)
constexpr int kAS = 3;                     // TMEM A stages (128 columns each)
constexpr int kScaleBias = 8;              // weights staged as value * 2^8 in FP16
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemD = kAS * 128;     // D columns [384, 384 + kN)

constexpr int kRawB = kN * kKT * 2;       // 8 KB token tile (B operand), first: 1024-aligned
constexpr int kRawW = 128 * 128;           // 16 KB weight tile
constexpr int kRawS = 128 * 8;             // 1 KB scale tile
constexpr int kRawStage = kRawB + kRawW + kRawS;   // 25 KB (multiple of 1024)
constexpr int kOffRaw = 0;
constexpr int kOffUp = kOffRaw + kNS * kRawStage;
constexpr int kOffBar = kOffUp + 64 * kN * 4;      // upbuf [kN][64] floats
constexpr int kNumBars = 2 * kNS + 2 * kAS + 2;    // ring full/empty, A full/empty, done, dfree
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmemUsed = kOffMisc + 64 + 1024;
constexpr int kSmem = kSmemUsed;  // > half of the SM: one CTA (one 512-column TMEM allocation) per SM

struct TcParams {
  const __half* xs;        // [slots, K] fp16 token rows per slot, 16-byte units of each 128-byte
                           // chunk XOR-swizzled by (slot position in its expert's list) % 8
  __half* act_s;           // gate_up output in the same slot layout (the down pass's xs)
  int K, R, I, mode, H;
  const uint8_t* w;        // tiled weights
  const uint8_t* s;        // tiled scales
  const int32_t* offsets;
  const int32_t* slot_token;
  const float* slot_weight;
  const int32_t* active;
  float* out;
  int* err;
  int debug;  // diagnostics only: bit0 skips the MMAs, bit1 skips dequantization + tcgen05.st,
              // bit2 skips the token-row copies, bit3 skips the weight/scale copies
};

__device__ __forceinline__ void bar_sync_conv() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

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

__global__ void __launch_bounds__(kThreads, 1) moe_fp4_tc_kernel(const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* raw_empty = raw_full + kNS;
  uint64_t* a_full = raw_empty + kNS;
  uint64_t* a_empty = a_full + kAS;
  uint64_t* done = a_empty + kAS;
  uint64_t* dfree = done + 1;
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
    pm::mbar_init(done, 1);
    pm::mbar_init(dfree, kConvWarps);
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
  const size_t tile_w = (size_t)kRawW, tile_s = (size_t)kRawS;
  uint32_t g_tile = 0, g_pass = 0;
  const uint32_t idesc = pm::make_idesc_f16(128, kN, 0, 0, 0);

  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int e = p.active[1 + it / nrt];
    const int rt = it % nrt;
    const int lo = p.offsets[e], hi = p.offsets[e + 1];
    const uint8_t* Wt = p.w + ((size_t)e * nrt + rt) * ktiles * tile_w;
    const uint8_t* St = p.s + ((size_t)e * nrt + rt) * ktiles * tile_s;
    for (int s0 = lo; s0 < hi; s0 += kN) {
      const int nt = min(kN, hi - s0);
      if (warp == kConvWarps + 1) {
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
            const bool cw = !(p.debug & 8), cb = !(p.debug & 4);
            pm::mbar_arrive_expect_tx(&raw_full[st], (cw ? kRawW + kRawS : 0) + (cb ? nt * kKT * 2 : 0));
            if (cw) {
              pm::bulk_g2s(dst + kRawB, Wt + kt * tile_w, kRawW, &raw_full[st]);
              pm::bulk_g2s(dst + kRawB + kRawW, St + kt * tile_s, kRawS, &raw_full[st]);
            }
            // token t, chunk c (64 k = 128 B) -> B tile row t (K-major SW128, chunk stride kN * 128)
            for (int j = 0; j < nt * 4 && cb; ++j) {
              const int t = j >> 2, c = j & 3;
              const __half* src = p.xs + (size_t)(s0 + t) * p.K + kt * kKT + 64 * c;
              pm::bulk_g2s(dst + c * (kN * 128) + (t >> 3) * 1024 + (t & 7) * 128, src, 128, &raw_full[st]);
            }
          }
        }
        __syncwarp();
      } else if (warp < kConvWarps) {
        // ---------------- converters: lane quarter q4, k-quarter kq (64 k = 32 TMEM columns)
        const int q4 = warp & 3, kq = warp >> 2;
        const int hh = kq;  // epilogue: warps 0-3 own the D columns
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
          // A: row lrow, k-half hh (64 B = 128 values) -> 64 TMEM columns
          const uint8_t* raw = smem + kOffRaw + rs * kRawStage + kRawB;
          const uint32_t sc2w = *reinterpret_cast<const uint16_t*>(raw + kRawW + lrow * 8 + kq * 2);
          uint4 wq[2];
#pragma unroll
          for (int c = 0; c < 2; ++c)
            wq[c] = *reinterpret_cast<const uint4*>(raw + lrow * 128 + (((kq * 2 + c) ^ (lrow & 7)) << 4));
          __syncwarp();
          if (lane == 0) pm::mbar_arrive(&raw_empty[rs]);
          const uint32_t col0 = st * 128 + kq * 32;  // A stage st: columns [128 st, 128 st + 128)
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
        // ---------------- epilogue
        bool ok = !*abort_flag;
        if (ok && !pm::mbar_wait(done, g_pass & 1, p.err, 33)) { *abort_flag = 1; ok = false; }
        pm::tc_fence_after();
        float d[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) d[i] = 0.f;
        if (ok && hh == 0) pm::tmem_ld16(tmem + kTmemD + ((uint32_t)(32 * q4) << 16), d);
        const float unscale = pm::exp2i(-kScaleBias);
        if (p.mode == 0) {
          if (lrow >= 64 && hh == 0) {
#pragma unroll
            for (int i = 0; i < kN; ++i) upbuf[i * 64 + (lrow - 64)] = d[i] * unscale;
          }
          bar_sync_conv();
          if (ok && lrow < 64 && hh == 0) {
#pragma unroll
            for (int i = 0; i < kN; ++i) {
              const int t = i;
              if (t < nt) {
                const float gv = d[i] * unscale;
                const float a = gv / (1.f + __expf(-gv)) * upbuf[t * 64 + lrow];
                // column k = 64 rt + lrow of slot s0 + t; slot position t: unit (k % 64) / 8 ^ (t % 8)
                const int k = rt * 64 + lrow;
                const int col = (k & ~63) | ((((k >> 3) & 7) ^ (t & 7)) << 3) | (k & 7);
                p.act_s[(size_t)(s0 + t) * p.I + col] = __float2half_rn(a);
              }
            }
          }
          bar_sync_conv();
        } else if (ok && hh == 0) {
#pragma unroll
          for (int i = 0; i < kN; ++i) {
            const int t = i;
            if (t < nt)
              atomicAdd(p.out + (size_t)p.slot_token[s0 + t] * p.H + rt * 128 + lrow,
                        p.slot_weight[s0 + t] * d[i] * unscale);
          }
        }
        pm::tc_fence_before();
        __syncwarp();
        if (lane == 0) pm::mbar_arrive(dfree);
      } else {
        // ---------------- MMA issuer (warp kConvWarps)
        if (lane == 0) {
          bool ok = !*abort_flag;
          if (ok && g_pass > 0 && !pm::mbar_wait(dfree, (g_pass - 1) & 1, p.err, 34)) { *abort_flag = 1; ok = false; }
          for (int kt = 0; kt < ktiles && ok; ++kt) {
            const uint32_t g = g_tile + kt;
            const int st = g % kAS;
            const int rs = g % kNS;
            if (!pm::mbar_wait(&a_full[st], (g / kAS) & 1, p.err, 35)) { *abort_flag = 1; break; }
            pm::tc_fence_after();
            const uint32_t b0 = pm::smem_u32(smem + kOffRaw + rs * kRawStage);
#pragma unroll
            for (int j = 0; j < kKT / 16 && !(p.debug & 1); ++j) {
              const uint64_t bd = pm::make_sdesc(b0 + (j >> 2) * (kN * 128) + ((j * 32) & 127), 16, 1024);
              pm::umma_f16_tmem_a(tmem + kTmemD, tmem + st * 128 + 8 * j, bd, idesc, (kt > 0 || j > 0) ? 1u : 0u);
            }
            pm::umma_commit(&a_empty[st]);
            pm::umma_commit(&raw_empty[rs]);
          }
          pm::umma_commit(done);
        }
        __syncwarp();
      }
      g_tile += ktiles;
      ++g_pass;
    }
  }
  pm::tc_fence_before();
  __syncthreads();
  if (warp == 0) pm::tmem_dealloc(tmem, kTmemCols);
}

// Gather the routed token rows into fp16 per-slot rows, swizzled for the B-tile bulk copies.
__global__ void moe_gather_slots_kernel(const __nv_bfloat16* __restrict__ x, int K, const int32_t* __restrict__ offsets,
                                        const int32_t* __restrict__ slot_token, const int32_t* __restrict__ active,
                                        int E, __half* __restrict__ xs) {
  const int units = K / 8;
  const int n = offsets[E];
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < n * units; idx += gridDim.x * blockDim.x) {
    const int slot = idx / units, u = idx % units;
    // slot position inside its expert's list: binary search on offsets
    int lo = 0, hi = E;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (offsets[mid] <= slot) lo = mid; else hi = mid;
    }
    const int t = slot - offsets[lo];
    const uint4 v = *reinterpret_cast<const uint4*>(x + (size_t)slot_token[slot] * K + 8 * u);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
    __half2 h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(b[i]);
      h[i] = __floats2half2_rn(f.x, f.y);
    }
    const int pu = (u & ~7) | ((u ^ t) & 7);
    *reinterpret_cast<uint4*>(xs + (size_t)slot * K + 8 * pu) = *reinterpret_cast<uint4*>(h);
  }
}

}  // namespace

void launch_moe_fp4_tc(const __nv_bfloat16* x, int T, int H, int I, int E, int max_slots, const int32_t* offsets,
                       const int32_t* slot_token, const float* slot_weight, const int32_t* active, const uint8_t* w13t,
                       const uint8_t* s13t, const uint8_t* w2t, const uint8_t* s2t, __half* xs, __half* act_s,
                       float* out, int num_sms, int* err, int debug, cudaStream_t stream) {
  if (T == 0) return;
  moe_gather_slots_kernel<<<num_sms * 4, 256, 0, stream>>>(x, H, offsets, slot_token, active, E, xs);
  cudaFuncSetAttribute(moe_fp4_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  TcParams gu{xs, act_s, H, 2 * I, I, 0, H, w13t, s13t, offsets, slot_token, slot_weight, active, out, err, debug};
  moe_fp4_tc_kernel<<<num_sms, kThreads, kSmem, stream>>>(gu);
  TcParams dn{act_s, act_s, I, H, I, 1, H, w2t, s2t, offsets, slot_token, slot_weight, active, out, err, debug};
  moe_fp4_tc_kernel<<<num_sms, kThreads, kSmem, stream>>>(dn);
}
