// MXFP4 routed experts for decode-sized token counts (<= 16 tokens per expert per pass).
//
// Reference behaviour: FlashInfer `Mxfp4FlashinferCutlassMoEMethod`.  At decode batch sizes
// an expert sees ~1-4 tokens, so the layer is a stream of the active experts' E2M1 weights.  This
// is the BF16-activation variant (expert_format "bf16"); the default MXFP8 x MXFP4 block-scaled
// tcgen05 kernel is csrc/moe_mxf4.cu.  Here the weights are dequantized straight into register A
// fragments of m16n8k16 MMAs, so each weight byte is touched once after landing in shared memory.
//
// Weight layout (packmla/ops/moe.py: tile_fp4_frag), per tile of 128 rows x 256 k (16 KB + 1 KB):
//   warp (k-slice ks in 0..3 = 64 k, row half rh = 64 rows) owns 4 m16 tiles x 4 k16 steps;
//   weights [ks][rh][mt][lane][16 B]: for k16 step s, bytes 4 s .. 4 s + 3 are the E2M1 pairs
//     (row g, k 2q) (row g + 8, k 2q) (row g, k 2q + 8) (row g + 8, k 2q + 8)  (g = lane / 4,
//     q = lane % 4, k relative to the step) -- exactly the A fragment a0..a7 after cvt.e2m1x2;
//   scales  [ks][rh][g][mt][block][2 B]: UE8M0 of rows (g, g + 8) for the two 32-k blocks.
// Token rows: padded per-expert slots gathered by moe_gather_slots_kernel (8 KB per 16-token, 256-k tile).
//
// CTA = 8 MMA warps + 1 loader warp (cp.async.bulk ring of 6 stages x 25 KB).  Per pass the
// warps' K-slice partials (4 x [128 rows x 16 tokens]) are summed through shared memory; gate/up
// passes write silu(gate) * up as the down pass's token rows, down passes scatter-add
// weight * y into the FP32 output.
#include "launchers.h"
#include "common/sm100.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kLoadWarp = 8;
constexpr int kThreads = 32 * (kWarps + 1);
constexpr int kKT = 256;
constexpr int kN = 16;
constexpr int kNS = 6;
constexpr int kScaleBias = 8;
constexpr int kRawB = kN * kKT * 2;                 // 8 KB token tile
constexpr int kRawW = 128 * 128;                    // 16 KB weight tile
constexpr int kRawS = 128 * 8;                      // 1 KB scales
constexpr int kRawStage = kRawB + kRawW + kRawS;    // 25 KB
constexpr int kOffRaw = 0;
constexpr int kOffRed = kOffRaw + kNS * kRawStage;  // float red[4][128][16] = 32 KB
constexpr int kOffBar = kOffRed + 4 * 128 * kN * 4;
constexpr int kOffMisc = kOffBar + 2 * kNS * 8;
constexpr int kSmem = kOffMisc + 64 + 1024;

struct MmaParams {
  const __half* xs;
  __half* act_s;
  int K, R, I, mode, H;
  const uint8_t* w;  // fragment-ordered tiles
  const uint8_t* s;
  const int32_t* offsets;
  const int32_t* pad;
  const int32_t* slot_token;
  const float* slot_weight;
  const int32_t* active;
  float* out;
  int* err;
};

__device__ __forceinline__ size_t xs_offset(int row, int k, int K) {
  const int g = row >> 4, r16 = row & 15, c = k >> 6, u = (k >> 3) & 7;
  return ((((size_t)g * (K >> 6) + c) * 16 + r16) * 128) + (size_t)((u ^ (r16 & 7)) << 4) + (size_t)((k & 7) << 1);
}

__device__ __forceinline__ void bar_sync_mma() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// a[0..3] = fp16x2 A fragment registers of one k16 step from 4 E2M1 bytes, scaled by (s_g, s_g8).
__device__ __forceinline__ void frag_a(uint32_t w, __half2 sg, __half2 sg8, uint32_t (&a)[4]) {
  uint32_t r0, r1, r2, r3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(w));
  __half2 h0 = __hmul2(*reinterpret_cast<__half2*>(&r0), sg);
  __half2 h1 = __hmul2(*reinterpret_cast<__half2*>(&r1), sg8);
  __half2 h2 = __hmul2(*reinterpret_cast<__half2*>(&r2), sg);
  __half2 h3 = __hmul2(*reinterpret_cast<__half2*>(&r3), sg8);
  a[0] = *reinterpret_cast<uint32_t*>(&h0);
  a[1] = *reinterpret_cast<uint32_t*>(&h1);
  a[2] = *reinterpret_cast<uint32_t*>(&h2);
  a[3] = *reinterpret_cast<uint32_t*>(&h3);
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(kThreads, 1) moe_fp4_mma_kernel(const MmaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* empty = full + kNS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc);
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kNS; ++i) {
      pm::mbar_init(&full[i], 1);
      pm::mbar_init(&empty[i], kWarps);
    }
    pm::fence_mbar_init();
    *abort_flag = 0;
  }
  __syncthreads();
  const int nrt = p.R / 128;
  const int items = p.active[0] * nrt;
  const int ktiles = p.K / kKT;
  uint32_t g_tile = 0;
  const int ks = warp & 3, rh = warp >> 2;  // k-slice (64 k) and row half (64 rows)
  const int g = lane >> 2, q = lane & 3;

  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int e = p.active[1 + it / nrt];
    const int rt = it % nrt;
    const int lo = p.offsets[e], hi = p.offsets[e + 1];
    const int pad0 = p.pad[e];
    const uint8_t* Wt = p.w + ((size_t)e * nrt + rt) * ktiles * kRawW;
    const uint8_t* St = p.s + ((size_t)e * nrt + rt) * ktiles * kRawS;
    for (int s0 = lo; s0 < hi; s0 += kN) {
      const int nt = min(kN, hi - s0);
      const int prow = pad0 + (s0 - lo);
      if (warp == kLoadWarp) {
        if (lane == 0) {
          for (int kt = 0; kt < ktiles; ++kt) {
            const uint32_t gt = g_tile + kt;
            const int st = gt % kNS;
            if (gt >= (uint32_t)kNS && !pm::mbar_wait(&empty[st], ((gt / kNS) - 1) & 1, p.err, 60)) {
              *abort_flag = 1;
              break;
            }
            if (*abort_flag) break;
            uint8_t* dst = smem + kOffRaw + st * kRawStage;
            pm::mbar_arrive_expect_tx(&full[st], kRawStage);
            pm::bulk_g2s(dst, reinterpret_cast<const uint8_t*>(p.xs) + xs_offset(prow, kt * kKT, p.K), kRawB, &full[st]);
            pm::bulk_g2s(dst + kRawB, Wt + (size_t)kt * kRawW, kRawW, &full[st]);
            pm::bulk_g2s(dst + kRawB + kRawW, St + (size_t)kt * kRawS, kRawS, &full[st]);
          }
        }
        __syncwarp();
      } else {
        float acc[4][2][4];
#pragma unroll
        for (int mt = 0; mt < 4; ++mt)
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[mt][j][i] = 0.f;
        for (int kt = 0; kt < ktiles; ++kt) {
          const uint32_t gt = g_tile + kt;
          const int st = gt % kNS;
          if (*abort_flag) break;
          if (!pm::mbar_wait(&full[st], (gt / kNS) & 1, p.err, 61)) { *abort_flag = 1; break; }
          const uint8_t* stage = smem + kOffRaw + st * kRawStage;
          // B fragments: token n = lane / 4 (+ 8 j), k = 16 s + 2 q (+ 8); chunk ks of the SW128 token tile.
          // The second n8 tile (tokens 8..15) is skipped when the pass has at most 8 tokens.
          const bool two = nt > 8;
          uint32_t bfr[4][2][2];
#pragma unroll
          for (int s = 0; s < 4; ++s)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              if (j == 1 && !two) { bfr[s][1][0] = bfr[s][1][1] = 0u; continue; }
              const int n = g + 8 * j;
              const int k0 = 16 * s + 2 * q;  // within the 64-k chunk
              const uint8_t* rowp = stage + ks * (kN * 128) + (n >> 3) * 1024 + (n & 7) * 128;
              bfr[s][j][0] = *reinterpret_cast<const uint32_t*>(rowp + ((((k0 >> 3) ^ (n & 7)) << 4) | ((k0 & 7) << 1)));
              const int k1 = k0 + 8;
              bfr[s][j][1] = *reinterpret_cast<const uint32_t*>(rowp + ((((k1 >> 3) ^ (n & 7)) << 4) | ((k1 & 7) << 1)));
            }
          const uint8_t* wbase = stage + kRawB + ((ks * 2 + rh) * 4) * 512;
          const uint4 sc = *reinterpret_cast<const uint4*>(stage + kRawB + kRawW + ((ks * 2 + rh) * 8 + g) * 16);
          const uint32_t scw[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
          for (int mt = 0; mt < 4; ++mt) {
            const uint4 wq = *reinterpret_cast<const uint4*>(wbase + mt * 512 + lane * 16);
            const uint32_t ws[4] = {wq.x, wq.y, wq.z, wq.w};
            // scale bytes of this m-tile: (block 0: row g, row g+8), (block 1: row g, row g+8)
            __half2 sg[2], sg8[2];
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
              sg[blk] = __float2half2_rn(pm::exp2i((int)((scw[mt] >> (16 * blk)) & 0xFF) - 127 + kScaleBias));
              sg8[blk] = __float2half2_rn(pm::exp2i((int)((scw[mt] >> (16 * blk + 8)) & 0xFF) - 127 + kScaleBias));
            }
#pragma unroll
            for (int s = 0; s < 4; ++s) {
              uint32_t a[4];
              frag_a(ws[s], sg[s >> 1], sg8[s >> 1], a);
              mma16816(acc[mt][0], a, bfr[s][0][0], bfr[s][0][1]);
              if (two) mma16816(acc[mt][1], a, bfr[s][1][0], bfr[s][1][1]);
            }
          }
          __syncwarp();
          if (lane == 0) pm::mbar_arrive(&empty[st]);
        }
        // K-slice partials -> shared: red[ks][row][token]
        const float unscale = pm::exp2i(-kScaleBias);
#pragma unroll
        for (int mt = 0; mt < 4; ++mt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int r0 = rh * 64 + mt * 16 + g;
            const int n0 = 8 * j + 2 * q;
            red[(ks * 128 + r0) * kN + n0] = acc[mt][j][0] * unscale;
            red[(ks * 128 + r0) * kN + n0 + 1] = acc[mt][j][1] * unscale;
            red[(ks * 128 + r0 + 8) * kN + n0] = acc[mt][j][2] * unscale;
            red[(ks * 128 + r0 + 8) * kN + n0 + 1] = acc[mt][j][3] * unscale;
          }
        bar_sync_mma();
        const bool ok = !*abort_flag;
        if (p.mode == 0) {
          // 64 gate rows x 16 tokens: thread -> (row r, tokens 4 m .. 4 m + 3)
          const int r = tid >> 2, tb = (tid & 3) * 4;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int t = tb + i;
            if (ok && t < nt) {
              float gv = 0.f, uv = 0.f;
#pragma unroll
              for (int k4 = 0; k4 < 4; ++k4) {
                gv += red[(k4 * 128 + r) * kN + t];
                uv += red[(k4 * 128 + 64 + r) * kN + t];
              }
              const float a = gv / (1.f + __expf(-gv)) * uv;
              const int k = rt * 64 + r;
              *reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(p.act_s) + xs_offset(prow + t, k, p.I)) =
                  __float2half_rn(a);
            }
          }
        } else {
          // 128 rows x 16 tokens: thread -> (row r, tokens 8 m .. 8 m + 7)
          const int r = tid >> 1, tb = (tid & 1) * 8;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int t = tb + i;
            if (ok && t < nt) {
              float y = 0.f;
#pragma unroll
              for (int k4 = 0; k4 < 4; ++k4) y += red[(k4 * 128 + r) * kN + t];
              atomicAdd(p.out + (size_t)p.slot_token[s0 + t] * p.H + rt * 128 + r, p.slot_weight[s0 + t] * y);
            }
          }
        }
        bar_sync_mma();
      }
      g_tile += ktiles;
    }
  }
  __syncthreads();
}

// Gather the routed token rows (bf16) into the padded fp16 slot layout of `xs_offset`.
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
void launch_moe_fp4_mma(const __nv_bfloat16* x, int T, int H, int I, int E, const int32_t* offsets, const int32_t* pad,
                        const int32_t* slot_token, const float* slot_weight, const int32_t* active, const uint8_t* w13f,
                        const uint8_t* s13f, const uint8_t* w2f, const uint8_t* s2f, __half* xs, __half* act_s,
                        float* out, int num_sms, int* err, cudaStream_t stream) {
  if (T == 0) return;
  launch_moe_gather_slots(x, H, offsets, pad, slot_token, E, xs, num_sms, stream);
  cudaFuncSetAttribute(moe_fp4_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  MmaParams gu{xs, act_s, H, 2 * I, I, 0, H, w13f, s13f, offsets, pad, slot_token, slot_weight, active, out, err};
  moe_fp4_mma_kernel<<<num_sms, kThreads, kSmem, stream>>>(gu);
  MmaParams dn{act_s, act_s, I, H, I, 1, H, w2f, s2f, offsets, pad, slot_token, slot_weight, active, out, err};
  moe_fp4_mma_kernel<<<num_sms, kThreads, kSmem, stream>>>(dn);
}
