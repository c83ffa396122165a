// Dense projections with MXFP8 weights on the 5th-generation tensor cores.
//
// Reference behaviour: the reference serves V4-Flash's dense layers with FP8 E4M3 weights and FP8
// activations (SGLang's FP8 linear over DeepGEMM; `quant=fp8` in the serve logs it records).  Here the
// weights are MXFP8 (E4M3 codes, one UE8M0 scale per 32 values along K: Blackwell's native block-scaled
// format) and the activations are quantized per token to MXFP8 on the way in, so every projection is one
// tcgen05.mma kind::mxf8f6f4.block_scale stream with the scales applied inside the MMA.
//
//   1. quant (CTA per token row): x[b, t] BF16 -> E4M3 codes of the A operand image [b][K/128][Tp][128]
//      (16-byte units XOR-swizzled by row % 8) and the row's four scale bytes per 128-K group [b][K/128][Tp].
//   2. GEMM (persistent, one CTA per SM; unit = (batch, 256-row weight tile, 128-token tile, K split)):
//      warp 0 streams per 128-K group the 256 x 128 weight tile (TMA, 128-byte swizzle), its scales (bulk
//      copy of a pre-arranged 1 KB block), the token tile's A rows and their scales; warps 6-9 move the
//      scale words into TMEM; warp 1 issues four MMAs per group with M = 128 token rows and N = 256 weight
//      rows (so each instruction consumes 8 KB of weights: the weights are the operand that streams);
//      warps 2-5 take D = [tokens x 256] out of TMEM.  With one split they write BF16 y; with several,
//      every split adds its fp32 partial into an accumulator (vector reductions) and the split that
//      finishes last converts the tile to BF16 and zeroes its part of the accumulator again, so it is
//      zero on entry to the next call.
// Decode-sized projections (T <= 128 tokens, N of a few thousand) use K splits so that tiles x splits
// covers the SMs; prefill-sized ones tile the tokens and keep one split (consecutive units share a weight
// tile, which the other CTAs then read from L2).
//
// Scale factors in TMEM follow the block-scaled MoE kernel (csrc/moe_mxf4.cu): token m at lane m, column
// base + m / 32; weight row n at lane 32 q + n % 32 of every lane quadrant q, column base + 8 + n / 32.
#include <cuda.h>

#include "launchers.h"
#include "common/sm100.cuh"

namespace {

constexpr int kThreads = 320;  // warp 0 TMA producer, 1 MMA issuer, 2-5 epilogue, 6-9 scale factors
constexpr int kStages = 4;
constexpr uint32_t kColD = 0, kColSf = 256, kTmemCols = 512;
constexpr int kAImgMax = 65536;  // fused mode: the unit's quantized activations [groups][Tp][128] in shared memory
constexpr int kASfMax = 16384;   //   and their scale words [groups][Tp]

// Shared-memory layout.  Non-fused: a ring of stages {A 128 x 128 | W 256 x 128 | W scales | A scales}.
// Fused: the activation image and its scales, then a ring of stages {W | W scales}.
template <bool FUSED>
struct DenseCfg {
  static constexpr uint32_t kOffW = FUSED ? 0 : 128 * 128;
  static constexpr uint32_t kOffWs = kOffW + 256 * 128;
  static constexpr uint32_t kOffAs = kOffWs + 1024;
  static constexpr uint32_t kStageBytes = FUSED ? kOffAs + 1024 : kOffAs + 1024;  // (fused: 1 KB pad)
  static constexpr uint32_t kRingOff = FUSED ? kAImgMax + kASfMax : 0;
  static constexpr uint32_t kBarOff = kRingOff + kStages * kStageBytes;
  static constexpr uint32_t kSmemBytes = kBarOff + 256 + 1024;
  static_assert(kStageBytes % 1024 == 0 && kRingOff % 1024 == 0, "stage layout");
  static_assert(kSmemBytes <= 232448, "shared memory");
};

struct GemmParams {
  int T, K, N, batch, G, Tp, tiles_n, tiles_t, splits;
  const __nv_bfloat16* x;  // fused mode: the activations (x_stride_b / x_stride_t elements)
  int64_t x_stride_b, x_stride_t;
  const uint8_t* a_img;    // non-fused: [batch][G][Tp][128]
  const uint32_t* a_sf;    // non-fused: [batch][G][Tp]
  const uint8_t* w_sf;     // [batch][tiles_n][G][256][4]
  __nv_bfloat16* y;
  int64_t y_stride_t, y_stride_b;
  float* part;             // [batch][splits][Tp][tiles_n * 256]
  int32_t* counters;       // [batch][tiles_n]
  int* err;
};

// 32 BF16 values -> 8 words of E4M3 codes and the block's UE8M0 exponent (the rule of ue8m0_exp).
__device__ __forceinline__ int quant32(const __nv_bfloat16* src, bool live, uint32_t (&w)[8]) {
  float v[32];
  if (live) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = *reinterpret_cast<const uint4*>(src + 8 * i);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(b2[j]);
        v[8 * i + 2 * j] = f.x;
        v[8 * i + 2 * j + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const int e = pm::ue8m0_exp(amax);
  const float s = pm::exp2i(-e);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    w[i] = (uint32_t)pm::f32x2_to_e4m3x2(v[4 * i] * s, v[4 * i + 1] * s) |
           ((uint32_t)pm::f32x2_to_e4m3x2(v[4 * i + 2] * s, v[4 * i + 3] * s) << 16);
  return e;
}

// ----------------------------------------------------------------------------- activation quantization
// CTA per (batch, token row); thread per 32-value block.  Rows T .. Tp - 1 are padding (zero codes).
__global__ void __launch_bounds__(128) dense_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride_b,
                                                          int64_t x_stride_t, int T, int K, int Tp,
                                                          uint8_t* __restrict__ a_img, uint32_t* __restrict__ a_sf) {
  pm::griddep_wait();
  const int b = blockIdx.y, t = blockIdx.x, G = K / 128;
  const __nv_bfloat16* src = x + (int64_t)b * x_stride_b + (int64_t)t * x_stride_t;
  uint8_t* scale_bytes = reinterpret_cast<uint8_t*>(a_sf);
  for (int kb = threadIdx.x; kb < K / 32; kb += blockDim.x) {
    uint32_t w[8];
    const int e = quant32(src + kb * 32, t < T, w);
    const int g = kb >> 2;
    uint8_t* dst = a_img + (((int64_t)b * G + g) * Tp + t) * 128;
    const int u0 = (kb & 3) * 2;
    *reinterpret_cast<uint4*>(dst + ((u0 ^ (t & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(dst + (((u0 + 1) ^ (t & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
    scale_bytes[(((int64_t)b * G + g) * Tp + t) * 4 + (kb & 3)] = (uint8_t)(e + 127);
  }
}

// ----------------------------------------------------------------------------- GEMM
template <bool FUSED>
__global__ void __launch_bounds__(kThreads, 1) dense_mx_kernel(const __grid_constant__ CUtensorMap tmW,
                                                               const GemmParams p) {
  using C = DenseCfg<FUSED>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* ring = smem + C::kRingOff;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* empty = full + kStages;
  uint64_t* sf_ready = empty + kStages;
  uint64_t* d_full = sf_ready + kStages;
  uint64_t* d_empty = d_full + 1;
  uint64_t* drain = d_empty + 1;
  uint64_t* a_ready = drain + 1;  // fused: the unit's activation image is written (8 warps)
  uint64_t* a_free = a_ready + 1; // fused: the unit's MMAs are done with the image
  uint32_t* tslot = reinterpret_cast<uint32_t*>(a_free + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
  volatile int* last_flag = abort_flag + 1;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (warp == 0) {
    pm::tmem_alloc(tslot, kTmemCols);
    pm::tmem_relinquish();
  }
  if (tid == 32) {
    for (int s = 0; s < kStages; ++s) {
      pm::mbar_init(full + s, 1);
      pm::mbar_init(empty + s, 1);
      pm::mbar_init(sf_ready + s, 4);
    }
    pm::mbar_init(d_full, 1);
    pm::mbar_init(d_empty, 4);
    pm::mbar_init(drain, 1);
    pm::mbar_init(a_ready, 8);
    pm::mbar_init(a_free, 1);
    *abort_flag = 0;
    pm::fence_mbar_init();
  }
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  const uint32_t tmem = *tslot;
  // Inputs of the previous launch (the activations; the quantized image in non-fused mode) are read only
  // after griddepcontrol.wait.  In fused mode the TMA producer reads weights only, so it starts at once.
  if (!FUSED || warp != 0) pm::griddep_wait();
  const int nunits = p.batch * p.tiles_n * p.tiles_t * p.splits, G = p.G;
  // unit u -> (b, n tile, token tile, split), split fastest then token tile
  auto decode_unit = [&](int u, int& b, int& nt, int& tt, int& ks) {
    ks = u % p.splits;
    int r = u / p.splits;
    tt = r % p.tiles_t;
    r /= p.tiles_t;
    nt = r % p.tiles_n;
    b = r / p.tiles_n;
  };
  auto group_range = [&](int ks, int& g0, int& g1) {
    g0 = (ks * G) / p.splits;
    g1 = ((ks + 1) * G) / p.splits;
  };
  uint8_t* a_img = smem;                                            // fused: [g - g0][Tp][128]
  uint32_t* a_sfi = reinterpret_cast<uint32_t*>(smem + kAImgMax);   // fused: [g - g0][Tp]

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0;
      uint32_t issued_ph[kStages];
      int n_issued = 0;
      for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x) {
        int b, nt, tt, ks, g0, g1;
        decode_unit(u, b, nt, tt, ks);
        group_range(ks, g0, g1);
        const int rows = min(128, p.Tp - 128 * tt);  // token rows of the tile (multiple of 8)
        for (int g = g0; g < g1; ++g) {
          if (!pm::mbar_wait(empty + st, ph ^ 1, p.err, 40)) { *abort_flag = 1; break; }
          uint8_t* sb = ring + st * C::kStageBytes;
          const uint32_t a_bytes = FUSED ? 0u : (uint32_t)rows * 132u;
          pm::mbar_arrive_expect_tx(full + st, 256u * 128u + 1024u + a_bytes);
          pm::tma_load_2d(sb + C::kOffW, &tmW, 128 * g, b * p.N + 256 * nt, full + st);
          pm::bulk_g2s(sb + C::kOffWs, p.w_sf + (((int64_t)b * p.tiles_n + nt) * G + g) * 1024, 1024u, full + st);
          if (!FUSED) {
            const int64_t arow = ((int64_t)b * G + g) * p.Tp + 128 * tt;
            pm::bulk_g2s(sb, p.a_img + arow * 128, (uint32_t)rows * 128u, full + st);
            pm::bulk_g2s(sb + C::kOffAs, p.a_sf + arow, (uint32_t)rows * 4u, full + st);
          }
          issued_ph[st] = ph;
          ++n_issued;
          if (++st == kStages) { st = 0; ph ^= 1; }
        }
      }
      if (*abort_flag) {  // let the copies already issued land before the CTA can exit
        for (int i = 1; i <= kStages && i <= n_issued; ++i) {
          const int s = (st - i + kStages) % kStages;
          pm::mbar_wait(full + s, issued_ph[s], nullptr, 0, 20000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int st = 0, lu = 0;
      uint32_t ph = 0;
      bool any = false;
      for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x, ++lu) {
        int b, nt, tt, ks, g0, g1;
        decode_unit(u, b, nt, tt, ks);
        group_range(ks, g0, g1);
        if (!pm::mbar_wait(d_empty, (lu & 1) ^ 1, p.err, 41)) { *abort_flag = 1; break; }
        if (FUSED && !pm::mbar_wait(a_ready, lu & 1, p.err, 46)) { *abort_flag = 1; break; }
        pm::tc_fence_after();
        for (int g = g0; g < g1; ++g) {
          if (!pm::mbar_wait(full + st, ph, p.err, 42) || !pm::mbar_wait(sf_ready + st, ph, p.err, 43)) {
            *abort_flag = 1;
            break;
          }
          pm::tc_fence_after();
          const uint32_t sb = pm::smem_u32(ring + st * C::kStageBytes);
          const uint32_t ab = FUSED ? pm::smem_u32(a_img + (g - g0) * p.Tp * 128) : sb;
          const uint32_t sf_col = tmem + kColSf + 16 * st;
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const uint32_t idesc = pm::make_idesc_mxf8(128, 256, 0, 0, s, s);  // E4M3 x E4M3
            pm::umma_mxf8(tmem + kColD, pm::make_sdesc(ab + 32 * s, 16, 1024),
                          pm::make_sdesc(sb + C::kOffW + 32 * s, 16, 1024), idesc, sf_col, sf_col + 8,
                          (g > g0 || s) ? 1u : 0u);
          }
          pm::umma_commit(empty + st);
          any = true;
          if (++st == kStages) { st = 0; ph ^= 1; }
        }
        if (*abort_flag) break;
        pm::umma_commit(d_full);
        if (FUSED) pm::umma_commit(a_free);
      }
      if (*abort_flag && any) {
        pm::umma_commit(drain);
        pm::mbar_wait(drain, 0, nullptr, 0, 20000000ull);
      }
    }
  } else {
    // ------------------------------------------------------------------ warps 2-9
    const bool epi = warp < 6;  // 2-5: epilogue; 6-9: scale factors; fused mode: all 8 quantize first
    const int q = warp & 3;     // TMEM lane quadrant this warp may access
    const int wtid = tid - 64;  // 0 .. 255
    const int n_pad = p.tiles_n * 256;
    int st = 0, lu = 0;
    uint32_t ph = 0;
    for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x, ++lu) {
      int b, nt, tt, ks, g0, g1;
      decode_unit(u, b, nt, tt, ks);
      group_range(ks, g0, g1);
      const int rows = min(128, p.Tp - 128 * tt);
      if (FUSED) {
        // the unit's activations -> E4M3 image and scale words (the previous unit's MMAs are done with them)
        if (lu > 0 && !pm::mbar_wait(a_free, (lu - 1) & 1, p.err, 47)) { *abort_flag = 1; break; }
        const int kbs = (g1 - g0) * 4;  // 32-value blocks per row
        for (int i = wtid; i < rows * kbs; i += 256) {
          const int r = i / kbs, kb = i % kbs, t = 128 * tt + r;
          uint32_t w[8];
          const int e = quant32(p.x + (int64_t)b * p.x_stride_b + (int64_t)t * p.x_stride_t + (int64_t)(g0 * 4 + kb) * 32,
                                t < p.T, w);
          uint8_t* dst = a_img + ((kb >> 2) * p.Tp + r) * 128;
          const int u0 = (kb & 3) * 2;
          *reinterpret_cast<uint4*>(dst + ((u0 ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(dst + (((u0 + 1) ^ (r & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
          reinterpret_cast<uint8_t*>(a_sfi)[((kb >> 2) * p.Tp + r) * 4 + (kb & 3)] = (uint8_t)(e + 127);
        }
        pm::fence_proxy_async_smem();  // the image is read by the MMAs (async proxy)
        __syncwarp();
        if (lane == 0) pm::mbar_arrive(a_ready);
      }
      if (!epi) {
        // ---------------------------------------------------------------- scale factors -> TMEM
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        if (FUSED && !pm::mbar_wait(a_ready, lu & 1, p.err, 48)) { *abort_flag = 1; break; }
        for (int g = g0; g < g1 && !*abort_flag; ++g) {
          if (!pm::mbar_wait(full + st, ph, p.err, 44)) { *abort_flag = 1; break; }
          const uint8_t* sb = ring + st * C::kStageBytes;
          const uint32_t* ws = reinterpret_cast<const uint32_t*>(sb + C::kOffWs);
          const uint32_t* as = FUSED ? a_sfi + (g - g0) * p.Tp : reinterpret_cast<const uint32_t*>(sb + C::kOffAs);
          const int m = 32 * q + lane;  // token row of A: lane m, column base + m / 32 = base + q
          const uint32_t tk = m < rows ? as[m] : 0u;
          uint32_t v[16];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = i == q ? tk : 0u;
#pragma unroll
          for (int c = 0; c < 8; ++c) v[8 + c] = ws[32 * c + lane];  // weight row 32 c + lane
          pm::tc_fence_after();
          pm::tmem_st16u(tmem + lane_base + kColSf + 16 * st, v);
          pm::tmem_wait_st();
          pm::tc_fence_before();
          __syncwarp();
          if (lane == 0) pm::mbar_arrive(sf_ready + st);
          if (++st == kStages) { st = 0; ph ^= 1; }
        }
        continue;
      }
      // ---------------------------------------------------------------- epilogue (warps 2-5)
      const int etid = tid - 64;  // 0 .. 127
      if (!pm::mbar_wait(d_full, lu & 1, p.err, 45)) { *abort_flag = 1; break; }
      if (*abort_flag) break;
      pm::tc_fence_after();
      const int m = 32 * q + lane, t = 128 * tt + m;
      const bool live = t < p.T;
      const int ncols = min(256, p.N - 256 * nt);
      const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16) + kColD;
      for (int h = 0; h < 2; ++h) {
        float v[128];
        pm::tmem_ld32x4(lane_addr + 128 * h, lane_addr + 128 * h + 32, lane_addr + 128 * h + 64,
                        lane_addr + 128 * h + 96, v);
        if (h == 1) {  // the accumulator is free for the next unit
          pm::tc_fence_before();
          __syncwarp();
          if (lane == 0) pm::mbar_arrive(d_empty);
        }
        if (!live) continue;
        if (p.splits == 1) {
          __nv_bfloat16* yrow = p.y + (int64_t)b * p.y_stride_b + (int64_t)t * p.y_stride_t + 256 * nt + 128 * h;
#pragma unroll
          for (int i = 0; i < 128; i += 8) {
            if (128 * h + i + 8 <= ncols) {
              uint32_t w4[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[i + 2 * k], v[i + 2 * k + 1]);
                w4[k] = *reinterpret_cast<const uint32_t*>(&h2);
              }
              *reinterpret_cast<uint4*>(yrow + i) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            } else {
              for (int k = 0; k < 8; ++k)
                if (128 * h + i + k < ncols) yrow[i + k] = __float2bfloat16_rn(v[i + k]);
            }
          }
        } else {  // this split's partial row
          float* prow = p.part + (((int64_t)b * p.splits + ks) * p.Tp + m) * n_pad + 256 * nt + 128 * h;
#pragma unroll
          for (int i = 0; i < 128; i += 4)
            *reinterpret_cast<float4*>(prow + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
      }
      if (p.splits > 1) {
        // the split that finishes a tile last sums the partials in split order into BF16 y
        __threadfence();
        pm::named_bar_sync(1, 128);
        if (etid == 0) {
          const int prev = atomicAdd(p.counters + (int64_t)b * p.tiles_n + nt, 1);
          *last_flag = prev == p.splits - 1;
        }
        pm::named_bar_sync(1, 128);
        if (*last_flag) {
          __threadfence();
          const int nrows = min(128, p.T - 128 * tt);
          for (int idx = etid; idx < nrows * 64; idx += 128) {
            const int r = idx >> 6, c4 = (idx & 63) * 4;
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int k = 0; k < p.splits; ++k) {
              const float4 v = __ldcg(reinterpret_cast<const float4*>(
                  p.part + (((int64_t)b * p.splits + k) * p.Tp + r) * n_pad + 256 * nt + c4));
              a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
            }
            __nv_bfloat16* yrow = p.y + (int64_t)b * p.y_stride_b + (int64_t)(128 * tt + r) * p.y_stride_t + 256 * nt;
            if (c4 + 4 <= ncols) {
              const __nv_bfloat162 lo = __floats2bfloat162_rn(a.x, a.y), hi = __floats2bfloat162_rn(a.z, a.w);
              *reinterpret_cast<uint2*>(yrow + c4) =
                  make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
            } else {
              const float av[4] = {a.x, a.y, a.z, a.w};
              for (int k = 0; k < 4; ++k)
                if (c4 + k < ncols) yrow[c4 + k] = __float2bfloat16_rn(av[k]);
            }
          }
          if (etid == 0) p.counters[(int64_t)b * p.tiles_n + nt] = 0;
          pm::named_bar_sync(1, 128);  // last_flag is read by every thread before the next unit sets it
        }
      }
    }
  }
  pm::tc_fence_before();
  __syncthreads();
  if (warp == 0) pm::tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

namespace {
template <typename... KArgs, typename... Args>
void launch_pdl2(void (*kernel)(KArgs...), dim3 grid, int block, size_t smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

bool misaligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; }
}  // namespace

bool dense_mx_fused_quant(int T, int K, int splits) {
  const int Tp = (T + 7) & ~7, G = K / 128;
  const int g_unit = (G + splits - 1) / splits;  // the most groups a split holds
  return Tp <= 128 && Tp * 128 * g_unit <= kAImgMax && Tp * 4 * g_unit <= kASfMax;
}

// Returns 0, or -2 for unsupported sizes, -3 for misaligned operands, or the tensor-map encoder's error.
int launch_dense_mx(const DenseMxArgs& a, cudaStream_t stream) {
  if (a.T == 0 || a.N == 0 || a.batch == 0) return 0;
  if (a.T < 0 || a.N < 0 || a.batch < 0 || a.K <= 0 || a.K % 128 || a.splits < 1 || (a.splits > 1 && a.T > 128))
    return -2;
  const int G = a.K / 128;
  if (a.splits > G) return -2;
  const int Tp = (a.T + 7) & ~7;
  const int tiles_n = (a.N + 255) / 256, tiles_t = (Tp + 127) / 128;
  const bool fused = dense_mx_fused_quant(a.T, a.K, a.splits);
  if (misaligned16(a.x) || (a.x_stride_t * 2) % 16 || (a.x_stride_b * 2) % 16 || misaligned16(a.w) || a.K % 16 ||
      misaligned16(a.w_sf) || misaligned16(a.y) || (a.y_stride_t * 2) % 16 || (a.y_stride_b * 2) % 16 ||
      (!fused && (misaligned16(a.a_img) || misaligned16(a.a_sf))) ||
      (a.splits > 1 && (misaligned16(a.part) || !a.counters)))
    return -3;
  CUtensorMap mw;
  if (const int rc = make_tmap_u8_sw128(&mw, a.w, (uint64_t)a.K, (uint64_t)a.batch * a.N, (uint64_t)a.K, 256)) return rc;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(dense_mx_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, DenseCfg<true>::kSmemBytes);
    cudaFuncSetAttribute(dense_mx_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         DenseCfg<false>::kSmemBytes);
    attr = true;
  }
  if (!fused)
    launch_pdl2(dense_quant_kernel, dim3(Tp, a.batch), 128, 0, stream, a.x, a.x_stride_b, a.x_stride_t, a.T, a.K, Tp,
                a.a_img, a.a_sf);
  GemmParams p{a.T, a.K, a.N, a.batch, G, Tp, tiles_n, tiles_t, a.splits, a.x, a.x_stride_b, a.x_stride_t,
               a.a_img, a.a_sf, a.w_sf, a.y, a.y_stride_t, a.y_stride_b, a.part, a.counters, a.err};
  const int units = a.batch * tiles_n * tiles_t * a.splits;
  const dim3 grid(units < a.num_sms ? units : a.num_sms);
  if (fused)
    launch_pdl2(dense_mx_kernel<true>, grid, kThreads, (size_t)DenseCfg<true>::kSmemBytes, stream, mw, p);
  else
    launch_pdl2(dense_mx_kernel<false>, grid, kThreads, (size_t)DenseCfg<false>::kSmemBytes, stream, mw, p);
  return 0;
}
