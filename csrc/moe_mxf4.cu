// MXFP4 routed experts x MXFP8 activations on the 5th-generation tensor cores.
//
// Reference behaviour: the reference serves the experts through FlashInfer's MXFP4 MoE
// (`moe_runner_backend='flashinfer_mxfp4'`, `flashinfer_mxfp4_moe_precision='default'` in
// benchmarks/lswb-replay/*/kernel/*/server/serve_kernel.log).  On sm_100 that precision quantizes the
// activations to MXFP8 (E4M3 values, one UE8M0 scale per 32) for both expert GEMMs, which is what this
// file does: the weights stay packed MXFP4 in HBM and are never dequantized in registers.
//
//   1. route (csrc/moe_fp4.cu, align 32): per-expert slot lists sorted by token, padded row ranges that
//      start on multiples of 32, and the chunk table {expert, first row, tokens <= MT, first slot} with
//      MT = 16 for decode-sized batches and 128 for prefill-sized ones (see MxCfg).
//   2. quant (CTA per slot): h[token] -> E4M3 + UE8M0 per 32 values, written straight into the operand
//      images the MMA kernel streams; also zeroes `out` for the scatter-add of pass 4.
//   3. gate/up (persistent, one CTA per SM): unit = (chunk, 128 gate rows + the matching 128 up rows).
//      Per K-group of 128 a TMA producer warp streams both weight tiles (tensor map of type
//      16U4_ALIGN16B: packed FP4 in HBM, the tcgen05 unpacked layout in shared memory, 128-byte
//      swizzle) into one 256-row B operand, the chunk's activation rows (A operand) and the group's
//      weight scales; one thread issues tcgen05.mma kind::mxf8f6f4.block_scale with M = 128 token rows,
//      N = 256 weight rows, so D = [tokens x (gate | up)]; an epilogue warp computes silu(g) * u per
//      token, quantizes it to MXFP8 per 32 intermediate values and writes the down pass's operand rows.
//   4. down (same kernel, mode 1): unit = (chunk, 256 output rows); the epilogue scatter-adds routing
//      weight * y into out (fp32 reductions).
//
// Why weights are the N operand: a tcgen05.mma costs the same ~170-220 issue cycles for any N from 8 to
// 256 (measured with the tc probe; it is the M x K work that sets the pace), so with the weights as the
// 128-row A operand the tensor pipe, not HBM, capped the weight stream at ~4.5 TB/s.  As the 256-row B
// operand every instruction consumes twice the weights.  The A operand keeps M = 128 rows although a
// decode chunk has <= 16 tokens: its descriptor walks 1 KB per 8 rows, so rows past the chunk read
// neighbouring shared memory and only fill accumulator rows nobody reads.
//
// Operand images: activations [K/128][rows][128] E4M3 codes (K-major, 128 K-bytes per row, 16-byte units
// XOR-swizzled by row % 8; the rows of one chunk are contiguous per K-group) and their UE8M0 scales
// [rows][K/32]; weight scales [units][K/128][256][4] (per unit's 256 weight rows and K-group, the 4 k-block
// scales of each row, rows contiguous), made once when the experts are loaded.  Weights come through a
// 4-D tensor map [E][gate | up][I][H] (gate/up) or a 2-D map with a 256-row box (down), so one TMA fills
// a stage's 256-row B operand.
//
// Scale factors go to TMEM with tcgen05.st from a scale warp per lane quadrant, one ring slot per stage
// (token m at lane m, column base + m / 32; weight row n at lane 32 q + n % 32 of every quadrant q,
// column base + 8 + n / 32; every scale address given to tcgen05.mma is a multiple of 4 columns), and
// are signalled to the MMA issuer through an mbarrier.
#include <cuda.h>

#include "launchers.h"
#include "common/sm100.cuh"

namespace {

constexpr int kPrefetch = 10;  // stages fetched into L2 ahead of the shared-memory ring
constexpr int kThreads = 320;  // warp 0 TMA producer, 1 MMA issuer, 2-5 epilogue, 6-9 scale factors
constexpr int kMaxG = 32;      // K-groups of 128 (K <= 4096)
constexpr uint32_t kStageW = 32768;           // 256 weight rows x 128 B (B operand)
constexpr uint32_t kStageS = 1024;            // weight scales: 256 rows x 4 B
constexpr uint32_t kColD = 0, kColSf = 256, kTmemCols = 512;

// Stage geometry for chunks of at most MT tokens (A rows with data).  MT = 16 serves decode: the A copy is
// 2 KB and six stages keep the weight stream deep.  MT = 128 serves prefill (hundreds of tokens per
// expert): each 256-row weight tile then feeds a full 128-row A operand, so an expert's weights are
// streamed once per 128 routed tokens instead of once per 16; four stages fit.
template <int MT>
struct MxCfg {
  static constexpr int kStages = MT <= 16 ? 6 : 4;
  static constexpr uint32_t kOffW = MT <= 16 ? 2048 : (uint32_t)MT * 128;  // A first, then B
  static constexpr uint32_t kStageBytes = kOffW + kStageW + kStageS;      // multiple of 1024
  static constexpr uint32_t kBarOff = kStages * kStageBytes;
  static constexpr uint32_t kSmemBytes = kBarOff + 256 + 1024;
  static_assert((uint32_t)MT * 128 <= kOffW && kOffW % 1024 == 0 && kStageBytes % 1024 == 0, "stage layout");
  // TMEM columns: D [128 token lanes x 256] fp32, scale ring (kStages x {tokens: 4, unused: 4, weights: 8}).
  static_assert(kColSf + 16 * kStages <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory");
};

struct MxParams {
  int K, G, J, rows_exp, rows_total, H;  // H: output row stride (mode 1) / act K (mode 0, = I)
  int rows_total_w;                      // weight rows (E * rows_exp) of the tensor map
  const uint8_t* sfw;                    // weight scales [units of 256 rows][K/128][256][4]
  const uint8_t* b_img;                  // [G][rows_total][128]
  const uint8_t* sfb;                    // token scales [rows_total][K/32]
  const int4* chunks;
  const int32_t* n_chunks;
  uint8_t* act_img;                      // mode 0: [I/128][rows_total][128]
  uint8_t* act_sf;                       // mode 0: [rows_total][I/32]
  const int32_t* slot_token;
  const float* slot_weight;
  float* out;                            // mode 1: [T, H]
  int* err;
  unsigned long long* prof;              // optional wait-time counters (ns), see launch_moe_mxf4
};

// Bounded wait that adds the SM cycles it spent to *acc (when profiling).
__device__ __forceinline__ bool timed_wait(uint64_t* bar, uint32_t parity, int* err, int site, uint64_t* acc) {
  if (acc == nullptr) return pm::mbar_wait(bar, parity, err, site);
  const uint64_t t0 = clock64();
  const bool ok = pm::mbar_wait(bar, parity, err, site);
  *acc += clock64() - t0;
  return ok;
}

// ----------------------------------------------------------------------------- activation quantization
// CTA per slot p: h[token(p)] -> operand image rows of the padded row of p.  Threads own k-blocks of 32.
__global__ void __launch_bounds__(128) mx_quant_kernel(const __nv_bfloat16* __restrict__ h, int H, int E,
                                                       const int32_t* __restrict__ offsets,
                                                       const int32_t* __restrict__ pad,
                                                       const int32_t* __restrict__ slot_token, int rows_total,
                                                       uint8_t* __restrict__ xq, uint8_t* __restrict__ xs,
                                                       float* __restrict__ out, int T) {
  const int p = blockIdx.x, tid = threadIdx.x;
  if (p < T)
    for (int i = tid * 4; i < H; i += 128 * 4) *reinterpret_cast<float4*>(out + (size_t)p * H + i) = float4{0, 0, 0, 0};
  if (p >= offsets[E]) return;
  int lo = 0, hi = E;  // expert e with offsets[e] <= p < offsets[e + 1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (offsets[mid] <= p) lo = mid; else hi = mid;
  }
  const int row = pad[lo] + p - offsets[lo];
  const __nv_bfloat16* src = h + (size_t)slot_token[p] * H;
  for (int kb = tid; kb < H / 32; kb += 128) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = *reinterpret_cast<const uint4*>(src + kb * 32 + 8 * i);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(b2[j]);
        v[8 * i + 2 * j] = f.x;
        v[8 * i + 2 * j + 1] = f.y;
      }
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const int e = pm::ue8m0_exp(amax);
    const float s = pm::exp2i(-e);
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      w[i] = (uint32_t)pm::f32x2_to_e4m3x2(v[4 * i] * s, v[4 * i + 1] * s) |
             ((uint32_t)pm::f32x2_to_e4m3x2(v[4 * i + 2] * s, v[4 * i + 3] * s) << 16);
    uint8_t* dst = xq + ((size_t)(kb >> 2) * rows_total + row) * 128;
    const int u0 = (kb & 3) * 2;
    *reinterpret_cast<uint4*>(dst + (((u0) ^ (row & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(dst + (((u0 + 1) ^ (row & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
    xs[(size_t)row * (H / 32) + kb] = (uint8_t)(e + 127);
  }
}

// ----------------------------------------------------------------------------- expert GEMM
template <int MODE, int MT>
__global__ void __launch_bounds__(kThreads, 1) mx_expert_kernel(const __grid_constant__ CUtensorMap tmW,
                                                                const MxParams p) {
  using C = MxCfg<MT>;
  constexpr int kStages = C::kStages;
  constexpr uint32_t kStageBytes = C::kStageBytes, kOffW = C::kOffW, kBarOff = C::kBarOff;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* empty = full + kStages;
  uint64_t* sf_ready = empty + kStages;
  uint64_t* d_full = sf_ready + kStages;
  uint64_t* d_empty = d_full + 1;
  uint64_t* drain = d_empty + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
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
    *abort_flag = 0;
    pm::fence_mbar_init();
  }
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  const uint32_t tmem = *tslot;
  const int nunits = p.n_chunks[0] * p.J;
  const int G = p.G, KB = p.K / 32;  // K-groups, scale bytes per row

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint64_t w_empty = 0, t_start = clock64(), t_pissue = 0;
      uint64_t* acc = p.prof ? &w_empty : nullptr;
      int st = 0;
      uint32_t ph = 0;
      uint32_t issued_ph[kStages];
      int n_issued = 0;
      // weight box of unit u, K-group g: gate/up map {k, row in expert, tile, expert} or down {k, row}
      auto load_w = [&](uint8_t* dst, int e, int j, int g, uint64_t* bar) {
        if (MODE == 0) pm::tma_load_4d(dst, &tmW, 128 * g, 128 * j, 0, e, bar);
        else pm::tma_load_2d(dst, &tmW, 128 * g, e * p.rows_exp + 256 * j, bar);
      };
      auto prefetch_w = [&](int e, int j, int g) {
        if (MODE == 0) pm::tma_prefetch_4d(&tmW, 128 * g, 128 * j, 0, e);
        else pm::tma_prefetch_2d(&tmW, 128 * g, e * p.rows_exp + 256 * j);
      };
      // L2 prefetch cursor (unit pu, group pg) kPrefetch stages ahead of the loads; chunk entries are
      // read one unit ahead so their load latency stays off the issue path
      int pu = blockIdx.x, pg = 0;
      int pe = pu < nunits ? p.chunks[pu / p.J].x : 0;
      auto prefetch_next = [&]() {
        if (pu >= nunits) return;
        prefetch_w(pe, pu % p.J, pg);
        if (++pg == G) {
          pg = 0;
          pu += gridDim.x;
          if (pu < nunits) pe = p.chunks[pu / p.J].x;
        }
      };
      for (int i = 0; i < kPrefetch; ++i) prefetch_next();
      int4 ct_next = blockIdx.x < nunits ? p.chunks[blockIdx.x / p.J] : make_int4(0, 0, 0, 0);
      for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x) {
        const int4 ct = ct_next;
        if (u + (int)gridDim.x < nunits) ct_next = p.chunks[(u + gridDim.x) / p.J];
        const int n8 = (ct.z + 7) & ~7, j = u % p.J;
        // self-check of the copy geometry (records the unit and skips instead of faulting)
        if ((ct.y & 15) || ct.z < 1 || ct.z > MT || ct.y + n8 > p.rows_total ||
            (ct.x + 1) * p.rows_exp > p.rows_total_w || (reinterpret_cast<uintptr_t>(p.b_img) & 15)) {
          pm::report_error(p.err, pm::kBadArgument, 100000 + u);
          *abort_flag = 1;
          break;
        }
        const uint8_t* sw = p.sfw + (size_t)(ct.x * p.J + j) * G * 1024;
        const uint8_t* act = p.b_img + (size_t)ct.y * 128;
        for (int g = 0; g < G; ++g) {
          if (!timed_wait(empty + st, ph ^ 1, p.err, 22, acc)) { *abort_flag = 1; break; }
          const uint64_t t_p0 = p.prof ? clock64() : 0;
          uint8_t* sb = smem + st * kStageBytes;
          pm::mbar_arrive_expect_tx(full + st, 2 * 8192 + n8 * 128 + 1024);
          pm::bulk_g2s(sb, act + (size_t)g * p.rows_total * 128, n8 * 128, full + st);
          load_w(sb + kOffW, ct.x, j, g, full + st);
          pm::bulk_g2s(sb + kOffW + kStageW, sw + g * 1024, 1024, full + st);
          issued_ph[st] = ph;
          ++n_issued;
          prefetch_next();
          if (p.prof) t_pissue += clock64() - t_p0;
          if (++st == kStages) { st = 0; ph ^= 1; }
        }
      }
      if (p.prof) {
        atomicAdd(p.prof + 0, (unsigned long long)w_empty);
        atomicAdd(p.prof + 4, (unsigned long long)(clock64() - t_start));
        atomicAdd(p.prof + 7, (unsigned long long)t_pissue);
      }
      if (*abort_flag) {
        // let the copies already issued land before the CTA can exit
        for (int i = 1; i <= kStages && i <= n_issued; ++i) {
          const int s = (st - i + kStages) % kStages;
          pm::mbar_wait(full + s, issued_ph[s], nullptr, 0, 20000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint64_t w_full = 0, w_d = 0, w_sf = 0, t_issue = 0;
      uint64_t* acc_f = p.prof ? &w_full : nullptr;
      uint64_t* acc_d = p.prof ? &w_d : nullptr;
      uint64_t* acc_s = p.prof ? &w_sf : nullptr;
      int st = 0, lu = 0;
      uint32_t ph = 0;
      bool any = false;
      for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x, ++lu) {
        if (!timed_wait(d_empty, (lu & 1) ^ 1, p.err, 24, acc_d)) {
          *abort_flag = 1;
          break;
        }
        pm::tc_fence_after();
        for (int g = 0; g < G; ++g) {
          if (!timed_wait(full + st, ph, p.err, 25, acc_f) || !timed_wait(sf_ready + st, ph, p.err, 27, acc_s)) {
            *abort_flag = 1;
            break;
          }
          const uint64_t t_i0 = p.prof ? clock64() : 0;
          pm::tc_fence_after();
          const uint32_t sb = pm::smem_u32(smem + st * kStageBytes);
          const uint32_t sf_col = tmem + kColSf + 16 * st;
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const uint32_t idesc = pm::make_idesc_mxf8(128, 256, 0, 5, s, s);
            pm::umma_mxf8(tmem + kColD, pm::make_sdesc(sb + 32 * s, 16, 1024),
                          pm::make_sdesc(sb + kOffW + 32 * s, 16, 1024), idesc, sf_col, sf_col + 8, (g | s) ? 1u : 0u);
          }
          pm::umma_commit(empty + st);
          if (p.prof) t_issue += clock64() - t_i0;
          any = true;
          if (++st == kStages) { st = 0; ph ^= 1; }
        }
        if (*abort_flag) break;
        pm::umma_commit(d_full);
      }
      if (p.prof) {
        atomicAdd(p.prof + 1, (unsigned long long)w_full);
        atomicAdd(p.prof + 2, (unsigned long long)w_d);
        atomicAdd(p.prof + 5, (unsigned long long)w_sf);
        atomicAdd(p.prof + 6, (unsigned long long)t_issue);
      }
      if (*abort_flag && any) {
        pm::umma_commit(drain);
        pm::mbar_wait(drain, 0, nullptr, 0, 20000000ull);
      }
    }
  } else if (warp >= 6) {
    // ------------------------------------------------------------------ scale-factor warps (6-9)
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    int st = 0;
    uint32_t ph = 0;
    for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x) {
      const int4 ct = p.chunks[u / p.J];
      // token scale words of this lane's token (row 32 q + lane of A), one per K-group
      uint32_t tk[kMaxG];
      {
        const bool has = 32 * q + lane < ct.z;
        const uint4* src = reinterpret_cast<const uint4*>(p.sfb + (size_t)(ct.y + (has ? 32 * q + lane : 0)) * KB);
#pragma unroll
        for (int i = 0; i < kMaxG / 4; ++i) {
          if (4 * i < G) {
            const uint4 t = has ? src[i] : make_uint4(0, 0, 0, 0);
            tk[4 * i] = t.x; tk[4 * i + 1] = t.y; tk[4 * i + 2] = t.z; tk[4 * i + 3] = t.w;
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kMaxG; ++g) {
        if (g < G && !*abort_flag) {
          // the stage's weight scales arrive with its data; the slot is free once its MMAs are done
          if (!pm::mbar_wait(full + st, ph, p.err, 29)) { *abort_flag = 1; break; }
          const uint32_t* ws = reinterpret_cast<const uint32_t*>(smem + st * kStageBytes + kOffW + kStageW);
          // token m = 32 q + lane lives at lane m, column base + m / 32 = base + q
          uint32_t v[16];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = i == q ? tk[g] : 0u;
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
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-5)
    const int q = warp & 3;  // TMEM lane quadrant: tokens 32 q .. 32 q + 31
    uint64_t w_dfull = 0;
    uint64_t* acc_e = (p.prof && lane == 0 && q == 0) ? &w_dfull : nullptr;
    int lu = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++lu) {
      const int j = u % p.J;
      const int4 ct = p.chunks[u / p.J];
      if (!timed_wait(d_full, lu & 1, p.err, 26, acc_e)) { *abort_flag = 1; break; }
      if (*abort_flag) break;
      pm::tc_fence_after();
      const int m = 32 * q + lane;  // token row of D
      const bool live = m < ct.z;
      const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16) + kColD;
      if (32 * q >= ct.z) {  // no token of this chunk in the quadrant
        pm::tc_fence_before();
        __syncwarp();
        if (lane == 0) pm::mbar_arrive(d_empty);
        continue;
      }
      if (MODE == 0) {
        // D columns: gate rows 0-127, up rows 128-255 of the tile -> intermediate 128 j + c.  All loads
        // first (warp-collective), release the accumulator, then math on the chunk's token rows only
        // (the other rows hold garbage that would send the division down its slow path).
        const int row = ct.y + m;
        for (int h = 0; h < 2; ++h) {
          float gu[128];  // gate columns 64 h .. 64 h + 63, then the matching up columns
          pm::tmem_ld32x4(lane_addr + 64 * h, lane_addr + 64 * h + 32, lane_addr + 128 + 64 * h,
                          lane_addr + 160 + 64 * h, gu);
          const float* g = gu;
          const float* up = gu + 64;
          if (h == 1) {
            pm::tc_fence_before();
            __syncwarp();
            if (lane == 0) pm::mbar_arrive(d_empty);
          }
          if (live) {
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
              float a[32];
              float amax = 0.f;
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const float x = g[32 * blk + i];
                a[i] = __fdividef(x, 1.f + __expf(-x)) * up[32 * blk + i];
                amax = fmaxf(amax, fabsf(a[i]));
              }
              const int e = pm::ue8m0_exp(amax);
              const float sc = pm::exp2i(-e);
              uint32_t w8[8];
#pragma unroll
              for (int i = 0; i < 8; ++i)
                w8[i] = (uint32_t)pm::f32x2_to_e4m3x2(a[4 * i] * sc, a[4 * i + 1] * sc) |
                        ((uint32_t)pm::f32x2_to_e4m3x2(a[4 * i + 2] * sc, a[4 * i + 3] * sc) << 16);
              uint8_t* dst = p.act_img + ((size_t)j * p.rows_total + row) * 128;
              const int u0 = 4 * h + 2 * blk;  // 16-byte unit of intermediate 64 h + 32 blk
              *reinterpret_cast<uint4*>(dst + ((u0 ^ (row & 7)) << 4)) = make_uint4(w8[0], w8[1], w8[2], w8[3]);
              *reinterpret_cast<uint4*>(dst + (((u0 + 1) ^ (row & 7)) << 4)) = make_uint4(w8[4], w8[5], w8[6], w8[7]);
              p.act_sf[(size_t)row * (p.H / 32) + 4 * j + 2 * h + blk] = (uint8_t)(e + 127);
            }
          }
        }
      } else {
        // D columns: output rows 256 j + c
        const int t = live ? p.slot_token[ct.w + m] : 0;
        const float w = live ? p.slot_weight[ct.w + m] : 0.f;
        float* o = p.out + (size_t)t * p.H + 256 * j;
        for (int h = 0; h < 2; ++h) {
          float v[128];
          pm::tmem_ld32x4(lane_addr + 128 * h, lane_addr + 128 * h + 32, lane_addr + 128 * h + 64,
                          lane_addr + 128 * h + 96, v);
          if (h == 1) {
            pm::tc_fence_before();
            __syncwarp();
            if (lane == 0) pm::mbar_arrive(d_empty);
          }
          if (live) {  // vector fp32 reductions (sm_90+), 4 outputs per instruction
#pragma unroll
            for (int i = 0; i < 128; i += 4)
              atomicAdd(reinterpret_cast<float4*>(o + 128 * h + i),
                        make_float4(w * v[i], w * v[i + 1], w * v[i + 2], w * v[i + 3]));
          }
        }
      }
    }
    if (acc_e) atomicAdd(p.prof + 3, (unsigned long long)w_dfull);
  }
  pm::tc_fence_before();
  __syncthreads();
  if (warp == 0) pm::tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

int launch_moe_mxf4(const MoeMxArgs& a, cudaStream_t stream) {
  if (a.T == 0) return 0;
  if (a.H % 512 || a.I % 512 || a.H / 128 > kMaxG || a.I / 128 > kMaxG || a.rows_total % 32) return -2;
  if ((reinterpret_cast<uintptr_t>(a.w13) | reinterpret_cast<uintptr_t>(a.w2)) & 31) return -4;
  const int n = a.T * a.k;
  // chunks of 128 tokens once experts average 64 or more routed tokens (prefill), else of 16 (decode)
  const int mt = n >= 64 * a.E ? 128 : 16;
  launch_moe_route_chunks(a.topk_ids, a.topk_w, a.T, a.k, a.expert_base, a.E, a.offsets, a.slot_token,
                          a.slot_weight, a.active, a.pad, a.chunks, a.n_chunks, mt, stream);
  mx_quant_kernel<<<max(n, a.T), 128, 0, stream>>>(a.h, a.H, a.E, a.offsets, a.pad, a.slot_token, a.rows_total, a.xq,
                                                   a.xs, a.out, a.T);
  CUtensorMap m13, m2;
  {
    // gate/up: [E][2][I][H] with a {128, 128, 2, 1} box = the 128 gate rows and the 128 up rows of a unit
    const uint64_t dims[4] = {(uint64_t)a.H, (uint64_t)a.I, 2, (uint64_t)a.E};
    const uint64_t strides[3] = {(uint64_t)a.H / 2, (uint64_t)a.I * a.H / 2, (uint64_t)2 * a.I * a.H / 2};
    const uint32_t box[4] = {128, 128, 2, 1};
    const int rc = make_tmap_fp4_unpacked_nd(&m13, a.w13, 4, dims, strides, box);
    if (rc) return rc;
  }
  {
    const int rc = make_tmap_fp4_unpacked(&m2, a.w2, a.I, (uint64_t)a.E * a.H, a.I / 2, 256);
    if (rc) return rc;
  }
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(mx_expert_kernel<0, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, MxCfg<16>::kSmemBytes);
    cudaFuncSetAttribute(mx_expert_kernel<1, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, MxCfg<16>::kSmemBytes);
    cudaFuncSetAttribute(mx_expert_kernel<0, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         MxCfg<128>::kSmemBytes);
    cudaFuncSetAttribute(mx_expert_kernel<1, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         MxCfg<128>::kSmemBytes);
    attr = true;
  }
  if ((reinterpret_cast<uintptr_t>(a.xq) | reinterpret_cast<uintptr_t>(a.xs) | reinterpret_cast<uintptr_t>(a.act_q) |
       reinterpret_cast<uintptr_t>(a.act_s) | reinterpret_cast<uintptr_t>(a.sfw13) | reinterpret_cast<uintptr_t>(a.sfw2) |
       reinterpret_cast<uintptr_t>(a.chunks) | reinterpret_cast<uintptr_t>(a.out)) & 15)
    return -3;
  MxParams p0{a.H, a.H / 128, a.I / 128, 2 * a.I, a.rows_total, a.I, a.E * 2 * a.I, a.sfw13, a.xq, a.xs, a.chunks, a.n_chunks,
              a.act_q, a.act_s, a.slot_token, a.slot_weight, a.out, a.err, a.prof};
  if (mt == 128) mx_expert_kernel<0, 128><<<a.num_sms, kThreads, MxCfg<128>::kSmemBytes, stream>>>(m13, p0);
  else mx_expert_kernel<0, 16><<<a.num_sms, kThreads, MxCfg<16>::kSmemBytes, stream>>>(m13, p0);
  MxParams p1{a.I, a.I / 128, a.H / 256, a.H, a.rows_total, a.H, a.E * a.H, a.sfw2, a.act_q, a.act_s, a.chunks, a.n_chunks,
              nullptr, nullptr, a.slot_token, a.slot_weight, a.out, a.err, a.prof ? a.prof + 8 : nullptr};
  if (mt == 128) mx_expert_kernel<1, 128><<<a.num_sms, kThreads, MxCfg<128>::kSmemBytes, stream>>>(m2, p1);
  else mx_expert_kernel<1, 16><<<a.num_sms, kThreads, MxCfg<16>::kSmemBytes, stream>>>(m2, p1);
  return 0;
}
