// MXFP4 routed experts x MXFP8 activations on the 5th-generation tensor cores.
//
// Reference behaviour: the reference serves the experts through FlashInfer's MXFP4 MoE
// (`moe_runner_backend='flashinfer_mxfp4'`, `flashinfer_mxfp4_moe_precision='default'` in
// benchmarks/lswb-replay/*/kernel/*/server/serve_kernel.log).  On sm_100 that precision quantizes the
// activations to MXFP8 (E4M3 values, one UE8M0 scale per 32) for both expert GEMMs, which is what this
// file does: the weights stay packed MXFP4 in HBM and are never dequantized in registers.
//
//   1. route (csrc/moe_fp4.cu, align 32): per-expert slot lists sorted by token, padded row ranges that
//      start on multiples of 32, and the chunk table {expert, first row, tokens <= 32, first slot}.
//   2. quant (CTA per slot): h[token] -> E4M3 + UE8M0 per 32 values, written straight into the operand
//      images the MMA kernel streams; also zeroes `out` for the scatter-add of pass 4.
//   3. gate/up (persistent, one CTA per SM): unit = (chunk, 128 gate rows + the matching 128 up rows).
//      A TMA producer warp streams both weight tiles per K-group of 128 (tensor map of type
//      16U4_ALIGN16B: packed FP4 in HBM, the tcgen05 unpacked layout in shared memory, 128-byte
//      swizzle), the activation slice and the weight scale-factor blocks; one thread issues
//      tcgen05.cp (scale factors -> TMEM) and tcgen05.mma kind::mxf8f6f4.block_scale (gate -> D0,
//      up -> D1, N = tokens rounded to 8); four epilogue warps compute silu(g) * u, quantize it to
//      MXFP8 per 32 intermediate values and write the down pass's operand images.
//   4. down (same kernel, mode 1): unit = (chunk, 256 output rows as two 128-row tiles); the epilogue
//      scatter-adds routing weight * y into out (fp32 reductions).
//
// Operand images (all K-major, 128 K-bytes per row, 16-byte units XOR-swizzled by row % 8):
//   activations  [K/128][rows][128]        E4M3 codes; the rows of one chunk are contiguous per K-group
//   act scales   [rows/32][K/128][32][16]  UE8M0: row r of block (row block, g) holds the 4 k-block
//                                          scales of K-group g of one token in bytes 0-3 (the tcgen05.cp
//                                          source of one 4-column TMEM cell group; bytes 4-15 unused)
//   weight scales[tiles][K/128][32][16]    row r = the 4 k-block scales of rows r, 32 + r, 64 + r, 96 + r
//                                          of the 128-row tile (TMEM lane m reads column m / 32)
#include <cuda.h>

#include "launchers.h"
#include "common/sm100.cuh"

namespace {

constexpr int kStages = 5;
constexpr int kThreads = 192;  // warp 0 TMA producer, warp 1 MMA issuer, warps 2-5 epilogue
constexpr int kMaxTok = 32;    // tokens per chunk (MMA N <= 32)
constexpr int kMaxG = 32;      // K-groups of 128 (K <= 4096)
constexpr uint32_t kStageA = 16384, kStageB = kMaxTok * 128;
constexpr uint32_t kStageBytes = 2 * kStageA + kStageB + 2 * 512;  // 37888 (multiple of 1024)
constexpr uint32_t kSfbBytes = kMaxG * 512;                         // 16384
constexpr uint32_t kBarOff = kStages * kStageBytes + 2 * kSfbBytes;
constexpr uint32_t kSmemBytes = kBarOff + 256 + 1024;
// TMEM columns: D buffers (2 x {D0: 32, D1: 32}), SFB (2 x 4 per K-group), SFA ring (kStages x 8).
// Every scale-factor address handed to tcgen05.mma is a multiple of 4 columns.
constexpr uint32_t kColD = 0, kColSfb = 128, kColSfa = 384, kTmemCols = 512;
static_assert(kColSfb + 2 * 4 * kMaxG <= kColSfa, "TMEM budget");
static_assert(kColSfa + 8 * kStages <= kTmemCols, "TMEM budget");

struct MxParams {
  int K, G, J, rows_exp, rows_total, H;  // H: output row stride (mode 1) / act K (mode 0, = I)
  int rows_total_w;                      // weight rows (E * rows_exp) of the tensor map
  const uint8_t* sfa;                    // [tiles][G][512]
  const uint8_t* b_img;                  // [G][rows_total][128]
  const uint8_t* sfb_img;                // [rows_total/32][G][512]
  const int4* chunks;
  const int32_t* n_chunks;
  uint8_t* act_img;                      // mode 0: [I/128][rows_total][128]
  uint8_t* act_sf;                       // mode 0: [rows_total/32][I/128][512]
  const int32_t* slot_token;
  const float* slot_weight;
  float* out;                            // mode 1: [T, H]
  int* err;
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
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
    xs[((size_t)(row >> 5) * (H / 128) + (kb >> 2)) * 512 + (row & 31) * 16 + (kb & 3)] = (uint8_t)(e + 127);
  }
}

// ----------------------------------------------------------------------------- expert GEMM
template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) mx_expert_kernel(const __grid_constant__ CUtensorMap tmW,
                                                                const MxParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* empty = full + kStages;
  uint64_t* sfb_full = empty + kStages;
  uint64_t* sfb_empty = sfb_full + 2;
  uint64_t* d_full = sfb_empty + 2;
  uint64_t* d_empty = d_full + 2;
  uint64_t* drain = d_empty + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (warp == 0) {
    pm::tmem_alloc(tslot, kTmemCols);
    pm::tmem_relinquish();
  }
  if (tid == 32) {
    for (int s = 0; s < kStages; ++s) { pm::mbar_init(full + s, 1); pm::mbar_init(empty + s, 1); }
    for (int b = 0; b < 2; ++b) {
      pm::mbar_init(sfb_full + b, 1);
      pm::mbar_init(sfb_empty + b, 1);
      pm::mbar_init(d_full + b, 1);
      pm::mbar_init(d_empty + b, 4);
    }
    pm::mbar_init(drain, 1);
    *abort_flag = 0;
    pm::fence_mbar_init();
  }
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  const uint32_t tmem = *tslot;
  const int nunits = p.n_chunks[0] * p.J;
  const int G = p.G;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int st = 0, lu = 0;
      uint32_t ph = 0;
      uint32_t issued_ph[kStages];
      int n_issued = 0;
      for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x, ++lu) {
        const int j = u % p.J;
        const int4 ct = p.chunks[u / p.J];
        const int n8 = (ct.z + 7) & ~7;
        const int ub = lu & 1;
        const int row0 = ct.x * p.rows_exp + (MODE == 0 ? 128 * j : 256 * j);
        const int row1 = MODE == 0 ? row0 + p.rows_exp / 2 : row0 + 128;
        const uint8_t* sfb_src = p.sfb_img + (size_t)(ct.y >> 5) * G * 512;
        // self-check of the copy geometry (records the unit and skips instead of faulting)
        if ((ct.y & 31) || ct.z < 1 || ct.z > kMaxTok || ct.y + n8 > p.rows_total || row1 + 128 > p.rows_total_w ||
            (reinterpret_cast<uintptr_t>(sfb_src) & 15) || (reinterpret_cast<uintptr_t>(p.b_img) & 15) ||
            (reinterpret_cast<uintptr_t>(p.sfa) & 15)) {
          pm::report_error(p.err, pm::kBadArgument, 100000 + u);
          *abort_flag = 1;
          break;
        }
        if (!pm::mbar_wait(sfb_empty + ub, ((lu >> 1) & 1) ^ 1, p.err, 21)) { *abort_flag = 1; break; }
        pm::mbar_arrive_expect_tx(sfb_full + ub, (uint32_t)G * 512);
        pm::bulk_g2s(smem + kStages * kStageBytes + ub * kSfbBytes, sfb_src, (uint32_t)G * 512, sfb_full + ub);
        for (int g = 0; g < G; ++g) {
          if (!pm::mbar_wait(empty + st, ph ^ 1, p.err, 22)) { *abort_flag = 1; break; }
          uint8_t* sb = smem + st * kStageBytes;
          pm::mbar_arrive_expect_tx(full + st, 2 * 8192 + n8 * 128 + 2 * 512);
          pm::tma_load_2d(sb, &tmW, 128 * g, row0, full + st);
          pm::tma_load_2d(sb + kStageA, &tmW, 128 * g, row1, full + st);
          pm::bulk_g2s(sb + 2 * kStageA, p.b_img + ((size_t)g * p.rows_total + ct.y) * 128, n8 * 128, full + st);
          pm::bulk_g2s(sb + 2 * kStageA + kStageB, p.sfa + ((size_t)(row0 >> 7) * G + g) * 512, 512, full + st);
          pm::bulk_g2s(sb + 2 * kStageA + kStageB + 512, p.sfa + ((size_t)(row1 >> 7) * G + g) * 512, 512,
                       full + st);
          issued_ph[st] = ph;
          ++n_issued;
          if (++st == kStages) { st = 0; ph ^= 1; }
        }
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
      int st = 0, lu = 0;
      uint32_t ph = 0;
      bool any = false;
      for (int u = blockIdx.x; u < nunits && !*abort_flag; u += gridDim.x, ++lu) {
        const int4 ct = p.chunks[u / p.J];
        const int n8 = (ct.z + 7) & ~7;
        const int ub = lu & 1, db = lu & 1;
        const uint32_t uph = (lu >> 1) & 1;
        if (!pm::mbar_wait(sfb_full + ub, uph, p.err, 23) || !pm::mbar_wait(d_empty + db, uph ^ 1, p.err, 24)) {
          *abort_flag = 1;
          break;
        }
        pm::tc_fence_after();
        const uint32_t sfb_col = tmem + kColSfb + 4 * kMaxG * ub;
        const uint32_t sfb_src = pm::smem_u32(smem + kStages * kStageBytes + ub * kSfbBytes);
        for (int g = 0; g < G; ++g) pm::tmem_cp_32x128_x4(sfb_col + 4 * g, sfb_src + 512 * g);
        const uint32_t d0 = tmem + kColD + 64 * db, d1 = d0 + 32;
        for (int g = 0; g < G; ++g) {
          if (!pm::mbar_wait(full + st, ph, p.err, 25)) { *abort_flag = 1; break; }
          pm::tc_fence_after();
          const uint32_t sb = pm::smem_u32(smem + st * kStageBytes);
          const uint32_t sfa_col = tmem + kColSfa + 8 * st;
          pm::tmem_cp_32x128_x4(sfa_col, sb + 2 * kStageA + kStageB);
          pm::tmem_cp_32x128_x4(sfa_col + 4, sb + 2 * kStageA + kStageB + 512);
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const uint32_t idesc = pm::make_idesc_mxf8(128, n8, 5, 0, s, s);
            const uint64_t bd = pm::make_sdesc(sb + 2 * kStageA + 32 * s, 16, 1024);
            const uint32_t acc = (g | s) ? 1u : 0u;
            pm::umma_mxf8(d0, pm::make_sdesc(sb + 32 * s, 16, 1024), bd, idesc, sfa_col, sfb_col + 4 * g, acc);
            pm::umma_mxf8(d1, pm::make_sdesc(sb + kStageA + 32 * s, 16, 1024), bd, idesc, sfa_col + 4,
                          sfb_col + 4 * g, acc);
          }
          pm::umma_commit(empty + st);
          any = true;
          if (++st == kStages) { st = 0; ph ^= 1; }
        }
        if (*abort_flag) break;
        pm::umma_commit(d_full + db);
        pm::umma_commit(sfb_empty + ub);
      }
      if (*abort_flag && any) {
        pm::umma_commit(drain);
        pm::mbar_wait(drain, 0, nullptr, 0, 20000000ull);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-5)
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    int lu = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++lu) {
      const int j = u % p.J;
      const int4 ct = p.chunks[u / p.J];
      const int db = lu & 1;
      if (!pm::mbar_wait(d_full + db, (lu >> 1) & 1, p.err, 26)) { *abort_flag = 1; break; }
      if (*abort_flag) break;
      pm::tc_fence_after();
      const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16) + kColD + 64 * db;
      float a0[16], a1[16], b0[16], b1[16];
      pm::tmem_ld16(lane_addr, a0);
      pm::tmem_ld16(lane_addr + 32, b0);
      if (ct.z > 16) {
        pm::tmem_ld16(lane_addr + 16, a1);
        pm::tmem_ld16(lane_addr + 48, b1);
      }
      pm::tc_fence_before();
      __syncwarp();
      if (lane == 0) pm::mbar_arrive(d_empty + db);
      if (MODE == 0) {
        // intermediate index i = 128 j + 32 q + lane; its k-block (4 j + q) is this warp's 32 lanes
        const int pos = 32 * q + lane;
        const int I = p.H;
#pragma unroll
        for (int n = 0; n < kMaxTok; ++n) {
          if (n < ct.z) {
            const float g = n < 16 ? a0[n & 15] : a1[n & 15];
            const float up = n < 16 ? b0[n & 15] : b1[n & 15];
            const float a = g / (1.f + __expf(-g)) * up;
            const int e = pm::ue8m0_exp(warp_max(fabsf(a)));
            const uint16_t c2 = pm::f32x2_to_e4m3x2(a * pm::exp2i(-e), 0.f);
            const int row = ct.y + n;
            p.act_img[((size_t)j * p.rows_total + row) * 128 + ((((pos >> 4) ^ (row & 7))) << 4) + (pos & 15)] =
                (uint8_t)(c2 & 0xFF);
            if (lane == 0)
              p.act_sf[((size_t)(row >> 5) * (I / 128) + j) * 512 + (row & 31) * 16 + q] = (uint8_t)(e + 127);
          }
        }
      } else {
        const int h0 = 256 * j + 32 * q + lane;
#pragma unroll
        for (int n = 0; n < kMaxTok; ++n) {
          if (n < ct.z) {
            const int t = p.slot_token[ct.w + n];
            const float w = p.slot_weight[ct.w + n];
            float* o = p.out + (size_t)t * p.H;
            atomicAdd(o + h0, w * (n < 16 ? a0[n & 15] : a1[n & 15]));
            atomicAdd(o + h0 + 128, w * (n < 16 ? b0[n & 15] : b1[n & 15]));
          }
        }
      }
    }
  }
  pm::tc_fence_before();
  __syncthreads();
  if (warp == 0) pm::tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

int launch_moe_mxf4(const MoeMxArgs& a, cudaStream_t stream) {
  if (a.T == 0) return 0;
  if (a.H % 512 || a.I % 512 || a.H / 128 > kMaxG || a.I / 128 > kMaxG || a.rows_total % 32) return -2;
  const int n = a.T * a.k;
  launch_moe_route_chunks(a.topk_ids, a.topk_w, a.T, a.k, a.expert_base, a.E, a.offsets, a.slot_token,
                          a.slot_weight, a.active, a.pad, a.chunks, a.n_chunks, stream);
  mx_quant_kernel<<<max(n, a.T), 128, 0, stream>>>(a.h, a.H, a.E, a.offsets, a.pad, a.slot_token, a.rows_total, a.xq,
                                                   a.xs, a.out, a.T);
  CUtensorMap m13, m2;
  int rc = make_tmap_fp4_unpacked(&m13, a.w13, a.H, (uint64_t)a.E * 2 * a.I, a.H / 2, 128);
  if (rc) return rc;
  rc = make_tmap_fp4_unpacked(&m2, a.w2, a.I, (uint64_t)a.E * a.H, a.I / 2, 128);
  if (rc) return rc;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(mx_expert_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    cudaFuncSetAttribute(mx_expert_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    attr = true;
  }
  if ((reinterpret_cast<uintptr_t>(a.xq) | reinterpret_cast<uintptr_t>(a.xs) | reinterpret_cast<uintptr_t>(a.act_q) |
       reinterpret_cast<uintptr_t>(a.act_s) | reinterpret_cast<uintptr_t>(a.sfa13) | reinterpret_cast<uintptr_t>(a.sfa2) |
       reinterpret_cast<uintptr_t>(a.chunks) | reinterpret_cast<uintptr_t>(a.out)) & 15)
    return -3;
  MxParams p0{a.H, a.H / 128, a.I / 128, 2 * a.I, a.rows_total, a.I, a.E * 2 * a.I, a.sfa13, a.xq, a.xs, a.chunks, a.n_chunks,
              a.act_q, a.act_s, a.slot_token, a.slot_weight, a.out, a.err};
  mx_expert_kernel<0><<<a.num_sms, kThreads, kSmemBytes, stream>>>(m13, p0);
  MxParams p1{a.I, a.I / 128, a.H / 256, a.H, a.rows_total, a.H, a.E * a.H, a.sfa2, a.act_q, a.act_s, a.chunks, a.n_chunks,
              nullptr, nullptr, a.slot_token, a.slot_weight, a.out, a.err};
  mx_expert_kernel<1><<<a.num_sms, kThreads, kSmemBytes, stream>>>(m2, p1);
  return 0;
}
