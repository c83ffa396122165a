// Sparse MLA decode attention on tcgen05 (Native and Direct-Packed KV), plus split combine.
//
// Reference behaviour: FlashMLA sparse FP8 decode, Native <1,64,0> and Direct Packed <1,64,1>
// (K1/K2, third_party/README.md:355-361) and `flash_fwd_mla_combine_kernel` (K3).  Semantics:
// joint softmax over [SWA rows ; selected C4 rows] with a per-head sink, K = V = latent row,
// output tail inverse-rotated with the query position (training/losses.py:121-126).
//
// Design (sm_100a): one CTA = (query b, group of 64 heads, KV split).  Per tile of 128 KV rows:
//   1. 8 warps gather the rows (Native 584 B or Packed 328 B) and expand them into a dense BF16
//      tile [128 x 512] in shared memory, 128-byte swizzled (Packed: bitmap POPC prefix,
//      E4M3 x UE8M0 dequant, BF16 round, tail RoPE with the record position).
//   2. one thread issues S^T = K Q^T   (tcgen05.mma kind::f16, M=128 rows, N=64 heads, K=512)
//      into TMEM columns [256, 320).
//   3. 8 warps read S^T with tcgen05.ld, do the online softmax per head (column reductions by
//      shuffles), write P^T (BF16) to shared memory; O^T is rescaled in TMEM only when a head's
//      running max grows by more than 2^8 (exact: the final division uses the same reference max).
//   4. one thread issues O^T += V^T P^T (four M=128 d-blocks, N=64, K=128) into TMEM [0, 256);
//      V^T is the same shared tile read through an MN-major descriptor.
// The partial (O unnormalized, m, l) per split goes to global memory; the combine kernel merges
// splits, adds the sink, normalizes, inverse-rotates the tail and writes BF16 O and LSE.
#include "launchers.h"
#include "common/sm100.cuh"

namespace {

constexpr int kD = 512;
constexpr int kHG = 64;           // heads per CTA group
constexpr int kTile = 128;        // KV rows per tile
constexpr int kThreads = 256;
constexpr int kPage = 64;
constexpr int kNativeData = 576;
constexpr int kNativePageBytes = kPage * 584;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;

// shared memory map (bytes, from a 1024-aligned base)
constexpr int kQBytes = kHG * kD * 2;        // 65536
constexpr int kKVBytes = kTile * kD * 2;     // 131072
constexpr int kPBytes = kTile * kHG * 2;     // 16384
constexpr int kStageBytes = 592;             // per-warp raw row staging
constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + kQBytes;
constexpr int kOffP = kOffKV + kKVBytes;
constexpr int kOffStage = kOffP + kPBytes;
constexpr int kOffRed = kOffStage + 8 * kStageBytes;  // float red[8][32]
constexpr int kOffHead = kOffRed + 8 * 32 * 4;          // m_used[64], l[64], alpha[64]
constexpr int kOffMisc = kOffHead + 3 * 64 * 4;         // bars, tmem addr, flags
constexpr int kOffRowValid = kOffMisc + 64;            // uint8 rowvalid[128]
constexpr int kSmemBytes = kOffRowValid + 128 + 1024;   // + alignment slack

constexpr uint32_t kTmemO = 0;
constexpr uint32_t kTmemS = 256;
constexpr uint32_t kTmemCols = 512;


__device__ __forceinline__ uint4 zero4() { return make_uint4(0, 0, 0, 0); }

// 8 E4M3 bytes * 2^e -> 8 BF16 packed in uint4 (exact).
__device__ __forceinline__ uint4 dequant8(uint2 codes, float s) {
  uint32_t w[2] = {codes.x, codes.y};
  __nv_bfloat162 out[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint16_t pair = (uint16_t)(w[k >> 1] >> (16 * (k & 1)));
    const float2 f = __half22float2(pm::e4m3x2_to_h2(pair));
    out[k] = __floats2bfloat162_rn(f.x * s, f.y * s);
  }
  return *reinterpret_cast<uint4*>(out);
}

struct RowRef {
  int kind;  // 0 = masked, 1 = native (swa pool), 2 = native (csa pool), 3 = packed
  int slot;
  int pos;
};

__device__ __forceinline__ RowRef row_ref(const DecodeParams& p, int b, int i, int nswa, int ntot) {
  RowRef r{0, -1, 0};
  if (i >= ntot) return r;
  if (i < nswa) {
    const int s = p.swa_slots[(int64_t)b * p.swa_cap + i];
    if (s >= 0 && s < p.swa_pool_slots) { r.kind = 1; r.slot = s; }
    else if (s >= p.swa_pool_slots) pm::report_error(p.err, pm::kIndexOutOfRange, i);
    return r;
  }
  const int j = i - nswa;
  const int s = p.csa_slots[(int64_t)b * p.csa_cap + j];
  const int pos = p.csa_pos[(int64_t)b * p.csa_cap + j];
  if (s < 0) return r;
  if (s >= p.csa_pool_rows || (p.csa_packed && (pos < 0 || pos >= p.freq_rows))) {
    pm::report_error(p.err, pm::kIndexOutOfRange, i);
    return r;
  }
  r.kind = p.csa_packed ? 3 : 2;
  r.slot = s;
  r.pos = pos;
  return r;
}

// Raw bytes of one row, as two 16-byte pieces per lane:
//   A -> stage[16 lane]       (native data units 0..31; packed values 0..15, bitmap 16..19, scales 20)
//   B -> stage[512 + 16 lane] (native data units 32..35 for lanes 0..3, scales for lane 4)
// Packed rows: lanes 24..31, which rotate the tail units 56..63, also prefetch their four RoPE
// (cos, sin) pairs into A and B, so no dependent global load sits on the expansion path.
__device__ __forceinline__ void load_row_raw(const DecodeParams& p, int kind, int slot, int pos, int lane, uint4& A,
                                             uint4& B) {
  A = zero4();
  B = zero4();
  if (kind == 1 || kind == 2) {
    const uint8_t* pool = kind == 1 ? p.swa_pool : p.csa_pool;
    const int64_t page = slot / kPage, rip = slot % kPage;
    const uint8_t* data = pool + page * kNativePageBytes + rip * kNativeData;
    A = *reinterpret_cast<const uint4*>(data + 16 * lane);
    if (lane < 4) B = *reinterpret_cast<const uint4*>(data + 512 + 16 * lane);
    if (lane == 4) {
      const uint2 s = *reinterpret_cast<const uint2*>(pool + page * kNativePageBytes + kPage * kNativeData + rip * 8);
      B = make_uint4(s.x, s.y, 0, 0);
    }
  } else if (kind == 3) {
    if (lane < 16) A = *reinterpret_cast<const uint4*>(p.csa_values + (int64_t)slot * 256 + 16 * lane);
    else if (lane < 20)
      A = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(p.csa_bitmap + (int64_t)slot * 8) + 16 * (lane - 16));
    else if (lane == 20) {
      const uint2 s = *reinterpret_cast<const uint2*>(p.csa_scales + (int64_t)slot * 8);
      A = make_uint4(s.x, s.y, 0, 0);
    } else if (lane >= 24) {
      const float* f = p.freqs + (int64_t)pos * 64 + 8 * (lane - 24);
      A = *reinterpret_cast<const uint4*>(f);
      B = *reinterpret_cast<const uint4*>(f + 4);
    }
  }
}

// Exclusive prefix of kept-coordinate counts over bitmap words: lane w (< 8) holds it for word w.
__device__ __forceinline__ int wprefix_of(int wpre, int w) { return __shfl_sync(0xffffffffu, wpre, w); }

// Warp-cooperative: staged raw row -> 64 units of 8 BF16 in the swizzled dense tile (row `trow`).
__device__ __forceinline__ void expand_row(const DecodeParams& p, int kind, int pos, int trow, uint8_t* stage,
                                           uint8_t* kv, int lane, const uint4& A, const uint4& B) {
  *reinterpret_cast<uint4*>(stage + 16 * lane) = A;
  if (lane < 5) *reinterpret_cast<uint4*>(stage + 512 + 16 * lane) = B;
  __syncwarp();
  int wpre = 0;
  if (kind == 3) {
    const int pc = lane < 8 ? __popcll(reinterpret_cast<const uint64_t*>(stage + 256)[lane]) : 0;
    int incl = pc;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    wpre = incl - pc;
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int u = lane + 32 * h;
    uint4 outv = zero4();
    if (kind == 1 || kind == 2) {
      if (u < 56) {
        const uint2 codes = *reinterpret_cast<const uint2*>(stage + 8 * u);
        const int e = (int)stage[576 + (u >> 3)] - 127;
        outv = dequant8(codes, pm::exp2i(e));
      } else {
        outv = *reinterpret_cast<const uint4*>(stage + 448 + 16 * (u - 56));
      }
    } else if (kind == 3) {
      const uint64_t* words = reinterpret_cast<const uint64_t*>(stage + 256);
      const int w = u >> 3, shift = 8 * (u & 7);
      const uint64_t word = words[w];
      const int rank = wprefix_of(wpre, w) + __popcll(word & ((1ull << shift) - 1ull));
      const uint32_t bits = (uint32_t)(word >> shift) & 0xFFu;
      const float s = pm::exp2i((int)stage[320 + w] - 127);
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int k = __popc(bits & ((1u << i) - 1u));
        const uint16_t c = stage[min(rank + k, 255)];
        const float f = __half2float(__low2half(pm::e4m3x2_to_h2(c))) * s;
        v[i] = (bits >> i) & 1u ? f : 0.f;
      }
      if (u >= 56) {  // RoPE tail: pairs (2i, 2i+1), pair index 4 (u - 56) + i; (cos, sin) in A, B
        const float cs[8] = {__uint_as_float(A.x), __uint_as_float(A.y), __uint_as_float(A.z), __uint_as_float(A.w),
                             __uint_as_float(B.x), __uint_as_float(B.y), __uint_as_float(B.z), __uint_as_float(B.w)};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float c = cs[2 * i], sn = cs[2 * i + 1];
          const float re = __bfloat162float(__float2bfloat16_rn(v[2 * i]));
          const float im = __bfloat162float(__float2bfloat16_rn(v[2 * i + 1]));
          v[2 * i] = __fsub_rn(__fmul_rn(re, c), __fmul_rn(im, sn));
          v[2 * i + 1] = __fadd_rn(__fmul_rn(re, sn), __fmul_rn(im, c));
        }
      }
      __nv_bfloat162 o2[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) o2[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      outv = *reinterpret_cast<uint4*>(o2);
    }
    *reinterpret_cast<uint4*>(kv + pm::sw128_offset(trow, 16 * u, kTile * 128)) = outv;
  }
  __syncwarp();
}

// Lane L returns op-reduction over the 32 lanes of v[L] (31 shuffles instead of 160).
template <bool kMax>
__device__ __forceinline__ float transpose_reduce(float (&v)[32], int lane) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = upper ? v[i] : v[i + o];
      const float keep = upper ? v[i + o] : v[i];
      const float got = __shfl_xor_sync(0xffffffffu, send, o);
      v[i] = kMax ? fmaxf(keep, got) : keep + got;
    }
  }
  return v[0];
}

__global__ void __launch_bounds__(kThreads, 1) sparse_mla_decode_kernel(const DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem + kOffQ;
  uint8_t* sKV = smem + kOffKV;
  uint8_t* sP = smem + kOffP;
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  float* m_used = reinterpret_cast<float*>(smem + kOffHead);
  float* l_sum = m_used + 64;
  float* alpha = l_sum + 64;
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(smem + kOffMisc);
  uint64_t* bar_o = bar_s + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_s + 2);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] rescale needed, [1] abort
  uint8_t* rowvalid = smem + kOffRowValid;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int unit = blockIdx.x;
  const int split = unit % p.num_splits;
  const int g = (unit / p.num_splits) % p.num_groups;
  const int b = unit / (p.num_splits * p.num_groups);
  const int h0 = g * kHG;

  if (warp == 0) {
    pm::tmem_alloc(tmem_slot, kTmemCols);
    pm::tmem_relinquish();
  }
  if (tid == 0) {
    pm::mbar_init(bar_s, 1);
    pm::mbar_init(bar_o, 1);
    pm::fence_mbar_init();
    flags[0] = 0;
    flags[1] = 0;
  }
  if (tid < 64) { m_used[tid] = -INFINITY; l_sum[tid] = 0.f; alpha[tid] = 1.f; }

  // Q group -> shared (K-major, SW128, chunk stride 64 rows * 128 B)
  for (int idx = tid; idx < kHG * 64; idx += kThreads) {
    const int row = idx >> 6, u = idx & 63;
    uint4 v = zero4();
    if (h0 + row < p.H)
      v = *reinterpret_cast<const uint4*>(p.q + (int64_t)b * p.q_stride_b + (int64_t)(h0 + row) * p.q_stride_h + 8 * u);
    *reinterpret_cast<uint4*>(sQ + pm::sw128_offset(row, 16 * u, kHG * 128)) = v;
  }
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int nswa = min(p.swa_len[b], p.swa_cap);
  const int ntot = nswa + min(p.csa_len[b], p.csa_cap);
  const int row0 = split * p.rows_per_split;
  const int row1 = min(ntot, row0 + p.rows_per_split);
  const int ntiles = row1 > row0 ? (row1 - row0 + kTile - 1) / kTile : 0;

  const uint32_t q_base = pm::smem_u32(sQ), kv_base = pm::smem_u32(sKV), p_base = pm::smem_u32(sP);
  const uint32_t idesc_s = pm::make_idesc_f16(128, kHG, 1, 0, 0);
  const uint32_t idesc_o = pm::make_idesc_f16(128, kHG, 1, 1, 1);
  bool ok = true;

  uint8_t* stage = smem + kOffStage + warp * kStageBytes;
  struct Batch {
    uint4 A[8], B[8];
    int kind[8], pos[8];
  } bk;
  // rows warp + 8 (8 k + j), j = 0..7, of tile tt: index lookups by lanes 0..7, then raw loads
  auto load_batch = [&](int tt, int k) {
    const int tb = row0 + tt * kTile;
    const int tv = min(kTile, row1 - tb);
    RowRef mine{0, -1, 0};
    const int r = warp + 8 * (8 * k + (lane & 7));
    if (lane < 8 && r < tv) mine = row_ref(p, b, tb + r, nswa, ntot);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      bk.kind[j] = __shfl_sync(0xffffffffu, mine.kind, j);
      const int slot = __shfl_sync(0xffffffffu, mine.slot, j);
      bk.pos[j] = __shfl_sync(0xffffffffu, mine.pos, j);
      if (p.debug & 4) { bk.A[j] = zero4(); bk.B[j] = zero4(); }
      else load_row_raw(p, bk.kind[j], slot, bk.pos[j], lane, bk.A[j], bk.B[j]);
    }
  };

  for (int t = 0; t < ntiles && ok; ++t) {
    const int tbase = row0 + t * kTile;
    const int tvalid = min(kTile, row1 - tbase);
    // ---- 1. gather + expand 128 rows (warp w: rows w + 8 i), two batches of 8 rows; batch 0 of
    //         this tile was loaded while the previous tile's P.V MMAs ran
    if (t == 0) load_batch(0, 0);
#pragma unroll 1
    for (int k = 0; k < 2; ++k) {
      if (k == 1) load_batch(t, 1);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = warp + 8 * (8 * k + j);
        if (!(p.debug & 2)) expand_row(p, bk.kind[j], bk.pos[j], r, stage, sKV, lane, bk.A[j], bk.B[j]);
        if (lane == 0) rowvalid[r] = bk.kind[j] != 0;
      }
    }
    pm::fence_proxy_async_smem();
    pm::tc_fence_before();
    __syncthreads();
    pm::tc_fence_after();
    // ---- 2. S^T = K Q^T
    if (tid == 0) {
#pragma unroll 1
      for (int k = 0; k < kD / 16 && !(p.debug & 1); ++k) {
        const uint32_t koff = (k * 32) & 127;
        const uint64_t ad = pm::make_sdesc(kv_base + (k >> 2) * (kTile * 128) + koff, 16, 1024);
        const uint64_t bd = pm::make_sdesc(q_base + (k >> 2) * (kHG * 128) + koff, 16, 1024);
        pm::umma_f16(tmem + kTmemS, ad, bd, idesc_s, k > 0);
      }
      pm::umma_commit(bar_s);
    }
    if (!pm::mbar_wait(bar_s, t & 1, p.err, 1)) { flags[1] = 1; }
    pm::tc_fence_after();
    // ---- 3. softmax over rows (lanes) per head (columns)
    const int quarter = warp & 3, chalf = warp >> 2;
    const int n = 32 * quarter + lane;  // KV row within tile
    float s[32];
    {
      float a[16], c[16];
      const uint32_t ta = tmem + kTmemS + 32 * chalf + ((uint32_t)(32 * quarter) << 16);
      pm::tmem_ld16(ta, a);
      pm::tmem_ld16(ta + 16, c);
      pm::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i) { s[i] = a[i]; s[16 + i] = c[i]; }
    }
    const bool row_ok = rowvalid[n] != 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) s[i] = row_ok ? s[i] * p.scale_log2 : -INFINITY;
    // column max: transpose-reduce over lanes, then across the 4 quarter-warps of this column half
    {
      float mx[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) mx[i] = s[i];
      red[warp * 32 + lane] = transpose_reduce<true>(mx, lane);
    }
    __syncthreads();
    if (tid < 64) {
      const int h = tid, hc = h >> 5, hl = h & 31;
      float tmax = -INFINITY;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) tmax = fmaxf(tmax, red[(hc * 4 + q4) * 32 + hl]);
      const float mu = m_used[h];
      float a = 1.f;
      if (tmax > mu + kRescaleThreshold || mu == -INFINITY) {
        a = (mu == -INFINITY) ? 0.f : exp2f(mu - tmax);
        m_used[h] = tmax;
        if (mu != -INFINITY) flags[0] = 1;
      }
      alpha[h] = a;
    }
    __syncthreads();
    // p = 2^(s - m_used), write P^T (MN-major SW128: row n = 64 heads * 2 B)
    float psum[32];
    {
      __nv_bfloat162 pk[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float m0 = m_used[32 * chalf + i], m1 = m_used[32 * chalf + i + 1];
        const float p0 = (s[i] == -INFINITY || m0 == -INFINITY) ? 0.f : exp2f(s[i] - m0);
        const float p1 = (s[i + 1] == -INFINITY || m1 == -INFINITY) ? 0.f : exp2f(s[i + 1] - m1);
        pk[i >> 1] = __floats2bfloat162_rn(p0, p1);
        // sum the BF16-rounded probabilities so l matches what the PV MMA accumulates
        const float2 r = __bfloat1622float2(pk[i >> 1]);
        psum[i] = r.x;
        psum[i + 1] = r.y;
      }
#pragma unroll
      for (int uu = 0; uu < 4; ++uu)
        *reinterpret_cast<uint4*>(sP + pm::sw128_offset(n, 64 * chalf + 16 * uu, 0)) =
            *reinterpret_cast<uint4*>(&pk[4 * uu]);
    }
    red[warp * 32 + lane] = transpose_reduce<false>(psum, lane);
    // rescale O^T columns if some head's reference max moved (rare)
    if (flags[0] && t > 0) {
      // warp w: lane quarter w%4, d-blocks 2*(w/4) .. +1, 64 head columns each
#pragma unroll 1
      for (int db = 2 * chalf; db < 2 * chalf + 2; ++db) {
#pragma unroll 1
        for (int c0 = 0; c0 < kHG; c0 += 16) {
          float v[16];
          const uint32_t ta = tmem + kTmemO + db * kHG + c0 + ((uint32_t)(32 * quarter) << 16);
          pm::tmem_ld16(ta, v);
          pm::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] *= alpha[c0 + i];
          pm::tmem_st16(ta, v);
        }
      }
      pm::tmem_wait_st();
    }
    pm::fence_proxy_async_smem();
    pm::tc_fence_before();
    __syncthreads();
    pm::tc_fence_after();
    if (tid < 64) {
      const int h = tid, hc = h >> 5, hl = h & 31;
      float ts = 0.f;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) ts += red[(hc * 4 + q4) * 32 + hl];
      l_sum[h] = l_sum[h] * alpha[h] + ts;
      if (h == 0) flags[0] = 0;
    }
    // ---- 4. O^T += V^T P^T
    if (tid == 0 && !flags[1]) {
#pragma unroll 1
      for (int db = 0; db < 4 && !(p.debug & 1); ++db) {
#pragma unroll 1
        for (int k = 0; k < kTile / 16; ++k) {
          const uint64_t ad = pm::make_sdesc(kv_base + (2 * db) * (kTile * 128) + k * 2048, kTile * 128, 1024);
          const uint64_t bd = pm::make_sdesc(p_base + k * 2048, 8192, 1024);
          pm::umma_f16(tmem + kTmemO + db * kHG, ad, bd, idesc_o, (t > 0 || k > 0) ? 1u : 0u);
        }
      }
      pm::umma_commit(bar_o);
    }
    if (t + 1 < ntiles) load_batch(t + 1, 0);  // overlaps the P.V MMAs
    if (!flags[1]) {
      if (!pm::mbar_wait(bar_o, t & 1, p.err, 2)) flags[1] = 1;
    }
    pm::tc_fence_after();
    __syncthreads();
    ok = !flags[1];
  }

  // ---- epilogue: partial O (unnormalized, relative to m_used), m, l
  const int64_t part = ((int64_t)b * p.num_splits + split);
  if (ok && ntiles > 0) {
    const int quarter = warp & 3, chalf = warp >> 2;
#pragma unroll 1
    for (int db = 2 * chalf; db < 2 * chalf + 2; ++db) {
      const int d = 128 * db + 32 * quarter + lane;
#pragma unroll 1
      for (int c0 = 0; c0 < kHG; c0 += 16) {
        float v[16];
        pm::tmem_ld16(tmem + kTmemO + db * kHG + c0 + ((uint32_t)(32 * quarter) << 16), v);
        pm::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int h = h0 + c0 + i;
          if (h < p.H) p.part_o[(part * p.H + h) * kD + d] = v[i];
        }
      }
    }
  }
  if (tid < 64 && h0 + tid < p.H) {
    const bool empty = !(ok && ntiles > 0);
    p.part_ml[(part * p.H + h0 + tid) * 2 + 0] = empty ? -INFINITY : m_used[tid];
    p.part_ml[(part * p.H + h0 + tid) * 2 + 1] = empty ? 0.f : l_sum[tid];
  }
  pm::tc_fence_before();
  __syncthreads();
  if (warp == 0) pm::tmem_dealloc(tmem, kTmemCols);
}

// ----------------------------------------------------------------------------- combine
// One warp per (b, h): lane owns 16 coordinates.
__global__ void __launch_bounds__(256) mla_combine_kernel(const float* __restrict__ part_o,
                                                          const float* __restrict__ part_ml,
                                                          const float* __restrict__ sink, float scale_log2_unused,
                                                          const int32_t* __restrict__ q_pos,
                                                          const float* __restrict__ freqs, int64_t freq_rows, int B,
                                                          int H, int splits, __nv_bfloat16* __restrict__ out,
                                                          float* __restrict__ lse, int* err) {
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (wid >= B * H) return;
  const int b = wid / H, h = wid % H;
  const float sink2 = sink ? sink[h] * kLog2e : -INFINITY;
  float M = sink2;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_ml[(((int64_t)b * splits + s) * H + h) * 2]);
  float L = (sink2 == -INFINITY) ? 0.f : exp2f(sink2 - M);
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.f;
  for (int s = 0; s < splits; ++s) {
    const int64_t base = ((int64_t)b * splits + s) * H + h;
    const float m = part_ml[base * 2], l = part_ml[base * 2 + 1];
    if (m == -INFINITY) continue;
    const float w = exp2f(m - M);
    L += w * l;
    const float* o = part_o + base * kD;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(o + 128 * j + 4 * lane);
      acc[4 * j + 0] += w * v.x; acc[4 * j + 1] += w * v.y; acc[4 * j + 2] += w * v.z; acc[4 * j + 3] += w * v.w;
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  float o[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i] = __bfloat162float(__float2bfloat16_rn(acc[i] * inv));
  // inverse-rotate the tail (coords 448..511 live in chunk j = 3, lanes 16..31)
  if (lane >= 16) {
    int pos = q_pos ? q_pos[b] : 0;
    if (pos < 0 || pos >= freq_rows) { pm::report_error(err, pm::kIndexOutOfRange, b); pos = 0; }
    const float* f = freqs + (int64_t)pos * 64;
#pragma unroll
    for (int pp = 0; pp < 2; ++pp) {
      const int pair = 2 * (lane - 16) + pp;
      const float c = f[2 * pair], sn = -f[2 * pair + 1];
      const float re = o[12 + 2 * pp], im = o[13 + 2 * pp];
      o[12 + 2 * pp] = __fsub_rn(__fmul_rn(re, c), __fmul_rn(im, sn));
      o[13 + 2 * pp] = __fadd_rn(__fmul_rn(re, sn), __fmul_rn(im, c));
    }
  }
  __nv_bfloat16* orow = out + ((int64_t)b * H + h) * kD;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat162 v0 = __floats2bfloat162_rn(o[4 * j], o[4 * j + 1]);
    __nv_bfloat162 v1 = __floats2bfloat162_rn(o[4 * j + 2], o[4 * j + 3]);
    uint2 pk = make_uint2(*reinterpret_cast<uint32_t*>(&v0), *reinterpret_cast<uint32_t*>(&v1));
    *reinterpret_cast<uint2*>(orow + 128 * j + 4 * lane) = pk;
  }
  if (lse && lane == 0) lse[(int64_t)b * H + h] = (L > 0.f) ? (M + log2f(L)) / kLog2e : -INFINITY;
}

}  // namespace

void launch_sparse_mla_decode(const DecodeParams& p, const float* sink, const int32_t* q_pos,
                              __nv_bfloat16* out, float* lse, cudaStream_t stream) {
  if (p.B == 0) return;
  cudaFuncSetAttribute(sparse_mla_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  const int grid = p.B * p.num_groups * p.num_splits;
  sparse_mla_decode_kernel<<<grid, kThreads, kSmemBytes, stream>>>(p);
  const int warps = p.B * p.H;
  mla_combine_kernel<<<(warps + 7) / 8, 256, 0, stream>>>(p.part_o, p.part_ml, sink, p.scale_log2, q_pos, p.freqs,
                                                          p.freq_rows, p.B, p.H, p.num_splits, out, lse, p.err);
}
