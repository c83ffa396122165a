// Sparse MLA decode attention on tcgen05 (Native and Direct-Packed KV), plus split combine.
//
// Reference behaviour: FlashMLA sparse FP8 decode, Native <1,64,0> and Direct Packed <1,64,1>
// (third_party/README.md:355-361) and `flash_fwd_mla_combine_kernel`.  Semantics:
// joint softmax over [SWA rows ; selected C4 rows] with a per-head sink, K = V = latent row,
// output tail inverse-rotated with the query position (training/losses.py:121-126).
//
// Design (sm_100a): one CTA = (query b, group of 64 heads, KV split).  Per tile of 128 KV rows:
//   1. 8 warps gather the rows (Native 584 B or Packed 328 B) and expand them into a dense BF16
//      tile [128 x 512] in shared memory, 128-byte swizzled (Packed: bitmap POPC prefix,
//      E4M3 x UE8M0 dequant, BF16 round, tail RoPE with the record position).  A warp takes 4 rows
//      per step with 8 lanes per row: the lanes copy the raw record (and a Packed row's RoPE
//      table row) into the warp's staging, then each lane expands one 64-coordinate word (one
//      UE8M0 scale tile) 8 coordinates at a time: the unit's kept bytes are placed with one byte
//      permute from a mask-indexed table; the next step's record loads are in flight meanwhile.
//      A query's rows are split over the CTAs of its splits in whole tiles, as evenly as possible.
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
constexpr int kStageRow = 592;               // raw row staging: record (<= 584 B) or packed + RoPE row
constexpr int kStageBytes = 4 * kStageRow;   // per warp: 4 rows
constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + kQBytes;
constexpr int kOffP = kOffKV + kKVBytes;
// the gather staging is live only during a tile's gather, P only from its softmax to its P.V MMA
// (complete before the next gather starts): the two share one region
constexpr int kOffStage = kOffP;
constexpr int kPStageBytes = kPBytes > 8 * kStageBytes ? kPBytes : 8 * kStageBytes;
constexpr int kOffRed = kOffP + kPStageBytes;  // float red[8][32]
constexpr int kOffHead = kOffRed + 8 * 32 * 4;          // m_used[64], l[64], alpha[64]
constexpr int kOffMisc = kOffHead + 3 * 64 * 4;         // bars, tmem addr, flags
constexpr int kOffRowValid = kOffMisc + 64;            // uint8 rowvalid[128]
constexpr int kOffExpand = kOffRowValid + 128;         // uint4 expand_lut[256]
constexpr int kSmemBytes = kOffExpand + 256 * 16 + 1024;  // + alignment slack

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

// 8 E4M3 bytes (little-endian in codes.x, codes.y) * s -> 8 floats (exact).
__device__ __forceinline__ void dequant8f(uint2 codes, float s, float (&f)[8]) {
  const uint32_t w[2] = {codes.x, codes.y};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 v = __half22float2(pm::e4m3x2_to_h2((uint16_t)(w[k >> 1] >> (16 * (k & 1)))));
    f[2 * k] = v.x * s;
    f[2 * k + 1] = v.y * s;
  }
}

// Byte expansion of a Packed 8-coordinate unit with kept-mask m: the unit's kept values are the 8
// bytes starting at its rank (lo, hi); entry m = {selector of coords 0-3, selector of coords 4-7,
// mask 0-3, mask 4-7} for __byte_perm, so codes = perm(lo, hi, sel) & mask (E4M3 zero = 0x00).
__device__ __forceinline__ uint4 expand_lut_entry(int m) {
  uint32_t sel[2] = {0, 0}, msk[2] = {0, 0};
  int r = 0;
  for (int i = 0; i < 8; ++i) {
    if ((m >> i) & 1) {
      sel[i >> 2] |= (uint32_t)r << (4 * (i & 3));
      msk[i >> 2] |= 0xFFu << (8 * (i & 3));
      ++r;
    }
  }
  return make_uint4(sel[0], sel[1], msk[0], msk[1]);
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

// ----------------------------------------------------------------------------- tile gather
// One gather step of a warp: rows 4 warp + j + 32 k (j = lane / 8) of the tile, lane v = lane % 8 of
// the row.  Raw 16-byte units of the row are spread over its 8 lanes (unit v + 8 i).
//   Native (584 B): units 0..35 = data (448 E4M3 + 128 B BF16 tail), scale row (8 B) by lane v = 0.
//   Packed (328 B): units 0..15 values, 16..19 bitmap, scales by v = 0; the record's RoPE table row
//   (64 floats) staged at byte 336 (a staged row is 592 bytes).
struct StepRegs {
  uint4 U[5];
  uint2 sc;
  int kind, pos;
};

__device__ __forceinline__ RowRef step_ref(const DecodeParams& p, int b, int tbase, int tvalid, int nswa, int ntot,
                                           int r) {
  return r < tvalid ? row_ref(p, b, tbase + r, nswa, ntot) : RowRef{0, -1, 0};
}

// Raw loads of one step from its (already resolved) row reference.
__device__ __forceinline__ void fetch_step(const DecodeParams& p, const RowRef& rr, int v, StepRegs& R) {
  R.kind = rr.kind;
  R.pos = rr.pos;
  R.sc = make_uint2(0, 0);
#pragma unroll
  for (int i = 0; i < 5; ++i) R.U[i] = zero4();
  if (rr.kind == 1 || rr.kind == 2) {
    const uint8_t* pool = rr.kind == 1 ? p.swa_pool : p.csa_pool;
    const int64_t page = rr.slot / kPage, rip = rr.slot % kPage;
    const uint8_t* data = pool + page * kNativePageBytes + rip * kNativeData;
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      const int u = v + 8 * i;
      if (u < 36) R.U[i] = *reinterpret_cast<const uint4*>(data + 16 * u);
    }
    if (v == 0) R.sc = *reinterpret_cast<const uint2*>(pool + page * kNativePageBytes + kPage * kNativeData + rip * 8);
  } else if (rr.kind == 3) {
    const uint4* vals = reinterpret_cast<const uint4*>(p.csa_values + (int64_t)rr.slot * 256);
    const uint4* bits = reinterpret_cast<const uint4*>(p.csa_bitmap + (int64_t)rr.slot * 8);
    const uint4* fq = reinterpret_cast<const uint4*>(p.freqs + (int64_t)rr.pos * 64);
    R.U[0] = vals[v];
    R.U[1] = vals[v + 8];
    if (v < 4) R.U[2] = bits[v];
    R.U[3] = fq[v];
    R.U[4] = fq[v + 8];
    if (v == 0) R.sc = *reinterpret_cast<const uint2*>(p.csa_scales + (int64_t)rr.slot * 8);
  }
}

// Stage the row, then expand word v (coordinates 64 v .. 64 v + 63) of it into tile row `trow`, one
// 16-byte unit (8 coordinates) at a time (rolled loops keep the kernel within the instruction cache).
__device__ __forceinline__ void expand_step(const StepRegs& R, int trow, int v, uint8_t* __restrict__ srow,
                                            uint8_t* __restrict__ kv, uint8_t* __restrict__ rowvalid,
                                            const uint4* __restrict__ expand_lut) {
  if (R.kind == 1 || R.kind == 2) {
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      const int u = v + 8 * i;
      if (u < 36) *reinterpret_cast<uint4*>(srow + 16 * u) = R.U[i];
    }
    if (v == 0) *reinterpret_cast<uint2*>(srow + 576) = R.sc;
  } else if (R.kind == 3) {
    *reinterpret_cast<uint4*>(srow + 16 * v) = R.U[0];
    *reinterpret_cast<uint4*>(srow + 16 * (v + 8)) = R.U[1];
    if (v < 4) *reinterpret_cast<uint4*>(srow + 256 + 16 * v) = R.U[2];
    if (v == 0) *reinterpret_cast<uint2*>(srow + 320) = R.sc;
    *reinterpret_cast<uint4*>(srow + 336 + 16 * v) = R.U[3];
    *reinterpret_cast<uint4*>(srow + 336 + 16 * (v + 8)) = R.U[4];
  }
  __syncwarp();
  if (v == 0) rowvalid[trow] = R.kind != 0;
  if (R.kind == 1 || R.kind == 2) {
    // lane v expands unit v of every 64-coordinate word i: seven dequantized NoPE units and one copied
    // (already rotated) BF16 tail unit per lane, uniform across the warp; the 8 lanes of a row store
    // 128 contiguous bytes per word
#pragma unroll 2
    for (int i = 0; i < 8; ++i) {
      const uint4 o = i < 7 ? dequant8(*reinterpret_cast<const uint2*>(srow + 64 * i + 8 * v),
                                       pm::exp2i((int)srow[576 + i] - 127))
                            : *reinterpret_cast<const uint4*>(srow + 448 + 16 * v);
      *reinterpret_cast<uint4*>(kv + pm::sw128_offset(trow, 16 * (8 * i + v), kTile * 128)) = o;
    }
  } else if (R.kind == 3) {
    // lane v expands unit v of every 64-coordinate word i (coordinates 64 i + 8 v .. + 7): each lane
    // rotates exactly one RoPE unit (word 7) and the seven NoPE units skip the rotation, with the
    // branch uniform across the warp
    const uint64_t* words = reinterpret_cast<const uint64_t*>(srow + 256);
    const uint64_t below = (1ull << (8 * v)) - 1ull;  // bits of the word before this lane's unit
    int prefix = 0;                                    // kept values before word i
#pragma unroll 2
    for (int i = 0; i < 8; ++i) {
      const uint64_t word = words[i];
      const uint32_t bits = (uint32_t)(word >> (8 * v)) & 0xFFu;
      const int rank = prefix + __popcll(word & below);
      prefix += __popcll(word);
      // the 8 value bytes from `rank` (reads may run past the values into the staged bitmap: masked)
      const uint32_t* vw = reinterpret_cast<const uint32_t*>(srow + (rank & ~3));
      const uint32_t sh = 8u * (uint32_t)(rank & 3);
      const uint32_t lo = __funnelshift_r(vw[0], vw[1], sh), hi = __funnelshift_r(vw[1], vw[2], sh);
      const uint4 e = expand_lut[bits];
      const uint2 codes = make_uint2(__byte_perm(lo, hi, e.x) & e.z, __byte_perm(lo, hi, e.y) & e.w);
      float f[8];
      dequant8f(codes, pm::exp2i((int)srow[320 + i] - 127), f);
      __nv_bfloat162 o2[4];
      if (i < 7) {
#pragma unroll
        for (int k = 0; k < 4; ++k) o2[k] = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
      } else {
        const float* cs = reinterpret_cast<const float*>(srow + 336) + 8 * v;  // pairs 4 v .. 4 v + 3
        const float4 cs01 = *reinterpret_cast<const float4*>(cs), cs23 = *reinterpret_cast<const float4*>(cs + 4);
        const float cc[4] = {cs01.x, cs01.z, cs23.x, cs23.z}, ss[4] = {cs01.y, cs01.w, cs23.y, cs23.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float re = __bfloat162float(__float2bfloat16_rn(f[2 * k]));
          const float im = __bfloat162float(__float2bfloat16_rn(f[2 * k + 1]));
          o2[k] = __floats2bfloat162_rn(__fsub_rn(__fmul_rn(re, cc[k]), __fmul_rn(im, ss[k])),
                                        __fadd_rn(__fmul_rn(re, ss[k]), __fmul_rn(im, cc[k])));
        }
      }
      *reinterpret_cast<uint4*>(kv + pm::sw128_offset(trow, 16 * (8 * i + v), kTile * 128)) =
          *reinterpret_cast<uint4*>(o2);
    }
  } else {
#pragma unroll 2
    for (int i = 0; i < 8; ++i)
      *reinterpret_cast<uint4*>(kv + pm::sw128_offset(trow, 16 * (8 * i + v), kTile * 128)) = zero4();
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
  uint4* expand_lut = reinterpret_cast<uint4*>(smem + kOffExpand);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // optional phase counters (thread 0, ns of the GPU global timer): [0] setup, [1] gather + expand,
  // [2] S MMA, [3] softmax, [4] O MMA (with the next tile's first gather), [5] epilogue, [6] CTAs,
  // [7] tiles, [8] earliest CTA start, [9] latest CTA end; [16 + 2 i] CTA i's total, [17 + 2 i] gather
  unsigned long long ph[6] = {0, 0, 0, 0, 0, 0};
  uint64_t tp = p.prof ? pm::globaltimer_ns() : 0;
  const uint64_t t_cta0 = tp;
  auto mark = [&](int i) {
    if (p.prof && tid == 0) {
      const uint64_t t = pm::globaltimer_ns();
      ph[i] += t - tp;
      tp = t;
    }
  };
  const int unit = blockIdx.x;
  const int split = unit % p.num_splits;
  const int g = (unit / p.num_splits) % p.num_groups;
  const int b = unit / (p.num_splits * p.num_groups);
  const int h0 = g * kHG;

  const int nswa = min(p.swa_len[b], p.swa_cap);
  const int ntot = nswa + min(p.csa_len[b], p.csa_cap);
  // this query's rows split into whole tiles of `trows` rows (128, or 64 when a small batch needs more
  // CTAs), as evenly as the split count allows; a 64-row tile leaves MMA rows 64-127 zero and masked
  const int trows = p.tile_rows == 64 ? 64 : kTile;
  const int tiles_q = (ntot + trows - 1) / trows;
  const int tiles_per_split = (tiles_q + p.num_splits - 1) / p.num_splits;
  const int row0 = split * tiles_per_split * trows;
  const int row1 = min(ntot, row0 + tiles_per_split * trows);
  const int ntiles = row1 > row0 ? (row1 - row0 + trows - 1) / trows : 0;

  uint8_t* srow = smem + kOffStage + warp * kStageBytes + (lane >> 3) * kStageRow;
  const int v8 = lane & 7;
  // step k of a tile: rows 4 warp + lane / 8 + 32 k
  auto step_row = [&](int k) { return 4 * warp + (lane >> 3) + 32 * k; };
  // row references of the 4 steps of tile tt (4 independent index loads in flight together)
  RowRef rr[4];
  auto resolve = [&](int tt) {
    const int tb = row0 + tt * trows, tv = min(trows, row1 - tb);
#pragma unroll
    for (int k = 0; k < 4; ++k) rr[k] = step_ref(p, b, tb, tv, nswa, ntot, step_row(k));
  };
  // four register sets, one per gather step: all record loads of a tile are in flight together, and the
  // loads of tile t + 1 are issued while the P.V MMAs of tile t run; no register copy ever waits on loads
  // still in flight
  StepRegs ra, rb, rc, rd;
  auto fetch_all = [&](int n) {
    fetch_step(p, rr[0], v8, ra);
    fetch_step(p, rr[1], v8, rb);
    if (n == 4) {
      fetch_step(p, rr[2], v8, rc);
      fetch_step(p, rr[3], v8, rd);
    }
  };

  // tile 0's index and record loads go out first: their latency overlaps the TMEM allocation, the
  // LUT set-up and the Q load below
  if (ntiles > 0) {
    resolve(0);
    fetch_all(4);
  }
  __syncwarp();  // the lanes took row-dependent branches; tcgen05.alloc is warp-collective

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
  for (int m = tid; m < 256; m += kThreads) expand_lut[m] = expand_lut_entry(m);

  // Q group -> shared (K-major, SW128, chunk stride 64 rows * 128 B): all 16 loads of a thread in
  // flight before the first store
  {
    uint4 qv[kHG * 64 / kThreads];
#pragma unroll
    for (int i = 0; i < kHG * 64 / kThreads; ++i) {
      const int idx = tid + kThreads * i, row = idx >> 6, u = idx & 63;
      qv[i] = h0 + row < p.H ? *reinterpret_cast<const uint4*>(p.q + (int64_t)b * p.q_stride_b +
                                                               (int64_t)(h0 + row) * p.q_stride_h + 8 * u)
                             : zero4();
    }
#pragma unroll
    for (int i = 0; i < kHG * 64 / kThreads; ++i) {
      const int idx = tid + kThreads * i, row = idx >> 6, u = idx & 63;
      *reinterpret_cast<uint4*>(sQ + pm::sw128_offset(row, 16 * u, kHG * 128)) = qv[i];
    }
  }
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  mark(0);
  const uint32_t q_base = pm::smem_u32(sQ), kv_base = pm::smem_u32(sKV), p_base = pm::smem_u32(sP);
  const uint32_t idesc_s = pm::make_idesc_f16(128, kHG, 1, 0, 0);
  const uint32_t idesc_o = pm::make_idesc_f16(128, kHG, 1, 1, 1);
  bool ok = true;

  for (int t = 0; t < ntiles && ok; ++t) {
    // ---- 1. gather + expand 128 rows (64-row tiles: steps 2-3 only on the first tile, zero rows)
    const int nsteps = (trows == kTile || t == 0) ? 4 : 2;  // tile 0's loads were issued at set-up
    uint64_t tg = p.prof && tid == 0 ? pm::globaltimer_ns() : 0;
    auto sub = [&](int slot) {  // finer split of the gather for thread 0: [11] expand
      if (p.prof && tid == 0) {
        const uint64_t tn = pm::globaltimer_ns();
        atomicAdd(p.prof + slot, (unsigned long long)(tn - tg));
        tg = tn;
      }
    };
    auto expand = [&](const StepRegs& R, int k) {
      expand_step(R, step_row(k), v8, srow, sKV, rowvalid, expand_lut);
    };
    expand(ra, 0);
    expand(rb, 1);
    if (nsteps == 4) {
      expand(rc, 2);
      expand(rd, 3);
    }
    sub(11);
    pm::fence_proxy_async_smem();
    pm::tc_fence_before();
    __syncthreads();
    pm::tc_fence_after();
    sub(12);  // [12] waiting for the other warps at the end of the gather
    mark(1);
    // ---- 2. S^T = K Q^T
    if (tid == 0) {
#pragma unroll 1
      for (int k = 0; k < kD / 16; ++k) {
        const uint32_t koff = (k * 32) & 127;
        const uint64_t ad = pm::make_sdesc(kv_base + (k >> 2) * (kTile * 128) + koff, 16, 1024);
        const uint64_t bd = pm::make_sdesc(q_base + (k >> 2) * (kHG * 128) + koff, 16, 1024);
        pm::umma_f16(tmem + kTmemS, ad, bd, idesc_s, k > 0);
      }
      pm::umma_commit(bar_s);
    }
    if (!pm::mbar_wait(bar_s, t & 1, p.err, 1)) { flags[1] = 1; }
    pm::tc_fence_after();
    mark(2);
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
    mark(3);
    // ---- 4. O^T += V^T P^T
    if (tid == 0 && !flags[1]) {
#pragma unroll 1
      for (int db = 0; db < 4; ++db) {
#pragma unroll 1
        for (int k = 0; k < trows / 16; ++k) {
          const uint64_t ad = pm::make_sdesc(kv_base + (2 * db) * (kTile * 128) + k * 2048, kTile * 128, 1024);
          const uint64_t bd = pm::make_sdesc(p_base + k * 2048, 8192, 1024);
          pm::umma_f16(tmem + kTmemO + db * kHG, ad, bd, idesc_o, (t > 0 || k > 0) ? 1u : 0u);
        }
      }
      pm::umma_commit(bar_o);
    }
    if (t + 1 < ntiles) {  // overlaps the P.V MMAs
      resolve(t + 1);
      fetch_all(trows == kTile ? 4 : 2);
    }
    if (!flags[1]) {
      if (!pm::mbar_wait(bar_o, t & 1, p.err, 2)) flags[1] = 1;
    }
    pm::tc_fence_after();
    __syncthreads();
    ok = !flags[1];
    mark(4);
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
  mark(5);
  if (p.prof && tid == 0) {
    for (int i = 0; i < 6; ++i) atomicAdd(p.prof + i, ph[i]);
    atomicAdd(p.prof + 6, 1ull);
    atomicAdd(p.prof + 7, (unsigned long long)ntiles);
    atomicMin(p.prof + 8, (unsigned long long)t_cta0);
    atomicMax(p.prof + 9, (unsigned long long)pm::globaltimer_ns());
    if (blockIdx.x < 1024) {
      p.prof[16 + 2 * blockIdx.x] = pm::globaltimer_ns() - t_cta0;
      p.prof[17 + 2 * blockIdx.x] = ph[1];
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
