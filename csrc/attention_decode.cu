// Sparse MLA decode attention on tcgen05 (Native and Direct-Packed KV), plus split combine.
//
// Reference behaviour: FlashMLA sparse FP8 decode, Native <1,64,0> and Direct Packed <1,64,1>
// (third_party/README.md:355-361) and `flash_fwd_mla_combine_kernel`.  Semantics: joint softmax over
// [SWA rows ; selected C4 rows] with a per-head sink, K = V = latent row, output tail inverse-rotated
// with the query position (training/losses.py:121-126).
//
// Design (sm_100a).  One CTA = (query b, group of 64 heads, KV split); 512 threads:
//   * all 16 warps gather and expand the KV rows into shared memory, 128-row tiles at a time, and run each
//     tile's softmax; warp 0 owns TMEM and issues the MMAs from one elected lane of the converged warp.
//     Sixteen warps (four per scheduler) hide the latency of the expansion's dependent chains; at 128
//     registers a lane holds two raw rows and 16 scores.
// Per tile (a 128-row, 128-byte-swizzled K-major FP16 buffer):
//   S^T (128 rows x 64 heads, fp32) = K Q^T: tcgen05.mma kind::f16 M=128 N=64, 32 instructions over K = 512;
//   softmax over the tile (one thread per row and 16 heads: 16 warps cover the four TMEM lane quadrants and
//     the four head quarters), P^T in FP16 to shared memory;
//   O^T (512 d x 64 heads, fp32, 256 TMEM columns) += V^T P^T: four d-blocks of M=128, K = 128 rows, V^T
//     read through an MN-major descriptor of the same buffer.
// The next tile's rows are resolved and loaded into registers while the current tile's
// softmax and P.V run, and the indices of the tile after it are loaded, so a tile's expansion starts with its
// data at hand.  O^T is rescaled in TMEM only when a head's running max grows by more than 2^8 (exact: the
// final division uses the same reference max).
//
// Expansion (8 lanes per row, two rows per lane and tile):
//   Native 584 B rows: each lane loads the 16-byte units v, v + 8, v + 16, v + 24, v + 32 of the record
//     and expands exactly those bytes (E4M3 x UE8M0 -> FP16, the BF16 tail -> FP16), so no staging.
//   Packed 328 B rows: the values are staged per row in the P buffer (free while a tile is expanded) and
//     the bitmap words are shuffled from the group's lanes; lane v expands the 8-coordinate unit v of
//     every 64-coordinate word (bitmap POPC prefix, one byte permute from a mask-indexed table, E4M3 x
//     UE8M0), and the tail word is rounded to BF16, rotated with the record's RoPE row and rounded again.
// FP16 operands: E4M3 x 2^e is exact in FP16 for e in [-15, 7], and the BF16 tail values are exact in
// FP16 in its normal range, so S and O are the same sums the BF16 dequantization gives; a scale outside
// that range takes an fp32 path (values below FP16's range round, above it saturate and report an error).
// With one split the epilogue normalizes (sink included), inverse-rotates the tail and writes BF16 O and
// the LSE; with several, it writes fp32 partials that the combine kernel merges.  Either way the group's
// rows are staged in the free K buffer and leave in one bulk copy (contiguous [heads][512] rows).
// Set-up: TMEM, barriers and the expansion table are prepared before griddepcontrol.wait (programmatic
// dependent launch); Q arrives by bulk copies into the K buffer and is converted to FP16 from there, so
// the first tile's index and row loads own the load path while Q streams in.
#include <cuda_fp4.h>

#include "launchers.h"
#include "common/sm100.cuh"

namespace {

constexpr int kD = 512;
constexpr int kHG = 64;            // heads per CTA (N of the MMAs)
constexpr int kTileRows = 128;     // KV rows per tile (the M of the score MMA)
constexpr int kBufRows = 128;
constexpr int kThreads = 512;      // 16 warps: all expand, all run the softmax, warp 0 also issues the MMAs
constexpr int kPage = 64;
constexpr int kNativeData = 576;
constexpr int kNativePageBytes = kPage * 584;
constexpr int kFp4NativeData = 256;                       // FP4 Native data row: 512 E2M1 codes
constexpr int kFp4PackedData = 192;                       // FP4 Packed data row: 256 codes + 8 bitmap words
constexpr int kFp4NativePage = kPage * (kFp4NativeData + 32);
constexpr int kFp4PackedPage = kPage * (kFp4PackedData + 32);
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;

// shared memory map (bytes, from a 1024-aligned base)
constexpr int kQBytes = kHG * kD * 2;          // 65536: Q, FP16, K-major SW128, chunk stride 64 x 128 B
constexpr int kKBytes = kBufRows * kD * 2;     // 131072: K, chunk stride 128 x 128 B
constexpr int kKChunk = kBufRows * 128;        // 16384
constexpr int kQChunk = kHG * 128;             // 8192
constexpr int kPBytes = kBufRows * kHG * 2;    // 16384: P^T, FP16, one 128 B row per buffer row
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kQBytes;
constexpr int kOffP = kOffK + kKBytes;
constexpr int kOffRed = kOffP + kPBytes;               // float red[4][64]
constexpr int kOffHead = kOffRed + 4 * 64 * 4;          // m_used[64], l[64], alpha[64], fac[64], sink2[64]
constexpr int kOffBar = kOffHead + 5 * 64 * 4;          // mbarriers
constexpr int kOffMisc = kOffBar + 16 * 8;              // tmem slot, flags
constexpr int kOffRowValid = kOffMisc + 32;             // uint8[128]
constexpr int kOffLut = kOffRowValid + 128;             // uint4[256] byte-expansion table
constexpr int kSmemBytes = kOffLut + 256 * 16 + 1024;   // + alignment slack

constexpr uint32_t kTmemO = 0;
constexpr uint32_t kTmemS = 256;
constexpr uint32_t kTmemCols = 512;

// barrier indices
enum : int { kBarSFull = 0, kBarPvDone = 1, kBarQ = 2, kBarMerge = 3 };

__device__ __forceinline__ uint4 zero4() { return make_uint4(0, 0, 0, 0); }

// Byte expansion of a Packed 8-coordinate unit with kept-mask m: the unit's kept values are the 8 bytes
// starting at its rank (lo, hi); entry m = {selector of coords 0-3, selector of coords 4-7, mask 0-3,
// mask 4-7} for __byte_perm, so codes = perm(lo, hi, sel) & mask (E4M3 zero = 0x00).
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

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// 2^x with the hardware approximation (ex2.approx.f32: subnormal results kept, 2 ulp), as exp2f promises.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Scale exponents e whose products with E4M3 values are exact in FP16 (see the header comment).
__device__ __forceinline__ bool fast_scale(int e) { return e >= -15 && e <= 7; }

// 2^e as an FP16 bit pattern, e in [-15, 7] (2^-15 is subnormal).
__device__ __forceinline__ unsigned short f16_pow2(int e) {
  return (unsigned short)(e >= -14 ? (e + 15) << 10 : 1u << (e + 24));
}

// 8 E4M3 codes (little-endian in c.x, c.y) x 2^e -> 8 FP16 (uint4).
__device__ __forceinline__ uint4 dq8(uint2 c, int e, int* err) {
  const uint32_t w[2] = {c.x, c.y};
  uint32_t o[4];
  if (fast_scale(e)) {
    const __half2 s2 = __half2half2(__ushort_as_half(f16_pow2(e)));
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = h2_bits(__hmul2(pm::e4m3x2_to_h2((uint16_t)(w[k >> 1] >> (16 * (k & 1)))), s2));
  } else {
    if (e > 7) pm::report_error(err, pm::kBadArgument, e);
    const float s = pm::exp2i(e);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(pm::e4m3x2_to_h2((uint16_t)(w[k >> 1] >> (16 * (k & 1)))));
      asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(o[k]) : "f"(f.y * s), "f"(f.x * s));
    }
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// 8 BF16 (uint4) -> 8 FP16 (exact in FP16's normal range; saturating).
__device__ __forceinline__ uint4 bf16x8_to_f16(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float lo = __uint_as_float(w[k] << 16), hi = __uint_as_float(w[k] & 0xFFFF0000u);
    asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(o[k]) : "f"(hi), "f"(lo));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

struct RowRef {
  int kind;  // 0 = masked, 1 = native (swa pool), 2 = native (csa pool), 3 = packed, 4/5 = FP4 native/packed,
             // 6/7 = GLM-5.3 native/packed
  int slot;
  int pos;
};

// Row i of query b's list [SWA rows ; C4 rows], in two steps so the index loads can be issued long
// before their values are needed: idx_load only loads (no use of the values), idx_resolve checks them.
struct RowIdx {
  int slot;  // raw slot (SWA or C4)
  int pos;   // raw RoPE position (Packed C4 rows)
};
__device__ __forceinline__ RowIdx idx_load(const DecodeParams& p, int b, int i, int nswa, int ntot) {
  RowIdx x{-1, 0};
  if (i >= ntot) return x;
  if (i < nswa) {
    x.slot = p.swa_slots[(int64_t)b * p.swa_cap + i];
  } else {
    const int64_t j = (int64_t)b * p.csa_cap + (i - nswa);
    x.slot = p.csa_slots[j];
    if (p.csa_packed) x.pos = p.csa_pos[j];
  }
  return x;
}
// `i` is the row's index in the list (the same one given to idx_load).
__device__ __forceinline__ RowRef idx_resolve(const DecodeParams& p, const RowIdx& x, int i, int nswa, int ntot) {
  RowRef r{0, -1, 0};
  if (i >= ntot) return r;
  const int s = x.slot;
  if (i < nswa) {
    if (s >= 0 && s < p.swa_pool_slots) { r.kind = 1; r.slot = s; }
    else if (s >= p.swa_pool_slots) pm::report_error(p.err, pm::kIndexOutOfRange, i);
    return r;
  }
  if (s < 0) return r;
  if (s >= p.csa_pool_rows || (p.csa_packed && (x.pos < 0 || x.pos >= p.freq_rows))) {
    pm::report_error(p.err, pm::kIndexOutOfRange, i);
    return r;
  }
  r.kind = p.csa_glm ? 5 + p.csa_glm : (p.csa_fp4 ? 3 + p.csa_fp4 : (p.csa_packed ? 3 : 2));
  r.slot = s;
  r.pos = x.pos;
  return r;
}

// Raw bytes of one row held by one of its 8 lanes (lane v):
//   Native: u[i] = 16-byte unit v + 8 i of the record (units 0..27 E4M3, 28..35 BF16 tail; i = 4 only v < 4).
//   Packed: u[0], u[1] = value units v, v + 8; u[2] = bitmap unit v (v < 4); u[3], u[4] = 16-byte units
//           2 v, 2 v + 1 of the record's RoPE row (the cos/sin of pairs 4 v .. 4 v + 3).
//   FP4 Native: u[0], u[1] = code units v, v + 8 (32 coordinates each); sc = E4M3 scale bytes 2 v, 2 v + 1
//           (sc.x) and 2 v + 16, 2 v + 17 (sc.y).
//   FP4 Packed: u[0] = code unit v (v < 8: the 128 survivor code bytes); u[2] = bitmap words 2 v, 2 v + 1
//           (v < 4); u[3], u[4] = the 32 E4M3 scale bytes.
//   GLM Native: u[i] = 16-byte unit v + 8 i of the 512-code row.
//   GLM Packed: u[0], u[1] = value units v, v + 8; u[2] = bitmap unit v (v < 4).
//   sc: the row's 8 UE8M0 scale bytes (FP8 rows).
struct Raw {
  uint4 u[5];
  uint2 sc;
  int kind;
};

__device__ __forceinline__ void fetch(const DecodeParams& p, const RowRef& rr, int v, Raw& R) {
  R.kind = rr.kind;
  R.sc = make_uint2(0, 0);
#pragma unroll
  for (int i = 0; i < 5; ++i) R.u[i] = zero4();
  if (rr.kind == 1 || rr.kind == 2) {
    const uint8_t* pool = rr.kind == 1 ? p.swa_pool : p.csa_pool;
    const int64_t page = rr.slot / kPage, rip = rr.slot % kPage;
    const uint4* data = reinterpret_cast<const uint4*>(pool + page * kNativePageBytes + rip * kNativeData);
#pragma unroll
    for (int i = 0; i < 4; ++i) R.u[i] = data[v + 8 * i];
    if (v < 4) R.u[4] = data[v + 32];
    R.sc = *reinterpret_cast<const uint2*>(pool + page * kNativePageBytes + kPage * kNativeData + rip * 8);
  } else if (rr.kind == 3) {
    const uint4* vals = reinterpret_cast<const uint4*>(p.csa_values + (int64_t)rr.slot * 256);
    const uint4* bits = reinterpret_cast<const uint4*>(p.csa_bitmap + (int64_t)rr.slot * 8);
    const uint4* fq = reinterpret_cast<const uint4*>(p.freqs + (int64_t)rr.pos * 64);
    R.u[0] = vals[v];
    R.u[1] = vals[v + 8];
    if (v < 4) R.u[2] = bits[v];
    R.u[3] = fq[2 * v];
    R.u[4] = fq[2 * v + 1];
    R.sc = *reinterpret_cast<const uint2*>(p.csa_scales + (int64_t)rr.slot * 8);
  } else if (rr.kind == 4) {
    const int64_t page = rr.slot / kPage, rip = rr.slot % kPage;
    const uint8_t* pg = p.csa_pool + page * kFp4NativePage;
    const uint4* data = reinterpret_cast<const uint4*>(pg + rip * kFp4NativeData);
    R.u[0] = data[v];
    R.u[1] = data[v + 8];
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(pg + kPage * kFp4NativeData + rip * 32);
    R.sc = make_uint2(sc[v], sc[v + 8]);
  } else if (rr.kind == 5) {
    const int64_t page = rr.slot / kPage, rip = rr.slot % kPage;
    const uint8_t* pg = p.csa_pool + page * kFp4PackedPage;
    const uint4* data = reinterpret_cast<const uint4*>(pg + rip * kFp4PackedData);
    R.u[0] = data[v];
    if (v < 4) R.u[2] = data[8 + v];
    const uint4* sc = reinterpret_cast<const uint4*>(pg + kPage * kFp4PackedData + rip * 32);
    R.u[3] = sc[0];
    R.u[4] = sc[1];
  } else if (rr.kind == 6) {
    const uint4* data = reinterpret_cast<const uint4*>(p.csa_pool + (int64_t)rr.slot * kD);
#pragma unroll
    for (int i = 0; i < 4; ++i) R.u[i] = data[v + 8 * i];
  } else if (rr.kind == 7) {
    const uint4* vals = reinterpret_cast<const uint4*>(p.csa_values + (int64_t)rr.slot * 256);
    const uint4* bits = reinterpret_cast<const uint4*>(p.csa_bitmap + (int64_t)rr.slot * 8);
    R.u[0] = vals[v];
    R.u[1] = vals[v + 8];
    if (v < 4) R.u[2] = bits[v];
  }
}

// Two E2M1 codes (low nibble = the lower coordinate) -> FP16x2 bits, times an FP16x2 scale.  E2M1 x E4M3
// products have at most 6 significant bits and lie in [2^-10, 2688]: exact in FP16.
__device__ __forceinline__ uint32_t fp4x2_scaled(uint32_t byte, __half2 s2) {
  const __half2_raw r = __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)byte, __NV_E2M1);
  return h2_bits(__hmul2(__half2(r), s2));
}

__device__ __forceinline__ int scale_exp(uint2 sc, int word) {
  const uint32_t w = word < 4 ? sc.x : sc.y;
  return (int)((w >> (8 * (word & 3))) & 0xFF) - 127;
}

// Expand one row (lane v of its 8 lanes) into K-buffer row `brow`.  Out of line: the four passes of a stage
// share one copy of this code, which keeps the kernel small enough for the instruction cache.
__device__ __noinline__ void expand_row(const Raw R, int brow, int v, uint8_t* __restrict__ stg,
                                           uint8_t* __restrict__ sK, uint8_t* __restrict__ rowvalid,
                                           const uint4* __restrict__ lut, int* err) {
  // 128-byte swizzle: 16-byte unit u of a row's 64-coordinate chunk c sits at
  // c * kKChunk + (row / 8) * 1024 + (row % 8) * 128 + ((u ^ row % 8) * 16)
  uint8_t* const row_base = sK + (brow >> 3) * 1024 + (brow & 7) * 128;
  const int rsw = brow & 7;
  auto out = [&](int byte_in_row) -> uint4* {
    return reinterpret_cast<uint4*>(row_base + (byte_in_row >> 7) * kKChunk + (((byte_in_row >> 4) & 7) ^ rsw) * 16);
  };
  // unit v of every chunk (the Packed and masked paths): one swizzled column, chunk i at + i * kKChunk
  uint8_t* const col_v = row_base + ((v ^ rsw) << 4);
  if (v == 0) rowvalid[brow] = R.kind != 0;
  if (R.kind == 1 || R.kind == 2) {
    // NoPE units v + 8 i (16 codes = coordinates 16 u .. 16 u + 15 of word u / 4)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int u = v + 8 * i;
      if (u < 28) {
        const int e = scale_exp(R.sc, u >> 2);
        *out(32 * u) = dq8(make_uint2(R.u[i].x, R.u[i].y), e, err);
        *out(32 * u + 16) = dq8(make_uint2(R.u[i].z, R.u[i].w), e, err);
      }
    }
    // the lane's tail unit (8 BF16 coordinates, already rotated)
    const int ut = v >= 4 ? v + 24 : v + 32;
    *out(896 + 16 * (ut - 28)) = bf16x8_to_f16(v >= 4 ? R.u[3] : R.u[4]);
  } else if (R.kind == 6) {
    // GLM Native: raw E4M3 units v + 8 i (coordinates 16 u .. 16 u + 15), exact in FP16
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int u = v + 8 * i;
      *out(32 * u) = dq8(make_uint2(R.u[i].x, R.u[i].y), 0, err);
      *out(32 * u + 16) = dq8(make_uint2(R.u[i].z, R.u[i].w), 0, err);
    }
  } else if (R.kind == 3 || R.kind == 7) {
    // the values are staged (256 bytes); the 8 bitmap words come from lanes 0..3 of the row's group
    // (GLM Packed rows: raw E4M3 survivors, no scales and no RoPE word)
    const bool glm = R.kind == 7;
    const uint32_t gmask = 0xFFu << (8 * ((threadIdx.x & 31) >> 3));
    *reinterpret_cast<uint4*>(stg + 16 * v) = R.u[0];
    *reinterpret_cast<uint4*>(stg + 16 * (v + 8)) = R.u[1];
    uint64_t word[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t x = __shfl_sync(gmask, R.u[2].x, j, 8), y = __shfl_sync(gmask, R.u[2].y, j, 8);
      const uint32_t z = __shfl_sync(gmask, R.u[2].z, j, 8), w = __shfl_sync(gmask, R.u[2].w, j, 8);
      word[2 * j] = ((uint64_t)y << 32) | x;
      word[2 * j + 1] = ((uint64_t)w << 32) | z;
    }
    __syncwarp(gmask);
    // every word's rank base (kept values before it) from an add chain
    const uint64_t below = (1ull << (8 * v)) - 1ull;  // bits of the word before this lane's unit
    int prefix = 0;                                    // kept values before word i
    // fully unrolled: the words' loads, permutes and conversions are independent and interleave
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t bits = (uint32_t)(word[i] >> (8 * v)) & 0xFFu;
      const int rank = prefix + __popcll(word[i] & below);
      prefix += __popcll(word[i]);
      // the 8 value bytes from `rank` (bytes read past the row's values are masked off)
      const uint32_t* vw = reinterpret_cast<const uint32_t*>(stg + (rank & ~3));
      const uint32_t sh = 8u * (uint32_t)(rank & 3);
      const uint32_t lo = __funnelshift_r(vw[0], vw[1], sh), hi = __funnelshift_r(vw[1], vw[2], sh);
      const uint4 e = lut[bits];
      const uint2 codes = make_uint2(__byte_perm(lo, hi, e.x) & e.z, __byte_perm(lo, hi, e.y) & e.w);
      const int ex = glm ? 0 : scale_exp(R.sc, i);
      uint4 o;
      if (i < 7 || glm) {
        o = dq8(codes, ex, err);
      } else {
        // dequantize (exact in fp32), round to BF16, rotate with the record's pair (cos, sin), round again
        const float s = pm::exp2i(ex);
        const uint32_t cw[2] = {codes.x, codes.y};
        const float cs[8] = {__uint_as_float(R.u[3].x), __uint_as_float(R.u[3].y), __uint_as_float(R.u[3].z),
                             __uint_as_float(R.u[3].w), __uint_as_float(R.u[4].x), __uint_as_float(R.u[4].y),
                             __uint_as_float(R.u[4].z), __uint_as_float(R.u[4].w)};
        uint32_t ow[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __half22float2(pm::e4m3x2_to_h2((uint16_t)(cw[k >> 1] >> (16 * (k & 1)))));
          const float re = __bfloat162float(__float2bfloat16_rn(f.x * s));
          const float im = __bfloat162float(__float2bfloat16_rn(f.y * s));
          const float c = cs[2 * k], sn = cs[2 * k + 1];
          const float rr = __bfloat162float(__float2bfloat16_rn(__fsub_rn(__fmul_rn(re, c), __fmul_rn(im, sn))));
          const float ri = __bfloat162float(__float2bfloat16_rn(__fadd_rn(__fmul_rn(re, sn), __fmul_rn(im, c))));
          asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(ow[k]) : "f"(ri), "f"(rr));
        }
        o = make_uint4(ow[0], ow[1], ow[2], ow[3]);
      }
      *reinterpret_cast<uint4*>(col_v + i * kKChunk) = o;
    }
    __syncwarp(0xFFu << (8 * ((threadIdx.x & 31) >> 3)));
  } else if (R.kind == 4) {
    // FP4 Native (values already rotated): code unit u = v + 8 h covers coordinates 32 u .. 32 u + 31, scale
    // groups 2 u and 2 u + 1, output units 4 u .. 4 u + 3 (4 code bytes each)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 c = R.u[h];
      const __half2 s2 = pm::e4m3x2_to_h2((uint16_t)(h ? R.sc.y : R.sc.x));
      const __half2 sg[2] = {__low2half2(s2), __high2half2(s2)};
      const uint32_t cw[4] = {c.x, c.y, c.z, c.w};
      const int u = v + 8 * h;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] = fp4x2_scaled((cw[m] >> (8 * k)) & 0xFFu, sg[m >> 1]);
        *out(16 * (4 * u + m)) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  } else if (R.kind == 5) {
    // FP4 Packed: the 128 code bytes are staged; the 8 MSB-first bitmap words come from lanes 0..3 of the
    // row's group and are bit-reversed (coordinate b at bit b); lane v expands unit v of every word
    const uint32_t gmask = 0xFFu << (8 * ((threadIdx.x & 31) >> 3));
    *reinterpret_cast<uint4*>(stg + 16 * v) = R.u[0];
    uint64_t word[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t x = __shfl_sync(gmask, R.u[2].x, j, 8), y = __shfl_sync(gmask, R.u[2].y, j, 8);
      const uint32_t z = __shfl_sync(gmask, R.u[2].z, j, 8), w = __shfl_sync(gmask, R.u[2].w, j, 8);
      word[2 * j] = __brevll(((uint64_t)y << 32) | x);
      word[2 * j + 1] = __brevll(((uint64_t)w << 32) | z);
    }
    __syncwarp(gmask);
    const uint32_t sw[8] = {R.u[3].x, R.u[3].y, R.u[3].z, R.u[3].w, R.u[4].x, R.u[4].y, R.u[4].z, R.u[4].w};
    const uint64_t below = (1ull << (8 * v)) - 1ull;
    int prefix = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t bits = (uint32_t)(word[i] >> (8 * v)) & 0xFFu;
      const int rank = prefix + __popcll(word[i] & below);
      prefix += __popcll(word[i]);
      // 8 codes from nibble `rank` (nibbles past the survivors are masked off), one per byte, then the
      // kept ones moved to their coordinates with the byte-permute table
      const uint32_t* vw = reinterpret_cast<const uint32_t*>(stg + 4 * (rank >> 3));
      const uint32_t nib = __funnelshift_r(vw[0], vw[1], 4u * (uint32_t)(rank & 7));
      const uint32_t ev = nib & 0x0F0F0F0Fu, od = (nib >> 4) & 0x0F0F0F0Fu;
      const uint32_t lo = __byte_perm(ev, od, 0x5140), hi = __byte_perm(ev, od, 0x7362);
      const uint4 e = lut[bits];
      const uint32_t b0 = __byte_perm(lo, hi, e.x) & e.z, b1 = __byte_perm(lo, hi, e.y) & e.w;
      const uint32_t p0 = b0 | (b0 >> 4), p1 = b1 | (b1 >> 4);  // bytes 0 and 2: code pairs
      const uint32_t sb = (sw[i] >> (8 * (v >> 1))) & 0xFFu;    // scale group 4 i + v / 2
      const __half2 s2 = pm::e4m3x2_to_h2((uint16_t)(sb | (sb << 8)));
      *reinterpret_cast<uint4*>(col_v + i * kKChunk) =
          make_uint4(fp4x2_scaled(p0 & 0xFFu, s2), fp4x2_scaled((p0 >> 16) & 0xFFu, s2),
                     fp4x2_scaled(p1 & 0xFFu, s2), fp4x2_scaled((p1 >> 16) & 0xFFu, s2));
    }
    __syncwarp(gmask);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) *reinterpret_cast<uint4*>(col_v + i * kKChunk) = zero4();
  }
}

// Lanes L and L + 16 return the op-reduction over the 32 lanes of v[L % 16]: the two lane halves are folded,
// then a transposing butterfly over 16 lanes (31 shuffles instead of 80).
template <bool kMax>
__device__ __forceinline__ float transpose_reduce16(float (&v)[16], int lane) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float got = __shfl_xor_sync(0xffffffffu, v[i], 16);
    v[i] = kMax ? fmaxf(v[i], got) : v[i] + got;
  }
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) {
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
  uint8_t* sK = smem + kOffK;
  uint8_t* sP = smem + kOffP;
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  float* m_used = reinterpret_cast<float*>(smem + kOffHead);
  float* l_sum = m_used + 64;
  float* alpha = l_sum + 64;
  float* fac = alpha + 64;
  float* sink2v = fac + 64;  // the heads' sink logits in log2 units (-inf without a sink)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* flags = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);  // [0] rescale, [1] abort
  uint8_t* rowvalid = smem + kOffRowValid;
  uint4* lut = reinterpret_cast<uint4*>(smem + kOffLut);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int unit = blockIdx.x;
  // optional global-timer stamps of the last split of query 0, head group 0 (a split with a tile whenever
  // any has one), in ns: [0] start (after the dependency wait), [1] set-up done,
  // [2 + 2 t] tile t expanded, [3 + 2 t] its softmax done, [18 + t] S(t) issued, [26 + t] P.V(t) issued,
  // [34] epilogue start, [35] end, [36..41] inside tile 0's softmax, [44] tile 1's rows issued,
  // [48..51] epilogue steps, [54..56] set-up steps; [57] / [58] / [59]: latest end / latest start /
  // earliest start over all CTAs (atomics)
  auto stamp = [&](int i) {
    if (p.prof != nullptr && blockIdx.x == p.num_splits - 1 && i < 64) p.prof[i] = pm::globaltimer_ns();
  };
  const int split = unit % p.num_splits;
  const int g = (unit / p.num_splits) % p.num_groups;
  const int b = unit / (p.num_splits * p.num_groups);
  const int h0 = g * kHG;
  const int nh = min(kHG, p.H - h0);

  // set-up that reads no input: TMEM, barriers, the expansion table (overlaps the previous kernel's tail
  // under programmatic dependent launch)
  if (warp == 0) {
    pm::tmem_alloc(tmem_slot, kTmemCols);
    pm::tmem_relinquish();
  }
  if (tid == 0) {
    pm::mbar_init(&bars[kBarSFull], 1);
    pm::mbar_init(&bars[kBarPvDone], 1);
    pm::mbar_init(&bars[kBarQ], 1);
    pm::mbar_init(&bars[kBarMerge], 1);
    pm::fence_mbar_init();
    flags[0] = 0;
    flags[1] = 0;
  }
  if (tid < 64) { m_used[tid] = -INFINITY; l_sum[tid] = 0.f; alpha[tid] = 1.f; }
  for (int m = tid; m < 256; m += kThreads) lut[m] = expand_lut_entry(m);
  __syncthreads();
  pm::griddep_wait();  // inputs are complete from here on
  if (tid == 0) {
    stamp(0);
    if (p.prof != nullptr) {
      const unsigned long long now = pm::globaltimer_ns();
      atomicMax(reinterpret_cast<unsigned long long*>(p.prof + 58), now);
      atomicMin(reinterpret_cast<unsigned long long*>(p.prof + 59), now);
    }
    // the group's Q rows (BF16, 1 KB each) -> the K buffer as staging: one bulk copy when the rows are
    // contiguous (the TMA unit takes each copy in turn, so per-row copies would cost ~2 us of issue)
    pm::mbar_arrive_expect_tx(&bars[kBarQ], (uint32_t)nh * 1024u);
    if (p.q_stride_h == kD)
      pm::bulk_g2s(sK, p.q + (int64_t)b * p.q_stride_b + (int64_t)h0 * kD, (uint32_t)nh * 1024u, &bars[kBarQ]);
  }
  if (p.q_stride_h != kD && warp == kThreads / 32 - 1) {  // strided rows: one copy per row, from the last warp
    __syncwarp();
    for (int r = lane; r < nh; r += 32)
      pm::bulk_g2s(sK + r * 1024, p.q + (int64_t)b * p.q_stride_b + (int64_t)(h0 + r) * p.q_stride_h, 1024u,
                   &bars[kBarQ]);
  }

  // inputs the epilogue needs, loaded now so no late global load sits before a cluster barrier
  if (tid < kHG) sink2v[tid] = (p.sink && h0 + tid < p.H) ? p.sink[h0 + tid] * kLog2e : -INFINITY;
  const int qpos_raw = p.q_pos ? p.q_pos[b] : 0;
  const int nswa = p.swa_cap > 0 ? min(p.swa_len[b], p.swa_cap) : 0;
  const int ntot = nswa + min(p.csa_len[b], p.csa_cap);
  const int tiles_q = (ntot + kTileRows - 1) / kTileRows;
  const int t0 = (split * tiles_q) / p.num_splits;  // 32-bit: tiles_q is at most a few thousand
  const int t1 = ((split + 1) * tiles_q) / p.num_splits;
  const int nt = t1 - t0;
  const bool clustered = decode_splits_clustered(p.num_splits);  // the splits are one cluster, merged on chip

  // bounded wait; after the first timeout every later wait returns at once (the CTA runs to its end
  // on garbage data instead of waiting again)
  auto wait = [&](int bar, uint32_t parity, int site) {
    if (flags[1]) return;
    if (!pm::mbar_wait(&bars[bar], parity, p.err, site)) flags[1] = 1;
  };

  const int wq = warp & 3, v8 = lane & 7, rsub = lane >> 3;
  uint8_t* stg = sP + (4 * warp + rsub) * 256;  // Packed value staging (the P buffer is free while expanding)

  // A tile's 128 rows: pass pp of warp w holds rows 64 pp + 4 w + lane / 8 (8 lanes per row).  The raw
  // indices of the next tile are loaded a tile ahead (ix0, ix1); they are resolved and their rows loaded
  // into ra, rb while the current tile's softmax and P.V run.
  const int lrow = 4 * warp + rsub;
  RowIdx ix0, ix1;
  Raw ra, rb;
  auto idx2 = [&](int t) {
    const int base = (t0 + t) * kTileRows + lrow;
    ix0 = idx_load(p, b, base, nswa, ntot);
    ix1 = idx_load(p, b, base + 64, nswa, ntot);
  };
  auto load2 = [&](int t) {
    const int base = (t0 + t) * kTileRows + lrow;
    const RowRef f0 = idx_resolve(p, ix0, base, nswa, ntot), f1 = idx_resolve(p, ix1, base + 64, nswa, ntot);
    fetch(p, f0, v8, ra);
    fetch(p, f1, v8, rb);
    if (tid == 0 && t == 1) stamp(44);
  };
  if (nt > 0) {  // the first tile's rows are in flight while Q is converted, the second tile's indices too
    idx2(0);
    load2(0);
    if (tid == 0) stamp(54);
    if (nt > 1) idx2(1);
  }
  if (tid == 0) stamp(55);
  // Q: staged BF16 rows -> shared FP16 (K-major SW128); heads past H are zero
  wait(kBarQ, 0, 31);
#pragma unroll 4
  for (int i = 0; i < kHG * 64 / kThreads; ++i) {
    const int idx = tid + kThreads * i, row = idx >> 6, u = idx & 63;
    const uint4 v = row < nh ? *reinterpret_cast<const uint4*>(sK + row * 1024 + 16 * u) : zero4();
    *reinterpret_cast<uint4*>(sQ + pm::sw128_offset(row, 16 * u, kQChunk)) = bf16x8_to_f16(v);
  }
  if (tid == 0) stamp(56);
  pm::fence_proxy_async_smem();
  pm::tc_fence_before();
  __syncthreads();  // Q complete; the staging (K buffer) is free for tile 0
  pm::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) stamp(1);

  const uint32_t q_base = pm::smem_u32(sQ), k_base = pm::smem_u32(sK), p_base = pm::smem_u32(sP);
  const uint32_t idesc_s = pm::make_idesc_f16(128, kHG, 0, 0, 0);
  const uint32_t idesc_o = pm::make_idesc_f16(128, kHG, 0, 1, 1);
  const int ch = warp >> 2;         // softmax: this warp's head columns 16 ch .. 16 ch + 15; epilogue: d-block
  const int brow = 32 * wq + lane;  // softmax: this thread's tile row (TMEM lane)
  if (clustered && nt == 0) pm::cluster_arrive_relaxed();
#pragma unroll 1
  for (int t = 0; t < nt; ++t) {
    if (t > 0) {  // the buffer and P are free once the previous tile's P.V MMAs complete
      wait(kBarPvDone, (t - 1) & 1, 32);
      pm::tc_fence_after();
    }
    expand_row(ra, lrow, v8, stg, sK, rowvalid, lut, p.err);
    expand_row(rb, lrow + 64, v8, stg, sK, rowvalid, lut, p.err);
    pm::fence_proxy_async_smem();
    pm::tc_fence_before();
    pm::named_bar_sync(1, kThreads);  // every row (and row flag) of the tile is written
    if (tid == 0 && t < 8) stamp(2 + 2 * t);
    if (warp == 0) {  // S^T = K Q^T, issued by one elected lane of the converged warp
      pm::tc_fence_after();
      if (lane == 0 && t < 8) stamp(18 + t);
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t ad = pm::make_sdesc(k_base + c * kKChunk + 32 * k, 16, 1024);
          const uint64_t bd = pm::make_sdesc(q_base + c * kQChunk + 32 * k, 16, 1024);
          pm::umma_f16_warp(tmem + kTmemS, ad, bd, idesc_s, (c | k) ? 1u : 0u);
        }
      }
      pm::umma_commit_warp(&bars[kBarSFull]);
    }
    // the next tile's rows go out now (they land during this tile's scores, softmax and P.V), and the
    // indices of the tile after it
    if (t + 1 < nt) {
      load2(t + 1);
      if (t + 2 < nt) idx2(t + 2);
    }
    // ---- softmax of the tile
    if (tid == 0 && t == 0) stamp(36);
    wait(kBarSFull, t & 1, 33);
    pm::tc_fence_after();
    // cluster merge: past the last score MMA this CTA's Q buffer and expansion table can take the other
    // splits' partials (first phase of the cluster barrier; waited before those are sent)
    if (clustered && t == nt - 1) pm::cluster_arrive_relaxed();
    if (tid == 0 && t == 0) stamp(37);
    const bool row_ok = rowvalid[brow] != 0;
    const uint32_t s_addr = tmem + kTmemS + 16 * ch + ((uint32_t)(32 * wq) << 16);
    float sv[16];
    pm::tmem_ld16(s_addr, sv);
#pragma unroll
    for (int i = 0; i < 16; ++i) sv[i] = row_ok ? sv[i] * p.scale_log2 : -INFINITY;
    {  // per-head maxima over the tile's rows (scores in log2 units, masked rows -inf)
      float mx[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) mx[i] = sv[i];
      const float r = transpose_reduce16<true>(mx, lane);
      if (lane < 16) red[wq * 64 + 16 * ch + lane] = r;
    }
    pm::named_bar_sync(1, kThreads);
    if (tid == 0 && t == 0) stamp(38);
    if (tid < 64) {
      const int hh = tid;
      const float tmax = fmaxf(fmaxf(red[hh], red[64 + hh]), fmaxf(red[128 + hh], red[192 + hh]));
      const float mu = m_used[hh];
      float a = 1.f;
      if (tmax > mu + kRescaleThreshold || mu == -INFINITY) {
        a = (mu == -INFINITY) ? 0.f : exp2f(mu - tmax);
        m_used[hh] = tmax;
        if (mu != -INFINITY) flags[0] = 1;
      }
      alpha[hh] = a;
    }
    pm::named_bar_sync(1, kThreads);
    if (tid == 0 && t == 0) stamp(40);
    if (flags[0]) {
      // O^T is complete once the previous tile's P.V is (waited above); this warp rescales its lane
      // quadrant's columns of its head quarter in every d-block
#pragma unroll 1
      for (int db = 0; db < 4; ++db) {
        float o[16];
        const uint32_t ta = tmem + kTmemO + db * kHG + 16 * ch + ((uint32_t)(32 * wq) << 16);
        pm::tmem_ld16(ta, o);
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] *= alpha[16 * ch + i];
        pm::tmem_st16(ta, o);
      }
      pm::tmem_wait_st();
    }
    {  // P = 2^(s - m_used) in FP16 (row = tile row, this warp's 16 heads) and the per-head sums of the
       // FP16-rounded values (what the P.V MMA accumulates); red now takes the sums
      __half2 pk[8];
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const float m0 = m_used[16 * ch + i], m1 = m_used[16 * ch + i + 1];
        // a masked row (-inf) or a head without any row yet (-inf max) contributes 0
        const float p0 = (sv[i] == -INFINITY || m0 == -INFINITY) ? 0.f : fast_exp2(sv[i] - m0);
        const float p1 = (sv[i + 1] == -INFINITY || m1 == -INFINITY) ? 0.f : fast_exp2(sv[i + 1] - m1);
        pk[i >> 1] = __floats2half2_rn(p0, p1);
        const float2 r = __half22float2(pk[i >> 1]);
        sv[i] = r.x;
        sv[i + 1] = r.y;
      }
      if (tid == 0 && t == 0) stamp(41);
#pragma unroll
      for (int uu = 0; uu < 2; ++uu)
        *reinterpret_cast<uint4*>(sP + pm::sw128_offset(brow, 32 * ch + 16 * uu, 0)) =
            *reinterpret_cast<uint4*>(&pk[4 * uu]);
      const float r = transpose_reduce16<false>(sv, lane);
      if (lane < 16) red[wq * 64 + 16 * ch + lane] = r;
    }
    if (tid == 0 && t == 0) stamp(39);
    pm::fence_proxy_async_smem();
    pm::tc_fence_before();
    pm::named_bar_sync(1, kThreads);
    if (warp == 0) {  // O^T += V^T P^T over the tile's 128 rows
      pm::tc_fence_after();
      if (lane == 0 && t < 8) stamp(26 + t);
#pragma unroll 1
      for (int db = 0; db < 4; ++db) {
#pragma unroll
        for (int k16 = 0; k16 < 8; ++k16) {  // 16-row groups of the tile
          const uint64_t ad = pm::make_sdesc(k_base + (2 * db) * kKChunk + k16 * 2048, kKChunk, 1024);
          const uint64_t bd = pm::make_sdesc(p_base + k16 * 2048, 8192, 1024);
          pm::umma_f16_warp(tmem + kTmemO + db * kHG, ad, bd, idesc_o, (t > 0 || k16 > 0) ? 1u : 0u);
        }
      }
      pm::umma_commit_warp(&bars[kBarPvDone]);
    }
    if (tid < 64) {
      const int hh = tid;
      l_sum[hh] = l_sum[hh] * alpha[hh] + (red[hh] + red[64 + hh]) + (red[128 + hh] + red[192 + hh]);
      if (hh == 0) flags[0] = 0;
    }
    if (tid == 0 && t < 8) stamp(3 + 2 * t);
  }
  {
    // ------------------------------------------------------------------ epilogue (all 16 warps)
    const bool direct = p.num_splits == 1;
    if (nt > 0) {
      wait(kBarPvDone, (nt - 1) & 1, 36);
      pm::tc_fence_after();
    }
    pm::named_bar_sync(1, kThreads);  // the last tile's sums are in l
    const int64_t part = (int64_t)b * p.num_splits + split;
    if (tid == 0) stamp(34);
    if (tid < 64) {
      const int hh = tid, head = h0 + hh;
      const float m = m_used[hh], l = l_sum[hh];
      if (direct) {
        const float sink2 = sink2v[hh];
        const float M = fmaxf(m, sink2);
        const float w = (m == -INFINITY) ? 0.f : exp2f(m - M);
        const float L = l * w + ((sink2 == -INFINITY) ? 0.f : exp2f(sink2 - M));
        fac[hh] = L > 0.f ? w / L : 0.f;
        if (head < p.H && p.lse) p.lse[(int64_t)b * p.H + head] = L > 0.f ? (M + log2f(L)) / kLog2e : -INFINITY;
      } else if (clustered) {
        fac[hh] = l > 0.f ? 1.f / l : 0.f;  // the staged partial is O / l (FP16 range, like V's values)
      } else if (head < p.H) {
        const bool empty = nt == 0 || m == -INFINITY;
        p.part_ml[(part * p.H + head) * 2 + 0] = empty ? -INFINITY : m;
        p.part_ml[(part * p.H + head) * 2 + 1] = empty ? 0.f : l;
      }
    }
    pm::named_bar_sync(1, kThreads);
    pm::griddep_launch_dependents();  // the combine (or the next kernel) may be scheduled now
    if (tid == 0) stamp(48);
    // O^T: warp w reads lane quadrant w % 4 (d = 128 db + 32 (w % 4) + lane) of d-block db = w / 4, and
    // stages it as [head][512] rows in the (free) K buffer: fp32 partials, or the normalized BF16 output;
    // one bulk copy then writes the group's contiguous rows
    float* sPart = reinterpret_cast<float*>(sK);                // [64 heads][512] fp32 = the whole buffer
    __nv_bfloat16* sOut = reinterpret_cast<__nv_bfloat16*>(sK);  // [64 heads][512] BF16
    __half* sPartH = reinterpret_cast<__half*>(sK);              // [64 heads][512] FP16 O / l (cluster merge)
    int qp = 0;
    if ((direct || clustered) && !p.no_rope) {
      qp = qpos_raw;
      if (qp < 0 || qp >= p.freq_rows) { pm::report_error(p.err, pm::kIndexOutOfRange, b); qp = 0; }
    }
    // cluster merge: this thread's output coordinates d0 .. d0 + 7 (the same for each of its positions) and,
    // for the tail, their inverse-RoPE pairs, loaded now so they have arrived by the cluster barrier
    const int d0 = 8 * (tid % (kD / 8));
    float rc[4] = {1.f, 1.f, 1.f, 1.f}, rs[4] = {0.f, 0.f, 0.f, 0.f};
    if (clustered && d0 >= 448 && !p.no_rope) {
      const float4* f = reinterpret_cast<const float4*>(p.freqs + (int64_t)qp * 64 + (d0 - 448));
      const float4 f0 = f[0], f1 = f[1];  // (cos, sin) of pairs (d0 - 448) / 2 .. + 3
      rc[0] = f0.x; rs[0] = -f0.y; rc[1] = f0.z; rs[1] = -f0.w;
      rc[2] = f1.x; rs[2] = -f1.y; rc[3] = f1.z; rs[3] = -f1.w;
    }
#pragma unroll 1
    for (int db = ch; db < ch + 1; ++db) {
      const int d = 128 * db + 32 * wq + lane;
#pragma unroll 1
      for (int hf = 0; hf < 2; ++hf) {
        float o[32];
        if (nt > 0) {
          pm::tmem_ld32(tmem + kTmemO + db * kHG + 32 * hf + ((uint32_t)(32 * wq) << 16), o);
          if (tid == 0 && db == 0 && hf == 0) stamp(49);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (clustered) {
#pragma unroll
          for (int i = 0; i < 32; ++i) sPartH[(32 * hf + i) * kD + d] = __float2half_rn(o[i] * fac[32 * hf + i]);
          continue;
        }
        if (!direct) {
#pragma unroll
          for (int i = 0; i < 32; ++i) sPart[(32 * hf + i) * kD + d] = o[i];
          continue;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __bfloat162float(__float2bfloat16_rn(o[i] * fac[32 * hf + i]));
        if (d >= 448 && !p.no_rope) {  // inverse RoPE of the tail: pair (d, d + 1) = lanes (2 k, 2 k + 1)
          const int pair = (d - 448) >> 1;
          const float c = p.freqs[(int64_t)qp * 64 + 2 * pair], sn = -p.freqs[(int64_t)qp * 64 + 2 * pair + 1];
          const bool odd = d & 1;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float other = __shfl_xor_sync(0xffffffffu, o[i], 1);
            const float re = odd ? other : o[i], im = odd ? o[i] : other;
            o[i] = odd ? __fadd_rn(__fmul_rn(re, sn), __fmul_rn(im, c))
                       : __fsub_rn(__fmul_rn(re, c), __fmul_rn(im, sn));
          }
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) sOut[(32 * hf + i) * kD + d] = __float2bfloat16_rn(o[i]);
      }
    }
    if (tid == 0) stamp(50);
    if (tid == 0 && p.prof != nullptr) {  // latest / earliest "staged" over all CTAs
      const unsigned long long now = pm::globaltimer_ns();
      atomicMax(reinterpret_cast<unsigned long long*>(p.prof + 47), now);
      atomicMin(reinterpret_cast<unsigned long long*>(p.prof + 46), now);
    }
    pm::fence_proxy_async_smem();  // the staged rows are read by the bulk copy (async proxy)
    pm::named_bar_sync(1, kThreads);
    if (!clustered) {
      if (tid == 0 && nh > 0) {
        if (direct)
          pm::bulk_s2g(p.out + ((int64_t)b * p.H + h0) * kD, sOut, (uint32_t)nh * kD * 2u);
        else
          pm::bulk_s2g(p.part_o + (part * p.H + h0) * kD, sPart, (uint32_t)nh * kD * 4u);
        pm::bulk_commit();
        pm::bulk_wait_read_all();  // the staging is read before the CTA exits; the writes complete with the grid
        stamp(51);
      }
    } else {
      // Split merge inside the cluster.  CTA r (= split r) owns heads [r * hpc, (r + 1) * hpc), hpc = 64 / cs.
      // Every split that has rows sends each owner its staged FP16 O / l rows of the owner's heads (one bulk
      // copy into the owner's Q buffer, slot = sender) and their (m, l) (into the owner's expansion table);
      // both complete on the owner's merge barrier.  The owner weights the splits, sums, and writes BF16 O
      // and the LSE.  Splits without rows send nothing (the set is the same for every CTA).
      const int cs = p.num_splits, hpc = kHG / cs, hb = split * hpc;
      const int lcs = __ffs(cs) - 1;  // cs is a power of two
      uint32_t active = 0;            // bit j: split j has rows (the split ranges of t0 / t1, in 32-bit shifts)
      for (int j = 0; j < cs; ++j)
        if ((((j + 1) * tiles_q) >> lcs) > ((j * tiles_q) >> lcs)) active |= 1u << j;
      const uint32_t n_active = __popc(active);
      const bool sender = (active >> split) & 1;
      float* stat = reinterpret_cast<float*>(lut);  // [cs][hpc][2] (m, l) as received
      if (tid == 0) pm::mbar_arrive_expect_tx(&bars[kBarMerge], n_active * (uint32_t)hpc * (kD * 2u + 8u));
      pm::cluster_wait();  // every CTA is past its last score MMA: its Q buffer and table may be written
      if (tid == 0) stamp(52);
      if (sender) {
        if (tid < cs)  // one bulk copy per owner r = tid: heads r * hpc .. + hpc of the staging
          pm::bulk_s2cluster(pm::dsmem_addr(sQ + split * hpc * (kD * 2), tid), sPartH + tid * hpc * kD,
                             (uint32_t)hpc * kD * 2u, pm::dsmem_addr(&bars[kBarMerge], tid));
        if (tid < kHG) {  // (m, l) of head tid to its owner
          const int r = tid / hpc, i = tid % hpc;
          pm::st_async_f32x2(pm::dsmem_addr(stat + (split * hpc + i) * 2, r), m_used[tid], l_sum[tid],
                             pm::dsmem_addr(&bars[kBarMerge], r));
        }
      }
      // the partials arrive within microseconds: poll before the bounded sleeping wait (wake-ups from a
      // suspended try_wait come late)
      for (int spin = 0; spin < 4096 && !pm::mbar_test_wait(&bars[kBarMerge], 0); ++spin) {
      }
      wait(kBarMerge, 0, 37);
      pm::cluster_arrive_relaxed();  // this CTA's receiving is complete (second phase, waited before exit)
      if (tid == 0) stamp(53);
      float* wts = red;  // [cs][hpc]: w_j l_j / L of head hb + i from split j
      float lse_v = 0.f;
      if (tid < hpc) {
        const float sink2 = sink2v[hb + tid];
        float M = sink2;
        for (int j = 0; j < cs; ++j)
          if ((active >> j) & 1) M = fmaxf(M, stat[(j * hpc + tid) * 2]);
        float L = (sink2 == -INFINITY) ? 0.f : exp2f(sink2 - M);
        for (int j = 0; j < cs; ++j) {
          const float m = stat[(j * hpc + tid) * 2];
          const float wl = (!((active >> j) & 1) || m == -INFINITY) ? 0.f : exp2f(m - M) * stat[(j * hpc + tid) * 2 + 1];
          wts[j * hpc + tid] = wl;
          L += wl;
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        for (int j = 0; j < cs; ++j) wts[j * hpc + tid] *= inv;
        lse_v = L > 0.f ? (M + log2f(L)) / kLog2e : -INFINITY;
      }
      pm::named_bar_sync(1, kThreads);
      if (tid == 0) stamp(45);
      const __half* recv = reinterpret_cast<const __half*>(sQ);  // [cs][hpc][512] FP16 O / l
#pragma unroll 1
      for (int pos = tid; pos < hpc * (kD / 8); pos += kThreads) {
        const int hl = pos / (kD / 8), hh = hb + hl;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j < cs && ((active >> j) & 1)) {
            const float wgt = wts[j * hpc + hl];
            const uint4 v = *reinterpret_cast<const uint4*>(recv + (j * hpc + hl) * kD + d0);
            const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[k]));
              acc[2 * k] += wgt * f.x;
              acc[2 * k + 1] += wgt * f.y;
            }
          }
        }
        uint32_t ob[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {  // BF16 output; the tail inverse-rotated (pairs (d, d + 1)) and rounded again
          float re = __bfloat162float(__float2bfloat16_rn(acc[2 * k]));
          float im = __bfloat162float(__float2bfloat16_rn(acc[2 * k + 1]));
          if (d0 >= 448 && !p.no_rope) {
            const float r2 = __fsub_rn(__fmul_rn(re, rc[k]), __fmul_rn(im, rs[k]));
            const float i2 = __fadd_rn(__fmul_rn(re, rs[k]), __fmul_rn(im, rc[k]));
            re = r2;
            im = i2;
          }
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(re, im);
          ob[k] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        if (h0 + hh < p.H)
          *reinterpret_cast<uint4*>(p.out + ((int64_t)b * p.H + h0 + hh) * kD + d0) = make_uint4(ob[0], ob[1], ob[2], ob[3]);
      }
      if (tid < hpc && h0 + hb + tid < p.H && p.lse) p.lse[(int64_t)b * p.H + h0 + hb + tid] = lse_v;
      if (tid == 0) stamp(51);
      pm::cluster_wait();  // every CTA has received: no bulk copy still reads this CTA's staging
    }
  }
  pm::tc_fence_before();
  __syncthreads();
  if (tid == 0) stamp(35);
  if (tid == 0 && p.prof != nullptr)
    atomicMax(reinterpret_cast<unsigned long long*>(p.prof + 57), pm::globaltimer_ns());
  if (warp == 0) pm::tmem_dealloc(tmem, kTmemCols);
}

// ----------------------------------------------------------------------------- combine
// One warp per (b, h): lane owns 16 coordinates.
__global__ void __launch_bounds__(256) mla_combine_kernel(const float* __restrict__ part_o,
                                                          const float* __restrict__ part_ml,
                                                          const float* __restrict__ sink,
                                                          const int32_t* __restrict__ q_pos,
                                                          const float* __restrict__ freqs, int64_t freq_rows, int B,
                                                          int H, int splits, __nv_bfloat16* __restrict__ out,
                                                          float* __restrict__ lse, int* err, int no_rope) {
  pm::griddep_wait();  // the decode kernel's partials are complete
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
  if (lane >= 16 && !no_rope) {
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

// Both kernels are launched with programmatic stream serialization: the decode kernel's input-free set-up
// overlaps the previous kernel's tail, and the combine is scheduled while the decode epilogue runs; each
// waits (griddepcontrol.wait) for its predecessor's completion before it touches global memory.  `cluster`
// > 1 groups consecutive CTAs into thread-block clusters of that size.
template <typename... KArgs, typename... Args>
static void launch_pdl(void (*kernel)(KArgs...), int grid, int block, size_t smem, int cluster, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    n = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

void launch_sparse_mla_decode(const DecodeParams& params, const float* sink, const int32_t* q_pos,
                              __nv_bfloat16* out, float* lse, cudaStream_t stream) {
  if (params.B == 0) return;
  DecodeParams p = params;
  p.sink = sink;
  p.q_pos = q_pos;
  p.out = out;
  p.lse = lse;
  cudaFuncSetAttribute(sparse_mla_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  const int grid = p.B * p.num_groups * p.num_splits;
  const bool clustered = decode_splits_clustered(p.num_splits);
  launch_pdl(sparse_mla_decode_kernel, grid, kThreads, (size_t)kSmemBytes, clustered ? p.num_splits : 1, stream, p);
  if (p.num_splits > 1 && !clustered) {
    const int warps = p.B * p.H;
    launch_pdl(mla_combine_kernel, (warps + 7) / 8, 256, 0, 1, stream, p.part_o, p.part_ml, sink, q_pos, p.freqs,
               p.freq_rows, p.B, p.H, p.num_splits, out, lse, p.err, p.no_rope);
  }
}

int decode_max_active_clusters(int cluster) {
  cudaFuncSetAttribute(sparse_mla_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster * 64);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, sparse_mla_decode_kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}
