// KV store kernels: FP32 compressor rows -> Native (584 B) or Packed (328 B) C4 records.
//
// One warp per row.  Lane l owns coordinates {128 j + 4 l + i : j, i in 0..3}, loaded as four
// float4.  The 64-coordinate tile of (j, l) is 2 j + (l >= 16), so per-tile reductions are
// half-warp butterflies.  Arithmetic order is the contract of packmla/formats/codec.py:
// squares rounded then summed in (j, i) order, butterfly over lanes, r = 1/sqrt(ss/512 + eps)
// with IEEE ops, y = bf16((x*r)*w), UE8M0 from the exact exponent rule, E4M3 via cvt.rn.satfinite.
//
// Reference behaviour: Native store = `fused_norm_rope_flashmla`, Packed store =
// `_pack_fused_fp32_kernel` (third_party/README.md:257; docs/agents/numerical-and-validation.md:22-26).
#include "launchers.h"
#include "common/sm100.cuh"

namespace {

constexpr int kD = 512, kNope = 448, kPage = 64, kNativeData = 576;
constexpr int kNativePageBytes = kPage * 584;

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

using pm::ue8m0_exp;

__device__ __forceinline__ float half_max(float v) {
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum of squares in the canonical lane order; every lane returns the full sum.
__device__ __forceinline__ float lane_sumsq(const float (&x)[16]) {
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 16; ++k) acc = __fadd_rn(acc, __fmul_rn(x[k], x[k]));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  return acc;
}

__device__ __forceinline__ void load_row(const float* __restrict__ row, int lane, float (&x)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float4 v = *reinterpret_cast<const float4*>(row + 128 * j + 4 * lane);
    x[4 * j + 0] = v.x; x[4 * j + 1] = v.y; x[4 * j + 2] = v.z; x[4 * j + 3] = v.w;
  }
}

// ----------------------------------------------------------------------------- native
__global__ void __launch_bounds__(256) native_store_kernel(
    const float* __restrict__ raw, int64_t raw_stride, const float* __restrict__ weight, float eps,
    const int64_t* __restrict__ slots, const int64_t* __restrict__ positions, const float* __restrict__ freqs,
    int64_t freq_rows, uint8_t* __restrict__ pool, int64_t pool_slots, int rows, int* err) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int64_t slot = slots[warp];
  if (slot < 0) return;  // invalid destination: nothing written
  if (slot >= pool_slots) { if (lane == 0) pm::report_error(err, pm::kIndexOutOfRange, warp); return; }
  const int64_t pos = positions[warp];
  if (pos < 0 || pos >= freq_rows) { if (lane == 0) pm::report_error(err, pm::kIndexOutOfRange, warp); return; }

  float x[16];
  load_row(raw + (int64_t)warp * raw_stride, lane, x);
  const float ss = lane_sumsq(x);
  const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.f / 512.f), eps)));
  float y[16];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float w = weight[128 * j + 4 * lane + i];
      y[4 * j + i] = bf16_round(__fmul_rn(__fmul_rn(x[4 * j + i], r), w));
    }

  const int64_t page = slot / kPage, rip = slot % kPage;
  uint8_t* data = pool + page * kNativePageBytes + rip * kNativeData;
  uint8_t* scales = pool + page * kNativePageBytes + kPage * kNativeData + rip * 8;
  int codes[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) amax = fmaxf(amax, fabsf(y[4 * j + i]));
    amax = half_max(amax);
    const int e = ue8m0_exp(amax);
    codes[j] = e + 127;
    const bool tail = (j == 3) && (lane >= 16);
    if (!tail) {
      const float inv = pm::exp2i(-e);
      uint16_t lo = pm::f32x2_to_e4m3x2(y[4 * j + 0] * inv, y[4 * j + 1] * inv);
      uint16_t hi = pm::f32x2_to_e4m3x2(y[4 * j + 2] * inv, y[4 * j + 3] * inv);
      *reinterpret_cast<uint32_t*>(data + 128 * j + 4 * lane) = (uint32_t)lo | ((uint32_t)hi << 16);
    } else {
      const int c0 = 4 * (lane - 16);  // tail coordinate offset of y[12]
      const float* f = freqs + pos * 64;
      __nv_bfloat16 out[4];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const int pair = c0 / 2 + p;
        const float c = f[2 * pair], s = f[2 * pair + 1];
        const float re = y[12 + 2 * p], im = y[13 + 2 * p];
        out[2 * p] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(re, c), __fmul_rn(im, s)));
        out[2 * p + 1] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(re, s), __fmul_rn(im, c)));
      }
      *reinterpret_cast<uint2*>(data + kNope + 2 * c0) = *reinterpret_cast<uint2*>(out);
    }
  }
  // tile t = 2 j + half: lanes 0 and 16 hold codes of both halves
  int c_hi[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) c_hi[j] = __shfl_sync(0xffffffffu, codes[j], 16);
  if (lane == 0) {
    const uint32_t lo_word =
        (uint32_t)codes[0] | ((uint32_t)c_hi[0] << 8) | ((uint32_t)codes[1] << 16) | ((uint32_t)c_hi[1] << 24);
    const uint32_t hi_word = (uint32_t)codes[2] | ((uint32_t)c_hi[2] << 8) | ((uint32_t)codes[3] << 16);  // pad 0
    *reinterpret_cast<uint2*>(scales) = make_uint2(lo_word, hi_word);
  }
}

// ----------------------------------------------------------------------------- packed
// kRaw: GLM-5.3 Packed rows (raw E4M3 survivors, no scale plane): the same selection and masked norm, codes
// of y itself.
template <bool kRaw>
__global__ void __launch_bounds__(256) packed_store_kernel(
    const float* __restrict__ raw, int64_t raw_stride, const float* __restrict__ weight, float eps,
    const int64_t* __restrict__ slots, uint8_t* __restrict__ values, uint64_t* __restrict__ bitmap,
    uint8_t* __restrict__ scales, int64_t pool_rows, int keep_n, int rows, int* err) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int64_t slot = slots[warp];
  if (slot < 0) return;
  if (slot >= pool_rows) { if (lane == 0) pm::report_error(err, pm::kIndexOutOfRange, warp); return; }

  float x[16];
  load_row(raw + (int64_t)warp * raw_stride, lane, x);
  uint32_t key[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) key[k] = __float_as_uint(x[k]) & 0x7FFFFFFFu;

  // T = largest value with count(key >= T) >= keep_n  (the keep_n-th largest magnitude)
  uint32_t T = 0;
#pragma unroll 1
  for (int bit = 30; bit >= 0; --bit) {
    const uint32_t cand = T | (1u << bit);
    int c = 0;
#pragma unroll
    for (int k = 0; k < 16; ++k) c += key[k] >= cand;
    c = __reduce_add_sync(0xffffffffu, c);
    if (c >= keep_n) T = cand;
  }
  int gt = 0;
#pragma unroll
  for (int k = 0; k < 16; ++k) gt += key[k] > T;
  gt = __reduce_add_sync(0xffffffffu, gt);
  const int need = keep_n - gt;  // equal-to-T elements to keep, lowest coordinates first

  bool keep[16];
  int eq_before = 0;  // equal elements in earlier chunks (warp-uniform)
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int cnt = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) cnt += key[4 * j + i] == T;
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int rank = eq_before + incl - cnt;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t kk = key[4 * j + i];
      bool kp = kk > T;
      if (kk == T) { kp = rank < need; ++rank; }
      keep[4 * j + i] = kp;
    }
    eq_before += __shfl_sync(0xffffffffu, incl, 31);
  }

  float xm[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) xm[k] = keep[k] ? x[k] : 0.f;
  const float ss = lane_sumsq(xm);
  const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.f / 512.f), eps)));
  float y[16];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float w = weight[128 * j + 4 * lane + i];
      y[4 * j + i] = bf16_round(__fmul_rn(__fmul_rn(xm[4 * j + i], r), w));
    }

  uint8_t* vrow = values + slot * keep_n;
  int out_before = 0;
  int codes[4];
  uint64_t words[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int e = 0;
    if (!kRaw) {
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) amax = fmaxf(amax, fabsf(y[4 * j + i]));
      amax = half_max(amax);
      e = ue8m0_exp(amax);
    }
    codes[j] = e + 127;
    const float inv = pm::exp2i(-e);
    uint16_t lo = pm::f32x2_to_e4m3x2(y[4 * j + 0] * inv, y[4 * j + 1] * inv);
    uint16_t hi = pm::f32x2_to_e4m3x2(y[4 * j + 2] * inv, y[4 * j + 3] * inv);
    const uint32_t packed4 = (uint32_t)lo | ((uint32_t)hi << 16);
    int cnt = 0;
    uint32_t nib = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) { cnt += keep[4 * j + i]; nib |= (uint32_t)keep[4 * j + i] << i; }
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int pos = out_before + incl - cnt;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (keep[4 * j + i]) vrow[pos++] = (uint8_t)(packed4 >> (8 * i));
    out_before += __shfl_sync(0xffffffffu, incl, 31);
    // bitmap word for tile 2j + half: OR of nibble << 4*(lane%16) over the half-warp
    uint64_t w = (uint64_t)nib << (4 * (lane & 15));
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) w |= __shfl_xor_sync(0xffffffffu, w, o);
    words[j] = w;
  }
  if (lane == 0 || lane == 16) {
    const int half = lane >> 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) bitmap[slot * 8 + 2 * j + half] = words[j];
  }
  if (kRaw) return;
  int c_hi[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) c_hi[j] = __shfl_sync(0xffffffffu, codes[j], 16);
  if (lane == 0) {
    uint32_t lo_word = (uint32_t)codes[0] | ((uint32_t)c_hi[0] << 8) | ((uint32_t)codes[1] << 16) | ((uint32_t)c_hi[1] << 24);
    uint32_t hi_word = (uint32_t)codes[2] | ((uint32_t)c_hi[2] << 8) | ((uint32_t)codes[3] << 16) | ((uint32_t)c_hi[3] << 24);
    *reinterpret_cast<uint2*>(scales + slot * 8) = make_uint2(lo_word, hi_word);
  }
}

// ----------------------------------------------------------------------------- GLM-5.3 Native
// 512 raw E4M3 codes of y = bf16((x r) w) per row, rows contiguous ([rows, 512] bytes).
__global__ void __launch_bounds__(256) glm_native_store_kernel(
    const float* __restrict__ raw, int64_t raw_stride, const float* __restrict__ weight, float eps,
    const int64_t* __restrict__ slots, uint8_t* __restrict__ pool, int64_t pool_rows, int rows, int* err) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int64_t slot = slots[warp];
  if (slot < 0) return;
  if (slot >= pool_rows) { if (lane == 0) pm::report_error(err, pm::kIndexOutOfRange, warp); return; }
  float x[16];
  load_row(raw + (int64_t)warp * raw_stride, lane, x);
  const float ss = lane_sumsq(x);
  const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.f / 512.f), eps)));
  uint8_t* row = pool + slot * kD;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float y[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      y[i] = bf16_round(__fmul_rn(__fmul_rn(x[4 * j + i], r), weight[128 * j + 4 * lane + i]));
    const uint16_t lo = pm::f32x2_to_e4m3x2(y[0], y[1]), hi = pm::f32x2_to_e4m3x2(y[2], y[3]);
    *reinterpret_cast<uint32_t*>(row + 128 * j + 4 * lane) = (uint32_t)lo | ((uint32_t)hi << 16);
  }
}

// GLM-5.3 Adapter: Packed rows (256 survivors + LSB-first bitmap) -> Native rows (dropped coordinates 0).
// One warp per row; lane l writes coordinates 16 l .. 16 l + 15 (bits 16 (l % 4) .. of word l / 4).
__global__ void __launch_bounds__(256) glm_packed_to_native_kernel(
    const uint8_t* __restrict__ values, const uint64_t* __restrict__ bitmap, int64_t pool_rows,
    const int64_t* __restrict__ rows_in, uint8_t* __restrict__ out, int rows, int* err) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int64_t r = rows_in[warp];
  uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)warp * kD) + lane;
  if (r < 0 || r >= pool_rows) {
    if (r >= pool_rows && lane == 0) pm::report_error(err, pm::kIndexOutOfRange, warp);
    *dst = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint64_t* bw = bitmap + r * 8;
  const int w = lane >> 2, sh = 16 * (lane & 3);
  int rank = 0;
  for (int k = 0; k < w; ++k) rank += __popcll(bw[k]);
  const uint64_t word = bw[w];
  rank += __popcll(word & ((1ull << sh) - 1ull));
  const uint32_t bits = (uint32_t)(word >> sh) & 0xFFFFu;
  const uint8_t* v = values + r * 256;
  alignas(16) uint8_t c[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const bool kept = ((bits >> k) & 1u) && rank < 256;  // a row with more than 256 bits set reads no further
    c[k] = kept ? v[rank] : (uint8_t)0;
    rank += kept;
  }
  *dst = *reinterpret_cast<const uint4*>(c);
}

}  // namespace

void launch_native_store(const float* raw, int64_t raw_stride, const float* weight, float eps, const int64_t* slots,
                         const int64_t* positions, const float* freqs, int64_t freq_rows, uint8_t* pool,
                         int64_t pool_slots, int rows, int* err, cudaStream_t stream) {
  if (rows == 0) return;
  native_store_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(raw, raw_stride, weight, eps, slots, positions, freqs,
                                                          freq_rows, pool, pool_slots, rows, err);
}

void launch_packed_store(const float* raw, int64_t raw_stride, const float* weight, float eps, const int64_t* slots,
                         uint8_t* values, uint64_t* bitmap, uint8_t* scales, int64_t pool_rows, int keep, int rows,
                         int* err, cudaStream_t stream) {
  if (rows == 0) return;
  packed_store_kernel<false><<<(rows + 7) / 8, 256, 0, stream>>>(raw, raw_stride, weight, eps, slots, values, bitmap,
                                                                 scales, pool_rows, keep, rows, err);
}

void launch_glm_store(const float* raw, int64_t raw_stride, const float* weight, float eps, const int64_t* slots,
                      bool packed, uint8_t* pool, uint8_t* values, uint64_t* bitmap, int64_t pool_rows, int rows,
                      int* err, cudaStream_t stream) {
  if (rows == 0) return;
  if (packed)
    packed_store_kernel<true><<<(rows + 7) / 8, 256, 0, stream>>>(raw, raw_stride, weight, eps, slots, values, bitmap,
                                                                  nullptr, pool_rows, 256, rows, err);
  else
    glm_native_store_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(raw, raw_stride, weight, eps, slots, pool, pool_rows,
                                                                rows, err);
}

void launch_glm_packed_to_native(const uint8_t* values, const uint64_t* bitmap, int64_t pool_rows,
                                 const int64_t* rows_in, uint8_t* out, int rows, int* err, cudaStream_t stream) {
  if (rows == 0) return;
  glm_packed_to_native_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(values, bitmap, pool_rows, rows_in, out, rows, err);
}
