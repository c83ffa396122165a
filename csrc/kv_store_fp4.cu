// FP4 C4 records of the V4.1 cache: FP32 compressor rows -> Native (288 B) or Packed (224 B) records.
//
// Reference behaviour: the V4.1 fork's FP4 cache store (third_party/README.md:120-141); the bytes follow
// packmla/formats/fp4.py (the CPU oracle these kernels are tested against byte for byte):
//   * rows are normalized like the FP8 stores (bf16((x * r) * w)), the 64-coordinate tail is rotated with
//     the record's RoPE row and rounded to BF16 again: FP4 records hold rotated values;
//   * one E4M3 scale per 16 coordinates, E4M3(amax / 6) rounded to nearest even (saturating), and E2M1
//     codes of x / scale rounded to nearest, ties to the even code, saturating at 6 (cvt.rn.satfinite),
//     with a negative zero stored as +0;
//   * Native data row: 256 code bytes, coordinate 2 i in the low nibble of byte i;
//     Packed data row: the 256 largest dequantized magnitudes' codes in coordinate order (even ranks in low
//     nibbles, 128 B) and 8 bitmap words, MSB-first (coordinate 64 w + b is bit 63 - b of word w);
//   * a page holds its 64 data rows, then its 64 scale rows (32 B each).
// One warp per row; lane l owns coordinates {128 j + 4 l + i}, so a 16-coordinate scale group is four lanes.
#include "launchers.h"
#include "common/sm100.cuh"

namespace {

constexpr int kPage = 64;

__device__ __forceinline__ float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// sum of squares in the order of packmla.formats.codec (per lane in (j, i) order, then a butterfly)
__device__ __forceinline__ float lane_sumsq(const float (&x)[16]) {
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 16; ++k) acc = __fadd_rn(acc, __fmul_rn(x[k], x[k]));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  return acc;
}

// E4M3 code of a non-negative fp32 value (round to nearest even, saturating) and its fp32 value
__device__ __forceinline__ uint32_t e4m3_code(float v, float* value) {
  const uint16_t c = pm::f32x2_to_e4m3x2(v, 0.f);
  *value = __low2float(pm::e4m3x2_to_h2(c));
  return c & 0xFFu;
}

// E2M1 code of x (nearest, ties to even, saturating; negative zero -> +0)
__device__ __forceinline__ uint32_t e2m1_code(float x) {
  uint16_t r;
  // the first source goes to the high nibble, the second (x) to the low one
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tmov.b16 %0, {t, t};\n\t}" : "=h"(r) : "f"(0.f), "f"(x));
  const uint32_t c = r & 0xFu;
  return (c & 7u) ? c : 0u;
}

// value of an E2M1 code: magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6 (exponent (c >> 1) - 1, one mantissa bit)
__device__ __forceinline__ float e2m1_value(uint32_t c) {
  const uint32_t m = c & 7u;
  const float mag = m < 2u ? 0.5f * (float)m : pm::exp2i((int)(m >> 1) - 1) * (1.f + 0.5f * (float)(m & 1u));
  return (c & 8u) ? -mag : mag;
}

__global__ void __launch_bounds__(256) fp4_store_kernel(
    const float* __restrict__ raw, int64_t raw_stride, const float* __restrict__ weight, float eps,
    const int64_t* __restrict__ slots, const int64_t* __restrict__ positions, const float* __restrict__ freqs,
    int64_t freq_rows, uint8_t* __restrict__ pool, int64_t pool_slots, int packed, int rows, int* err) {
  __shared__ uint8_t stage[8][256];  // Packed: survivor codes by rank, one byte each (per warp)
  const int wl = threadIdx.x >> 5;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int64_t slot = slots[warp];
  if (slot < 0) return;  // invalid destination: nothing written
  if (slot >= pool_slots) { if (lane == 0) pm::report_error(err, pm::kIndexOutOfRange, warp); return; }
  const int64_t pos = positions[warp];
  if (pos < 0 || pos >= freq_rows) { if (lane == 0) pm::report_error(err, pm::kIndexOutOfRange, warp); return; }

  float x[16];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 v = *reinterpret_cast<const float4*>(raw + (int64_t)warp * raw_stride + 128 * j + 4 * lane);
    x[4 * j + 0] = v.x; x[4 * j + 1] = v.y; x[4 * j + 2] = v.z; x[4 * j + 3] = v.w;
  }
  const float ss = lane_sumsq(x);
  const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.f / 512.f), eps)));
  float y[16];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) y[4 * j + i] = bf16_round(__fmul_rn(__fmul_rn(x[4 * j + i], r), weight[128 * j + 4 * lane + i]));
  if (lane >= 16) {  // the tail (coordinates 448 + 4 (lane - 16) + i): rotate, round to BF16
    const float* f = freqs + pos * 64;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int pair = 2 * (lane - 16) + p;
      const float c = f[2 * pair], s = f[2 * pair + 1];
      const float re = y[12 + 2 * p], im = y[13 + 2 * p];
      y[12 + 2 * p] = bf16_round(__fsub_rn(__fmul_rn(re, c), __fmul_rn(im, s)));
      y[13 + 2 * p] = bf16_round(__fadd_rn(__fmul_rn(re, s), __fmul_rn(im, c)));
    }
  }
  // scales and codes; group of lane l in block j: 8 j + l / 4
  uint32_t code[16], scode[4];
  float deq[16];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) amax = fmaxf(amax, fabsf(y[4 * j + i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    float s;
    scode[j] = e4m3_code(__fdiv_rn(amax, 6.f), &s);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      code[4 * j + i] = s > 0.f ? e2m1_code(__fdiv_rn(y[4 * j + i], s)) : 0u;
      deq[4 * j + i] = e2m1_value(code[4 * j + i]) * s;  // exact: at most 6 significant bits
    }
  }
  const int64_t page = slot / kPage, rip = slot % kPage;
  const int data_row = packed ? 192 : 256;
  uint8_t* base = pool + page * (int64_t)kPage * (data_row + 32);
  uint8_t* data = base + rip * data_row;
  uint8_t* scales = base + (int64_t)kPage * data_row + rip * 32;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if ((lane & 3) == 0) scales[8 * j + (lane >> 2)] = (uint8_t)scode[j];
  if (!packed) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint16_t*>(data + 64 * j + 2 * lane) =
          (uint16_t)(code[4 * j] | (code[4 * j + 1] << 4) | (code[4 * j + 2] << 8) | (code[4 * j + 3] << 12));
    return;
  }
  // Packed: the 256 largest dequantized magnitudes, ties to the lower coordinate
  uint32_t key[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) key[k] = __float_as_uint(deq[k]) & 0x7FFFFFFFu;
  uint32_t T = 0;  // the 256th largest magnitude
#pragma unroll 1
  for (int bit = 30; bit >= 0; --bit) {
    const uint32_t cand = T | (1u << bit);
    int c = 0;
#pragma unroll
    for (int k = 0; k < 16; ++k) c += key[k] >= cand;
    if (__reduce_add_sync(0xffffffffu, c) >= 256) T = cand;
  }
  int gt = 0;
#pragma unroll
  for (int k = 0; k < 16; ++k) gt += key[k] > T;
  const int need = 256 - __reduce_add_sync(0xffffffffu, gt);  // elements equal to T to keep, lowest first
  bool keep[16];
  int eq_before = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int cnt = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) cnt += key[4 * j + i] == T;
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int rank = eq_before + incl - cnt;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      bool kp = key[4 * j + i] > T;
      if (key[4 * j + i] == T) { kp = rank < need; ++rank; }
      keep[4 * j + i] = kp;
    }
    eq_before += __shfl_sync(0xffffffffu, incl, 31);
  }
  // survivor codes to their ranks (coordinate order: block j, then lane, then i), one byte each
  int out_before = 0;
  uint32_t wlo[4], whi[4];  // bitmap words 2 j (lanes 0-15) and 2 j + 1 (lanes 16-31), as 32-bit halves
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int cnt = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) cnt += keep[4 * j + i];
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int pos_r = out_before + incl - cnt;
    uint64_t bits = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (keep[4 * j + i]) {
        stage[wl][pos_r++] = (uint8_t)code[4 * j + i];
        bits |= 1ull << (63 - (4 * (lane & 15) + i));  // coordinate b of the word at bit 63 - b
      }
    }
    out_before += __shfl_sync(0xffffffffu, incl, 31);
    const bool lo_half = lane < 16;
    const uint32_t b_hi = (uint32_t)(bits >> 32), b_lo = (uint32_t)bits;
    wlo[j] = __reduce_or_sync(0xffffffffu, lo_half ? b_lo : 0u);
    whi[j] = __reduce_or_sync(0xffffffffu, lo_half ? b_hi : 0u);
    const uint32_t w1_lo = __reduce_or_sync(0xffffffffu, lo_half ? 0u : b_lo);
    const uint32_t w1_hi = __reduce_or_sync(0xffffffffu, lo_half ? 0u : b_hi);
    if (lane == 2 * j) *reinterpret_cast<uint2*>(data + 128 + 8 * (2 * j)) = make_uint2(wlo[j], whi[j]);
    if (lane == 2 * j + 1) *reinterpret_cast<uint2*>(data + 128 + 8 * (2 * j + 1)) = make_uint2(w1_lo, w1_hi);
  }
  __syncwarp();
  const uint8_t* st = stage[wl] + 8 * lane;  // ranks 8 l .. 8 l + 7 -> bytes 4 l .. 4 l + 3
  *reinterpret_cast<uint32_t*>(data + 4 * lane) =
      (uint32_t)(st[0] | (st[1] << 4)) | ((uint32_t)(st[2] | (st[3] << 4)) << 8) |
      ((uint32_t)(st[4] | (st[5] << 4)) << 16) | ((uint32_t)(st[6] | (st[7] << 4)) << 24);
}

}  // namespace

void launch_fp4_store(const float* raw, int64_t raw_stride, const float* weight, float eps, const int64_t* slots,
                      const int64_t* positions, const float* freqs, int64_t freq_rows, uint8_t* pool,
                      int64_t pool_slots, bool packed, int rows, int* err, cudaStream_t stream) {
  if (rows == 0) return;
  fp4_store_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(raw, raw_stride, weight, eps, slots, positions, freqs,
                                                       freq_rows, pool, pool_slots, packed ? 1 : 0, rows, err);
}
