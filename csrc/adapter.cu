// Adapter: Packed C4 records (values / bitmap / scales planes) -> Native 584 B records in a paged
// workspace, so a Native reader can consume Packed KV (reference: `packed_to_native.cu`, the CUDA
// Adapter mode that reconstructs the selected rows before stock FlashMLA, 64-bit addressing).  Any
// survivor count: the values plane holds `keep` bytes per row (64 .. 448; the default layout 256).
//
// One warp per record.  Lane l owns the 16 consecutive coordinates [16 l, 16 l + 16): bits
// 16 (l % 4) .. + 15 of bitmap word l / 4.  A warp prefix sum of the lanes' popcounts gives each lane
// the index of its first kept value.  Values are dequantized exactly (E4M3 x 2^(scale - 127), BF16),
// pruned coordinates are zero.  NoPE tiles (lanes 0-27, 4 lanes per 64-coordinate tile) are
// re-quantized with the exact UE8M0 rule (smallest e with 448 * 2^e >= max(amax, 1e-4)) and E4M3
// round-to-nearest-even; the RoPE tail (lanes 28-31) is rotated by the record's position as adjacent
// pairs (re c - im s, re s + im c, IEEE products) and rounded to BF16.  Same arithmetic as
// packmla/formats/codec.py `native_from_packed`.
#include "launchers.h"
#include "common/sm100.cuh"

namespace {
constexpr int kPage = 64, kNativeData = 576, kNativePageBytes = kPage * 584, kNope = 448;

__global__ void __launch_bounds__(256) packed_to_native_kernel(
    const uint8_t* __restrict__ values, const uint64_t* __restrict__ bitmap, const uint8_t* __restrict__ scales,
    int64_t src_rows_total, const int32_t* __restrict__ rows, const int32_t* __restrict__ positions,
    const float* __restrict__ freqs, int64_t freq_rows, uint8_t* __restrict__ out, const int64_t* __restrict__ dst,
    int64_t out_slots, int keep, int n, int* err) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n) return;
  const int64_t d = dst[warp];
  if (d < 0) return;
  const int64_t row = rows[warp];
  const int64_t pos = positions[warp];
  if (row < 0 || row >= src_rows_total || d >= out_slots || pos < 0 || pos >= freq_rows) {
    if (lane == 0) pm::report_error(err, pm::kIndexOutOfRange, warp);
    return;
  }
  const uint64_t word = bitmap[row * 8 + (lane >> 2)];
  const uint32_t bits = (uint32_t)(word >> (16 * (lane & 3))) & 0xFFFFu;
  const int cnt = __popc(bits);
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  int k = incl - cnt;  // index of this lane's first kept value
  const float scale = pm::exp2i((int)scales[row * 8 + (lane >> 2)] - 127);
  const uint8_t* vrow = values + row * keep;
  float x[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    x[i] = 0.f;
    if (bits & (1u << i)) {
      const uint16_t code = k < keep ? vrow[k] : 0;  // a corrupt bitmap (> keep bits) reads no further
      ++k;
      x[i] = __low2float(pm::e4m3x2_to_h2(code)) * scale;  // exact: E4M3 x power of two
    }
  }
  const int64_t page = d / kPage, rip = d % kPage;
  uint8_t* data = out + page * kNativePageBytes + rip * kNativeData;
  uint8_t* srow = out + page * kNativePageBytes + kPage * kNativeData + rip * 8;
  int code = 0;
  if (lane < 28) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(x[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0x0fffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0x0fffffffu, amax, 2));
    const int e = pm::ue8m0_exp(amax);
    code = e + 127;
    const float inv = pm::exp2i(-e);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w[i] = (uint32_t)pm::f32x2_to_e4m3x2(x[4 * i] * inv, x[4 * i + 1] * inv) |
             ((uint32_t)pm::f32x2_to_e4m3x2(x[4 * i + 2] * inv, x[4 * i + 3] * inv) << 16);
    *reinterpret_cast<uint4*>(data + 16 * lane) = make_uint4(w[0], w[1], w[2], w[3]);
  } else {
    const float* f = freqs + pos * 64;
    __nv_bfloat16 o[16];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const int pair = 8 * (lane - 28) + p;
      const float c = f[2 * pair], s = f[2 * pair + 1];
      const float re = x[2 * p], im = x[2 * p + 1];
      o[2 * p] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(re, c), __fmul_rn(im, s)));
      o[2 * p + 1] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(re, s), __fmul_rn(im, c)));
    }
    uint4* t = reinterpret_cast<uint4*>(data + kNope + 32 * (lane - 28));
    t[0] = *reinterpret_cast<uint4*>(o);
    t[1] = *reinterpret_cast<uint4*>(o + 8);
  }
  // scale bytes of the 7 NoPE tiles (lane 4 t holds tile t) + 1 pad byte
  uint32_t b[7];
#pragma unroll
  for (int t = 0; t < 7; ++t) b[t] = (uint32_t)__shfl_sync(0xffffffffu, code, 4 * t);
  if (lane == 0)
    *reinterpret_cast<uint2*>(srow) = make_uint2(b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24),
                                                 b[4] | (b[5] << 8) | (b[6] << 16));
}
}  // namespace

void launch_packed_to_native(const uint8_t* values, const uint64_t* bitmap, const uint8_t* scales, int64_t src_rows,
                             const int32_t* rows, const int32_t* positions, const float* freqs, int64_t freq_rows,
                             uint8_t* out, const int64_t* dst, int64_t out_slots, int keep, int n, int* err,
                             cudaStream_t stream) {
  if (n <= 0) return;
  packed_to_native_kernel<<<(n + 7) / 8, 256, 0, stream>>>(values, bitmap, scales, src_rows, rows, positions, freqs,
                                                           freq_rows, out, dst, out_slots, keep, n, err);
}
