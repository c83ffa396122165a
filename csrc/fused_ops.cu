// Fused element-wise / reduction kernels of the decode step (one launch each instead of chains of
// small framework kernels): residual add + RMSNorm, q-tail RoPE, compressor pooling, MoE routing,
// SiLU-and-multiply, MoE combine.  All bandwidth-trivial; the point is launch count inside the
// captured decode graph.
#include "launchers.h"
#include "common/sm100.cuh"

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ----------------------------------------------------------------------------- add + RMSNorm
// One CTA (256 threads) per row: x_out = x + d (if d), h = bf16(x_out * rsqrt(mean(x_out^2) + eps) * w).
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t xs,
                                                          const __nv_bfloat16* __restrict__ d, int64_t ds,
                                                          const float* __restrict__ dfp32, int64_t dfs,
                                                          __nv_bfloat16* __restrict__ x_out, int64_t xos,
                                                          const float* __restrict__ w, float eps,
                                                          __nv_bfloat16* __restrict__ h, int64_t hs, int n) {
  __shared__ float red[8];
  const int row = blockIdx.x, tid = threadIdx.x;
  const __nv_bfloat16* xr = x + (int64_t)row * xs;
  float v[32];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int i = tid * 2 + j * 512;
    v[2 * j] = v[2 * j + 1] = 0.f;
    if (i < n) {
      float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xr + i));
      if (d) {
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(d + (int64_t)row * ds + i));
        a.x += b.x;
        a.y += b.y;
      }
      if (dfp32) {
        const float2 b = *reinterpret_cast<const float2*>(dfp32 + (int64_t)row * dfs + i);
        a.x += b.x;
        a.y += b.y;
      }
      if (d || dfp32) {
        // the residual stream is bf16: round before the norm so h is computed from the stored stream
        const __nv_bfloat162 r = __floats2bfloat162_rn(a.x, a.y);
        if (x_out) *reinterpret_cast<__nv_bfloat162*>(x_out + (int64_t)row * xos + i) = r;
        a = __bfloat1622float2(r);
      }
      v[2 * j] = a.x;
      v[2 * j + 1] = a.y;
      ss += a.x * a.x + a.y * a.y;
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = rsqrtf(tot / n + eps);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int i = tid * 2 + j * 512;
    if (i < n) {
      const float a = v[2 * j] * r * w[i], b = v[2 * j + 1] * r * w[i + 1];
      *reinterpret_cast<__nv_bfloat162*>(h + (int64_t)row * hs + i) = __floats2bfloat162_rn(a, b);
    }
  }
}

// ----------------------------------------------------------------------------- q RoPE
// q [B, H, 512] bf16 (row stride qs, head stride 512): rotate coords 448..511 by freqs[pos[b]].
__global__ void rope_q_kernel(__nv_bfloat16* __restrict__ q, int64_t qs, int H, const int64_t* __restrict__ pos,
                              const float* __restrict__ freqs, int B) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;  // (b, h, pair)
  if (idx >= B * H * 32) return;
  const int pair = idx & 31, bh = idx >> 5, b = bh / H, hh = bh % H;
  __nv_bfloat16* p = q + b * qs + (int64_t)hh * 512 + 448 + 2 * pair;
  const float2 v = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(p));
  const float* f = freqs + pos[b] * 64 + 2 * pair;
  const float c = f[0], s = f[1];
  *reinterpret_cast<__nv_bfloat162*>(p) =
      __floats2bfloat162_rn(__fsub_rn(__fmul_rn(v.x, c), __fmul_rn(v.y, s)), __fadd_rn(__fmul_rn(v.x, s), __fmul_rn(v.y, c)));
}

// ----------------------------------------------------------------------------- compressor pooling
// Online-softmax pooling of one token per row into per-request state [slots, 3, D] = (max, sum, acc).
// proj [B, >= off + 2D] bf16 holds (value | gate) at column `off`; ape [ratio, D] fp32 is added to the
// gate at slot pos % ratio.  raw[b] = acc / sum after the update; the state resets when the group
// of `ratio` tokens completes.
__global__ void comp_pool_kernel(const __nv_bfloat16* __restrict__ proj, int64_t ps, int off, int D,
                                 const float* __restrict__ ape, int ratio, float* __restrict__ state,
                                 const int64_t* __restrict__ req, const int64_t* __restrict__ pos,
                                 float* __restrict__ raw, int64_t rs, int B) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= B * D) return;
  const int b = idx / D, d = idx % D;
  const int slot_in = (int)(pos[b] % ratio);
  const float val = __bfloat162float(proj[b * ps + off + d]);
  const float gate = __bfloat162float(proj[b * ps + off + D + d]) + ape[slot_in * D + d];
  float* st = state + req[b] * 3 * D;
  const float m = st[d], l = st[D + d], acc = st[2 * D + d];
  const float mn = fmaxf(m, gate);
  const float a = (m == -INFINITY) ? 0.f : expf(m - mn);
  const float e = expf(gate - mn);
  const float l2 = l * a + e, acc2 = acc * a + e * val;
  raw[b * rs + d] = acc2 / l2;
  const bool done = slot_in == ratio - 1;
  st[d] = done ? -INFINITY : mn;
  st[D + d] = done ? 0.f : l2;
  st[2 * D + d] = done ? 0.f : acc2;
}

// ----------------------------------------------------------------------------- routing
// Warp per token: s = sigmoid(logit); choose top-k of s + bias (ties: lower expert); w = s / sum * scale.
__global__ void route_topk_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ls, int E,
                                  const float* __restrict__ bias, int k, float scaling, int32_t* __restrict__ ids,
                                  float* __restrict__ wts, int T) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  const __nv_bfloat16* lr = logits + (int64_t)warp * ls;
  // each lane keeps its candidates in registers (E <= 512)
  float sc[16], key[16];
  int n = 0;
  for (int e = lane; e < E && n < 16; e += 32, ++n) {
    sc[n] = 1.f / (1.f + expf(-__bfloat162float(lr[e])));
    key[n] = sc[n] + (bias ? bias[e] : 0.f);
  }
  float total = 0.f;
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int bi = -1;
    for (int i = 0; i < n; ++i)
      if (key[i] > best) { best = key[i]; bi = i; }
    int be = bi >= 0 ? lane + 32 * bi : 0x7fffffff;
    // warp argmax (value desc, expert asc)
    float bv = best;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
    }
    float s = 0.f;
    if ((be & 31) == lane && be != 0x7fffffff) {
      const int i = be >> 5;
      s = sc[i];
      key[i] = -INFINITY;
    }
    s = __shfl_sync(0xffffffffu, s, be & 31);
    if (lane == 0) {
      ids[(int64_t)warp * k + j] = be;
      wts[(int64_t)warp * k + j] = s;
    }
    total += s;
  }
  __syncwarp();
  if (lane < k) wts[(int64_t)warp * k + lane] = wts[(int64_t)warp * k + lane] / total * scaling;
}

// ----------------------------------------------------------------------------- SiLU * up
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int64_t gs, int I, __nv_bfloat16* __restrict__ out,
                                int T) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= T * I) return;
  const int t = idx / I, i = idx % I;
  const float g = __bfloat162float(gu[t * gs + i]), u = __bfloat162float(gu[t * gs + I + i]);
  out[(int64_t)t * I + i] = __float2bfloat16_rn(g / (1.f + expf(-g)) * u);
}

}  // namespace

void launch_add_rmsnorm(const __nv_bfloat16* x, int64_t xs, const __nv_bfloat16* d, int64_t ds, const float* dfp32,
                        int64_t dfs, __nv_bfloat16* x_out, int64_t xos, const float* w, float eps, __nv_bfloat16* h,
                        int64_t hs, int rows, int n, cudaStream_t stream) {
  if (rows == 0) return;
  add_rmsnorm_kernel<<<rows, 256, 0, stream>>>(x, xs, d, ds, dfp32, dfs, x_out, xos, w, eps, h, hs, n);
}

void launch_rope_q(__nv_bfloat16* q, int64_t qs, int B, int H, const int64_t* pos, const float* freqs,
                   cudaStream_t stream) {
  const int n = B * H * 32;
  if (n == 0) return;
  rope_q_kernel<<<(n + 255) / 256, 256, 0, stream>>>(q, qs, H, pos, freqs, B);
}

void launch_comp_pool(const __nv_bfloat16* proj, int64_t ps, int off, int D, const float* ape, int ratio, float* state,
                      const int64_t* req, const int64_t* pos, float* raw, int64_t rs, int B, cudaStream_t stream) {
  const int n = B * D;
  if (n == 0) return;
  comp_pool_kernel<<<(n + 255) / 256, 256, 0, stream>>>(proj, ps, off, D, ape, ratio, state, req, pos, raw, rs, B);
}

void launch_route_topk(const __nv_bfloat16* logits, int64_t ls, int T, int E, const float* bias, int k, float scaling,
                       int32_t* ids, float* wts, cudaStream_t stream) {
  if (T == 0) return;
  route_topk_kernel<<<(T + 7) / 8, 256, 0, stream>>>(logits, ls, E, bias, k, scaling, ids, wts, T);
}

void launch_silu_mul(const __nv_bfloat16* gu, int64_t gs, int T, int I, __nv_bfloat16* out, cudaStream_t stream) {
  const int n = T * I;
  if (n == 0) return;
  silu_mul_kernel<<<(n + 255) / 256, 256, 0, stream>>>(gu, gs, I, out, T);
}
