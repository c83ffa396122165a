// MXFP4 routed experts for decode-sized batches (memory-bound on the expert weights).
//
// Reference behaviour: FlashInfer `Mxfp4FlashinferCutlassMoEMethod` (server log
// "Preparing DSv4 MXFP4 experts").  Weights: E2M1 nibbles (low nibble = even k) with one
// UE8M0 scale per 32 consecutive k; activations BF16.
//
//   1. route:   one CTA builds, per local expert, the list of (token, weight) slots routed to it,
//               sorted by token (deterministic), plus the list of active experts.
//   2. gate_up: persistent CTAs over (active expert, block of 64 gate + 64 up rows).  Each warp
//               streams 16 weight rows with 16-byte loads (16 in flight per lane), dequantizes
//               with cvt.rn.f16x2.e2m1x2, multiplies by the expert's tokens (FP16 in swizzled
//               shared memory) with HFMA2 over 32-element blocks, applies the block scale in
//               FP32, and writes act = silu(gate) * up (BF16) per slot.
//   3. down:    same streaming over W2 rows; out[token] += weight * (act . W2 row) (FP32 atomics).
#include "launchers.h"
#include "common/sm100.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kMT = 8;  // tokens per pass

__device__ __forceinline__ int swz(int u) { return (u & ~7) | ((u ^ (u >> 3)) & 7); }

// ----------------------------------------------------------------------------- routing
__global__ void __launch_bounds__(1024) moe_route_kernel(const int32_t* __restrict__ ids,
                                                         const float* __restrict__ w, int n, int k, int base,
                                                         int E, int32_t* __restrict__ offsets,
                                                         int32_t* __restrict__ slot_token,
                                                         float* __restrict__ slot_weight, int32_t* __restrict__ active,
                                                         int32_t* __restrict__ pad, int align,
                                                         int4* __restrict__ chunks, int32_t* __restrict__ n_chunks) {
  extern __shared__ int sh[];
  int* cnt = sh;         // [E]
  int* cur = sh + E;     // [E]
  const int tid = threadIdx.x;
  for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    const int e = ids[i] - base;
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0, na = 0, pacc = 0, nc = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = acc;
      cur[e] = acc;
      if (pad) pad[e] = pacc;  // padded rows: each expert's list starts on a multiple of `align`
      if (cnt[e] > 0) active[1 + na++] = e;
      if (chunks)  // chunk table: {expert, first padded row, tokens (<= 16), first slot}
        for (int c = 0; c < cnt[e]; c += 16) chunks[nc++] = make_int4(e, pacc + c, min(16, cnt[e] - c), acc + c);
      acc += cnt[e];
      pacc += (cnt[e] + align - 1) / align * align;
    }
    offsets[E] = acc;
    if (pad) pad[E] = pacc;
    if (n_chunks) n_chunks[0] = nc;
    active[0] = na;
  }
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    const int e = ids[i] - base;
    if (e >= 0 && e < E) {
      const int p = atomicAdd(&cur[e], 1);
      slot_token[p] = i / k;
      slot_weight[p] = w[i];
    }
  }
  __syncthreads();
  // deterministic order: sort each expert's segment by token (segments are short)
  for (int e = tid; e < E; e += blockDim.x) {
    const int lo = offsets[e], hi = offsets[e + 1];
    for (int a = lo + 1; a < hi; ++a) {
      const int t = slot_token[a];
      const float ww = slot_weight[a];
      int b = a - 1;
      while (b >= lo && slot_token[b] > t) {
        slot_token[b + 1] = slot_token[b];
        slot_weight[b + 1] = slot_weight[b];
        --b;
      }
      slot_token[b + 1] = t;
      slot_weight[b + 1] = ww;
    }
  }
}

// Block-wide exclusive scan of one int4 per thread (blockDim.x == 1024); returns the prefix and
// writes the totals to *total (all threads).
__device__ __forceinline__ int4 block_scan4(int4 v, int4* warp_tot, int4* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int4 inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, inc.x, o), b = __shfl_up_sync(0xffffffffu, inc.y, o);
    const int c = __shfl_up_sync(0xffffffffu, inc.z, o), d = __shfl_up_sync(0xffffffffu, inc.w, o);
    if (lane >= o) { inc.x += a; inc.y += b; inc.z += c; inc.w += d; }
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int4 t = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a = __shfl_up_sync(0xffffffffu, t.x, o), b = __shfl_up_sync(0xffffffffu, t.y, o);
      const int c = __shfl_up_sync(0xffffffffu, t.z, o), d = __shfl_up_sync(0xffffffffu, t.w, o);
      if (lane >= o) { t.x += a; t.y += b; t.z += c; t.w += d; }
    }
    warp_tot[lane] = t;  // inclusive over warps
    if (lane == 31) *total = t;
  }
  __syncthreads();
  const int4 before = warp == 0 ? make_int4(0, 0, 0, 0) : warp_tot[warp - 1];
  return make_int4(before.x + inc.x - v.x, before.y + inc.y - v.y, before.z + inc.z - v.z, before.w + inc.w - v.w);
}

// Routing for up to 4096 slots and 1024 local experts, all in shared memory: the slot order inside an
// expert is the slot index order (token-major), found by counting earlier slots of the same expert,
// so the result is deterministic without a sort.  Writes the same lists as moe_route_kernel.
__global__ void __launch_bounds__(1024) moe_route_smem_kernel(const int32_t* __restrict__ ids,
                                                              const float* __restrict__ w, int n, int k, int base,
                                                              int E, int32_t* __restrict__ offsets,
                                                              int32_t* __restrict__ slot_token,
                                                              float* __restrict__ slot_weight,
                                                              int32_t* __restrict__ active, int32_t* __restrict__ pad,
                                                              int align, int4* __restrict__ chunks,
                                                              int32_t* __restrict__ n_chunks, int max_tok) {
  __shared__ int s_e[4096];
  __shared__ int cnt[1024];
  __shared__ int start[1024];
  __shared__ int4 warp_tot[32];
  __shared__ int4 total;
  const int tid = threadIdx.x;
  if (tid < 1024) cnt[tid] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += 1024) {
    const int e = ids[i] - base;
    const int le = (e >= 0 && e < E) ? e : -1;
    s_e[i] = le;
    if (le >= 0) atomicAdd(&cnt[le], 1);
  }
  __syncthreads();
  const int c = tid < E ? cnt[tid] : 0;
  const int4 pre = block_scan4(make_int4(c, (c + align - 1) / align * align, (c + max_tok - 1) / max_tok, c > 0 ? 1 : 0),
                               warp_tot, &total);
  if (tid < E) {
    offsets[tid] = pre.x;
    start[tid] = pre.x;
    if (pad) pad[tid] = pre.y;
    if (c > 0) active[1 + pre.w] = tid;
    if (chunks)
      for (int q = 0; q < c; q += max_tok)
        chunks[pre.z + q / max_tok] = make_int4(tid, pre.y + q, min(max_tok, c - q), pre.x + q);
  }
  if (tid == 0) {
    offsets[E] = total.x;
    if (pad) pad[E] = total.y;
    if (n_chunks) n_chunks[0] = total.z;
    active[0] = total.w;
  }
  __syncthreads();
  for (int i = tid; i < n; i += 1024) {
    const int e = s_e[i];
    if (e < 0) continue;
    int r = 0;
    for (int j = 0; j < i; ++j) r += (s_e[j] == e);
    const int p = start[e] + r;
    slot_token[p] = i / k;
    slot_weight[p] = w[i];
  }
}

// Routing for any number of slots, deterministic without a sort, in three launches:
//   count (CTA per local expert) -> plan (one CTA: offsets, padded rows, active list, chunk table)
//   -> place (CTA per local expert: an ordered stream compaction of the expert's slots, so each expert's
//   list is in slot order, i.e. sorted by token).  Every CTA reads all slot ids (L2 resident).
__global__ void __launch_bounds__(256) moe_count_kernel(const int32_t* __restrict__ ids, int n, int base,
                                                        int32_t* __restrict__ cnt) {
  __shared__ int wsum[8];
  const int e = blockIdx.x;
  int c = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) c += (ids[i] - base == e);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < 8; ++w) t += wsum[w];
    cnt[e] = t;
  }
}

// `pad` holds the counts on entry and the padded row starts on exit (each thread reads its count before
// the scan's barriers and writes its start after them).
__global__ void __launch_bounds__(1024) moe_plan_kernel(int E, int align, int max_tok, int32_t* __restrict__ offsets,
                                                        int32_t* __restrict__ active, int32_t* __restrict__ pad,
                                                        int4* __restrict__ chunks, int32_t* __restrict__ n_chunks) {
  __shared__ int4 warp_tot[32];
  __shared__ int4 total;
  const int tid = threadIdx.x;
  const int c = tid < E ? pad[tid] : 0;
  const int4 pre = block_scan4(make_int4(c, (c + align - 1) / align * align, (c + max_tok - 1) / max_tok, c > 0 ? 1 : 0),
                               warp_tot, &total);
  if (tid < E) {
    offsets[tid] = pre.x;
    pad[tid] = pre.y;
    if (c > 0) active[1 + pre.w] = tid;
    for (int q = 0; q < c; q += max_tok)
      chunks[pre.z + q / max_tok] = make_int4(tid, pre.y + q, min(max_tok, c - q), pre.x + q);
  }
  if (tid == 0) {
    offsets[E] = total.x;
    pad[E] = total.y;
    n_chunks[0] = total.z;
    active[0] = total.w;
  }
}

__global__ void __launch_bounds__(1024) moe_place_kernel(const int32_t* __restrict__ ids, const float* __restrict__ w,
                                                         int n, int k, int base, const int32_t* __restrict__ offsets,
                                                         int32_t* __restrict__ slot_token,
                                                         float* __restrict__ slot_weight) {
  __shared__ int wcnt[32];
  const int e = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int out = offsets[e];
  for (int i0 = 0; i0 < n; i0 += 1024) {
    const int i = i0 + tid;
    const bool hit = i < n && ids[i] - base == e;
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    if (lane == 0) wcnt[warp] = __popc(m);
    __syncthreads();
    int before = 0, all = 0;
    for (int ww = 0; ww < 32; ++ww) {
      const int v = wcnt[ww];
      before += ww < warp ? v : 0;
      all += v;
    }
    if (hit) {
      const int p = out + before + __popc(m & ((1u << lane) - 1u));
      slot_token[p] = i / k;
      slot_weight[p] = w[i];
    }
    out += all;
    __syncthreads();
  }
}

// 32 E2M1 values (16 bytes) . 32 FP16 activations -> fp32 partial (unscaled)
__device__ __forceinline__ float dot32(const uint4& wq, const uint4 (&x)[4]) {
  const uint32_t ww[4] = {wq.x, wq.y, wq.z, wq.w};
  __half2 acc = __float2half2_rn(0.f);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t xs[4] = {x[q].x, x[q].y, x[q].z, x[q].w};
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const __half2 wv = pm::e2m1x2_to_h2((uint8_t)(ww[q] >> (8 * b)));
      acc = __hfma2(wv, *reinterpret_cast<const __half2*>(&xs[b]), acc);
    }
  }
  const float2 f = __half22float2(acc);
  return f.x + f.y;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Stage up to kMT activation rows (bf16, length K) as swizzled fp16 in shared memory.
template <typename GetRow>
__device__ __forceinline__ void stage_rows(__half* sx, int K, int nt, GetRow get_row) {
  const int units = K / 8;  // 16-byte units per row
  for (int idx = threadIdx.x; idx < nt * units; idx += kThreads) {
    const int t = idx / units, u = idx % units;
    const uint4 v = *reinterpret_cast<const uint4*>(get_row(t) + 8 * u);
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
    __half2 hv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(b[i]);
      hv[i] = __floats2half2_rn(f.x, f.y);
    }
    *reinterpret_cast<uint4*>(sx + (size_t)t * K + 8 * swz(u)) = *reinterpret_cast<uint4*>(hv);
  }
}

// One warp: rows [row0, row0 + NR) of an expert matrix W [rows, K/2] (+ scales [rows, K/32]);
// result res[r][t] (lane 0 valid after reduction) for tokens t < nt.
template <int NR, int CH>
__device__ __forceinline__ void warp_rows(const uint8_t* __restrict__ W, const uint8_t* __restrict__ S, int K,
                                          const int* rows, const __half* sx, int nt, int lane,
                                          float (&res)[NR][kMT]) {
  // CH = 16-byte chunks per lane per row: K/32 chunks per row over 32 lanes
  uint4 raw[NR][CH];
  float sc[NR][CH];
#pragma unroll
  for (int r = 0; r < NR; ++r)
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int q = lane + 32 * c;
      raw[r][c] = __ldg(reinterpret_cast<const uint4*>(W + (size_t)rows[r] * (K / 2) + 16 * q));
      sc[r][c] = pm::exp2i((int)__ldg(S + (size_t)rows[r] * (K / 32) + q) - 127);
    }
#pragma unroll
  for (int r = 0; r < NR; ++r)
#pragma unroll
    for (int t = 0; t < kMT; ++t) res[r][t] = 0.f;
#pragma unroll
  for (int t = 0; t < kMT; ++t) {
    if (t < nt) {
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int q = lane + 32 * c;
        uint4 x[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) x[m] = *reinterpret_cast<const uint4*>(sx + (size_t)t * K + 8 * swz(4 * q + m));
#pragma unroll
        for (int r = 0; r < NR; ++r) res[r][t] += dot32(raw[r][c], x) * sc[r][c];
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kMT; ++t)
    if (t < nt) {
#pragma unroll
      for (int r = 0; r < NR; ++r) res[r][t] = warp_sum(res[r][t]);
    }
}

struct MoeParams {
  const __nv_bfloat16* x;  // [T, H]
  int T, H, I, E;
  const uint8_t* w13;  // [E, 2I, H/2]
  const uint8_t* s13;  // [E, 2I, H/32]
  const uint8_t* w2;   // [E, H, I/2]
  const uint8_t* s2;   // [E, H, I/32]
  const int32_t* offsets;
  const int32_t* slot_token;
  const float* slot_weight;
  const int32_t* active;
  __nv_bfloat16* act;  // [slots, I]
  float* out;          // [T, H]
};

// CH = H / 1024: 16-byte weight chunks per lane per row (32 lanes x 32 values per chunk)
template <int CH>
__global__ void __launch_bounds__(kThreads, 1) moe_gate_up_kernel(const MoeParams p) {
  extern __shared__ uint8_t smem_raw[];
  __half* sx = reinterpret_cast<__half*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = p.I / 64;
  const int items = p.active[0] * nblk;
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int e = p.active[1 + it / nblk];
    const int rb = it % nblk;
    const int lo = p.offsets[e], hi = p.offsets[e + 1];
    const uint8_t* W = p.w13 + (size_t)e * (2 * p.I) * (p.H / 2);
    const uint8_t* S = p.s13 + (size_t)e * (2 * p.I) * (p.H / 32);
    for (int s0 = lo; s0 < hi; s0 += kMT) {
      const int nt = min(kMT, hi - s0);
      __syncthreads();
      stage_rows(sx, p.H, nt, [&](int t) { return p.x + (size_t)p.slot_token[s0 + t] * p.H; });
      __syncthreads();
#pragma unroll 1
      for (int pass = 0; pass < 2; ++pass) {
        int rg[4], ru[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          rg[r] = rb * 64 + warp * 8 + pass * 4 + r;
          ru[r] = p.I + rg[r];
        }
        float g[4][kMT], u[4][kMT];
        warp_rows<4, CH>(W, S, p.H, rg, sx, nt, lane, g);
        warp_rows<4, CH>(W, S, p.H, ru, sx, nt, lane, u);
        if (lane == 0) {
#pragma unroll
          for (int t = 0; t < kMT; ++t)
            if (t < nt)
#pragma unroll
              for (int r = 0; r < 4; ++r) {
                const float gv = g[r][t];
                const float a = gv / (1.f + __expf(-gv)) * u[r][t];
                p.act[(size_t)(s0 + t) * p.I + rg[r]] = __float2bfloat16_rn(a);
              }
        }
      }
    }
  }
}

// CH = I / 1024
template <int CH>
__global__ void __launch_bounds__(kThreads, 1) moe_down_kernel(const MoeParams p) {
  extern __shared__ uint8_t smem_raw[];
  __half* sx = reinterpret_cast<__half*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = p.H / 128;
  const int items = p.active[0] * nblk;
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int e = p.active[1 + it / nblk];
    const int rb = it % nblk;
    const int lo = p.offsets[e], hi = p.offsets[e + 1];
    const uint8_t* W = p.w2 + (size_t)e * p.H * (p.I / 2);
    const uint8_t* S = p.s2 + (size_t)e * p.H * (p.I / 32);
    for (int s0 = lo; s0 < hi; s0 += kMT) {
      const int nt = min(kMT, hi - s0);
      __syncthreads();
      stage_rows(sx, p.I, nt, [&](int t) { return p.act + (size_t)(s0 + t) * p.I; });
      __syncthreads();
#pragma unroll 1
      for (int pass = 0; pass < 2; ++pass) {
        int rows[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) rows[r] = rb * 128 + warp * 16 + pass * 8 + r;
        float y[8][kMT];
        warp_rows<8, CH>(W, S, p.I, rows, sx, nt, lane, y);
        // lanes 0..7 each scatter one row
#pragma unroll
        for (int t = 0; t < kMT; ++t)
          if (t < nt) {
            const int tok = p.slot_token[s0 + t];
            const float wt = p.slot_weight[s0 + t];
#pragma unroll
            for (int r = 0; r < 8; ++r)
              if (lane == r) atomicAdd(p.out + (size_t)tok * p.H + rows[r], wt * y[r][t]);
          }
      }
    }
  }
}

}  // namespace

void launch_moe_route(const int32_t* topk_ids, const float* topk_w, int T, int k, int expert_base, int E,
                      int32_t* offsets, int32_t* slot_token, float* slot_weight, int32_t* active, int32_t* pad,
                      cudaStream_t stream) {
  if (T == 0) return;
  moe_route_kernel<<<1, 1024, 2 * E * sizeof(int), stream>>>(topk_ids, topk_w, T * k, k, expert_base, E, offsets,
                                                           slot_token, slot_weight, active, pad, 16, nullptr, nullptr);
}

void launch_moe_fp4(const __nv_bfloat16* x, int T, int H, int I, int k, const int32_t* topk_ids, const float* topk_w,
                    int expert_base, int E, const uint8_t* w13, const uint8_t* s13, const uint8_t* w2,
                    const uint8_t* s2, int32_t* offsets, int32_t* slot_token, float* slot_weight, int32_t* active,
                    __nv_bfloat16* act, float* out, int num_sms, cudaStream_t stream) {
  if (T == 0) return;
  moe_route_kernel<<<1, 1024, 2 * E * sizeof(int), stream>>>(topk_ids, topk_w, T * k, k, expert_base, E, offsets,
                                                           slot_token, slot_weight, active, nullptr, 16, nullptr,
                                                           nullptr);
  MoeParams p{x, T, H, I, E, w13, s13, w2, s2, offsets, slot_token, slot_weight, active, act, out};
  const int smem_gu = kMT * H * 2, smem_dn = kMT * I * 2;
  auto gate_up = [&](auto kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_gu);
    kern<<<num_sms, kThreads, smem_gu, stream>>>(p);
  };
  auto down = [&](auto kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_dn);
    kern<<<num_sms, kThreads, smem_dn, stream>>>(p);
  };
  switch (H / 1024) {  // the wrapper admits H, I in {1024, 2048, 4096}
    case 1: gate_up(moe_gate_up_kernel<1>); break;
    case 2: gate_up(moe_gate_up_kernel<2>); break;
    default: gate_up(moe_gate_up_kernel<4>); break;
  }
  switch (I / 1024) {
    case 1: down(moe_down_kernel<1>); break;
    case 2: down(moe_down_kernel<2>); break;
    default: down(moe_down_kernel<4>); break;
  }
}

void launch_moe_route_chunks(const int32_t* topk_ids, const float* topk_w, int T, int k, int expert_base, int E,
                             int32_t* offsets, int32_t* slot_token, float* slot_weight, int32_t* active, int32_t* pad,
                             int4* chunks, int32_t* n_chunks, int max_tok, cudaStream_t stream) {
  if (T * k <= 4096 && E <= 1024) {
    moe_route_smem_kernel<<<1, 1024, 0, stream>>>(topk_ids, topk_w, T * k, k, expert_base, E, offsets, slot_token,
                                                  slot_weight, active, pad, 32, chunks, n_chunks, max_tok);
    return;
  }
  if (E <= 1024) {
    moe_count_kernel<<<E, 256, 0, stream>>>(topk_ids, T * k, expert_base, pad);
    moe_plan_kernel<<<1, 1024, 0, stream>>>(E, 32, max_tok, offsets, active, pad, chunks, n_chunks);
    moe_place_kernel<<<E, 1024, 0, stream>>>(topk_ids, topk_w, T * k, k, expert_base, offsets, slot_token,
                                             slot_weight);
    return;
  }
  moe_route_kernel<<<1, 1024, 2 * E * sizeof(int), stream>>>(topk_ids, topk_w, T * k, k, expert_base, E, offsets,
                                                           slot_token, slot_weight, active, pad, 32, chunks, n_chunks);
}
