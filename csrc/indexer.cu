// Sparse-attention indexer on tcgen05: FP8 index keys, per-query top-k C4 records.
//
// Reference behaviour: the DSV4 indexer selects the top-512 C4 records per query
// (`srt/layers/attention/dsv4/indexer.py`, server `dsa_topk_backend "sgl-kernel"`, FP8 indexer by
// default: `enable_deepseek_v4_fp4_indexer false`).  Score of record r for query b:
//     score(b, r) = sum_h w[b, h] * relu(q[b, h] . k[r])
// Key storage (one row per C4 record, same physical id as the C4 KV record): 128 E4M3 codes
// whose 16-byte units are XOR-swizzled by (row % 8) -- so a page of 64 rows copied linearly
// lands in shared memory already in the 128-byte-swizzled K-major UMMA layout -- plus one fp32
// scale per row (amax / 448).
//
//   index_key_store:  warp per row: amax, scale, E4M3 codes, swizzled write (slot -1: no write).
//   index_logits:     CTA = (up to 4 queries, chunk of 128-record tiles).  The queries' heads are
//                     quantized to E4M3 per head (scale folded into w, since relu is positively
//                     homogeneous) into the B operand; each tile's two key pages arrive by
//                     cp.async.bulk (two stages); one tcgen05.mma kind::f8f6f4 chain
//                     S^T[128 records x 64 heads per query] (K = 128); the epilogue thread of record r
//                     reduces its TMEM row to one score per query.  Several queries share a CTA only
//                     when they share one physical-row list (a prefill chunk's queries of one request,
//                     passed with row stride 0): each key tile then serves all of them.
//   index_topk:       CTA per query: 4-pass 8-bit radix select of the k-th largest score, then a
//                     deterministic (index-ordered) compaction; writes physical slots and RoPE rows.
#include "launchers.h"
#include "common/sm100.cuh"

namespace {

constexpr int kD = 128;       // index dim
constexpr int kHmax = 64;     // heads (MMA N)
constexpr int kRows = 128;    // records per tile
constexpr int kPageRows = 64;
constexpr float kE4M3Max = 448.f;

// ----------------------------------------------------------------------------- key store
__global__ void index_key_store_kernel(const float* __restrict__ kraw, int64_t stride, const int64_t* __restrict__ slots,
                                       uint8_t* __restrict__ keys, float* __restrict__ kscales, int64_t nrows, int R,
                                       int* err) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= R) return;
  const int64_t slot = slots[warp];
  if (slot < 0) return;
  if (slot >= nrows) { if (lane == 0) pm::report_error(err, pm::kIndexOutOfRange, warp); return; }
  const float4 v = *reinterpret_cast<const float4*>(kraw + (int64_t)warp * stride + 4 * lane);
  float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = amax > 0.f ? amax / kE4M3Max : 1.f;
  const float inv = 1.f / scale;
  const uint16_t lo = pm::f32x2_to_e4m3x2(v.x * inv, v.y * inv);
  const uint16_t hi = pm::f32x2_to_e4m3x2(v.z * inv, v.w * inv);
  const int unit = (lane >> 2) ^ (int)(slot & 7);
  *reinterpret_cast<uint32_t*>(keys + slot * kD + 16 * unit + 4 * (lane & 3)) = (uint32_t)lo | ((uint32_t)hi << 16);
  if (lane == 0) kscales[slot] = scale;
}

// ----------------------------------------------------------------------------- logits
struct LogitParams {
  const __nv_bfloat16* q;  // [B, H, 128]
  const float* w;          // [B, H]
  int B, H;
  const uint8_t* keys;     // [nrows, 128] swizzled E4M3
  const float* kscales;    // [nrows]
  int64_t nrows;
  const int32_t* phys;     // [B, phys_stride] physical row of logical record r (or -1)
  int64_t phys_stride;
  const int64_t* count;    // [B] visible records
  int R;                   // records scored (multiple of 128 not required)
  int tiles_per_cta;
  int nq;                  // queries per CTA (1, 2 or 4; above 1 only with phys_stride == 0)
  float* scores;           // [B, score_stride]
  int64_t score_stride;
  int* err;
};

constexpr int kLogitThreads = 128;
constexpr int kKeyStage = kRows * kD + kRows * 4;  // 16 KB keys + 512 B scales
constexpr int kOffQ = 2 * kKeyStage;               // 2 stages (each 1024-aligned: 16896 = 16.5 KB -> pad)
constexpr int kStageStride = 17408;                // 17 KB, multiple of 1024
constexpr int kQmax = 4;                           // queries per CTA sharing one physical-row list
constexpr int kOffQ2 = 2 * kStageStride;
constexpr int kOffW = kOffQ2 + kQmax * kHmax * kD;  // B operand: 64 rows per query
constexpr int kOffBar = kOffW + kQmax * kHmax * 4;
constexpr int kLogitSmem = kOffBar + 64 + 1024;

__global__ void __launch_bounds__(kLogitThreads) index_logits_kernel(const LogitParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (pm::smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem + kOffQ2;
  float* sW = reinterpret_cast<float*>(smem + kOffW);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);  // [2]
  uint64_t* mdone = full + 2;                                    // [1]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mdone + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b0 = blockIdx.y * p.nq;
  const int nqb = min(p.nq, p.B - b0);  // this CTA's queries
  const int ncols = kHmax * p.nq;        // MMA N and TMEM columns (64, 128 or 256)
  const int tile0 = blockIdx.x * p.tiles_per_cta;
  const int ntile_total = (p.R + kRows - 1) / kRows;
  const int tile1 = min(ntile_total, tile0 + p.tiles_per_cta);
  if (tile0 >= tile1) return;
  int64_t cnt = 0;  // records to load: the largest visible count of the CTA's queries
  for (int qi = 0; qi < nqb; ++qi) cnt = max(cnt, min((int64_t)p.R, p.count[b0 + qi]));

  if (warp == 0) {
    pm::tmem_alloc(tslot, ncols);
    pm::tmem_relinquish();
  }
  if (tid == 0) {
    pm::mbar_init(&full[0], 1);
    pm::mbar_init(&full[1], 1);
    pm::mbar_init(mdone, 1);
    pm::fence_mbar_init();
  }
  // query heads -> E4M3 (per-head scale folded into w), B operand row 64 qi + h (swizzled by row % 8)
  for (int row = tid; row < ncols; row += kLogitThreads) {
    const int qi = row / kHmax, h = row % kHmax;
    const bool valid = qi < nqb && h < p.H;
    float vals[kD];
    float amax = 0.f;
    if (valid) {
      const __nv_bfloat16* qr = p.q + ((int64_t)(b0 + qi) * p.H + h) * kD;
#pragma unroll
      for (int i = 0; i < kD; i += 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(qr + i);
        const __nv_bfloat162* bb = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(bb[j]);
          vals[i + 2 * j] = f.x;
          vals[i + 2 * j + 1] = f.y;
          amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < kD; ++i) vals[i] = 0.f;
    }
    const float qs = amax > 0.f ? amax / kE4M3Max : 1.f;
    const float inv = 1.f / qs;
#pragma unroll
    for (int u = 0; u < kD / 16; ++u) {
      uint32_t wds[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = 16 * u + 4 * j;
        wds[j] = (uint32_t)pm::f32x2_to_e4m3x2(vals[i] * inv, vals[i + 1] * inv) |
                 ((uint32_t)pm::f32x2_to_e4m3x2(vals[i + 2] * inv, vals[i + 3] * inv) << 16);
      }
      *reinterpret_cast<uint4*>(sQ + pm::sw128_offset(row, 16 * u, 0)) = make_uint4(wds[0], wds[1], wds[2], wds[3]);
    }
    sW[row] = valid ? p.w[(int64_t)(b0 + qi) * p.H + h] * qs : 0.f;
  }
  pm::fence_proxy_async_smem();
  pm::tc_fence_before();
  __syncthreads();
  pm::tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t idesc = pm::make_idesc_f8(128, ncols, 0, 0);
  const int32_t* phys_b = p.phys + (int64_t)b0 * p.phys_stride;  // shared by the CTA's queries

  // issue the copies of tile `j` (two pages) into stage `st`; returns false if the tile is masked
  auto issue = [&](int j, int st) {
    uint8_t* dst = smem + st * kStageStride;
    const int r0 = j * kRows;
    uint32_t bytes = 0;
    int64_t pg[2] = {-1, -1};
    for (int h = 0; h < 2; ++h) {
      const int rr = r0 + h * kPageRows;
      if (rr < cnt) {
        const int ph = phys_b[rr];
        if (ph >= 0 && ph % kPageRows == 0 && ph + kPageRows <= p.nrows) pg[h] = ph;
        else if (ph >= 0) pm::report_error(p.err, pm::kBadArgument, rr);
      }
      if (pg[h] >= 0) bytes += kPageRows * (kD + 4);
    }
    pm::mbar_arrive_expect_tx(&full[st], bytes);
    for (int h = 0; h < 2; ++h)
      if (pg[h] >= 0) {
        pm::bulk_g2s(dst + h * kPageRows * kD, p.keys + pg[h] * kD, kPageRows * kD, &full[st]);
        pm::bulk_g2s(dst + kRows * kD + h * kPageRows * 4, p.kscales + pg[h], kPageRows * 4, &full[st]);
      }
  };

  if (tid == 0) issue(tile0, 0);
  for (int j = tile0; j < tile1; ++j) {
    const int it = j - tile0, st = it & 1;
    if (tid == 0 && j + 1 < tile1) issue(j + 1, st ^ 1);  // stage st^1 was released by the previous epilogue
    bool ok = pm::mbar_wait(&full[st], (it >> 1) & 1, p.err, 40);
    if (tid == 0 && ok) {
      pm::tc_fence_after();
      const uint32_t a0 = pm::smem_u32(smem + st * kStageStride), b0 = pm::smem_u32(sQ);
#pragma unroll
      for (int k = 0; k < kD / 32; ++k)
        pm::umma_f8(tmem, pm::make_sdesc(a0 + 32 * k, 16, 1024), pm::make_sdesc(b0 + 32 * k, 16, 1024), idesc, k > 0);
      pm::umma_commit(mdone);
    }
    ok = ok && pm::mbar_wait(mdone, it & 1, p.err, 41);
    pm::tc_fence_after();
    // epilogue: thread = record row, one score per query of the CTA
    const int r = j * kRows + tid;
    const int ph = r < cnt ? phys_b[r] : -1;
    const float ks = *reinterpret_cast<const float*>(smem + st * kStageStride + kRows * kD + tid * 4);
#pragma unroll 1
    for (int qi = 0; qi < nqb; ++qi) {
      float acc = 0.f;
      if (ok) {
#pragma unroll
        for (int c = 0; c < 64; c += 16) {
          float t[16];
          pm::tmem_ld16(tmem + qi * kHmax + c + ((uint32_t)(32 * warp) << 16), t);
#pragma unroll
          for (int i = 0; i < 16; ++i) acc += sW[qi * kHmax + c + i] * fmaxf(t[i], 0.f);
        }
      }
      if (r < p.R) {
        const int64_t cq = min((int64_t)p.R, p.count[b0 + qi]);
        p.scores[(int64_t)(b0 + qi) * p.score_stride + r] = (ok && ph >= 0 && r < cq) ? acc * ks : -INFINITY;
      }
    }
    pm::tc_fence_before();
    __syncthreads();  // TMEM row read and stage st consumed before it is refilled / overwritten
  }
  if (warp == 0) pm::tmem_dealloc(tmem, ncols);
}

// ----------------------------------------------------------------------------- top-k
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kTopkThreads = 1024;

__global__ void __launch_bounds__(kTopkThreads) index_topk_kernel(const float* __restrict__ scores, int64_t stride,
                                                                  int R, int k, const int32_t* __restrict__ phys,
                                                                  int64_t phys_stride, int ratio,
                                                                  int32_t* __restrict__ out_slots,
                                                                  int32_t* __restrict__ out_pos) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel_digit, sel_need;
  __shared__ int warp_cnt[32];
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* sc = scores + (int64_t)b * stride;
  uint32_t prefix = 0, pmask = 0;
  uint32_t need = (uint32_t)min(k, R);
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < R; i += kTopkThreads) {
      const uint32_t key = order_key(sc[i]);
      if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (warp == 0) {
      // suffix scan over 256 bins (lane owns bins 8 lane .. 8 lane + 7, scanned from the top)
      uint32_t c[8], tot = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) { c[i] = hist[8 * lane + i]; tot += c[i]; }
      // exclusive suffix sum over lanes: candidates in bins owned by higher lanes
      uint32_t incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_down_sync(0xffffffffu, incl, o);
        if (lane + o < 32) incl += v;
      }
      const uint32_t above = incl - tot;
      // find the bin where the running count from the top reaches `need`
      uint32_t run = above;
      int found = -1;
      uint32_t need_in = 0;
#pragma unroll
      for (int i = 7; i >= 0; --i) {
        if (found < 0 && run + c[i] >= need && run < need) { found = 8 * lane + i; need_in = need - run; }
        run += c[i];
      }
      const unsigned m = __ballot_sync(0xffffffffu, found >= 0);
      if (m) {
        const int src = 31 - __clz(m);  // at most one lane matches; take it
        const int fd = __shfl_sync(0xffffffffu, found, src);
        const uint32_t nn = __shfl_sync(0xffffffffu, need_in, src);
        if (lane == 0) { sel_digit = (uint32_t)fd; sel_need = nn; }
      } else if (lane == 0) {
        sel_digit = 0; sel_need = 0;  // fewer candidates than need: everything below is taken
      }
    }
    __syncthreads();
    prefix |= sel_digit << shift;
    pmask |= 255u << shift;
    need = sel_need;
    __syncthreads();
  }
  // threshold key = prefix; take all keys > prefix and the first `need` keys == prefix (by index)
  const int chunk = (R + kTopkThreads - 1) / kTopkThreads;
  const int i0 = tid * chunk, i1 = min(R, i0 + chunk);
  int n_gt = 0, n_eq = 0;
  for (int i = i0; i < i1; ++i) {
    const uint32_t key = order_key(sc[i]);
    n_gt += key > prefix;
    n_eq += key == prefix;
  }
  // block exclusive scans of n_eq (to cap ties) and of the selected counts
  auto block_excl = [&](int v) {
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) warp_cnt[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = warp_cnt[lane], wi = w;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o) wi += t;
      }
      warp_cnt[lane] = wi - w;
    }
    __syncthreads();
    const int r = warp_cnt[warp] + incl - v;
    __syncthreads();
    return r;
  };
  const int eq_before = block_excl(n_eq);
  const int take_eq = max(0, min(n_eq, (int)need - eq_before));
  const int mine = n_gt + take_eq;
  int pos = block_excl(mine);
  int eq_seen = 0;
  for (int i = i0; i < i1; ++i) {
    const float s = sc[i];
    const uint32_t key = order_key(s);
    bool take = key > prefix;
    if (key == prefix) { take = eq_seen < take_eq; ++eq_seen; }
    if (take && pos < k) {
      const bool valid = s != -INFINITY;
      out_slots[(int64_t)b * k + pos] = valid ? phys[(int64_t)b * phys_stride + i] : -1;
      out_pos[(int64_t)b * k + pos] = i * ratio;
      ++pos;
    }
  }
  // total selected = min(k, R); fill the remainder (R < k) with masked entries
  for (int j = min(k, R) + tid; j < k; j += kTopkThreads) {
    out_slots[(int64_t)b * k + j] = -1;
    out_pos[(int64_t)b * k + j] = 0;
  }
}

}  // namespace

void launch_index_key_store(const float* kraw, int64_t stride, const int64_t* slots, uint8_t* keys, float* kscales,
                            int64_t nrows, int R, int* err, cudaStream_t stream) {
  if (R == 0) return;
  index_key_store_kernel<<<(R + 7) / 8, 256, 0, stream>>>(kraw, stride, slots, keys, kscales, nrows, R, err);
}

void launch_index_logits(const __nv_bfloat16* q, const float* w, int B, int H, const uint8_t* keys,
                         const float* kscales, int64_t nrows, const int32_t* phys, int64_t phys_stride,
                         const int64_t* count, int R, float* scores, int64_t score_stride, int num_sms, int* err,
                         cudaStream_t stream) {
  if (B == 0 || R == 0) return;
  // queries that share one physical-row list (row stride 0) share CTAs: each key tile serves up to 4
  const int nq = phys_stride == 0 ? (B >= 4 ? 4 : (B >= 2 ? 2 : 1)) : 1;
  const int qblocks = (B + nq - 1) / nq;
  const int ntiles = (R + kRows - 1) / kRows;
  const int want_ctas = 2 * num_sms;
  const int chunks = max(1, min(ntiles, (want_ctas + qblocks - 1) / qblocks));
  const int per = (ntiles + chunks - 1) / chunks;
  LogitParams p{q, w, B, H, keys, kscales, nrows, phys, phys_stride, count, R, per, nq, scores, score_stride, err};
  cudaFuncSetAttribute(index_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kLogitSmem);
  index_logits_kernel<<<dim3((ntiles + per - 1) / per, qblocks), kLogitThreads, kLogitSmem, stream>>>(p);
}

void launch_index_topk(const float* scores, int64_t stride, int B, int R, int k, const int32_t* phys,
                       int64_t phys_stride, int ratio, int32_t* out_slots, int32_t* out_pos, cudaStream_t stream) {
  if (B == 0) return;
  index_topk_kernel<<<B, kTopkThreads, 0, stream>>>(scores, stride, R, k, phys, phys_stride, ratio, out_slots, out_pos);
}
