// Plain C++ launchers of the packmla kernels (no torch types): the .cu files compile without
// torch headers; csrc/torch_ops.cpp validates tensors and calls these.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

void launch_native_store(const float* raw, int64_t raw_stride, const float* weight, float eps, const int64_t* slots,
                         const int64_t* positions, const float* freqs, int64_t freq_rows, uint8_t* pool,
                         int64_t pool_slots, int rows, int* err, cudaStream_t stream);
void launch_packed_store(const float* raw, int64_t raw_stride, const float* weight, float eps, const int64_t* slots,
                         uint8_t* values, uint64_t* bitmap, uint8_t* scales, int64_t pool_rows, int keep, int rows,
                         int* err, cudaStream_t stream);
// GLM-5.3 MLA rows: Native = 512 raw E4M3 codes per row ([rows, 512]); Packed = the 256 largest-|raw|
// coordinates' codes ([rows, 256]) + an LSB-first 512-bit bitmap ([rows, 8] words).
void launch_glm_store(const float* raw, int64_t raw_stride, const float* weight, float eps, const int64_t* slots,
                      bool packed, uint8_t* pool, uint8_t* values, uint64_t* bitmap, int64_t pool_rows, int rows,
                      int* err, cudaStream_t stream);
void launch_glm_packed_to_native(const uint8_t* values, const uint64_t* bitmap, int64_t pool_rows,
                                 const int64_t* rows_in, uint8_t* out, int rows, int* err, cudaStream_t stream);

// Sparse MLA decode (csrc/attention_decode.cu).  A query's rows [SWA ; C4] are split into 64-row
// stages; split s of num_splits takes an even share of whole stages.
struct DecodeParams {
  const __nv_bfloat16* q;  // [B, H, 512]
  int64_t q_stride_b, q_stride_h;
  int B, H, num_groups, num_splits;
  // SWA (Native) rows
  const uint8_t* swa_pool;
  int64_t swa_pool_slots;
  const int32_t* swa_slots;  // [B, swa_cap]
  int swa_cap;
  const int32_t* swa_len;    // [B]
  // CSA rows
  int csa_packed;
  int csa_fp4;               // 0 = FP8 records; 1 = FP4 Native pages (288 B records), 2 = FP4 Packed (224 B)
  int csa_glm;               // 0, or GLM-5.3 rows: 1 = Native (csa_pool [rows, 512] E4M3), 2 = Packed (values, bitmap)
  int no_rope;               // 1: no RoPE tail (the output is not inverse-rotated; freqs and q_pos are not read)
  const uint8_t* csa_pool;   // native pages (csa_packed == 0; FP8 or, with csa_fp4, FP4)
  const uint8_t* csa_values; // packed planes
  const uint64_t* csa_bitmap;
  const uint8_t* csa_scales;
  int64_t csa_pool_rows;
  const int32_t* csa_slots;  // [B, csa_cap]
  const int32_t* csa_pos;    // [B, csa_cap] token position of the record (RoPE row)
  int csa_cap;
  const int32_t* csa_len;    // [B]
  const float* freqs;        // [P, 32, 2]
  int64_t freq_rows;
  float scale_log2;          // softmax scale * log2(e)
  float* part_o;             // [B, splits, H, 512] (num_splits > 1)
  float* part_ml;            // [B, splits, H, 2]   (decode_uses_partials(num_splits))
  int* err;
  // set by launch_sparse_mla_decode from its arguments
  const float* sink;         // [H]
  const int32_t* q_pos;      // [B]
  __nv_bfloat16* out;        // [B, H, 512]
  float* lse;                // [B, H]
  // optional: global-timer stamps of CTA 0 (ns, 40 entries; see attention_decode.cu), null otherwise
  unsigned long long* prof;
};

void launch_sparse_mla_decode(const DecodeParams& p, const float* sink, const int32_t* q_pos,
                              __nv_bfloat16* out, float* lse, cudaStream_t stream);

// Split-KV counts whose CTAs form one thread-block cluster and merge their partials in distributed shared
// memory (no partial buffers, no combine launch); other counts above one write fp32 partials (part_o,
// part_ml) that the combine kernel merges.
#ifdef __CUDACC__
__host__ __device__
#endif
inline bool decode_splits_clustered(int splits) { return splits == 2 || splits == 4 || splits == 8; }
inline bool decode_uses_partials(int splits) { return splits > 1 && !decode_splits_clustered(splits); }
// How many clusters of `cluster` decode CTAs can be resident at once on the current device (0 if the
// size cannot be launched).
int decode_max_active_clusters(int cluster);

void launch_umma_probe(const void* a, const void* b, int K, int N, int mode, float* d, int* err, cudaStream_t stream);

void launch_moe_fp4(const __nv_bfloat16* x, int T, int H, int I, int k, const int32_t* topk_ids, const float* topk_w,
                    int expert_base, int E, const uint8_t* w13, const uint8_t* s13, const uint8_t* w2,
                    const uint8_t* s2, int32_t* offsets, int32_t* slot_token, float* slot_weight, int32_t* active,
                    __nv_bfloat16* act, float* out, int num_sms, cudaStream_t stream);

void launch_moe_route(const int32_t* topk_ids, const float* topk_w, int T, int k, int expert_base, int E,
                      int32_t* offsets, int32_t* slot_token, float* slot_weight, int32_t* active, int32_t* pad,
                      cudaStream_t stream);
void launch_index_key_store(const float* kraw, int64_t stride, const int64_t* slots, uint8_t* keys, float* kscales,
                            int64_t nrows, int R, int* err, cudaStream_t stream);
void launch_index_logits(const __nv_bfloat16* q, const float* w, int B, int H, const uint8_t* keys,
                         const float* kscales, int64_t nrows, const int32_t* phys, int64_t phys_stride,
                         const int64_t* count, int R, float* scores, int64_t score_stride, int num_sms, int* err,
                         cudaStream_t stream);
void launch_index_topk(const float* scores, int64_t stride, int B, int R, int k, const int32_t* phys,
                       int64_t phys_stride, int ratio, int32_t* out_slots, int32_t* out_pos, cudaStream_t stream);

void launch_moe_gather_slots(const __nv_bfloat16* x, int K, const int32_t* offsets, const int32_t* pad,
                             const int32_t* slot_token, int E, __half* xs, int num_sms, cudaStream_t stream);
void launch_moe_fp4_mma(const __nv_bfloat16* x, int T, int H, int I, int E, const int32_t* offsets, const int32_t* pad,
                        const int32_t* slot_token, const float* slot_weight, const int32_t* active, const uint8_t* w13f,
                        const uint8_t* s13f, const uint8_t* w2f, const uint8_t* s2f, __half* xs, __half* act_s,
                        float* out, int num_sms, int* err, cudaStream_t stream);

void launch_add_rmsnorm(const __nv_bfloat16* x, int64_t xs, const __nv_bfloat16* d, int64_t ds, const float* dfp32,
                        int64_t dfs, __nv_bfloat16* x_out, int64_t xos, const float* w, float eps, __nv_bfloat16* h,
                        int64_t hs, int rows, int n, cudaStream_t stream);
void launch_rope_q(__nv_bfloat16* q, int64_t qs, int B, int H, const int64_t* pos, const float* freqs,
                   cudaStream_t stream);
void launch_comp_pool(const __nv_bfloat16* proj, int64_t ps, int off, int D, const float* ape, int ratio, float* state,
                      const int64_t* req, const int64_t* pos, float* raw, int64_t rs, int B, cudaStream_t stream);
void launch_route_topk(const __nv_bfloat16* logits, int64_t ls, int T, int E, const float* bias, int k, float scaling,
                       int32_t* ids, float* wts, cudaStream_t stream);
void launch_silu_mul(const __nv_bfloat16* gu, int64_t gs, int T, int I, __nv_bfloat16* out, cudaStream_t stream);
void launch_bs_probe(const uint8_t* a_img, const uint8_t* b_img, const uint32_t* sfa, const uint32_t* sfb,
                     uint32_t idesc, int kind, int N, uint32_t sfa_extra, uint32_t sfb_extra, float* d, int* err,
                     cudaStream_t stream);
int make_tmap_fp4_unpacked(void* out, const void* base, uint64_t k_elems, uint64_t rows, uint64_t row_bytes,
                           uint32_t box_rows);
int make_tmap_fp4_unpacked_nd(void* out, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                              const uint32_t* box);
int launch_bs_probe2(const uint8_t* a_packed, const uint8_t* b_img, const uint8_t* sfa_src, const uint8_t* sfb_src,
                     int N, int k_steps, uint32_t expect_tx, float* d, uint8_t* a_dump, int* err,
                     cudaStream_t stream);

void launch_moe_route_chunks(const int32_t* topk_ids, const float* topk_w, int T, int k, int expert_base, int E,
                             int32_t* offsets, int32_t* slot_token, float* slot_weight, int32_t* active, int32_t* pad,
                             int4* chunks, int32_t* n_chunks, int max_tok, cudaStream_t stream);

// MXFP4 experts x MXFP8 activations (csrc/moe_mxf4.cu).  Workspace images: xq [H/128, rows, 128],
// xs [rows, H/32], act_q [I/128, rows, 128], act_s [rows, I/32] (rows % 32 == 0).
struct MoeMxArgs {
  const __nv_bfloat16* h;
  int T, H, I, k, E, expert_base, rows_total, num_sms;
  const int32_t* topk_ids;
  const float* topk_w;
  const uint8_t* w13;    // [E, 2I, H/2] packed E2M1
  const uint8_t* sfw13;  // [E*I/128, H/128, 256 (gate 128 | up 128 rows), 4] UE8M0 weight-scale image
  const uint8_t* w2;     // [E, H, I/2]
  const uint8_t* sfw2;   // [E*H/256, I/128, 256, 4]
  int32_t* offsets;
  int32_t* slot_token;
  float* slot_weight;
  int32_t* active;
  int32_t* pad;
  int4* chunks;
  int32_t* n_chunks;
  uint8_t* xq;
  uint8_t* xs;
  uint8_t* act_q;
  uint8_t* act_s;
  float* out;  // [T, H] fp32 (zeroed by the kernel)
  int* err;
  // optional per-launch counters (SM cycles summed over CTAs): [0] producer waiting for a free stage,
  // [1] MMA issuer waiting for data, [2] MMA issuer waiting for a free accumulator, [3] epilogue
  // waiting for an accumulator, [4] producer lifetime, [5] MMA issuer waiting for weight scales,
  // [6] MMA issuer issuing (fence + MMAs + commit); gate/up at [0..7], down at [8..15]
  unsigned long long* prof;
};
int launch_moe_mxf4(const MoeMxArgs& a, cudaStream_t stream);

// ----------------------------------------------------------------------------- fused collectives
// Symmetric buffer of one TP group: every rank allocated the same layout and mapped every peer's copy.
struct SymmComm {
  const unsigned long long* peers;  // [world] device array: base address of each rank's buffer (own included)
  int rank, world;
  int64_t recv_off;     // bytes: bf16 [2][max_src][recv_elems] partial sums (call parity, source)
  int64_t recv_elems;
  int64_t gath_off;     // bytes: bf16 [recv_elems] reduced values (all-gather target)
  int64_t flag_rs_off;  // bytes: u32 [max_src][max_tiles]
  int64_t flag_ag_off;  // bytes: u32 [max_tiles]
  int max_src, max_tiles;
  int64_t lpart_off;    // bytes: fp32 [max_splits][recv_elems] split-K partials (read by this GPU only)
  unsigned int* epoch;  // local u32[2]: [0] completed calls, [1] CTA arrival counter
  int* err;
  int64_t timeout_ns;   // limit of every wait on a peer
};

struct GemmArParams {
  SymmComm c;
  int B, N, K, S, stages, nmb;  // K: local reduction width; S: K splits per tile; nmb: 128-token blocks
  int one_shot;                 // 1: every rank reduces (one hop); 0: reduce-scatter + all-gather
  __nv_bfloat16* out;           // [B, N]
  unsigned long long* prof;     // optional phase counters (ns): see comm_fused.cu
};

struct ArParams {
  SymmComm c;
  const __nv_bfloat16* a;  // optional bf16 addend [n]
  const float* f;          // optional fp32 addend [n]
  int64_t n, chunk;        // elements; elements per CTA (tile)
  int one_shot;
  __nv_bfloat16* out;      // [n]
};

int make_tmap_bf16_sw128(void* out, const void* base, uint64_t k_elems, uint64_t rows, uint64_t row_bytes,
                         uint32_t box_rows);
int make_tmap_u8_sw128(void* out, const void* base, uint64_t k_elems, uint64_t rows, uint64_t row_bytes,
                       uint32_t box_rows);

// Dense projections with MXFP8 weights (csrc/dense_mx.cu): y[b] = x[b] W[b]^T for `batch` independent
// (x, W) pairs, x [T, K] BF16 quantized per token to MXFP8 (E4M3 + UE8M0 per 32), W [N, K] E4M3 codes with
// their UE8M0 scales pre-arranged per (256-row tile, 128-K group).  With K splits every split stores its fp32
// partial and the split that finishes a tile last sums them in split order (deterministic) into BF16 y.
struct DenseMxArgs {
  const __nv_bfloat16* x;   // [batch][T][K] (x_stride_b elements between batches, rows of K contiguous)
  int64_t x_stride_b;
  int64_t x_stride_t;
  int T, K, N, batch;
  const uint8_t* w;         // [batch][N][K] E4M3 codes
  const uint8_t* w_sf;      // [batch][N/256 tiles][K/128][256][4] UE8M0 (tile rows past N: any value)
  __nv_bfloat16* y;         // [batch][T][N] (y_stride_t elements between rows)
  int64_t y_stride_t;
  int64_t y_stride_b;
  uint8_t* a_img;           // workspace [batch][K/128][Tp][128] (Tp = T rounded up to 8); unused when the
  uint32_t* a_sf;           //   GEMM quantizes x itself (dense_mx_fused_quant); [batch][K/128][Tp]
  float* part;              // workspace [batch][splits][Tp][N_pad] fp32 (only with splits > 1)
  int32_t* counters;        // workspace [batch][N/256 tiles], zero (left zero)
  int splits;               // K splits per tile (1 = direct BF16 output)
  int num_sms;
  int* err;
};
int launch_dense_mx(const DenseMxArgs& a, cudaStream_t stream);

// FP4 C4 records (csrc/kv_store_fp4.cu): rows -> normalized, tail-rotated, BF16-rounded, E2M1 with an E4M3
// scale per 16; Native 288 B (packed = false) or Packed 224 B (the 256 largest magnitudes) in pages of 64
// records (data rows, then scale rows).
void launch_fp4_store(const float* raw, int64_t raw_stride, const float* weight, float eps, const int64_t* slots,
                      const int64_t* positions, const float* freqs, int64_t freq_rows, uint8_t* pool,
                      int64_t pool_slots, bool packed, int rows, int* err, cudaStream_t stream);
// Whether the GEMM quantizes the activations itself for these sizes (one launch; x read in place).
bool dense_mx_fused_quant(int T, int K, int splits);
int gemm_ar_smem_bytes(int stages);
int launch_gemm_allreduce(const GemmArParams& p, const void* w, const void* x, int num_sms, cudaStream_t stream);
int launch_allreduce(const ArParams& p, int num_sms, cudaStream_t stream);

// HiCache: copy segments (src, dst, bytes) x nseg between device and mapped host memory.
int launch_segment_copy(const int64_t* segs_dev, int nseg, int num_sms, cudaStream_t stream);

// Adapter: Packed planes rows -> Native records at dst slots of a paged workspace.
void launch_packed_to_native(const uint8_t* values, const uint64_t* bitmap, const uint8_t* scales, int64_t src_rows,
                             const int32_t* rows, const int32_t* positions, const float* freqs, int64_t freq_rows,
                             uint8_t* out, const int64_t* dst, int64_t out_slots, int keep, int n, int* err,
                             cudaStream_t stream);
