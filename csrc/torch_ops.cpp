// Torch-facing wrappers: argument validation, then the plain launchers of csrc/*.cu.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include "launchers.h"

namespace {
constexpr int kD = 512;
constexpr int kPage = 64;
constexpr int kNativePageBytes = kPage * 584;

void check_rows(const torch::Tensor& raw) {
  TORCH_CHECK(raw.is_cuda() && raw.scalar_type() == torch::kFloat32, "raw must be CUDA float32");
  TORCH_CHECK(raw.dim() == 2 && raw.size(1) == kD && raw.stride(1) == 1, "raw must be [R, 512] row-contiguous");
  TORCH_CHECK(raw.stride(0) % 4 == 0 && (reinterpret_cast<uintptr_t>(raw.data_ptr()) % 16) == 0,
              "raw rows must be 16-byte aligned");
}
void check_err(const torch::Tensor& err) {
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == torch::kInt32 && err.numel() >= 4, "err must be CUDA int32[4]");
}
cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }
}  // namespace

void native_store(torch::Tensor raw, torch::Tensor weight, double eps, torch::Tensor slots, torch::Tensor positions,
                  torch::Tensor freqs, torch::Tensor pool, torch::Tensor err) {
  check_rows(raw);
  check_err(err);
  TORCH_CHECK(weight.is_cuda() && weight.scalar_type() == torch::kFloat32 && weight.numel() == kD && weight.is_contiguous());
  TORCH_CHECK(slots.scalar_type() == torch::kInt64 && positions.scalar_type() == torch::kInt64);
  TORCH_CHECK(slots.numel() == raw.size(0) && positions.numel() == raw.size(0));
  TORCH_CHECK(slots.is_contiguous() && positions.is_contiguous());
  TORCH_CHECK(freqs.scalar_type() == torch::kFloat32 && freqs.dim() == 3 && freqs.size(1) == 32 && freqs.size(2) == 2 &&
              freqs.is_contiguous(), "freqs must be float32 [P, 32, 2]");
  TORCH_CHECK(pool.scalar_type() == torch::kUInt8 && pool.is_contiguous() && pool.numel() % kNativePageBytes == 0,
              "pool must be uint8 pages of 64 native records");
  const c10::cuda::CUDAGuard g(raw.device());
  launch_native_store(raw.data_ptr<float>(), raw.stride(0), weight.data_ptr<float>(), (float)eps,
                      slots.data_ptr<int64_t>(), positions.data_ptr<int64_t>(), freqs.data_ptr<float>(), freqs.size(0),
                      pool.data_ptr<uint8_t>(), pool.numel() / kNativePageBytes * kPage, raw.size(0),
                      err.data_ptr<int>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void packed_store(torch::Tensor raw, torch::Tensor weight, double eps, torch::Tensor slots, torch::Tensor values,
                  torch::Tensor bitmap, torch::Tensor scales, torch::Tensor err) {
  check_rows(raw);
  check_err(err);
  TORCH_CHECK(weight.is_cuda() && weight.scalar_type() == torch::kFloat32 && weight.numel() == kD && weight.is_contiguous());
  TORCH_CHECK(slots.scalar_type() == torch::kInt64 && slots.numel() == raw.size(0) && slots.is_contiguous());
  TORCH_CHECK(values.scalar_type() == torch::kUInt8 && values.dim() == 2 && values.is_contiguous());
  TORCH_CHECK(values.size(1) >= 64 && values.size(1) <= 448 && values.size(1) % 64 == 0,
              "values rows hold the survivor count: 64 .. 448 in steps of 64");
  TORCH_CHECK(bitmap.scalar_type() == torch::kInt64 && bitmap.dim() == 2 && bitmap.size(1) == 8 && bitmap.is_contiguous());
  TORCH_CHECK(scales.scalar_type() == torch::kUInt8 && scales.dim() == 2 && scales.size(1) == 8 && scales.is_contiguous());
  TORCH_CHECK(bitmap.size(0) == values.size(0) && scales.size(0) == values.size(0));
  const c10::cuda::CUDAGuard g(raw.device());
  launch_packed_store(raw.data_ptr<float>(), raw.stride(0), weight.data_ptr<float>(), (float)eps,
                      slots.data_ptr<int64_t>(), values.data_ptr<uint8_t>(),
                      reinterpret_cast<uint64_t*>(bitmap.data_ptr<int64_t>()), scales.data_ptr<uint8_t>(),
                      values.size(0), (int)values.size(1), raw.size(0), err.data_ptr<int>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void sparse_mla_decode(torch::Tensor q, torch::Tensor swa_pool, torch::Tensor swa_slots, torch::Tensor swa_len,
                       bool csa_packed, torch::Tensor csa_pool, torch::Tensor csa_values, torch::Tensor csa_bitmap,
                       torch::Tensor csa_scales, torch::Tensor csa_slots, torch::Tensor csa_pos, torch::Tensor csa_len,
                       torch::Tensor freqs, torch::Tensor sink, double scale, torch::Tensor q_pos, int64_t num_splits,
                       torch::Tensor part_o, torch::Tensor part_ml, torch::Tensor out, torch::Tensor lse,
                       torch::Tensor err, c10::optional<torch::Tensor> prof, int64_t csa_fp4) {
  constexpr int kHG = 64;
  if (prof) TORCH_CHECK(prof->is_cuda() && prof->scalar_type() == torch::kInt64 && prof->numel() >= 64);
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.dim() == 3 && q.size(2) == kD && q.stride(2) == 1);
  TORCH_CHECK(q.stride(1) % 8 == 0 && q.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0,
              "q rows must be 16-byte aligned");
  check_err(err);
  const int B = q.size(0), H = q.size(1);
  TORCH_CHECK(swa_slots.scalar_type() == torch::kInt32 && swa_slots.dim() == 2 && swa_slots.size(0) == B && swa_slots.is_contiguous());
  TORCH_CHECK(csa_slots.scalar_type() == torch::kInt32 && csa_slots.dim() == 2 && csa_slots.size(0) == B && csa_slots.is_contiguous());
  TORCH_CHECK(csa_pos.scalar_type() == torch::kInt32 && csa_pos.sizes() == csa_slots.sizes() && csa_pos.is_contiguous());
  TORCH_CHECK(swa_len.scalar_type() == torch::kInt32 && swa_len.numel() == B && swa_len.is_contiguous());
  TORCH_CHECK(csa_len.scalar_type() == torch::kInt32 && csa_len.numel() == B && csa_len.is_contiguous());
  TORCH_CHECK(swa_pool.scalar_type() == torch::kUInt8 && swa_pool.numel() % kNativePageBytes == 0 && swa_pool.is_contiguous());
  TORCH_CHECK(freqs.scalar_type() == torch::kFloat32 && freqs.dim() == 3 && freqs.size(1) == 32 && freqs.is_contiguous());
  TORCH_CHECK(sink.scalar_type() == torch::kFloat32 && sink.numel() == H && sink.is_contiguous());
  TORCH_CHECK(q_pos.scalar_type() == torch::kInt32 && q_pos.numel() == B && q_pos.is_contiguous());
  TORCH_CHECK(num_splits >= 1);
  if (decode_uses_partials((int)num_splits)) {
    TORCH_CHECK(part_o.is_cuda() && part_o.scalar_type() == torch::kFloat32 &&
                part_o.numel() >= (int64_t)B * num_splits * H * kD, "part_o too small for the split partials");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(part_o.data_ptr()) % 16 == 0, "part_o must be 16-byte aligned");
    TORCH_CHECK(part_ml.is_cuda() && part_ml.scalar_type() == torch::kFloat32 &&
                part_ml.numel() >= (int64_t)B * num_splits * H * 2, "part_ml too small for the split partials");
  }
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous() && out.numel() == (int64_t)B * H * kD);
  TORCH_CHECK(reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "out must be 16-byte aligned (bulk-copied rows)");
  TORCH_CHECK(lse.scalar_type() == torch::kFloat32 && lse.is_contiguous() && lse.numel() == (int64_t)B * H);
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  DecodeParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.q_stride_b = q.stride(0);
  p.q_stride_h = q.stride(1);
  p.B = B;
  p.H = H;
  p.num_groups = (H + kHG - 1) / kHG;
  p.num_splits = (int)num_splits;
  p.swa_pool = swa_pool.data_ptr<uint8_t>();
  p.swa_pool_slots = swa_pool.numel() / kNativePageBytes * kPage;
  p.swa_slots = swa_slots.data_ptr<int32_t>();
  p.swa_cap = swa_slots.size(1);
  p.swa_len = swa_len.data_ptr<int32_t>();
  p.csa_packed = csa_packed ? 1 : 0;
  TORCH_CHECK(csa_fp4 >= 0 && csa_fp4 <= 2 && !(csa_fp4 && csa_packed), "csa_fp4: 0 (FP8), 1 (FP4 Native), 2 (FP4 Packed)");
  p.csa_fp4 = (int)csa_fp4;
  if (csa_fp4) {
    const int64_t page = kPage * (csa_fp4 == 1 ? 288 : 224);
    TORCH_CHECK(csa_pool.scalar_type() == torch::kUInt8 && csa_pool.numel() % page == 0 && csa_pool.is_contiguous() &&
                reinterpret_cast<uintptr_t>(csa_pool.data_ptr()) % 16 == 0, "csa_pool must hold FP4 pages of 64 records");
    p.csa_pool = csa_pool.data_ptr<uint8_t>();
    p.csa_pool_rows = csa_pool.numel() / page * kPage;
  } else if (csa_packed) {
    TORCH_CHECK(csa_values.scalar_type() == torch::kUInt8 && csa_values.dim() == 2 && csa_values.size(1) == 256 && csa_values.is_contiguous());
    TORCH_CHECK(csa_bitmap.scalar_type() == torch::kInt64 && csa_bitmap.size(0) == csa_values.size(0) && csa_bitmap.is_contiguous());
    TORCH_CHECK(csa_scales.scalar_type() == torch::kUInt8 && csa_scales.size(0) == csa_values.size(0) && csa_scales.is_contiguous());
    p.csa_values = csa_values.data_ptr<uint8_t>();
    p.csa_bitmap = reinterpret_cast<const uint64_t*>(csa_bitmap.data_ptr<int64_t>());
    p.csa_scales = csa_scales.data_ptr<uint8_t>();
    p.csa_pool_rows = csa_values.size(0);
  } else {
    TORCH_CHECK(csa_pool.scalar_type() == torch::kUInt8 && csa_pool.numel() % kNativePageBytes == 0 && csa_pool.is_contiguous());
    p.csa_pool = csa_pool.data_ptr<uint8_t>();
    p.csa_pool_rows = csa_pool.numel() / kNativePageBytes * kPage;
  }
  p.csa_slots = csa_slots.data_ptr<int32_t>();
  p.csa_pos = csa_pos.data_ptr<int32_t>();
  p.csa_cap = csa_slots.size(1);
  p.csa_len = csa_len.data_ptr<int32_t>();
  p.freqs = freqs.data_ptr<float>();
  p.freq_rows = freqs.size(0);
  p.scale_log2 = (float)scale * 1.4426950408889634f;
  p.part_o = decode_uses_partials((int)num_splits) ? part_o.data_ptr<float>() : nullptr;
  p.part_ml = decode_uses_partials((int)num_splits) ? part_ml.data_ptr<float>() : nullptr;
  p.err = err.data_ptr<int>();
  p.prof = prof ? reinterpret_cast<unsigned long long*>(prof->data_ptr<int64_t>()) : nullptr;
  launch_sparse_mla_decode(p, sink.data_ptr<float>(), q_pos.data_ptr<int32_t>(),
                           reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), lse.data_ptr<float>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

namespace {
void check_glm_rows(const torch::Tensor& t, int64_t width, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.size(1) == width && t.is_contiguous() &&
              reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, what);
}
}  // namespace

void glm_store(torch::Tensor raw, torch::Tensor weight, double eps, torch::Tensor slots, bool packed,
               torch::Tensor pool, torch::Tensor values, torch::Tensor bitmap, torch::Tensor err) {
  check_rows(raw);
  check_err(err);
  TORCH_CHECK(weight.is_cuda() && weight.scalar_type() == torch::kFloat32 && weight.numel() == kD && weight.is_contiguous());
  TORCH_CHECK(slots.scalar_type() == torch::kInt64 && slots.numel() == raw.size(0) && slots.is_contiguous());
  int64_t rows;
  if (packed) {
    TORCH_CHECK(values.scalar_type() == torch::kUInt8, "values must be uint8");
    check_glm_rows(values, 256, "values must be [rows, 256] contiguous, 16-byte aligned");
    TORCH_CHECK(bitmap.scalar_type() == torch::kInt64 && bitmap.size(0) == values.size(0), "bitmap must be int64 [rows, 8]");
    check_glm_rows(bitmap, 8, "bitmap must be [rows, 8] contiguous, 16-byte aligned");
    rows = values.size(0);
  } else {
    TORCH_CHECK(pool.scalar_type() == torch::kUInt8, "pool must be uint8");
    check_glm_rows(pool, kD, "pool must be [rows, 512] contiguous, 16-byte aligned");
    rows = pool.size(0);
  }
  const c10::cuda::CUDAGuard g(raw.device());
  launch_glm_store(raw.data_ptr<float>(), raw.stride(0), weight.data_ptr<float>(), (float)eps, slots.data_ptr<int64_t>(),
                   packed, packed ? nullptr : pool.data_ptr<uint8_t>(), packed ? values.data_ptr<uint8_t>() : nullptr,
                   packed ? reinterpret_cast<uint64_t*>(bitmap.data_ptr<int64_t>()) : nullptr, rows, raw.size(0),
                   err.data_ptr<int>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void glm_packed_to_native(torch::Tensor values, torch::Tensor bitmap, torch::Tensor rows, torch::Tensor out,
                          torch::Tensor err) {
  check_err(err);
  TORCH_CHECK(values.scalar_type() == torch::kUInt8, "values must be uint8");
  check_glm_rows(values, 256, "values must be [rows, 256] contiguous, 16-byte aligned");
  TORCH_CHECK(bitmap.scalar_type() == torch::kInt64 && bitmap.size(0) == values.size(0), "bitmap must be int64 [rows, 8]");
  check_glm_rows(bitmap, 8, "bitmap must be [rows, 8] contiguous, 16-byte aligned");
  TORCH_CHECK(rows.is_cuda() && rows.scalar_type() == torch::kInt64 && rows.dim() == 1 && rows.is_contiguous());
  TORCH_CHECK(out.scalar_type() == torch::kUInt8 && out.size(0) == rows.size(0), "out must be uint8 [R, 512]");
  check_glm_rows(out, kD, "out must be [R, 512] contiguous, 16-byte aligned");
  const c10::cuda::CUDAGuard g(values.device());
  launch_glm_packed_to_native(values.data_ptr<uint8_t>(), reinterpret_cast<const uint64_t*>(bitmap.data_ptr<int64_t>()),
                              values.size(0), rows.data_ptr<int64_t>(), out.data_ptr<uint8_t>(), (int)rows.size(0),
                              err.data_ptr<int>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void glm_sparse_decode(torch::Tensor q, int64_t csa_glm, torch::Tensor pool, torch::Tensor values, torch::Tensor bitmap,
                       torch::Tensor slots, torch::Tensor lens, double scale, int64_t num_splits, torch::Tensor part_o,
                       torch::Tensor part_ml, torch::Tensor out, torch::Tensor lse, torch::Tensor err) {
  constexpr int kHG = 64;
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.dim() == 3 && q.size(2) == kD && q.stride(2) == 1);
  TORCH_CHECK(q.stride(1) % 8 == 0 && q.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0,
              "q rows must be 16-byte aligned");
  check_err(err);
  const int B = q.size(0), H = q.size(1);
  TORCH_CHECK(slots.is_cuda() && slots.scalar_type() == torch::kInt32 && slots.dim() == 2 && slots.size(0) == B &&
              slots.is_contiguous(), "slots must be int32 [B, K]");
  TORCH_CHECK(lens.is_cuda() && lens.scalar_type() == torch::kInt32 && lens.numel() == B && lens.is_contiguous());
  TORCH_CHECK(csa_glm == 1 || csa_glm == 2, "csa_glm: 1 (GLM Native) or 2 (GLM Packed)");
  TORCH_CHECK(num_splits >= 1);
  if (decode_uses_partials((int)num_splits)) {
    TORCH_CHECK(part_o.is_cuda() && part_o.scalar_type() == torch::kFloat32 &&
                part_o.numel() >= (int64_t)B * num_splits * H * kD, "part_o too small for the split partials");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(part_o.data_ptr()) % 16 == 0, "part_o must be 16-byte aligned");
    TORCH_CHECK(part_ml.is_cuda() && part_ml.scalar_type() == torch::kFloat32 &&
                part_ml.numel() >= (int64_t)B * num_splits * H * 2, "part_ml too small for the split partials");
  }
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous() && out.numel() == (int64_t)B * H * kD);
  TORCH_CHECK(reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "out must be 16-byte aligned (bulk-copied rows)");
  TORCH_CHECK(lse.scalar_type() == torch::kFloat32 && lse.is_contiguous() && lse.numel() == (int64_t)B * H);
  DecodeParams p{};
  if (csa_glm == 1) {
    TORCH_CHECK(pool.scalar_type() == torch::kUInt8, "pool must be uint8");
    check_glm_rows(pool, kD, "pool must be [rows, 512] contiguous, 16-byte aligned");
    p.csa_pool = pool.data_ptr<uint8_t>();
    p.csa_pool_rows = pool.size(0);
  } else {
    TORCH_CHECK(values.scalar_type() == torch::kUInt8, "values must be uint8");
    check_glm_rows(values, 256, "values must be [rows, 256] contiguous, 16-byte aligned");
    TORCH_CHECK(bitmap.scalar_type() == torch::kInt64 && bitmap.size(0) == values.size(0), "bitmap must be int64 [rows, 8]");
    check_glm_rows(bitmap, 8, "bitmap must be [rows, 8] contiguous, 16-byte aligned");
    p.csa_values = values.data_ptr<uint8_t>();
    p.csa_bitmap = reinterpret_cast<const uint64_t*>(bitmap.data_ptr<int64_t>());
    p.csa_pool_rows = values.size(0);
  }
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.q_stride_b = q.stride(0);
  p.q_stride_h = q.stride(1);
  p.B = B;
  p.H = H;
  p.num_groups = (H + kHG - 1) / kHG;
  p.num_splits = (int)num_splits;
  // no SWA rows: swa_cap 0 (the length and slot pointers are never read)
  p.swa_slots = slots.data_ptr<int32_t>();
  p.swa_len = lens.data_ptr<int32_t>();
  p.csa_glm = (int)csa_glm;
  p.no_rope = 1;
  p.csa_slots = slots.data_ptr<int32_t>();
  p.csa_pos = slots.data_ptr<int32_t>();  // not read (no Packed FP8 rows)
  p.csa_cap = slots.size(1);
  p.csa_len = lens.data_ptr<int32_t>();
  p.scale_log2 = (float)scale * 1.4426950408889634f;
  p.part_o = decode_uses_partials((int)num_splits) ? part_o.data_ptr<float>() : nullptr;
  p.part_ml = decode_uses_partials((int)num_splits) ? part_ml.data_ptr<float>() : nullptr;
  p.err = err.data_ptr<int>();
  launch_sparse_mla_decode(p, nullptr, nullptr, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), lse.data_ptr<float>(),
                           stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

torch::Tensor umma_probe(torch::Tensor a, torch::Tensor b, int64_t mode, torch::Tensor err) {
  const auto want = mode == 3 ? torch::kUInt8 : torch::kBFloat16;
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == want && a.is_contiguous());
  TORCH_CHECK(b.is_cuda() && b.scalar_type() == want && b.is_contiguous());
  check_err(err);
  int K, N;
  TORCH_CHECK(mode >= 0 && mode <= 3, "probe mode 0..3");
  if (mode == 0 || mode == 2 || mode == 3) {
    TORCH_CHECK(a.dim() == 2 && a.size(0) == 128 && b.dim() == 2 && b.size(1) == a.size(1));
    K = a.size(1);
    N = b.size(0);
  } else {
    TORCH_CHECK(a.dim() == 2 && a.size(1) == 128 && b.dim() == 2 && b.size(0) == a.size(0));
    K = a.size(0);
    N = b.size(1);
  }
  TORCH_CHECK(K % (mode == 3 ? 32 : 16) == 0 && K <= 128 && (N == 16 || N == 32 || N == 64),
              "probe supports K<=128, N in {16,32,64}");
  const c10::cuda::CUDAGuard g(a.device());
  auto d = torch::zeros({128, N}, a.options().dtype(torch::kFloat32));
  launch_umma_probe(a.data_ptr(), b.data_ptr(), K, N, (int)mode, d.data_ptr<float>(), err.data_ptr<int>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return d;
}

void moe_fp4(torch::Tensor h, torch::Tensor topk_ids, torch::Tensor topk_w, int64_t expert_base, torch::Tensor w13,
             torch::Tensor s13, torch::Tensor w2, torch::Tensor s2, torch::Tensor offsets, torch::Tensor slot_token,
             torch::Tensor slot_weight, torch::Tensor active, torch::Tensor act, torch::Tensor out,
             torch::Tensor err) {
  TORCH_CHECK(h.is_cuda() && h.scalar_type() == torch::kBFloat16 && h.dim() == 2 && h.is_contiguous());
  check_err(err);
  const int T = h.size(0), H = h.size(1);
  TORCH_CHECK(topk_ids.scalar_type() == torch::kInt32 && topk_ids.dim() == 2 && topk_ids.size(0) == T && topk_ids.is_contiguous());
  TORCH_CHECK(topk_w.scalar_type() == torch::kFloat32 && topk_w.sizes() == topk_ids.sizes() && topk_w.is_contiguous());
  const int k = topk_ids.size(1);
  TORCH_CHECK(w13.scalar_type() == torch::kUInt8 && w13.dim() == 3 && w13.size(2) * 2 == H && w13.is_contiguous());
  const int E = w13.size(0), I = w13.size(1) / 2;
  TORCH_CHECK(s13.scalar_type() == torch::kUInt8 && s13.dim() == 3 && s13.size(0) == E && s13.size(1) == 2 * I &&
              s13.size(2) * 32 == H && s13.is_contiguous());
  TORCH_CHECK(w2.scalar_type() == torch::kUInt8 && w2.dim() == 3 && w2.size(0) == E && w2.size(1) == H &&
              w2.size(2) * 2 == I && w2.is_contiguous());
  TORCH_CHECK(s2.scalar_type() == torch::kUInt8 && s2.dim() == 3 && s2.size(0) == E && s2.size(1) == H &&
              s2.size(2) * 32 == I && s2.is_contiguous());
  TORCH_CHECK((H == 1024 || H == 2048 || H == 4096) && (I == 1024 || I == 2048 || I == 4096),
              "moe_fp4 supports hidden and intermediate sizes 1024, 2048 or 4096");
  TORCH_CHECK(E <= 4096, "too many local experts");
  TORCH_CHECK(offsets.scalar_type() == torch::kInt32 && offsets.numel() >= E + 1);
  TORCH_CHECK(active.scalar_type() == torch::kInt32 && active.numel() >= E + 1);
  TORCH_CHECK(slot_token.scalar_type() == torch::kInt32 && slot_token.numel() >= (int64_t)T * k);
  TORCH_CHECK(slot_weight.scalar_type() == torch::kFloat32 && slot_weight.numel() >= (int64_t)T * k);
  TORCH_CHECK(act.scalar_type() == torch::kBFloat16 && act.is_contiguous() && act.numel() >= (int64_t)T * k * I);
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.is_contiguous() && out.numel() == (int64_t)T * H);
  const c10::cuda::CUDAGuard g(h.device());
  static int num_sms = 0;
  if (num_sms == 0) C10_CUDA_CHECK(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, h.device().index()));
  launch_moe_fp4(reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), T, H, I, k, topk_ids.data_ptr<int32_t>(),
                 topk_w.data_ptr<float>(), (int)expert_base, E, w13.data_ptr<uint8_t>(), s13.data_ptr<uint8_t>(),
                 w2.data_ptr<uint8_t>(), s2.data_ptr<uint8_t>(), offsets.data_ptr<int32_t>(),
                 slot_token.data_ptr<int32_t>(), slot_weight.data_ptr<float>(), active.data_ptr<int32_t>(),
                 reinterpret_cast<__nv_bfloat16*>(act.data_ptr()), out.data_ptr<float>(), num_sms, stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int num_sms_of(const torch::Device& d) {
  static int cache[64] = {0};
  const int idx = d.index() < 0 ? 0 : d.index();
  if (cache[idx] == 0) C10_CUDA_CHECK(cudaDeviceGetAttribute(&cache[idx], cudaDevAttrMultiProcessorCount, idx));
  return cache[idx];
}

void index_key_store(torch::Tensor kraw, torch::Tensor slots, torch::Tensor keys, torch::Tensor kscales,
                     torch::Tensor err) {
  TORCH_CHECK(kraw.is_cuda() && kraw.scalar_type() == torch::kFloat32 && kraw.dim() == 2 && kraw.size(1) == 128 &&
              kraw.stride(1) == 1 && kraw.stride(0) % 4 == 0, "kraw must be float32 [R, 128]");
  TORCH_CHECK(slots.scalar_type() == torch::kInt64 && slots.numel() == kraw.size(0) && slots.is_contiguous());
  TORCH_CHECK(keys.scalar_type() == torch::kUInt8 && keys.dim() == 2 && keys.size(1) == 128 && keys.is_contiguous());
  TORCH_CHECK(kscales.scalar_type() == torch::kFloat32 && kscales.numel() == keys.size(0));
  check_err(err);
  const c10::cuda::CUDAGuard g(kraw.device());
  launch_index_key_store(kraw.data_ptr<float>(), kraw.stride(0), slots.data_ptr<int64_t>(), keys.data_ptr<uint8_t>(),
                         kscales.data_ptr<float>(), keys.size(0), kraw.size(0), err.data_ptr<int>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// scores[b, r] for r < R; then top-k physical slots / RoPE rows.
void index_select(torch::Tensor q, torch::Tensor w, torch::Tensor keys, torch::Tensor kscales, torch::Tensor phys,
                  torch::Tensor count, int64_t R, torch::Tensor scores, torch::Tensor out_slots, torch::Tensor out_pos,
                  torch::Tensor err) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.dim() == 3 && q.size(2) == 128 && q.is_contiguous());
  const int B = q.size(0), H = q.size(1);
  TORCH_CHECK(H <= 64, "at most 64 indexer heads");
  TORCH_CHECK(w.scalar_type() == torch::kFloat32 && w.is_contiguous() && w.numel() == (int64_t)B * H);
  TORCH_CHECK(keys.scalar_type() == torch::kUInt8 && keys.dim() == 2 && keys.size(1) == 128 && keys.is_contiguous());
  TORCH_CHECK(kscales.scalar_type() == torch::kFloat32 && kscales.numel() == keys.size(0) && kscales.is_contiguous());
  TORCH_CHECK(phys.scalar_type() == torch::kInt32 && phys.dim() == 2 && phys.size(0) == B && phys.stride(1) == 1);
  TORCH_CHECK(R >= 1 && R <= phys.size(1));
  TORCH_CHECK(count.scalar_type() == torch::kInt64 && count.numel() == B && count.is_contiguous());
  TORCH_CHECK(scores.scalar_type() == torch::kFloat32 && scores.dim() == 2 && scores.size(0) == B &&
              scores.size(1) >= R && scores.stride(1) == 1);
  TORCH_CHECK(out_slots.scalar_type() == torch::kInt32 && out_slots.dim() == 2 && out_slots.size(0) == B &&
              out_slots.is_contiguous());
  TORCH_CHECK(out_pos.scalar_type() == torch::kInt32 && out_pos.sizes() == out_slots.sizes() && out_pos.is_contiguous());
  check_err(err);
  const c10::cuda::CUDAGuard g(q.device());
  // the keys pool keeps one trailing row for writes without a destination: pages use the rest
  launch_index_logits(reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), w.data_ptr<float>(), B, H,
                      keys.data_ptr<uint8_t>(), kscales.data_ptr<float>(), keys.size(0), phys.data_ptr<int32_t>(),
                      phys.stride(0), count.data_ptr<int64_t>(), (int)R, scores.data_ptr<float>(), scores.stride(0),
                      num_sms_of(q.device()), err.data_ptr<int>(), stream());
  launch_index_topk(scores.data_ptr<float>(), scores.stride(0), B, (int)R, out_slots.size(1), phys.data_ptr<int32_t>(),
                    phys.stride(0), 4, out_slots.data_ptr<int32_t>(), out_pos.data_ptr<int32_t>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Fragment-ordered MXFP4 experts (packmla/ops/moe.py tile_fp4_frag): w13f [E, I/64, H/256, 16384],
// s13f [E, I/64, H/256, 1024], w2f [E, H/128, I/256, 16384], s2f [E, H/128, I/256, 1024].
void moe_fp4_mma(torch::Tensor h, torch::Tensor topk_ids, torch::Tensor topk_w, int64_t expert_base,
                 torch::Tensor w13f, torch::Tensor s13f, torch::Tensor w2f, torch::Tensor s2f, torch::Tensor offsets,
                 torch::Tensor slot_token, torch::Tensor slot_weight, torch::Tensor active, torch::Tensor pad,
                 torch::Tensor xs, torch::Tensor act_s, torch::Tensor out, torch::Tensor err) {
  TORCH_CHECK(h.is_cuda() && h.scalar_type() == torch::kBFloat16 && h.dim() == 2 && h.is_contiguous());
  check_err(err);
  const int T = h.size(0), H = h.size(1);
  TORCH_CHECK(topk_ids.scalar_type() == torch::kInt32 && topk_ids.dim() == 2 && topk_ids.size(0) == T && topk_ids.is_contiguous());
  TORCH_CHECK(topk_w.scalar_type() == torch::kFloat32 && topk_w.sizes() == topk_ids.sizes() && topk_w.is_contiguous());
  const int k = topk_ids.size(1);
  TORCH_CHECK(w13f.scalar_type() == torch::kUInt8 && w13f.dim() == 4 && w13f.size(3) == 16384 && w13f.is_contiguous());
  const int E = w13f.size(0), I = w13f.size(1) * 64;
  TORCH_CHECK(w13f.size(2) * 256 == H, "w13f k-tiles do not match hidden size");
  TORCH_CHECK(s13f.scalar_type() == torch::kUInt8 && s13f.dim() == 4 && s13f.size(0) == E && s13f.size(1) == I / 64 &&
              s13f.size(2) == H / 256 && s13f.size(3) == 1024 && s13f.is_contiguous());
  TORCH_CHECK(w2f.scalar_type() == torch::kUInt8 && w2f.dim() == 4 && w2f.size(0) == E && w2f.size(1) * 128 == H &&
              w2f.size(2) * 256 == I && w2f.size(3) == 16384 && w2f.is_contiguous());
  TORCH_CHECK(s2f.scalar_type() == torch::kUInt8 && s2f.dim() == 4 && s2f.size(0) == E && s2f.size(1) * 128 == H &&
              s2f.size(2) * 256 == I && s2f.size(3) == 1024 && s2f.is_contiguous());
  TORCH_CHECK(H % 256 == 0 && I % 256 == 0, "hidden and intermediate must be multiples of 256");
  TORCH_CHECK(E <= 4096, "too many local experts");
  TORCH_CHECK(offsets.scalar_type() == torch::kInt32 && offsets.numel() >= E + 1);
  TORCH_CHECK(active.scalar_type() == torch::kInt32 && active.numel() >= E + 1);
  TORCH_CHECK(pad.scalar_type() == torch::kInt32 && pad.numel() >= E + 1);
  TORCH_CHECK(slot_token.scalar_type() == torch::kInt32 && slot_token.numel() >= (int64_t)T * k);
  TORCH_CHECK(slot_weight.scalar_type() == torch::kFloat32 && slot_weight.numel() >= (int64_t)T * k);
  const int64_t prow = (int64_t)T * k + 16 * (int64_t)E;
  TORCH_CHECK(xs.scalar_type() == torch::kFloat16 && xs.is_contiguous() && xs.numel() >= prow * H);
  TORCH_CHECK(act_s.scalar_type() == torch::kFloat16 && act_s.is_contiguous() && act_s.numel() >= prow * I);
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.is_contiguous() && out.numel() == (int64_t)T * H);
  const c10::cuda::CUDAGuard g(h.device());
  launch_moe_route(topk_ids.data_ptr<int32_t>(), topk_w.data_ptr<float>(), T, k, (int)expert_base, E,
                   offsets.data_ptr<int32_t>(), slot_token.data_ptr<int32_t>(), slot_weight.data_ptr<float>(),
                   active.data_ptr<int32_t>(), pad.data_ptr<int32_t>(), stream());
  launch_moe_fp4_mma(reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), T, H, I, E, offsets.data_ptr<int32_t>(),
                     pad.data_ptr<int32_t>(), slot_token.data_ptr<int32_t>(), slot_weight.data_ptr<float>(),
                     active.data_ptr<int32_t>(), w13f.data_ptr<uint8_t>(), s13f.data_ptr<uint8_t>(),
                     w2f.data_ptr<uint8_t>(), s2f.data_ptr<uint8_t>(), reinterpret_cast<__half*>(xs.data_ptr()),
                     reinterpret_cast<__half*>(act_s.data_ptr()), out.data_ptr<float>(), num_sms_of(h.device()),
                     err.data_ptr<int>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

namespace {
const __nv_bfloat16* bf16_ptr(const torch::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
__nv_bfloat16* bf16_mut(const torch::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }
void check_rows_bf16(const torch::Tensor& t, int64_t rows, int64_t n, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16 && t.dim() == 2 && t.size(0) == rows &&
              t.size(1) == n && t.stride(1) == 1 && t.stride(0) % 2 == 0, name, " must be bf16 [rows, n]");
}
}  // namespace

// h = bf16(rmsnorm(x (+ d) (+ dfp32)) * w); x_out (optional) receives the bf16 residual x + d.
void add_rmsnorm(torch::Tensor x, c10::optional<torch::Tensor> d, c10::optional<torch::Tensor> dfp32,
                 c10::optional<torch::Tensor> x_out, torch::Tensor w, double eps, torch::Tensor h) {
  const int64_t rows = x.size(0), n = x.size(1);
  check_rows_bf16(x, rows, n, "x");
  check_rows_bf16(h, rows, n, "h");
  TORCH_CHECK(n % 2 == 0 && n <= 8192, "add_rmsnorm: width must be even and at most 8192");
  TORCH_CHECK(w.scalar_type() == torch::kFloat32 && w.numel() == n && w.is_contiguous());
  if (d) check_rows_bf16(*d, rows, n, "d");
  if (dfp32) TORCH_CHECK(dfp32->scalar_type() == torch::kFloat32 && dfp32->dim() == 2 && dfp32->size(0) == rows &&
                         dfp32->size(1) == n && dfp32->stride(1) == 1 && dfp32->stride(0) % 2 == 0);
  if (x_out) check_rows_bf16(*x_out, rows, n, "x_out");
  const c10::cuda::CUDAGuard g(x.device());
  launch_add_rmsnorm(bf16_ptr(x), x.stride(0), d ? bf16_ptr(*d) : nullptr, d ? d->stride(0) : 0,
                     dfp32 ? dfp32->data_ptr<float>() : nullptr, dfp32 ? dfp32->stride(0) : 0,
                     x_out ? bf16_mut(*x_out) : nullptr, x_out ? x_out->stride(0) : 0, w.data_ptr<float>(), (float)eps,
                     bf16_mut(h), h.stride(0), (int)rows, (int)n, stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope_q(torch::Tensor q, torch::Tensor pos, torch::Tensor freqs) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.dim() == 3 && q.size(2) == 512 &&
              q.stride(2) == 1 && q.stride(1) == 512);
  TORCH_CHECK(pos.scalar_type() == torch::kInt64 && pos.numel() == q.size(0) && pos.is_contiguous());
  TORCH_CHECK(freqs.scalar_type() == torch::kFloat32 && freqs.dim() == 3 && freqs.is_contiguous());
  const c10::cuda::CUDAGuard g(q.device());
  launch_rope_q(bf16_mut(q), q.stride(0), q.size(0), q.size(1), pos.data_ptr<int64_t>(), freqs.data_ptr<float>(),
                stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void comp_pool(torch::Tensor proj, int64_t off, int64_t D, torch::Tensor ape, torch::Tensor state, torch::Tensor req,
               torch::Tensor pos, torch::Tensor raw) {
  TORCH_CHECK(proj.is_cuda() && proj.scalar_type() == torch::kBFloat16 && proj.dim() == 2 && proj.stride(1) == 1);
  const int B = proj.size(0);
  TORCH_CHECK(off >= 0 && off + 2 * D <= proj.size(1));
  TORCH_CHECK(ape.scalar_type() == torch::kFloat32 && ape.dim() == 2 && ape.size(1) == D && ape.is_contiguous());
  TORCH_CHECK(state.scalar_type() == torch::kFloat32 && state.dim() == 3 && state.size(1) == 3 && state.size(2) == D &&
              state.is_contiguous());
  TORCH_CHECK(req.scalar_type() == torch::kInt64 && req.numel() == B && pos.scalar_type() == torch::kInt64 &&
              pos.numel() == B);
  TORCH_CHECK(raw.scalar_type() == torch::kFloat32 && raw.dim() == 2 && raw.size(0) == B && raw.size(1) == D &&
              raw.stride(1) == 1);
  const c10::cuda::CUDAGuard g(proj.device());
  launch_comp_pool(bf16_ptr(proj), proj.stride(0), (int)off, (int)D, ape.data_ptr<float>(), (int)ape.size(0),
                   state.data_ptr<float>(), req.data_ptr<int64_t>(), pos.data_ptr<int64_t>(), raw.data_ptr<float>(),
                   raw.stride(0), B, stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void route_topk(torch::Tensor logits, c10::optional<torch::Tensor> bias, int64_t k, double scaling, torch::Tensor ids,
                torch::Tensor wts) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == torch::kBFloat16 && logits.dim() == 2 &&
              logits.stride(1) == 1);
  const int T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(E <= 512 && k >= 1 && k <= 32 && k <= E);
  TORCH_CHECK(ids.scalar_type() == torch::kInt32 && ids.is_contiguous() && ids.numel() == (int64_t)T * k);
  TORCH_CHECK(wts.scalar_type() == torch::kFloat32 && wts.is_contiguous() && wts.numel() == (int64_t)T * k);
  if (bias) TORCH_CHECK(bias->scalar_type() == torch::kFloat32 && bias->numel() == E && bias->is_contiguous());
  const c10::cuda::CUDAGuard g(logits.device());
  launch_route_topk(bf16_ptr(logits), logits.stride(0), T, E, bias ? bias->data_ptr<float>() : nullptr, (int)k, (float)scaling,
                    ids.data_ptr<int32_t>(), wts.data_ptr<float>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void silu_mul(torch::Tensor gu, torch::Tensor out) {
  TORCH_CHECK(gu.is_cuda() && gu.scalar_type() == torch::kBFloat16 && gu.dim() == 2 && gu.stride(1) == 1);
  const int T = gu.size(0), I = gu.size(1) / 2;
  check_rows_bf16(out, T, I, "out");
  TORCH_CHECK(out.is_contiguous());
  const c10::cuda::CUDAGuard g(gu.device());
  launch_silu_mul(bf16_ptr(gu), gu.stride(0), T, I, bf16_mut(out), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// One block-scaled tcgen05 MMA on host-supplied shared-memory / TMEM images (layout self-test).
torch::Tensor bs_probe(torch::Tensor a_img, torch::Tensor b_img, torch::Tensor sfa, torch::Tensor sfb, int64_t idesc,
                       int64_t kind, int64_t sfa_extra, int64_t sfb_extra, torch::Tensor err) {
  TORCH_CHECK(a_img.is_cuda() && a_img.scalar_type() == torch::kUInt8 && a_img.is_contiguous() &&
              a_img.numel() == 128 * 128);
  TORCH_CHECK(b_img.scalar_type() == torch::kUInt8 && b_img.is_contiguous() && b_img.dim() == 2 &&
              b_img.size(1) == 128);
  const int N = b_img.size(0);
  TORCH_CHECK(N >= 8 && N <= 256 && N % 8 == 0);
  TORCH_CHECK(sfa.scalar_type() == torch::kInt32 && sfa.is_contiguous() && sfa.numel() == 128 * 16);
  TORCH_CHECK(sfb.scalar_type() == torch::kInt32 && sfb.is_contiguous() && sfb.numel() == 128 * 16);
  TORCH_CHECK(kind >= 0 && kind <= 2 && sfa_extra >= 0 && sfa_extra < 16 && sfb_extra >= 0 && sfb_extra < 16);
  const c10::cuda::CUDAGuard g(a_img.device());
  auto d = torch::zeros({128, N}, a_img.options().dtype(torch::kFloat32));
  launch_bs_probe(a_img.data_ptr<uint8_t>(), b_img.data_ptr<uint8_t>(),
                  reinterpret_cast<const uint32_t*>(sfa.data_ptr<int>()),
                  reinterpret_cast<const uint32_t*>(sfb.data_ptr<int>()), (uint32_t)idesc, (int)kind, N,
                  (uint32_t)sfa_extra, (uint32_t)sfb_extra, d.data_ptr<float>(), err.data_ptr<int>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return d;
}

// TMA-unpacked FP4 A, tcgen05.cp scale factors, k_steps block-scaled MMAs -> (D, shared image of A).
std::vector<torch::Tensor> bs_probe2(torch::Tensor a_packed, torch::Tensor b_img, torch::Tensor sfa_src,
                                     torch::Tensor sfb_src, int64_t k_steps, int64_t expect_tx, torch::Tensor err) {
  TORCH_CHECK(a_packed.is_cuda() && a_packed.scalar_type() == torch::kUInt8 && a_packed.is_contiguous() &&
              a_packed.numel() == 128 * 64);
  TORCH_CHECK(b_img.scalar_type() == torch::kUInt8 && b_img.is_contiguous() && b_img.dim() == 2 &&
              b_img.size(1) == 128);
  const int N = b_img.size(0);
  TORCH_CHECK(N >= 8 && N <= 256 && N % 8 == 0 && k_steps >= 1 && k_steps <= 4);
  TORCH_CHECK(sfa_src.numel() == 512 && sfb_src.numel() == 512 && sfa_src.is_contiguous() && sfb_src.is_contiguous());
  TORCH_CHECK(expect_tx == 8192 || expect_tx == 16384);
  const c10::cuda::CUDAGuard g(a_packed.device());
  auto d = torch::zeros({128, N}, a_packed.options().dtype(torch::kFloat32));
  auto dump = torch::zeros({128, 128}, a_packed.options());
  const int rc = launch_bs_probe2(a_packed.data_ptr<uint8_t>(), b_img.data_ptr<uint8_t>(), sfa_src.data_ptr<uint8_t>(),
                                  sfb_src.data_ptr<uint8_t>(), N, (int)k_steps, (uint32_t)expect_tx,
                                  d.data_ptr<float>(), dump.data_ptr<uint8_t>(), err.data_ptr<int>(), stream());
  TORCH_CHECK(rc == 0, "tensor map encoding failed: ", rc);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {d, dump};
}

// MXFP4 experts with MXFP8 activations: route + quantize + gate/up + down (4 launches).
void moe_mxf4(torch::Tensor h, torch::Tensor topk_ids, torch::Tensor topk_w, int64_t expert_base, torch::Tensor w13,
              torch::Tensor sfw13, torch::Tensor w2, torch::Tensor sfw2, torch::Tensor offsets, torch::Tensor slot_token,
              torch::Tensor slot_weight, torch::Tensor active, torch::Tensor pad, torch::Tensor chunks,
              torch::Tensor n_chunks, torch::Tensor xq, torch::Tensor xs, torch::Tensor act_q, torch::Tensor act_s,
              torch::Tensor out, torch::Tensor err, c10::optional<torch::Tensor> prof) {
  TORCH_CHECK(h.is_cuda() && h.scalar_type() == torch::kBFloat16 && h.dim() == 2 && h.is_contiguous());
  const int T = h.size(0), H = h.size(1);
  if (prof) TORCH_CHECK(prof->scalar_type() == torch::kInt64 && prof->is_contiguous() && prof->numel() >= 16);
  TORCH_CHECK(topk_ids.scalar_type() == torch::kInt32 && topk_ids.is_contiguous() && topk_ids.size(0) == T);
  const int k = topk_ids.size(1);
  TORCH_CHECK(topk_w.scalar_type() == torch::kFloat32 && topk_w.is_contiguous() && topk_w.numel() == (int64_t)T * k);
  TORCH_CHECK(w13.scalar_type() == torch::kUInt8 && w13.dim() == 3 && w13.is_contiguous() && w13.size(2) * 2 == H);
  const int E = w13.size(0), I = w13.size(1) / 2;
  TORCH_CHECK(H % 512 == 0 && I % 512 == 0 && H <= 4096 && I <= 4096, "moe_mxf4: H, I multiples of 512, <= 4096");
  TORCH_CHECK(w2.scalar_type() == torch::kUInt8 && w2.is_contiguous() && w2.size(0) == E && w2.size(1) == H &&
              w2.size(2) * 2 == I);
  TORCH_CHECK(sfw13.scalar_type() == torch::kUInt8 && sfw13.is_contiguous() &&
              sfw13.numel() == (int64_t)E * 2 * I * (H / 32));
  TORCH_CHECK(sfw2.scalar_type() == torch::kUInt8 && sfw2.is_contiguous() && sfw2.numel() == (int64_t)E * H * (I / 32));
  TORCH_CHECK(reinterpret_cast<uintptr_t>(w13.data_ptr()) % 32 == 0 && reinterpret_cast<uintptr_t>(w2.data_ptr()) % 32 == 0);
  const int rows = xq.dim() == 3 ? xq.size(1) : 0;
  TORCH_CHECK(rows % 32 == 0 && rows >= T * k + 31 * std::min(E, T * k), "moe_mxf4: workspace rows too small");
  TORCH_CHECK(xq.is_contiguous() && xq.size(0) == H / 128 && xq.size(2) == 128);
  TORCH_CHECK(act_q.is_contiguous() && act_q.dim() == 3 && act_q.size(0) == I / 128 && act_q.size(1) == rows);
  TORCH_CHECK(xs.is_contiguous() && xs.numel() == (int64_t)rows * H / 32);
  TORCH_CHECK(act_s.is_contiguous() && act_s.numel() == (int64_t)rows * I / 32);
  TORCH_CHECK(offsets.numel() >= E + 1 && pad.numel() >= E + 1 && active.numel() >= E + 1);
  TORCH_CHECK(slot_token.numel() >= (int64_t)T * k && slot_weight.numel() >= (int64_t)T * k);
  TORCH_CHECK(chunks.scalar_type() == torch::kInt32 && chunks.is_contiguous() && chunks.numel() >= (int64_t)T * k * 4);
  TORCH_CHECK(n_chunks.scalar_type() == torch::kInt32 && n_chunks.numel() >= 1);
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.is_contiguous() && out.size(0) == T && out.size(1) == H);
  const c10::cuda::CUDAGuard g(h.device());
  MoeMxArgs a{};
  a.h = bf16_ptr(h);
  a.T = T; a.H = H; a.I = I; a.k = k; a.E = E; a.expert_base = (int)expert_base; a.rows_total = rows;
  a.num_sms = num_sms_of(h.device());
  a.topk_ids = topk_ids.data_ptr<int32_t>(); a.topk_w = topk_w.data_ptr<float>();
  a.w13 = w13.data_ptr<uint8_t>(); a.sfw13 = sfw13.data_ptr<uint8_t>();
  a.w2 = w2.data_ptr<uint8_t>(); a.sfw2 = sfw2.data_ptr<uint8_t>();
  a.offsets = offsets.data_ptr<int32_t>(); a.slot_token = slot_token.data_ptr<int32_t>();
  a.slot_weight = slot_weight.data_ptr<float>(); a.active = active.data_ptr<int32_t>(); a.pad = pad.data_ptr<int32_t>();
  a.chunks = reinterpret_cast<int4*>(chunks.data_ptr<int32_t>()); a.n_chunks = n_chunks.data_ptr<int32_t>();
  a.xq = xq.data_ptr<uint8_t>(); a.xs = xs.data_ptr<uint8_t>();
  a.act_q = act_q.data_ptr<uint8_t>(); a.act_s = act_s.data_ptr<uint8_t>();
  a.out = out.data_ptr<float>(); a.err = err.data_ptr<int>();
  a.prof = prof ? reinterpret_cast<unsigned long long*>(prof->data_ptr<int64_t>()) : nullptr;
  const int rc = launch_moe_mxf4(a, stream());
  TORCH_CHECK(rc == 0, "moe_mxf4 launch failed: ", rc);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}


// ----------------------------------------------------------------------------- symmetric memory (CUDA IPC)
// A buffer every rank of a TP group allocates with the same size; the IPC handles are exchanged by the
// caller (torch.distributed) and opened here, so kernels can load and store a peer's copy over NVLink.
std::tuple<int64_t, torch::Tensor> symm_alloc(int64_t bytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&ptr, (size_t)bytes));
  C10_CUDA_CHECK(cudaMemset(ptr, 0, (size_t)bytes));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, ptr));
  auto t = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  std::memcpy(t.data_ptr(), &h, sizeof(h));
  return {reinterpret_cast<int64_t>(ptr), t};
}
int64_t symm_open(torch::Tensor handle, int64_t device) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t) && handle.scalar_type() == torch::kUInt8);
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(ptr);
}
void symm_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}
void symm_free(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr)));
}

namespace {
// layout = [recv_off, recv_elems, gath_off, flag_rs_off, flag_ag_off, max_src, max_tiles, lpart_off]
SymmComm make_comm(const torch::Tensor& peers, int64_t rank, int64_t world, const std::vector<int64_t>& layout,
                   const torch::Tensor& epoch, const torch::Tensor& err, int64_t timeout_ns) {
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == torch::kInt64 && peers.numel() == world && peers.is_contiguous(),
              "peers must be CUDA int64[world]");
  TORCH_CHECK(epoch.is_cuda() && epoch.scalar_type() == torch::kInt32 && epoch.numel() >= 2, "epoch must be CUDA int32[2]");
  check_err(err);
  TORCH_CHECK(layout.size() == 8, "layout must have 8 entries");
  TORCH_CHECK(rank >= 0 && rank < world && world >= 1 && world <= layout[5], "bad rank/world");
  SymmComm c;
  c.peers = reinterpret_cast<const unsigned long long*>(peers.data_ptr<int64_t>());
  c.rank = (int)rank;
  c.world = (int)world;
  c.recv_off = layout[0];
  c.recv_elems = layout[1];
  c.gath_off = layout[2];
  c.flag_rs_off = layout[3];
  c.flag_ag_off = layout[4];
  c.max_src = (int)layout[5];
  c.max_tiles = (int)layout[6];
  c.lpart_off = layout[7];
  c.epoch = reinterpret_cast<unsigned int*>(epoch.data_ptr<int>());
  c.err = err.data_ptr<int>();
  c.timeout_ns = timeout_ns;
  return c;
}
}  // namespace

void gemm_allreduce(torch::Tensor x, torch::Tensor w, torch::Tensor out, torch::Tensor peers, int64_t rank,
                    int64_t world, std::vector<int64_t> layout, torch::Tensor epoch, torch::Tensor err, int64_t splits,
                    int64_t one_shot, int64_t timeout_ns, c10::optional<torch::Tensor> prof) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.is_contiguous(),
              "x must be CUDA bf16 [B, K] contiguous");
  TORCH_CHECK(w.scalar_type() == torch::kBFloat16 && w.dim() == 2 && w.is_contiguous() && w.size(1) == x.size(1),
              "w must be bf16 [N, K] contiguous");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous() && out.size(0) == x.size(0) &&
              out.size(1) == w.size(0), "out must be bf16 [B, N]");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(x.data_ptr()) % 16) == 0 && (reinterpret_cast<uintptr_t>(w.data_ptr()) % 16) == 0 &&
              (reinterpret_cast<uintptr_t>(out.data_ptr()) % 16) == 0, "x, w and out must be 16-byte aligned");
  GemmArParams p;
  p.c = make_comm(peers, rank, world, layout, epoch, err, timeout_ns);
  p.B = (int)x.size(0);
  p.K = (int)x.size(1);
  p.N = (int)w.size(0);
  p.S = (int)splits;
  p.nmb = (p.B + 127) / 128;
  p.stages = 4;
  p.one_shot = one_shot ? 1 : 0;
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.prof = nullptr;
  if (prof) {
    TORCH_CHECK(prof->is_cuda() && prof->scalar_type() == torch::kInt64 && prof->numel() >= 8);
    p.prof = reinterpret_cast<unsigned long long*>(prof->data_ptr<int64_t>());
  }
  const int rc = launch_gemm_allreduce(p, w.data_ptr(), x.data_ptr(), num_sms_of(x.device()), stream());
  TORCH_CHECK(rc == 0, "gemm_allreduce: unsupported shape or launch failure (code ", rc, ", B=", p.B, " N=", p.N,
              " K=", p.K, " splits=", p.S, ")");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void allreduce(c10::optional<torch::Tensor> a, c10::optional<torch::Tensor> f, torch::Tensor out, torch::Tensor peers,
               int64_t rank, int64_t world, std::vector<int64_t> layout, torch::Tensor epoch, torch::Tensor err,
               int64_t chunk, int64_t one_shot, int64_t timeout_ns) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == torch::kBFloat16 && out.is_contiguous(), "out must be CUDA bf16");
  ArParams p;
  p.c = make_comm(peers, rank, world, layout, epoch, err, timeout_ns);
  p.n = out.numel();
  p.chunk = chunk;
  p.one_shot = one_shot ? 1 : 0;
  p.a = nullptr;
  p.f = nullptr;
  if (a) {
    TORCH_CHECK(a->scalar_type() == torch::kBFloat16 && a->is_contiguous() && a->numel() == p.n);
    p.a = reinterpret_cast<const __nv_bfloat16*>(a->data_ptr());
  }
  if (f) {
    TORCH_CHECK(f->scalar_type() == torch::kFloat32 && f->is_contiguous() && f->numel() == p.n);
    p.f = f->data_ptr<float>();
  }
  for (const void* q : {(const void*)p.a, (const void*)p.f, (const void*)out.data_ptr()})
    TORCH_CHECK((reinterpret_cast<uintptr_t>(q) % 16) == 0, "all-reduce operands must be 16-byte aligned");
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  const int rc = launch_allreduce(p, num_sms_of(out.device()), stream());
  TORCH_CHECK(rc == 0, "allreduce: unsupported size or launch failure (code ", rc, ")");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void segment_copy(torch::Tensor segs) {
  TORCH_CHECK(segs.is_cuda() && segs.scalar_type() == torch::kInt64 && segs.dim() == 2 && segs.size(1) == 3 &&
              segs.is_contiguous(), "segs must be CUDA int64 [n, 3] (src, dst, bytes)");
  const int rc = launch_segment_copy(segs.data_ptr<int64_t>(), (int)segs.size(0), num_sms_of(segs.device()),
                                     stream());
  TORCH_CHECK(rc == 0, "segment_copy launch failed");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void packed_to_native(torch::Tensor values, torch::Tensor bitmap, torch::Tensor scales, torch::Tensor rows,
                      torch::Tensor positions, torch::Tensor freqs, torch::Tensor out, torch::Tensor dst,
                      torch::Tensor err) {
  check_err(err);
  TORCH_CHECK(values.is_cuda() && values.scalar_type() == torch::kUInt8 && values.dim() == 2 && values.size(1) >= 64 &&
              values.size(1) <= 448 && values.size(1) % 64 == 0 && values.is_contiguous(),
              "values must be CUDA uint8 [rows, keep], keep 64 .. 448 in steps of 64");
  TORCH_CHECK(bitmap.scalar_type() == torch::kInt64 && bitmap.is_contiguous() && bitmap.size(0) == values.size(0) &&
              bitmap.size(1) == 8, "bitmap must be int64 [rows, 8]");
  TORCH_CHECK(scales.scalar_type() == torch::kUInt8 && scales.is_contiguous() && scales.size(0) == values.size(0) &&
              scales.size(1) == 8, "scales must be uint8 [rows, 8]");
  TORCH_CHECK(rows.scalar_type() == torch::kInt32 && positions.scalar_type() == torch::kInt32 && rows.is_contiguous() &&
              positions.is_contiguous() && rows.numel() == positions.numel(), "rows/positions must be int32 [n]");
  TORCH_CHECK(dst.scalar_type() == torch::kInt64 && dst.is_contiguous() && dst.numel() == rows.numel(),
              "dst must be int64 [n]");
  TORCH_CHECK(freqs.scalar_type() == torch::kFloat32 && freqs.dim() == 3 && freqs.size(1) == 32 && freqs.is_contiguous());
  TORCH_CHECK(out.scalar_type() == torch::kUInt8 && out.is_contiguous() && out.numel() % kNativePageBytes == 0,
              "out must be uint8 Native pages");
  launch_packed_to_native(values.data_ptr<uint8_t>(), reinterpret_cast<const uint64_t*>(bitmap.data_ptr<int64_t>()),
                          scales.data_ptr<uint8_t>(), values.size(0), rows.data_ptr<int32_t>(),
                          positions.data_ptr<int32_t>(), freqs.data_ptr<float>(), freqs.size(0), out.data_ptr<uint8_t>(),
                          dst.data_ptr<int64_t>(), out.numel() / kNativePageBytes * kPage, (int)values.size(1),
                          (int)rows.numel(), err.data_ptr<int>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ----------------------------------------------------------------------------- dense MXFP8 projections
void dense_mx(torch::Tensor x, torch::Tensor w, torch::Tensor w_sf, torch::Tensor y, torch::Tensor a_img,
              torch::Tensor a_sf, torch::Tensor part, torch::Tensor counters, int64_t splits, torch::Tensor err) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 3 && x.stride(2) == 1,
              "x must be bf16 [batch, T, K] with K contiguous");
  const int64_t batch = x.size(0), T = x.size(1), K = x.size(2);
  TORCH_CHECK(w.scalar_type() == torch::kUInt8 && w.dim() == 3 && w.size(0) == batch && w.size(2) == K && w.is_contiguous(),
              "w must be uint8 E4M3 codes [batch, N, K]");
  const int64_t N = w.size(1), G = K / 128, tiles_n = (N + 255) / 256, Tp = (T + 7) & ~7;
  TORCH_CHECK(K % 128 == 0, "K must be a multiple of 128");
  TORCH_CHECK(splits >= 1 && splits <= G && (splits == 1 || T <= 128), "splits must be 1..K/128 (1 above 128 tokens)");
  TORCH_CHECK(w_sf.scalar_type() == torch::kUInt8 && w_sf.is_contiguous() && w_sf.numel() == batch * tiles_n * G * 1024,
              "w_sf must be uint8 [batch, N/256 tiles, K/128, 256, 4]");
  TORCH_CHECK(y.scalar_type() == torch::kBFloat16 && y.dim() == 3 && y.size(0) == batch && y.size(1) == T &&
              y.size(2) == N && y.stride(2) == 1, "y must be bf16 [batch, T, N] with N contiguous");
  if (!dense_mx_fused_quant((int)T, (int)K, (int)splits)) {
    TORCH_CHECK(a_img.scalar_type() == torch::kUInt8 && a_img.is_contiguous() && a_img.numel() >= batch * G * Tp * 128,
                "a_img workspace too small");
    TORCH_CHECK(a_sf.scalar_type() == torch::kInt32 && a_sf.is_contiguous() && a_sf.numel() >= batch * G * Tp,
                "a_sf workspace too small");
  }
  if (splits > 1) {
    TORCH_CHECK(part.scalar_type() == torch::kFloat32 && part.is_contiguous() &&
                part.numel() >= batch * splits * Tp * tiles_n * 256, "part workspace too small");
    TORCH_CHECK(counters.scalar_type() == torch::kInt32 && counters.is_contiguous() && counters.numel() >= batch * tiles_n,
                "counters workspace too small");
  }
  if (T == 0 || N == 0 || batch == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  static int num_sms[64] = {0};
  const int dev = x.get_device();
  if (num_sms[dev] == 0) num_sms[dev] = at::cuda::getDeviceProperties(dev)->multiProcessorCount;
  DenseMxArgs a{};
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.x_stride_b = x.stride(0);
  a.x_stride_t = x.stride(1);
  a.T = (int)T; a.K = (int)K; a.N = (int)N; a.batch = (int)batch;
  a.w = w.data_ptr<uint8_t>();
  a.w_sf = w_sf.data_ptr<uint8_t>();
  a.y = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  a.y_stride_t = y.stride(1);
  a.y_stride_b = y.stride(0);
  a.a_img = a_img.data_ptr<uint8_t>();
  a.a_sf = reinterpret_cast<uint32_t*>(a_sf.data_ptr<int32_t>());
  a.part = splits > 1 ? part.data_ptr<float>() : nullptr;
  a.counters = splits > 1 ? counters.data_ptr<int32_t>() : nullptr;
  a.splits = (int)splits;
  a.num_sms = num_sms[dev];
  a.err = err.data_ptr<int>();
  const int rc = launch_dense_mx(a, stream());
  TORCH_CHECK(rc == 0, "dense_mx launch rejected (", rc, "): sizes or alignment");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void fp4_store(torch::Tensor raw, torch::Tensor weight, double eps, torch::Tensor slots, torch::Tensor positions,
               torch::Tensor freqs, torch::Tensor pool, bool packed, torch::Tensor err) {
  TORCH_CHECK(raw.is_cuda() && raw.scalar_type() == torch::kFloat32 && raw.dim() == 2 && raw.size(1) == 512 &&
              raw.stride(1) == 1 && raw.stride(0) % 4 == 0, "raw must be fp32 [R, 512] with 16-byte rows");
  TORCH_CHECK(weight.scalar_type() == torch::kFloat32 && weight.numel() == 512 && weight.is_contiguous());
  TORCH_CHECK(slots.scalar_type() == torch::kInt64 && slots.numel() == raw.size(0) && slots.is_contiguous());
  TORCH_CHECK(positions.scalar_type() == torch::kInt64 && positions.numel() == raw.size(0) && positions.is_contiguous());
  TORCH_CHECK(freqs.scalar_type() == torch::kFloat32 && freqs.dim() == 3 && freqs.size(1) == 32 && freqs.is_contiguous());
  const int64_t page_bytes = 64 * (packed ? 224 : 288);
  TORCH_CHECK(pool.scalar_type() == torch::kUInt8 && pool.is_contiguous() && pool.numel() % page_bytes == 0,
              "pool must be uint8 pages of 64 FP4 records");
  const c10::cuda::CUDAGuard g(raw.device());
  launch_fp4_store(raw.data_ptr<float>(), raw.stride(0), weight.data_ptr<float>(), (float)eps, slots.data_ptr<int64_t>(),
                   positions.data_ptr<int64_t>(), freqs.data_ptr<float>(), freqs.size(0), pool.data_ptr<uint8_t>(),
                   pool.numel() / page_bytes * 64, packed, (int)raw.size(0), err.data_ptr<int>(), stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "packmla sm_100a kernels";
  m.def("native_store", &native_store, "FP32 rows -> Native 584 B C4 records (paged)");
  m.def("packed_store", &packed_store, "FP32 rows -> Packed 328 B C4 records (planes)");
  m.def("umma_probe", &umma_probe, "tcgen05 operand-layout self-test (one MMA)");
  m.def("index_key_store", &index_key_store, "FP8 index keys (swizzled rows) + fp32 scales");
  m.def("index_select", &index_select, "FP8 tcgen05 indexer logits + radix top-k");
  m.def("bs_probe2", &bs_probe2, "TMA FP4 + tcgen05.cp scale-factor pipeline self-test");
  m.def("bs_probe", &bs_probe, "block-scaled tcgen05 MMA layout self-test");
  m.def("add_rmsnorm", &add_rmsnorm, "residual add + RMSNorm (bf16)");
  m.def("rope_q", &rope_q, "in-place RoPE of query tails");
  m.def("comp_pool", &comp_pool, "compressor online-softmax pooling of one token per row");
  m.def("route_topk", &route_topk, "sigmoid top-k MoE routing");
  m.def("silu_mul", &silu_mul, "silu(gate) * up");
  m.def("moe_mxf4", &moe_mxf4, "MXFP4 experts x MXFP8 activations (tcgen05 block-scaled)", py::arg("h"),
        py::arg("topk_ids"), py::arg("topk_w"), py::arg("expert_base"), py::arg("w13"), py::arg("sfw13"), py::arg("w2"),
        py::arg("sfw2"), py::arg("offsets"), py::arg("slot_token"), py::arg("slot_weight"), py::arg("active"),
        py::arg("pad"), py::arg("chunks"), py::arg("n_chunks"), py::arg("xq"), py::arg("xs"), py::arg("act_q"),
        py::arg("act_s"), py::arg("out"), py::arg("err"), py::arg("prof") = py::none());
  m.def("moe_fp4_mma", &moe_fp4_mma, "MXFP4 routed experts, register-fragment MMAs (decode-sized batches)");
  m.def("moe_fp4", &moe_fp4, "MXFP4 routed experts (route, gate/up+SiLU, down+scatter)");
  m.def("dense_mx", &dense_mx, "dense projections with MXFP8 weights: y[b] = x[b] W[b]^T (tcgen05 block-scaled)");
  m.def("fp4_store", &fp4_store, "FP4 C4 records (E2M1 + E4M3 per 16; Native 288 B / Packed 224 B) into paged pools");
  m.def("decode_max_active_clusters", [](int64_t cluster) {
    TORCH_CHECK(decode_splits_clustered((int)cluster), "cluster size must be 2, 4 or 8");
    return decode_max_active_clusters((int)cluster);
  }, "co-resident decode clusters of the given size on the current device");
  m.def("sparse_mla_decode", &sparse_mla_decode, "Sparse MLA decode (tcgen05) + split combine", py::arg("q"),
        py::arg("swa_pool"), py::arg("swa_slots"), py::arg("swa_len"), py::arg("csa_packed"), py::arg("csa_pool"),
        py::arg("csa_values"), py::arg("csa_bitmap"), py::arg("csa_scales"), py::arg("csa_slots"), py::arg("csa_pos"),
        py::arg("csa_len"), py::arg("freqs"), py::arg("sink"), py::arg("scale"), py::arg("q_pos"),
        py::arg("num_splits"), py::arg("part_o"), py::arg("part_ml"), py::arg("out"), py::arg("lse"), py::arg("err"),
        py::arg("prof") = py::none(), py::arg("csa_fp4") = 0);
  m.def("glm_store", &glm_store, "GLM-5.3 MLA rows (Native 512 B raw E4M3, or Packed 256 survivors + bitmap)");
  m.def("glm_packed_to_native", &glm_packed_to_native, "GLM-5.3 Adapter: Packed rows -> Native rows");
  m.def("glm_sparse_decode", &glm_sparse_decode, "Sparse MLA decode over GLM-5.3 Native or Packed rows (tcgen05)");
  m.def("packed_to_native", &packed_to_native, "Adapter: Packed planes rows -> Native records (paged workspace)");
  m.def("segment_copy", &segment_copy, "batched 16-byte-aligned copies between device and mapped host memory");
  m.def("symm_alloc", &symm_alloc, "cudaMalloc + IPC handle of a symmetric buffer");
  m.def("symm_open", &symm_open, "map a peer's symmetric buffer from its IPC handle");
  m.def("symm_close", &symm_close, "unmap a peer's symmetric buffer");
  m.def("symm_free", &symm_free, "free a symmetric buffer");
  m.def("gemm_allreduce", &gemm_allreduce, "tcgen05 row-parallel GEMM fused with an all-reduce over peers",
        py::arg("x"), py::arg("w"), py::arg("out"), py::arg("peers"), py::arg("rank"), py::arg("world"),
        py::arg("layout"), py::arg("epoch"), py::arg("err"), py::arg("splits"), py::arg("one_shot"),
        py::arg("timeout_ns"), py::arg("prof") = py::none());
  m.def("allreduce", &allreduce, "one- or two-shot all-reduce of (bf16 + fp32) addends over peers");
}
