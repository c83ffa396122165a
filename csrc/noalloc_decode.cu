// Allocation-free entry point of the sparse MLA decode kernel.
//
// This entry point has no counterpart in the reference project; it is an addition of packmla.
// Its C interface and contract (who it is for, the scratch limit, the first-call set-up, the shared
// scratch and its race) are declared in csrc/packmla_noalloc.h.
//
// Implementation notes: the split-KV scratch (partial outputs and softmax statistics of every
// (query, split, head) triple) is two file-scope __device__ arrays.  Host code cannot pass their
// names to a kernel: the name is a host-side stand-in for the symbol, so the device address is looked
// up once per device with cudaGetSymbolAddress (with that device current) and cached.
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "launchers.h"
#include "packmla_noalloc.h"

#define PACKMLA_NOALLOC_MAX_DEVICES 64

// The struct is also restated by bindings in other languages (tests/test_zz_no_alloc.py uses ctypes):
// pin its layout on the usual 64-bit ABI.
static_assert(sizeof(void*) == 8, "64-bit ABI expected");
static_assert(offsetof(PackmlaNoallocDecodeArgs, B) == 24 && offsetof(PackmlaNoallocDecodeArgs, swa_pool) == 32,
              "PackmlaNoallocDecodeArgs layout changed");
static_assert(offsetof(PackmlaNoallocDecodeArgs, csa_packed) == 72 && offsetof(PackmlaNoallocDecodeArgs, freqs) == 160,
              "PackmlaNoallocDecodeArgs layout changed");
static_assert(offsetof(PackmlaNoallocDecodeArgs, num_splits) == 200 && sizeof(PackmlaNoallocDecodeArgs) == 232,
              "PackmlaNoallocDecodeArgs layout changed");

namespace {

constexpr int kD = 512;
constexpr int kHG = 64;
constexpr int kPage = 64;
constexpr int kNativePageBytes = kPage * 584;

static __device__ __align__(256) float g_noalloc_part_o[PACKMLA_NOALLOC_MAX_PARTS * kD];
static __device__ __align__(256) float g_noalloc_part_ml[PACKMLA_NOALLOC_MAX_PARTS * 2];

std::mutex g_mutex;
void* g_part_o_addr[PACKMLA_NOALLOC_MAX_DEVICES] = {};
void* g_part_ml_addr[PACKMLA_NOALLOC_MAX_DEVICES] = {};
thread_local char g_last_error[256] = "";

int fail(const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
  return 1;
}

// Resolve the scratch arrays' device addresses on the current device (once per device).
int scratch_for_current_device(float** part_o, float** part_ml) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail("cudaGetDevice failed");
  if (dev < 0 || dev >= PACKMLA_NOALLOC_MAX_DEVICES) return fail("device index out of range");
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_part_o_addr[dev] == nullptr) {
    void* a = nullptr;
    void* b = nullptr;
    cudaError_t e1 = cudaGetSymbolAddress(&a, g_noalloc_part_o);
    if (e1 != cudaSuccess) return fail(cudaGetErrorString(e1));
    cudaError_t e2 = cudaGetSymbolAddress(&b, g_noalloc_part_ml);
    if (e2 != cudaSuccess) return fail(cudaGetErrorString(e2));
    g_part_o_addr[dev] = a;
    g_part_ml_addr[dev] = b;
  }
  *part_o = static_cast<float*>(g_part_o_addr[dev]);
  *part_ml = static_cast<float*>(g_part_ml_addr[dev]);
  return 0;
}

}  // namespace

extern "C" {

// Returns 0 on success; otherwise 1 and packmla_noalloc_last_error() describes the problem.
int packmla_sparse_mla_decode_noalloc(const PackmlaNoallocDecodeArgs* a, cudaStream_t stream) {
  if (a == nullptr) return fail("null argument block");
  if (a->B < 0 || a->H <= 0 || a->num_splits < 1) return fail("B >= 0, H > 0 and num_splits >= 1 required");
  if ((int64_t)a->B * a->num_splits * a->H > PACKMLA_NOALLOC_MAX_PARTS)
    return fail("B * num_splits * H exceeds the 4096 partial rows of the built-in scratch");
  if (a->B == 0) return 0;
  // the kernel reads q with 16-byte vector loads: the rows must start on 16-byte boundaries
  if (a->q == nullptr || (reinterpret_cast<uintptr_t>(a->q) & 15) != 0)
    return fail("q must be a non-null 16-byte aligned pointer");
  if (a->q_stride_b % 8 != 0 || a->q_stride_h % 8 != 0 || a->q_stride_b < 0 || a->q_stride_h < 0)
    return fail("q strides must be non-negative multiples of 8 elements");
  if (a->swa_cap < 0 || a->csa_cap < 0) return fail("swa_cap and csa_cap must be >= 0");
  if (a->freq_rows <= 0) return fail("freq_rows must be > 0");
  if (a->swa_pool == nullptr || a->swa_slots == nullptr || a->swa_len == nullptr || a->csa_slots == nullptr ||
      a->csa_pos == nullptr || a->csa_len == nullptr || a->freqs == nullptr || a->sink == nullptr ||
      a->q_pos == nullptr || a->out == nullptr || a->lse == nullptr)
    return fail("null input or output pointer");
  if (a->swa_pool_bytes <= 0 || a->swa_pool_bytes % kNativePageBytes != 0)
    return fail("swa_pool_bytes must be a positive number of whole pages");
  if (a->csa_packed) {
    if (a->csa_values == nullptr || a->csa_bitmap == nullptr || a->csa_scales == nullptr || a->csa_rows <= 0)
      return fail("Packed rows need values, bitmap and scales planes and csa_rows > 0");
  } else if (a->csa_pool == nullptr || a->csa_pool_bytes <= 0 || a->csa_pool_bytes % kNativePageBytes != 0) {
    return fail("Native rows need csa_pool with a positive number of whole pages");
  }
  if (((reinterpret_cast<uintptr_t>(a->swa_pool) | reinterpret_cast<uintptr_t>(a->csa_pool) |
        reinterpret_cast<uintptr_t>(a->csa_values) | reinterpret_cast<uintptr_t>(a->csa_bitmap) |
        reinterpret_cast<uintptr_t>(a->freqs) | reinterpret_cast<uintptr_t>(a->out)) & 15) != 0)
    return fail("pools, planes, freqs and out must be 16-byte aligned");
  if (decode_splits_clustered(a->num_splits)) {
    // every (query, head group) cluster must be co-resident, as in every validated launch
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= PACKMLA_NOALLOC_MAX_DEVICES)
      return fail("no current CUDA device");
    static int fit_cache[PACKMLA_NOALLOC_MAX_DEVICES][9] = {};
    int fit;
    {
      std::lock_guard<std::mutex> lock(g_mutex);
      if (fit_cache[dev][a->num_splits] == 0) fit_cache[dev][a->num_splits] = decode_max_active_clusters(a->num_splits);
      fit = fit_cache[dev][a->num_splits];
    }
    if ((int64_t)a->B * ((a->H + kHG - 1) / kHG) > fit)
      return fail("more split clusters than are co-resident on this device: use fewer splits");
  }
  float* part_o = nullptr;
  float* part_ml = nullptr;
  if (scratch_for_current_device(&part_o, &part_ml) != 0) return 1;
  DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(a->q);
  p.q_stride_b = a->q_stride_b;
  p.q_stride_h = a->q_stride_h;
  p.B = a->B;
  p.H = a->H;
  p.num_groups = (a->H + kHG - 1) / kHG;
  p.num_splits = a->num_splits;
  p.swa_pool = static_cast<const uint8_t*>(a->swa_pool);
  p.swa_pool_slots = a->swa_pool_bytes / kNativePageBytes * kPage;
  p.swa_slots = a->swa_slots;
  p.swa_cap = a->swa_cap;
  p.swa_len = a->swa_len;
  p.csa_packed = a->csa_packed ? 1 : 0;
  if (a->csa_packed) {
    p.csa_values = static_cast<const uint8_t*>(a->csa_values);
    p.csa_bitmap = static_cast<const uint64_t*>(a->csa_bitmap);
    p.csa_scales = static_cast<const uint8_t*>(a->csa_scales);
    p.csa_pool_rows = a->csa_rows;
  } else {
    p.csa_pool = static_cast<const uint8_t*>(a->csa_pool);
    p.csa_pool_rows = a->csa_pool_bytes / kNativePageBytes * kPage;
  }
  p.csa_slots = a->csa_slots;
  p.csa_pos = a->csa_pos;
  p.csa_cap = a->csa_cap;
  p.csa_len = a->csa_len;
  p.freqs = a->freqs;
  p.freq_rows = a->freq_rows;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.part_o = part_o;
  p.part_ml = part_ml;
  p.err = a->err;
  launch_sparse_mla_decode(p, a->sink, a->q_pos, static_cast<__nv_bfloat16*>(a->out), a->lse, stream);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(cudaGetErrorString(e));
  return 0;
}

const char* packmla_noalloc_last_error(void) { return g_last_error; }

int packmla_noalloc_max_parts(void) { return PACKMLA_NOALLOC_MAX_PARTS; }

size_t packmla_noalloc_args_size(void) { return sizeof(PackmlaNoallocDecodeArgs); }

}  // extern "C"
