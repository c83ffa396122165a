// Allocation-free entry point of the sparse MLA decode kernel.
//
// This entry point has no counterpart in the reference project; it is an addition of packmla.
//
// Who needs it: callers that cannot allocate GPU memory at the point where they run attention,
// for example a host runtime that reserved all device memory up front for its own allocator,
// a plugin interface that only hands out input and output buffers, or code that must not call
// cudaMalloc while another framework is recording a stream.  The regular entry point needs a
// split-KV scratch buffer (partial outputs and softmax statistics) that its caller allocates;
// this one keeps that scratch in a fixed array compiled into the library instead.
//
// Contract:
//   * The caller passes inputs and outputs; this function calls no cudaMalloc, cudaFree or any
//     allocating library routine.
//   * Scratch lives in file-scope __device__ arrays of a fixed maximum size: at most
//     PACKMLA_NOALLOC_MAX_PARTS = 4096 partial rows, where one partial row is one
//     (query, KV split, head) triple, i.e. B * num_splits * H <= 4096 (8 MiB of partial outputs
//     plus 32 KiB of statistics).  Every GPU that loads the library holds this memory until the
//     process exits.  Larger requests are rejected with an error code and message.
//   * The first call on a device resolves the scratch address on that device with
//     cudaGetSymbolAddress (host code cannot use the array's name as a device pointer).  Make that
//     first call before any stream capture on the device.  The caller's current device must be
//     the device that owns the tensors.
//   * Every call shares the one scratch array, which keeps the previous call's contents.  Nothing
//     in it needs to start at zero: the kernel writes the statistics of every (query, split, head)
//     it covers, and the combine step only reads partial outputs of splits that wrote them.
//     Calls that overlap on the GPU (for example on two streams without ordering between them)
//     race on the scratch and produce wrong results; order them on one stream.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "launchers.h"

#define PACKMLA_NOALLOC_MAX_PARTS 4096
#define PACKMLA_NOALLOC_MAX_DEVICES 64

namespace {

constexpr int kD = 512;
constexpr int kHG = 64;
constexpr int kTile = 128;
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

// Arguments of one decode call; pointer fields are device pointers except `err` may be null.
struct PackmlaNoallocDecodeArgs {
  const void* q;              // bf16 [B, H, 512]; tail rotated by the query position
  int64_t q_stride_b;         // elements
  int64_t q_stride_h;         // elements
  int32_t B;
  int32_t H;
  const void* swa_pool;       // Native pages (uint8), SWA rows
  int64_t swa_pool_bytes;
  const int32_t* swa_slots;   // [B, swa_cap]
  int32_t swa_cap;
  const int32_t* swa_len;     // [B]
  int32_t csa_packed;         // 1 = Packed planes, 0 = Native pages
  const void* csa_pool;       // Native pages (uint8) when csa_packed == 0
  int64_t csa_pool_bytes;
  const void* csa_values;     // Packed: uint8 [rows, 256]
  const void* csa_bitmap;     // Packed: uint64 [rows, 8]
  const void* csa_scales;     // Packed: uint8 [rows, 8]
  int64_t csa_rows;           // Packed rows
  const int32_t* csa_slots;   // [B, csa_cap]
  const int32_t* csa_pos;     // [B, csa_cap]
  int32_t csa_cap;
  const int32_t* csa_len;     // [B]
  const float* freqs;         // [freq_rows, 32, 2]
  int64_t freq_rows;
  const float* sink;          // [H]
  float scale;                // softmax scale
  const int32_t* q_pos;       // [B]
  int32_t num_splits;
  void* out;                  // bf16 [B, H, 512]
  float* lse;                 // [B, H]
  int* err;                   // int32[4] device error word, or null
};

// Returns 0 on success; otherwise 1 and packmla_noalloc_last_error() describes the problem.
int packmla_sparse_mla_decode_noalloc(const PackmlaNoallocDecodeArgs* a, cudaStream_t stream) {
  if (a == nullptr) return fail("null argument block");
  if (a->B < 0 || a->H <= 0 || a->num_splits < 1) return fail("B >= 0, H > 0 and num_splits >= 1 required");
  if ((int64_t)a->B * a->num_splits * a->H > PACKMLA_NOALLOC_MAX_PARTS)
    return fail("B * num_splits * H exceeds the 4096 partial rows of the built-in scratch");
  if (a->swa_pool_bytes % kNativePageBytes != 0) return fail("swa_pool_bytes must be whole pages");
  if (!a->csa_packed && a->csa_pool_bytes % kNativePageBytes != 0) return fail("csa_pool_bytes must be whole pages");
  if (a->B == 0) return 0;
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
  const int cap = a->swa_cap + a->csa_cap;
  p.rows_per_split = ((cap + a->num_splits - 1) / a->num_splits + kTile - 1) / kTile * kTile;
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

}  // extern "C"
