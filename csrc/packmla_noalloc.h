// Public C interface of packmla's allocation-free sparse MLA decode.
//
// This interface has no counterpart in the reference project; it is an addition of packmla.
//
// Who it is for: code that calls attention where it cannot allocate GPU memory -- a host runtime
// that reserved all device memory up front for its own allocator, or a plugin interface that hands
// the attention op only its input and output buffers.  The regular entry point needs a split-KV
// scratch buffer (partial outputs and softmax statistics) from its caller; this one keeps that
// scratch in a fixed array compiled into the library (csrc/noalloc_decode.cu).
//
// Contract of packmla_sparse_mla_decode_noalloc:
//   * The caller passes device pointers to inputs and outputs; the call performs no cudaMalloc,
//     cudaFree or other allocating library routine.
//   * Scratch is a file-scope device array of PACKMLA_NOALLOC_MAX_PARTS partial rows; one partial
//     row is one (query, KV split, head) triple, so B * num_splits * H must not exceed the limit.
//     Every GPU that loads the library holds the array (8 MiB + 32 KiB) until the process exits.
//     Split counts 2, 4 and 8 merge their partials inside a thread-block cluster and leave the array
//     untouched; the limit applies to every call all the same, so a caller's sizes do not depend on
//     which merge a split count takes.
//   * The first call on a device looks up the array's device address on that device (host code
//     cannot use the array's name as a device pointer).  Make that first call before any stream
//     capture on the device; the caller's current device must own the tensors.
//   * All calls share the one array and it keeps the previous call's contents.  Nothing in it must
//     start at zero: every call writes the statistics of each partial row it later reads.  Calls
//     that overlap on the GPU (two streams with no ordering between them) race on the array and
//     give wrong results; order them on one stream.
//   * Arguments are checked on the host before anything is launched; a rejected call returns
//     non-zero and packmla_noalloc_last_error() says why (per calling thread).
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime.h>

#define PACKMLA_NOALLOC_MAX_PARTS 4096

#ifdef __cplusplus
extern "C" {
#endif

// Arguments of one decode call.  Pointers are device pointers; `err` may be null.
typedef struct PackmlaNoallocDecodeArgs {
  const void* q;              // bf16 [B, H, 512], tail rotated by the query position; 16-byte aligned
  int64_t q_stride_b;         // elements, multiple of 8
  int64_t q_stride_h;         // elements, multiple of 8
  int32_t B;
  int32_t H;
  const void* swa_pool;       // Native pages (uint8) holding the SWA rows
  int64_t swa_pool_bytes;     // whole pages of 64 x 584 bytes
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
} PackmlaNoallocDecodeArgs;

// Returns 0 on success; otherwise non-zero, nothing was launched, and packmla_noalloc_last_error()
// describes the problem.
int packmla_sparse_mla_decode_noalloc(const PackmlaNoallocDecodeArgs* args, cudaStream_t stream);

// Message of the calling thread's last rejected call ("" if none).
const char* packmla_noalloc_last_error(void);

// PACKMLA_NOALLOC_MAX_PARTS, for callers that load the library dynamically.
int packmla_noalloc_max_parts(void);

// sizeof(PackmlaNoallocDecodeArgs) as compiled into the library, so a caller that restates the
// struct (a binding in another language) can check its layout.
size_t packmla_noalloc_args_size(void);

#ifdef __cplusplus
}  // extern "C"
#endif
