// HiCache transfer kernel: one launch copies a batch of (src, dst, bytes) segments between device
// memory and pinned, device-mapped host memory (reference: the kernel IO backend of SGLang's HiCache,
// `--hicache-io-backend kernel`, moving all three Packed planes of a page together).
//
// A page move touches ~5 planes x 21 C4 layers + C128 pages + the request's SWA ring and compressor
// state: hundreds of small copies, which one kernel issues in parallel instead of one copy call each.
// Segments are 16-byte aligned with sizes a multiple of 16 (checked on the host); every CTA takes
// segments round-robin and its threads move 16-byte vectors.
#include "launchers.h"

namespace {
__global__ void __launch_bounds__(256) segment_copy_kernel(const int64_t* __restrict__ segs, int nseg) {
  for (int i = blockIdx.x; i < nseg; i += gridDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(segs[3 * i]);
    uint4* dst = reinterpret_cast<uint4*>(segs[3 * i + 1]);
    const int64_t n = segs[3 * i + 2] >> 4;
    for (int64_t j = threadIdx.x; j < n; j += blockDim.x) dst[j] = src[j];
  }
}
}  // namespace

int launch_segment_copy(const int64_t* segs_dev, int nseg, int num_sms, cudaStream_t stream) {
  if (nseg <= 0) return 0;
  const int grid = nseg < 4 * num_sms ? nseg : 4 * num_sms;
  segment_copy_kernel<<<grid, 256, 0, stream>>>(segs_dev, nseg);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
