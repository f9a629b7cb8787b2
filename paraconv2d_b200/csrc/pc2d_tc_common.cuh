// Device helpers shared by the tcgen05 kernels: bounded warp-uniform waits and
// the staging of input "halos" (the rows of an NCHW plane that a tile of
// consecutive output pixels reads) into shared memory with 1-D bulk copies.
#pragma once

#include "pc2d_common.cuh"
#include "pc2d_sm100.cuh"

namespace pc2d {
namespace tc {

using namespace sm100;

constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s per barrier wait

// Warp-uniform bounded wait: every lane polls, the warp agrees on the result.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  const bool ok = mbar_wait(bar, parity, kWaitNs, abort_flag);
  return __all_sync(0xffffffffu, ok);
}

// A plane segment [src, src + count) of floats copied with a 1-D bulk copy:
// the copy starts at src rounded down to 16 bytes and covers whole 16-byte
// units, so it starts `lead` floats before src and may end up to 15 bytes
// after src + count.  Both rounded bounds stay inside the 16-byte units (and
// so the memory pages) that hold the segment's first and last elements.
struct BulkSpan {
  const void *src;  // 16-byte aligned
  uint32_t bytes;   // multiple of 16
  int lead;         // floats between the aligned start and the segment start
};

__device__ __forceinline__ BulkSpan bulk_span(const float *src, int64_t count) {
  const uintptr_t b = reinterpret_cast<uintptr_t>(src);
  const uintptr_t a = b & ~(uintptr_t)15;
  const uintptr_t e = (b + (uintptr_t)count * 4 + 15) & ~(uintptr_t)15;
  BulkSpan s;
  s.src = reinterpret_cast<const void *>(a);
  s.bytes = (uint32_t)(e - a);
  s.lead = (int)((b - a) >> 2);
  return s;
}

}  // namespace tc
}  // namespace pc2d
