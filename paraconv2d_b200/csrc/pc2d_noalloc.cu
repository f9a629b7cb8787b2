// pc2d_forward_noalloc: the forward pass without any caller-provided or
// runtime-allocated scratch.
//
// Who needs it: hosts that hand an operator only its input and output buffers
// and do not allow device allocation while it executes -- for example plugin
// or custom-op interfaces of inference runtimes that have no workspace
// mechanism, or real-time code that budgets all device memory up front.
// cudaMalloc can synchronise the device and can fail under memory pressure,
// and such hosts forbid it (or any allocating library call) on this path.
//
// How: the tensor-core forward needs a small scratch buffer (the weights
// split into tf32 hi/lo halves plus one constant per output channel, about
// 0.6 MB for a 64->64-channel 3x3 layer).  Here it lives in the file-scope
// device array below, of fixed size kNoAllocScratchBytes; every GPU that
// loads this library holds it until the process exits.
//
// Rules of use:
//   - problems whose scratch would exceed kNoAllocScratchBytes are rejected
//     with PC2D_ERR_WORKSPACE before anything is launched;
//   - the first call in a CUDA context (on a device's primary context: the
//     first call on that device) looks up the array's device address with
//     cudaGetSymbolAddress, with that context current.  That lookup allocates
//     nothing but may load the module; make the first call on each device
//     (and in each other context a host creates) before any stream capture.
//     The address is cached per context, because a module's addresses belong
//     to the context it was loaded into;
//   - all calls share the one array, which keeps the previous call's contents.
//     Nothing has to start at zero: the forward's prep kernels overwrite every
//     scratch byte it reads.  Calls that overlap on the GPU (different streams,
//     or different host threads, on one device) race on the array and must be
//     serialised by the caller.
#include "pc2d_common.cuh"

namespace pc2d {
namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)8 << 20;  // 8 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

PerContext<void *> g_noalloc_ptr;

// Device address of g_noalloc_scratch in the current context (looked up once
// per context); nullptr with a message on failure.
void *noalloc_scratch_ptr() {
  unsigned long long ctx = current_context_id();
  void *ptr = nullptr;
  if (ctx && g_noalloc_ptr.get(ctx, &ptr)) return ptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess || ptr == nullptr) {
    set_last_error("pc2d_forward_noalloc: cudaGetSymbolAddress of the scratch array failed (%s)", cudaGetErrorString(e));
    return nullptr;
  }
  // the lookup may have made the device's primary context current
  if (!ctx) ctx = current_context_id();
  if (ctx) g_noalloc_ptr.set(ctx, ptr);
  return ptr;
}

}  // namespace
}  // namespace pc2d

extern "C" int pc2d_forward_noalloc(int dtype, const void *input, const void *pars, double factor, int k0, int k1,
                                    int s0, int s1, int dl0, int dl1, int n, int channels, int height, int width,
                                    int m, void *output, void *hsum, void *stream) {
  using namespace pc2d;
  // Shape checks and the scratch size come from the regular entry points, so a
  // problem this call accepts is exactly one pc2d_forward accepts.  The size
  // check here gives a clear message; pc2d_forward checks again against the
  // kernel path it actually takes (the process-wide kernel family may change
  // between the two).
  const size_t need = pc2d_forward_workspace_size(dtype, n, channels, height, width, m, k0, k1, s0, s1, dl0, dl1);
  if (need > kNoAllocScratchBytes) {
    set_last_error("pc2d_forward_noalloc: this problem needs %zu bytes of scratch, more than the %zu-byte static "
                   "scratch array; use pc2d_forward with a caller workspace",
                   need, kNoAllocScratchBytes);
    return PC2D_ERR_WORKSPACE;
  }
  void *ws = noalloc_scratch_ptr();
  if (ws == nullptr) return PC2D_ERR_CUDA;
  // nothing on this call's path may allocate (the status word's host mirror
  // included)
  t_no_alloc = true;
  const int st = pc2d_forward(dtype, input, pars, factor, k0, k1, s0, s1, dl0, dl1, n, channels, height, width, m,
                              output, hsum, ws, kNoAllocScratchBytes, stream);
  t_no_alloc = false;
  return st;
}
