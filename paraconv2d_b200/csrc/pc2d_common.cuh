// Shared definitions of the ParaConv2d sm_100a kernels: the problem
// descriptor, launch helpers and the device-side error flag.
#pragma once

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
#include <stdint.h>

#include <mutex>
#include <utility>
#include <vector>

#include "paraconv2d.h"

namespace pc2d {

// A named range on the profiler timeline for the duration of a scope (NVTX
// push/pop; without an attached tool the calls return at once).  The C-ABI
// entry points open one per call ("pc2d_forward", "pc2d_backward", ...) and
// the backward one per kernel family it launches ("dgrad", "wgrad").
struct NvtxRange {
  explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange &) = delete;
  NvtxRange &operator=(const NvtxRange &) = delete;
};

// Unique id (cuCtxGetId) of the CUDA context current on the calling thread;
// 0 when no context is current or the driver cannot say.  Ids are never
// reused within a process, unlike context handles or device ordinals.
unsigned long long current_context_id();

// Values kept per CUDA context.  Device addresses of this library's
// __device__ variables and per-kernel attributes belong to the module loaded
// into one context; a host may make a context other than the device's
// primary one current, so caches are keyed on the context, not the device.
template <typename T>
class PerContext {
 public:
  bool get(unsigned long long id, T *v) {
    std::lock_guard<std::mutex> lock(mu_);
    for (auto &e : entries_)
      if (e.first == id) {
        *v = e.second;
        return true;
      }
    return false;
  }
  void set(unsigned long long id, T v) {
    std::lock_guard<std::mutex> lock(mu_);
    for (auto &e : entries_)
      if (e.first == id) {
        e.second = v;
        return;
      }
    entries_.emplace_back(id, v);
  }

 private:
  std::mutex mu_;
  std::vector<std::pair<unsigned long long, T>> entries_;
};

// Runs `fn` (a function returning a pc2d_status) once per context for each
// bit of `cache`: a cudaFuncSetAttribute call, typically.  Without a context
// id it runs every time.
template <typename F>
int once_per_context(PerContext<uint64_t> &cache, uint64_t bit, F &&fn) {
  unsigned long long ctx = current_context_id();
  uint64_t mask = 0;
  if (ctx && cache.get(ctx, &mask) && (mask & bit)) return PC2D_OK;
  const int st = fn();
  if (st != PC2D_OK) return st;
  if (!ctx) ctx = current_context_id();
  if (ctx) {
    mask = 0;
    cache.get(ctx, &mask);
    cache.set(ctx, mask | bit);
  }
  return PC2D_OK;
}

// One ParaConv2d problem (a padded input batch and one parameter vector).
// Field names follow the reference op (paraconv2d.cc:254-269).
struct Problem {
  int n, C, H, W;         // padded input [n][C][H][W]
  int m;                  // output channels
  int k0, k1, s0, s1, dl0, dl1;
  int P, Q;               // output extent
  int T;                  // taps per channel, k0*k1
  int64_t d;              // C*T, length of one window
  int64_t HW, PQ, CHW, NPQ, NHW;
};

inline Problem make_problem(int n, int C, int H, int W, int m, int k0, int k1, int s0, int s1,
                            int dl0, int dl1) {
  Problem p;
  p.n = n; p.C = C; p.H = H; p.W = W; p.m = m;
  p.k0 = k0; p.k1 = k1; p.s0 = s0; p.s1 = s1; p.dl0 = dl0; p.dl1 = dl1;
  p.P = (s0 > 0) ? ((H - dl0 * (k0 - 1) - 1) / s0) + 1 : 0;
  p.Q = (s1 > 0) ? ((W - dl1 * (k1 - 1) - 1) / s1) + 1 : 0;
  p.T = k0 * k1;
  p.d = (int64_t)C * p.T;
  p.HW = (int64_t)H * W;
  p.PQ = (int64_t)p.P * p.Q;
  p.CHW = (int64_t)C * p.HW;
  p.NPQ = (int64_t)n * p.PQ;
  p.NHW = (int64_t)n * p.HW;
  return p;
}

// Where the input gradient goes.  The kernels compute it over the padded
// input [n][C][H][W] the op receives.  For the op itself the whole of it is
// written, as is.  A module that pads its input before the op (reference
// ptparaconv2d.py:216-218) needs only the gradient of the unpadded input,
// times its input factor and grad factor: rows pt .. pt+Hu-1 and columns
// pl .. pl+Wu-1, written into an [n][C][Hu][Wu] array and multiplied by
// `scale`, which saves the module two passes over dx (slice, scale).
struct DxOut {
  int pt, pl, Hu, Wu;
  int64_t HWu, CHWu;
  double scale;
};

inline DxOut dx_full(const Problem &p) { return DxOut{0, 0, p.H, p.W, p.HW, p.CHW, 1.0}; }

// Index in the input-gradient array of padded pixel (y, x), channel 0, of
// image n; -1 when the pixel lies in the padding.
__host__ __device__ __forceinline__ int64_t dx_index(const DxOut &o, int64_t n, int y, int x) {
  const int yi = y - o.pt, xi = x - o.pl;
  if ((unsigned)yi >= (unsigned)o.Hu || (unsigned)xi >= (unsigned)o.Wu) return -1;
  return n * o.CHWu + (int64_t)yi * o.Wu + xi;
}

// Offset, within one input channel plane, of tap `tap` (= ix2*k1 + iy2) of the
// window of output pixel (0,0).  The window is flipped: tap (ix2, iy2) reads
// row (k0-1-ix2)*dl0 and column (k1-1-iy2)*dl1 (reference paraconv2d.cc:89-92,
// with 2*(k/2) = k-1 for the odd kernel sizes accepted here).
__host__ __device__ inline int tap_row(const Problem &p, int tap) { return (p.k0 - 1 - tap / p.k1) * p.dl0; }
__host__ __device__ inline int tap_col(const Problem &p, int tap) { return (p.k1 - 1 - tap % p.k1) * p.dl1; }

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Device-side status of the current context: the first nonzero pc2d_status
// a kernel records (a bounded mbarrier wait that gave up), and a mirror of it
// in pinned host memory mapped into the device, which the entry points read
// without synchronising.  It is a __device__ variable of the ABI translation
// unit; kernels get its address as an int* (the code is its first word) and
// record errors with record_device_error.  Read by pc2d_device_status().
struct DeviceStatus {
  int code;
  int pad;
  int *mirror;  // device address of the mapped host word, or null
};
int *device_status_ptr();

__device__ __forceinline__ void record_device_error(int *status, int code) {
  atomicCAS(status, 0, code);
  int *mirror = reinterpret_cast<DeviceStatus *>(status)->mirror;
  if (mirror) *reinterpret_cast<volatile int *>(mirror) = code;  // a plain store: host memory
}

// PC2D_ERR_TIMEOUT (with a message) when a kernel of this context has
// recorded a device-side error that pc2d_clear_device_status() has not
// cleared yet, else PC2D_OK.  Reads the host mirror: no synchronisation.
int pending_device_error();

// Set by pc2d_forward_noalloc for the duration of its call: nothing on that
// path may allocate, so the host mirror is not created there.
extern thread_local bool t_no_alloc;

// Host-side error message of the last failing ABI call on this thread.
void set_last_error(const char *fmt, ...);

// Optional per-kernel timing (pc2d_timing_*): brackets a launch with CUDA
// events when enabled.  Kernel families are indexed by KernelId.
enum KernelId { K_FORWARD = 0, K_DGRAD, K_WGRAD, K_SIMT_FORWARD, K_SIMT_DGRAD, K_SIMT_WGRAD, K_COUNT };
void timing_begin(KernelId id, cudaStream_t stream);
void timing_end(KernelId id, cudaStream_t stream);

// Launchers implemented by the kernel translation units.
template <typename T>
int simt_forward(const Problem &p, const T *x, const T *pars, double factor, T *out, T *hsum,
                 cudaStream_t stream);
template <typename T>
size_t simt_backward_workspace(const Problem &p, bool skip_input_grad);
// Zero-padded, scaled copy of an [n][C][H][W] input (pc2d_pad.cu).
int pad_scale(int dtype, const void *in, int n, int C, int H, int W, int pt, int pb, int pl, int pr, double scale,
              void *out, cudaStream_t stream);
// With leave_dx the input gradient is neither computed nor written; with
// skip_wgrad only the input gradient is computed.  dx is written as `dxo`
// describes (skip_input_grad: zeros, when dx is not null).
template <typename T>
int simt_backward(const Problem &p, const T *grad, const T *x, const T *pars, const T *hsum,
                  double factor, bool skip_input_grad, T *dx, T *dpars, void *ws, size_t ws_bytes,
                  cudaStream_t stream, const DxOut &dxo, bool leave_dx = false, bool skip_wgrad = false);

}  // namespace pc2d

#define PC2D_CUDA_CHECK(call)                                                          \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess) {                                                           \
      pc2d::set_last_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_),      \
                           __FILE__, __LINE__);                                         \
      return PC2D_ERR_CUDA;                                                            \
    }                                                                                  \
  } while (0)

#define PC2D_LAUNCH_CHECK(what)                                                        \
  do {                                                                                 \
    cudaError_t e_ = cudaGetLastError();                                               \
    if (e_ != cudaSuccess) {                                                           \
      pc2d::set_last_error("launch of %s failed: %s", what, cudaGetErrorString(e_));   \
      return PC2D_ERR_CUDA;                                                            \
    }                                                                                  \
  } while (0)
