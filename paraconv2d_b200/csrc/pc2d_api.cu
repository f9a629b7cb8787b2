// The C ABI of libpc2d_sm100.so (declared in include/paraconv2d.h): argument
// validation, workspace sizing and dispatch between the tcgen05 tensor-core
// kernels (fp32) and the CUDA-core kernels (fp32/fp64).
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <cstddef>
#include <cstring>
#include <mutex>
#include <vector>

#include <cuda.h>  // CUcontext, CUresult (types only; entry points resolved at run time)

#include "pc2d_common.cuh"
#include "pc2d_tc.cuh"

namespace pc2d {

__device__ DeviceStatus g_device_status = {0, 0, nullptr};
thread_local bool t_no_alloc = false;

namespace {
thread_local char t_last_error[512] = "";

// ------------------------------------------------------------ kernel timing
const char *const kKernelNames[K_COUNT] = {"forward", "dgrad", "wgrad", "simt_forward", "simt_dgrad", "simt_wgrad"};
struct TimingState {
  std::mutex mu;
  bool on = false;
  std::vector<cudaEvent_t> pool;  // events free for reuse
  struct Rec {
    int id;
    cudaEvent_t a, b;
  };
  std::vector<Rec> recs;
  cudaEvent_t pending[K_COUNT] = {};
};
TimingState g_timing;

cudaEvent_t timing_event() {
  if (!g_timing.pool.empty()) {
    cudaEvent_t e = g_timing.pool.back();
    g_timing.pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}
std::atomic<int> g_algo{PC2D_ALGO_AUTO};
PerContext<int *> g_status_ptrs;
PerContext<volatile int *> g_status_mirrors;  // host address of each context's mapped word

// cuCtxGetCurrent and cuCtxGetId, resolved once through the runtime (the
// library links the CUDA runtime only).
using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);
struct CtxFns {
  CtxGetCurrentFn get_current = nullptr;
  CtxGetIdFn get_id = nullptr;
};
const CtxFns &ctx_fns() {
  static CtxFns fns;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fns.get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fns.get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  return fns;
}
}  // namespace

unsigned long long current_context_id() {
  const CtxFns &f = ctx_fns();
  if (!f.get_current || !f.get_id) return 0;
  CUcontext ctx = nullptr;
  if (f.get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (f.get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

void set_last_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

void timing_begin(KernelId id, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(g_timing.mu);
  if (!g_timing.on) return;
  cudaEvent_t e = timing_event();
  if (e && cudaEventRecord(e, stream) == cudaSuccess) g_timing.pending[id] = e;
}

void timing_end(KernelId id, cudaStream_t stream) {
  std::lock_guard<std::mutex> lock(g_timing.mu);
  if (!g_timing.on || !g_timing.pending[id]) return;
  cudaEvent_t e = timing_event();
  if (e && cudaEventRecord(e, stream) == cudaSuccess) g_timing.recs.push_back({(int)id, g_timing.pending[id], e});
  g_timing.pending[id] = nullptr;
}

int *device_status_ptr() {
  unsigned long long ctx = current_context_id();
  int *cached = nullptr;
  if (ctx && g_status_ptrs.get(ctx, &cached)) return cached;
  void *ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, g_device_status) != cudaSuccess) return nullptr;
  // the lookup may have made the device's primary context current
  if (!ctx) ctx = current_context_id();
  // the host mirror of the status word: pinned, mapped into the device, made
  // once per context (not on the no-allocation path, which then runs without
  // it until a regular call has made it)
  if (ctx && !t_no_alloc) {
    void *host = nullptr, *dev = nullptr;
    if (cudaHostAlloc(&host, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) return nullptr;
    *reinterpret_cast<volatile int *>(host) = 0;
    if (cudaHostGetDevicePointer(&dev, host, 0) != cudaSuccess ||
        cudaMemcpyToSymbol(g_device_status, &dev, sizeof(dev), offsetof(DeviceStatus, mirror)) != cudaSuccess) {
      cudaFreeHost(host);
      return nullptr;
    }
    g_status_mirrors.set(ctx, reinterpret_cast<volatile int *>(host));
    g_status_ptrs.set(ctx, reinterpret_cast<int *>(ptr));
  }
  return reinterpret_cast<int *>(ptr);
}

int pending_device_error() {
  const unsigned long long ctx = current_context_id();
  volatile int *mirror = nullptr;
  if (!ctx || !g_status_mirrors.get(ctx, &mirror) || *mirror == 0) return PC2D_OK;
  set_last_error("a kernel of an earlier call gave up waiting on the device (%s); its results are invalid. "
                 "pc2d_clear_device_status() clears this state",
                 pc2d_status_string(*mirror));
  return PC2D_ERR_TIMEOUT;
}

namespace {

// Shape and argument checks shared by forward and backward.  The reference op
// performs none (its launches fail silently, paraconv2d.cu:101-219); these
// turn every invalid call into PC2D_ERR_INVALID_ARGUMENT with a message.
int validate(int dtype, int n, int C, int H, int W, int m, int k0, int k1, int s0, int s1, int dl0,
             int dl1, Problem *out) {
  if (dtype != PC2D_DTYPE_F32 && dtype != PC2D_DTYPE_F64) {
    set_last_error("unsupported dtype %d (float32 and float64 only, as the reference)", dtype);
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  if (n < 0 || C <= 0 || H <= 0 || W <= 0 || m < 0) {
    set_last_error("invalid input shape n=%d C=%d H=%d W=%d m=%d", n, C, H, W, m);
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  if (k0 <= 0 || k1 <= 0 || s0 <= 0 || s1 <= 0 || dl0 <= 0 || dl1 <= 0) {
    set_last_error("kernel_size, stride and dilation must be positive (got k=%dx%d s=%dx%d dl=%dx%d)", k0, k1,
                   s0, s1, dl0, dl1);
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  if (k0 % 2 == 0 || k1 % 2 == 0) {
    set_last_error("even kernel size %dx%d: the reference window for even sizes reads outside the window "
                   "(paraconv2d.cc:89-92); only odd sizes are supported", k0, k1);
    return PC2D_ERR_UNSUPPORTED;
  }
  Problem p = make_problem(n, C, H, W, m, k0, k1, s0, s1, dl0, dl1);
  if (p.P <= 0 || p.Q <= 0) {
    set_last_error("input %dx%d is smaller than the dilated kernel %dx%d", H, W, dl0 * (k0 - 1) + 1,
                   dl1 * (k1 - 1) + 1);
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  if (p.d > (int64_t)1 << 30 || p.NHW * C > ((int64_t)1 << 40) || p.NPQ * (int64_t)(m > 0 ? m : 1) > ((int64_t)1 << 40)) {
    set_last_error("problem too large");
    return PC2D_ERR_UNSUPPORTED;
  }
  *out = p;
  return PC2D_OK;
}

bool use_tc_fwd(const Problem &p, int dtype) {
  const int algo = g_algo.load();
  if (dtype != PC2D_DTYPE_F32 || algo == PC2D_ALGO_SIMT) return false;
  return tc_forward_supported(p);
}

bool use_tc_bwd(const Problem &p, int dtype) {
  const int algo = g_algo.load();
  if (dtype != PC2D_DTYPE_F32 || algo == PC2D_ALGO_SIMT) return false;
  return tc_backward_supported(p);
}

}  // namespace
}  // namespace pc2d

using namespace pc2d;

extern "C" {

int pc2d_abi_version(void) { return PC2D_ABI_VERSION; }

int pc2d_out_size(int in, int kernel, int stride, int dilation) {
  if (stride <= 0) return 0;
  return ((in - (dilation * (kernel - 1)) - 1) / stride) + 1;
}

int64_t pc2d_infer_m(int64_t npars, int channels, int k0, int k1) {
  const int64_t d = (int64_t)channels * k0 * k1;
  if (d <= 0 || npars <= 0 || npars % (2 * (d + 1)) != 0) return -1;
  return npars / (2 * (d + 1));
}

int pc2d_set_algo(int algo) {
  if (algo < PC2D_ALGO_AUTO || algo > PC2D_ALGO_TC) return -1;
  return g_algo.exchange(algo);
}

int pc2d_get_algo(void) { return g_algo.load(); }

size_t pc2d_forward_workspace_size(int dtype, int n, int channels, int height, int width, int m, int k0, int k1,
                                   int s0, int s1, int dl0, int dl1) {
  Problem p;
  if (validate(dtype, n, channels, height, width, m, k0, k1, s0, s1, dl0, dl1, &p) != PC2D_OK) return 0;
  if (use_tc_fwd(p, dtype)) return tc_forward_workspace(p);
  return 0;
}

int pc2d_forward(int dtype, const void *input, const void *pars, double factor, int k0, int k1, int s0, int s1,
                 int dl0, int dl1, int n, int channels, int height, int width, int m, void *output, void *hsum,
                 void *workspace, size_t workspace_bytes, void *stream) {
  NvtxRange range("pc2d_forward");
  Problem p;
  int st = validate(dtype, n, channels, height, width, m, k0, k1, s0, s1, dl0, dl1, &p);
  if (st != PC2D_OK) return st;
  if ((st = pending_device_error()) != PC2D_OK) return st;
  if (p.NPQ == 0 || m == 0) return PC2D_OK;
  if (!input || !pars || !output || !hsum) {
    set_last_error("null tensor pointer");
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (use_tc_fwd(p, dtype)) {
    const size_t need = tc_forward_workspace(p);
    if (workspace_bytes < need || (need > 0 && (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255)))) {
      set_last_error("forward workspace: need %zu bytes, 256-byte aligned (got %zu)", need, workspace_bytes);
      return PC2D_ERR_WORKSPACE;
    }
    return tc_forward(p, (const float *)input, (const float *)pars, factor, (float *)output, (float *)hsum, workspace,
                      s);
  }
  if (g_algo.load() == PC2D_ALGO_TC) {
    set_last_error("tensor-core forward requested but not available for this problem");
    return PC2D_ERR_UNSUPPORTED;
  }
  if (dtype == PC2D_DTYPE_F32)
    return simt_forward<float>(p, (const float *)input, (const float *)pars, factor, (float *)output,
                               (float *)hsum, s);
  return simt_forward<double>(p, (const double *)input, (const double *)pars, factor, (double *)output,
                              (double *)hsum, s);
}

size_t pc2d_backward_workspace_size(int dtype, int n, int channels, int height, int width, int m, int k0, int k1,
                                    int s0, int s1, int dl0, int dl1, int skip_input_grad) {
  Problem p;
  if (validate(dtype, n, channels, height, width, m, k0, k1, s0, s1, dl0, dl1, &p) != PC2D_OK) return 0;
  if (use_tc_bwd(p, dtype)) return tc_backward_workspace(p, skip_input_grad != 0);
  if (dtype == PC2D_DTYPE_F32) return simt_backward_workspace<float>(p, skip_input_grad != 0);
  return simt_backward_workspace<double>(p, skip_input_grad != 0);
}

}  // extern "C"

namespace {

// Backward pass with the input gradient written as `dxo` describes; with
// dx_optional, inputgrad may be null when skip_input_grad is set.
int backward_impl(int dtype, const void *grad, const void *input, const void *pars, const void *hsum, double factor,
                  int k0, int k1, int s0, int s1, int dl0, int dl1, int n, int channels, int height, int width, int m,
                  int skip_input_grad, const DxOut *dxo_in, bool dx_optional, void *inputgrad, void *parsgrad,
                  void *workspace, size_t workspace_bytes, void *stream) {
  Problem p;
  int st = validate(dtype, n, channels, height, width, m, k0, k1, s0, s1, dl0, dl1, &p);
  if (st != PC2D_OK) return st;
  if ((st = pending_device_error()) != PC2D_OK) return st;
  const DxOut dxo = dxo_in ? *dxo_in : dx_full(p);
  const bool need_dx = (int64_t)p.n * dxo.CHWu > 0 && !(dx_optional && skip_input_grad && !inputgrad);
  const bool need_dp = m > 0;
  if ((need_dx && !inputgrad) || (need_dp && !parsgrad) || (p.NPQ > 0 && m > 0 && (!grad || !input || !pars || !hsum))) {
    set_last_error("null tensor pointer");
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255)) {
    set_last_error("workspace must be 256-byte aligned");
    return PC2D_ERR_WORKSPACE;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (m == 0) {
    if (need_dx)
      PC2D_CUDA_CHECK(cudaMemsetAsync(inputgrad, 0, (dtype == PC2D_DTYPE_F32 ? 4 : 8) * (size_t)p.n * dxo.CHWu, s));
    return PC2D_OK;
  }
  if (use_tc_bwd(p, dtype)) {
    const size_t need = tc_backward_workspace(p, skip_input_grad != 0);
    if (workspace_bytes < need || (need > 0 && workspace == nullptr)) {
      set_last_error("backward workspace: need %zu bytes (got %zu)", need, workspace_bytes);
      return PC2D_ERR_WORKSPACE;
    }
    return tc_backward(p, (const float *)grad, (const float *)input, (const float *)pars, (const float *)hsum, factor,
                       skip_input_grad != 0, (float *)inputgrad, (float *)parsgrad, workspace, workspace_bytes, s, dxo);
  }
  if (g_algo.load() == PC2D_ALGO_TC) {
    set_last_error("tensor-core backward requested but not available for this problem");
    return PC2D_ERR_UNSUPPORTED;
  }
  if (dtype == PC2D_DTYPE_F32)
    return simt_backward<float>(p, (const float *)grad, (const float *)input, (const float *)pars,
                                (const float *)hsum, factor, skip_input_grad != 0, (float *)inputgrad,
                                (float *)parsgrad, workspace, workspace_bytes, s, dxo);
  return simt_backward<double>(p, (const double *)grad, (const double *)input, (const double *)pars,
                               (const double *)hsum, factor, skip_input_grad != 0, (double *)inputgrad,
                               (double *)parsgrad, workspace, workspace_bytes, s, dxo);
}

}  // namespace

extern "C" {

int pc2d_backward(int dtype, const void *grad, const void *input, const void *pars, const void *hsum, double factor,
                  int k0, int k1, int s0, int s1, int dl0, int dl1, int n, int channels, int height, int width, int m,
                  int skip_input_grad, void *inputgrad, void *parsgrad, void *workspace, size_t workspace_bytes,
                  void *stream) {
  NvtxRange range("pc2d_backward");
  return backward_impl(dtype, grad, input, pars, hsum, factor, k0, k1, s0, s1, dl0, dl1, n, channels, height, width,
                       m, skip_input_grad, nullptr, false, inputgrad, parsgrad, workspace, workspace_bytes, stream);
}

int pc2d_backward_interior(int dtype, const void *grad, const void *input, const void *pars, const void *hsum,
                           double factor, int k0, int k1, int s0, int s1, int dl0, int dl1, int n, int channels,
                           int height, int width, int m, int skip_input_grad, int pad_top, int pad_bottom,
                           int pad_left, int pad_right, double dx_scale, void *inputgrad, void *parsgrad,
                           void *workspace, size_t workspace_bytes, void *stream) {
  NvtxRange range("pc2d_backward_interior");
  if (pad_top < 0 || pad_bottom < 0 || pad_left < 0 || pad_right < 0 || pad_top + pad_bottom > height ||
      pad_left + pad_right > width) {
    set_last_error("invalid padding %d/%d/%d/%d of a %dx%d input", pad_top, pad_bottom, pad_left, pad_right, height,
                   width);
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  DxOut o;
  o.pt = pad_top;
  o.pl = pad_left;
  o.Hu = height - pad_top - pad_bottom;
  o.Wu = width - pad_left - pad_right;
  o.HWu = (int64_t)o.Hu * o.Wu;
  o.CHWu = (int64_t)(channels > 0 ? channels : 0) * o.HWu;
  o.scale = dx_scale;
  return backward_impl(dtype, grad, input, pars, hsum, factor, k0, k1, s0, s1, dl0, dl1, n, channels, height, width,
                       m, skip_input_grad, &o, true, inputgrad, parsgrad, workspace, workspace_bytes, stream);
}

int pc2d_pad_scale(int dtype, const void *input, int n, int channels, int height, int width, int pad_top,
                   int pad_bottom, int pad_left, int pad_right, double scale, void *output, void *stream) {
  NvtxRange range("pc2d_pad_scale");
  if (dtype != PC2D_DTYPE_F32 && dtype != PC2D_DTYPE_F64) {
    set_last_error("unsupported dtype %d (float32 and float64 only)", dtype);
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  if (n < 0 || channels < 0 || height < 0 || width < 0 || pad_top < 0 || pad_bottom < 0 || pad_left < 0 ||
      pad_right < 0) {
    set_last_error("invalid shape or padding");
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  const int64_t rows = (int64_t)n * channels * (height + pad_top + pad_bottom);
  const int Wp = width + pad_left + pad_right;
  if (rows == 0 || Wp == 0) return PC2D_OK;
  if (!output || (!input && (int64_t)n * channels * height * width > 0)) {
    set_last_error("null tensor pointer");
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  return pad_scale(dtype, input, n, channels, height, width, pad_top, pad_bottom, pad_left, pad_right, scale, output,
                   reinterpret_cast<cudaStream_t>(stream));
}

const char *pc2d_status_string(int status) {
  switch (status) {
    case PC2D_OK: return "PC2D_OK";
    case PC2D_ERR_INVALID_ARGUMENT: return "PC2D_ERR_INVALID_ARGUMENT";
    case PC2D_ERR_UNSUPPORTED: return "PC2D_ERR_UNSUPPORTED";
    case PC2D_ERR_WORKSPACE: return "PC2D_ERR_WORKSPACE";
    case PC2D_ERR_CUDA: return "PC2D_ERR_CUDA";
    case PC2D_ERR_TIMEOUT: return "PC2D_ERR_TIMEOUT";
    default: return "PC2D_UNKNOWN_STATUS";
  }
}

const char *pc2d_last_error(void) { return t_last_error; }

int pc2d_timing_enable(int on) {
  std::lock_guard<std::mutex> lock(g_timing.mu);
  g_timing.on = on != 0;
  return PC2D_OK;
}

int pc2d_timing_reset(void) {
  std::lock_guard<std::mutex> lock(g_timing.mu);
  for (auto &r : g_timing.recs) {
    cudaEventSynchronize(r.b);
    g_timing.pool.push_back(r.a);
    g_timing.pool.push_back(r.b);
  }
  g_timing.recs.clear();
  return PC2D_OK;
}

int pc2d_timing_read(const char *kernel, double *total_ms, int *launches) {
  int id = -1;
  for (int i = 0; i < K_COUNT; ++i)
    if (kernel && std::strcmp(kernel, kKernelNames[i]) == 0) id = i;
  if (id < 0 || !total_ms || !launches) {
    set_last_error("unknown kernel family '%s'", kernel ? kernel : "(null)");
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  std::lock_guard<std::mutex> lock(g_timing.mu);
  double t = 0.0;
  int n = 0;
  for (auto &r : g_timing.recs) {
    if (r.id != id) continue;
    PC2D_CUDA_CHECK(cudaEventSynchronize(r.b));
    float ms = 0.f;
    PC2D_CUDA_CHECK(cudaEventElapsedTime(&ms, r.a, r.b));
    t += ms;
    ++n;
  }
  *total_ms = t;
  *launches = n;
  return PC2D_OK;
}

int pc2d_device_status(void) {
  PC2D_CUDA_CHECK(cudaDeviceSynchronize());
  int v = 0;
  PC2D_CUDA_CHECK(cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int), offsetof(DeviceStatus, code)));
  if (v != 0) set_last_error("a device-side wait gave up (%s)", pc2d_status_string(v));
  return v;
}

int pc2d_clear_device_status(void) {
  const int zero = 0;
  PC2D_CUDA_CHECK(cudaDeviceSynchronize());
  PC2D_CUDA_CHECK(cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int), offsetof(DeviceStatus, code)));
  const unsigned long long ctx = current_context_id();
  volatile int *mirror = nullptr;
  if (ctx && g_status_mirrors.get(ctx, &mirror)) *mirror = 0;
  return PC2D_OK;
}

int pc2d_selftest_bounded_wait(unsigned int timeout_us, void *stream) {
  int *status = device_status_ptr();
  if (!status) {
    set_last_error("no device status word");
    return PC2D_ERR_CUDA;
  }
  return tc_selftest_bounded_wait(timeout_us, status, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
