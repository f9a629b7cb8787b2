// Fused SGD step on a layer's flat parameter vector [h0 | h | p | p0], with
// the learning-rate and weight-decay multipliers the module attaches to
// `pars` for the optimizer (reference ptparaconv2d.py:194-198 and its
// docstring: h_lr_factor / p_lr_factor multiply the learning rate of the
// h and p parameters, wd_factor multiplies the weight decay).
//
// Per element w with gradient g (torch.optim.SGD's update, momentum without
// dampening or Nesterov, weight decay added to the gradient):
//   d   = g + (weight_decay * wd_factor) * w
//   buf = momentum * buf + d          (buf = d on the first step; no buffer
//                                      when momentum is 0)
//   w   = w - (lr * lr_factor) * buf   lr_factor = h_lr_factor on [h0 | h],
//                                      p_lr_factor on [p | p0]
// One pass over pars, grad and the momentum buffer (HBM-bound): a grid-stride
// loop over 16-byte groups (four floats or two doubles) where the arrays are
// 16-byte aligned, then the remaining elements one by one.
#include <algorithm>

#include "pc2d_common.cuh"
#include "pc2d_tc.cuh"

namespace pc2d {
namespace {

constexpr int kStepThreads = 256;

template <typename T>
struct StepArgs {
  T *w;
  const T *g;
  T *buf;       // null: no momentum
  int64_t n;    // elements
  int64_t nh;   // elements of [h0 | h]: m * (1 + d)
  T lr_h, lr_p; // lr * h_lr_factor, lr * p_lr_factor
  T wd;         // weight_decay * wd_factor
  T mom;
  int first;    // 1: the buffer starts as d
};

template <typename T>
__device__ __forceinline__ T step_one(const StepArgs<T> &a, int64_t i, T w, T g, T *b) {
  const T d = g + a.wd * w;
  T v = d;
  if (a.buf) {
    v = a.first ? d : a.mom * *b + d;
    *b = v;
  }
  return w - (i < a.nh ? a.lr_h : a.lr_p) * v;
}

template <typename T>
__global__ void __launch_bounds__(kStepThreads) param_step_kernel(StepArgs<T> a) {
  const int64_t tid = (int64_t)blockIdx.x * kStepThreads + threadIdx.x;
  const int64_t nt = (int64_t)gridDim.x * kStepThreads;
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte vector
  const bool vec = ((reinterpret_cast<uintptr_t>(a.w) | reinterpret_cast<uintptr_t>(a.g) |
                     reinterpret_cast<uintptr_t>(a.buf)) & 15) == 0;
  int64_t done = 0;
  if (vec) {
    const int64_t nv = a.n / V;
    for (int64_t v = tid; v < nv; v += nt) {
      T w[V], g[V], b[V];
#pragma unroll
      for (int u = 0; u < V; ++u) {
        w[u] = a.w[v * V + u];
        g[u] = __ldg(a.g + v * V + u);
        b[u] = a.buf ? a.buf[v * V + u] : T(0);
      }
#pragma unroll
      for (int u = 0; u < V; ++u) w[u] = step_one(a, v * V + u, w[u], g[u], &b[u]);
#pragma unroll
      for (int u = 0; u < V; ++u) {
        a.w[v * V + u] = w[u];
        if (a.buf) a.buf[v * V + u] = b[u];
      }
    }
    done = nv * V;
  }
  for (int64_t i = done + tid; i < a.n; i += nt) {
    T b = a.buf ? a.buf[i] : T(0);
    a.w[i] = step_one(a, i, a.w[i], __ldg(a.g + i), &b);
    if (a.buf) a.buf[i] = b;
  }
}

template <typename T>
int launch_step(void *w, const void *g, void *buf, int64_t n, int64_t nh, double lr, double h_lr_factor,
                double p_lr_factor, double weight_decay, double wd_factor, double momentum, int first,
                cudaStream_t stream) {
  StepArgs<T> a;
  a.w = static_cast<T *>(w);
  a.g = static_cast<const T *>(g);
  a.buf = momentum != 0.0 ? static_cast<T *>(buf) : nullptr;
  a.n = n;
  a.nh = nh;
  a.lr_h = (T)(lr * h_lr_factor);
  a.lr_p = (T)(lr * p_lr_factor);
  a.wd = (T)(weight_decay * wd_factor);
  a.mom = (T)momentum;
  a.first = first ? 1 : 0;
  const int64_t per_block = (int64_t)kStepThreads * (16 / sizeof(T));
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + per_block - 1) / per_block,
                                                                  (int64_t)device_sm_count() * 8));
  param_step_kernel<T><<<grid, kStepThreads, 0, stream>>>(a);
  PC2D_LAUNCH_CHECK("param_step_kernel");
  return PC2D_OK;
}

}  // namespace
}  // namespace pc2d

using namespace pc2d;

extern "C" int pc2d_param_step(int dtype, void *pars, const void *grad, void *momentum_buf, int m, int d,
                               double lr, double h_lr_factor, double p_lr_factor, double weight_decay,
                               double wd_factor, double momentum, int first_step, void *stream) {
  NvtxRange range("pc2d_param_step");
  if (dtype != PC2D_DTYPE_F32 && dtype != PC2D_DTYPE_F64) {
    set_last_error("pc2d_param_step: unsupported dtype %d (float32 and float64 only)", dtype);
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  if (m < 0 || d < 0) {
    set_last_error("pc2d_param_step: invalid m %d or d %d", m, d);
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  const int64_t nh = (int64_t)m * (1 + d), n = 2 * nh;
  if (n == 0) return PC2D_OK;
  if (!pars || !grad || (momentum != 0.0 && !momentum_buf)) {
    set_last_error("pc2d_param_step: null pointer (pars, grad, or the momentum buffer with momentum != 0)");
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  int st = pending_device_error();
  if (st != PC2D_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == PC2D_DTYPE_F32)
    return launch_step<float>(pars, grad, momentum_buf, n, nh, lr, h_lr_factor, p_lr_factor, weight_decay, wd_factor,
                              momentum, first_step, s);
  return launch_step<double>(pars, grad, momentum_buf, n, nh, lr, h_lr_factor, p_lr_factor, weight_decay, wd_factor,
                             momentum, first_step, s);
}
