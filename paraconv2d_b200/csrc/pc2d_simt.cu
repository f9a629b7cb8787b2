// CUDA-core (FMA) kernels of the ParaConv2d forward and backward passes, in
// fp32 and fp64.  They serve the fp64 dispatch of the op (reference
// AT_DISPATCH_FLOATING_TYPES, paraconv2d.cc:322,419) and every fp32 shape the
// tcgen05 kernels do not take.
//
// Every kernel is a tiled implicit GEMM over the flipped window
// (reference paraconv2d.cc:89-92).  Reductions are hierarchical and
// deterministic: no floating-point atomics anywhere, so two runs give the same
// bits.
//
//   forward   rows = output pixels (n*P*Q), cols = output channels,
//             K = window (C*k0*k1); accumulates hsum = h0 + h.win and
//             q = sum (win - p)^2 directly (reference paraconv2d.cc:82-122).
//   dgrad     rows = input pixels (n*H*W), cols = input channels,
//             K = taps x output channels; dx = 2 (sum g*hsum*h + g*p
//             - x * sum g)  (reference paraconv2d.cc:153-183).
//   wgrad     rows = output channels, cols = window elements,
//             K = output pixels split across CTAs; the per-CTA partial
//             sums are reduced in fixed order by a second kernel that also
//             applies the 2f scale and the -p*sum(g) term of dp
//             (reference paraconv2d.cc:186-237).
#include <algorithm>

#include "pc2d_common.cuh"

namespace pc2d {
namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------------- forward
constexpr int FM = 64, FN = 64, FK = 16;

template <typename T>
__global__ void __launch_bounds__(kThreads)
simt_forward_kernel(const T *__restrict__ x, const T *__restrict__ pars, T factor, Problem p,
                    T *__restrict__ out, T *__restrict__ hsum) {
  __shared__ T xs[FK][FM];
  __shared__ T hw[FK][FN];
  __shared__ T pw[FK][FN];
  __shared__ int64_t pbase[FM];

  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int64_t g0 = (int64_t)blockIdx.x * FM;
  const int j0 = blockIdx.y * FN;
  const int m = p.m;
  const int d = (int)p.d;
  const T *h0 = pars;
  const T *h = pars + m;
  const T *pp = h + (int64_t)m * d;
  const T *p0 = pp + (int64_t)m * d;

  if (tid < FM) {
    const int64_t g = g0 + tid;
    if (g < p.NPQ) {
      const int64_t nn = g / p.PQ;
      const int64_t r = g - nn * p.PQ;
      const int oy = (int)(r / p.Q), ox = (int)(r - (int64_t)oy * p.Q);
      pbase[tid] = nn * p.CHW + (int64_t)oy * p.s0 * p.W + (int64_t)ox * p.s1;
    } else {
      pbase[tid] = -1;
    }
  }
  T acc_h[4][4], acc_q[4][4];
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const int j = j0 + ty + 16 * jj;
    const T init = (j < m) ? h0[j] : T(0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc_h[i][jj] = init;
      acc_q[i][jj] = T(0);
    }
  }
  __syncthreads();

  for (int kc = 0; kc < d; kc += FK) {
    for (int e = tid; e < FK * FM; e += kThreads) {
      const int kk = e / FM, px = e % FM;
      const int k = kc + kk;
      const int64_t b = pbase[px];
      T v = T(0);
      if (b >= 0 && k < d) {
        const int c = k / p.T, tap = k - c * p.T;
        v = x[b + (int64_t)c * p.HW + (int64_t)tap_row(p, tap) * p.W + tap_col(p, tap)];
      }
      xs[kk][px] = v;
    }
    for (int e = tid; e < FK * FN; e += kThreads) {
      const int jn = e / FK, kk = e % FK;
      const int j = j0 + jn, k = kc + kk;
      T hv = T(0), pv = T(0);
      if (j < m && k < d) {
        hv = h[(int64_t)j * d + k];
        pv = pp[(int64_t)j * d + k];
      }
      hw[kk][jn] = hv;
      pw[kk][jn] = pv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < FK; ++kk) {
      T a[4], bh[4], bp[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = xs[kk][tx + 16 * i];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        bh[jj] = hw[kk][ty + 16 * jj];
        bp[jj] = pw[kk][ty + 16 * jj];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          acc_h[i][jj] = fma(a[i], bh[jj], acc_h[i][jj]);
          const T t = a[i] - bp[jj];
          acc_q[i][jj] = fma(t, t, acc_q[i][jj]);
        }
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t g = g0 + tx + 16 * i;
    if (g >= p.NPQ) continue;
    const int64_t nn = g / p.PQ;
    const int64_t r = g - nn * p.PQ;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = j0 + ty + 16 * jj;
      if (j >= m) continue;
      const T hs = acc_h[i][jj];
      const T o = ((hs * hs - acc_q[i][jj]) - p0[j] * p0[j]) * factor;
      const int64_t oi = (nn * m + j) * p.PQ + r;
      out[oi] = o;
      hsum[oi] = hs;
    }
  }
}

// ---------------------------------------------------------------- dgrad
constexpr int DM = 64, DC = 64, DK = 16;

template <typename T>
__global__ void __launch_bounds__(kThreads)
simt_dgrad_kernel(const T *__restrict__ grad, const T *__restrict__ x, const T *__restrict__ pars,
                  const T *__restrict__ hsum, Problem p, DxOut dxo, T *__restrict__ dx) {
  __shared__ T a1s[DK][DM], a2s[DK][DM];
  __shared__ T bhs[DK][DC], bps[DK][DC];
  __shared__ int64_t obase[DM];
  __shared__ int pyx[DM][2];
  __shared__ int oidx[DM];

  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int64_t g0 = (int64_t)blockIdx.x * DM;
  const int c0 = blockIdx.y * DC;
  const int m = p.m;
  const int d = (int)p.d;
  const T *h = pars + m;
  const T *pp = h + (int64_t)m * d;

  if (tid < DM) {
    const int64_t g = g0 + tid;
    if (g < p.NHW) {
      const int64_t nn = g / p.HW;
      const int64_t r = g - nn * p.HW;
      const int y = (int)(r / p.W);
      pyx[tid][0] = y;
      pyx[tid][1] = (int)(r - (int64_t)y * p.W);
      obase[tid] = nn * m * p.PQ;
    } else {
      obase[tid] = -1;
      pyx[tid][0] = pyx[tid][1] = 0;
    }
  }
  T acc[4][4];
  T sgb[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    sgb[i] = T(0);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) acc[i][jj] = T(0);
  }

  for (int tap = 0; tap < p.T; ++tap) {
    __syncthreads();
    if (tid < DM) {
      int o = -1;
      if (obase[tid] >= 0) {
        const int yy = pyx[tid][0] - tap_row(p, tap);
        const int xx = pyx[tid][1] - tap_col(p, tap);
        if (yy >= 0 && xx >= 0 && yy % p.s0 == 0 && xx % p.s1 == 0) {
          const int oy = yy / p.s0, ox = xx / p.s1;
          if (oy < p.P && ox < p.Q) o = oy * p.Q + ox;
        }
      }
      oidx[tid] = o;
    }
    __syncthreads();
    for (int jc = 0; jc < m; jc += DK) {
      for (int e = tid; e < DK * DM; e += kThreads) {
        const int jj = e / DM, px = e % DM;
        const int j = jc + jj;
        const int o = oidx[px];
        T v1 = T(0), v2 = T(0);
        if (o >= 0 && j < m) {
          const int64_t idx = obase[px] + (int64_t)j * p.PQ + o;
          const T gv = grad[idx];
          v1 = gv * hsum[idx];
          v2 = gv;
        }
        a1s[jj][px] = v1;
        a2s[jj][px] = v2;
      }
      for (int e = tid; e < DK * DC; e += kThreads) {
        const int jj = e / DC, cc = e % DC;
        const int j = jc + jj, c = c0 + cc;
        T hv = T(0), pv = T(0);
        if (j < m && c < p.C) {
          const int64_t wi = (int64_t)j * d + (int64_t)c * p.T + tap;
          hv = h[wi];
          pv = pp[wi];
        }
        bhs[jj][cc] = hv;
        bps[jj][cc] = pv;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < DK; ++kk) {
        T a1[4], a2[4], bh[4], bp[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a1[i] = a1s[kk][tx + 16 * i];
          a2[i] = a2s[kk][tx + 16 * i];
          sgb[i] += a2[i];
        }
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          bh[jj] = bhs[kk][ty + 16 * jj];
          bp[jj] = bps[kk][ty + 16 * jj];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) acc[i][jj] = fma(a1[i], bh[jj], fma(a2[i], bp[jj], acc[i][jj]));
      }
      __syncthreads();
    }
  }

  const T two_s = T(2) * (T)dxo.scale;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t g = g0 + tx + 16 * i;
    if (g >= p.NHW) continue;
    const int64_t nn = g / p.HW;
    const int64_t r = g - nn * p.HW;
    const int y = (int)(r / p.W);
    const int64_t ob = dx_index(dxo, nn, y, (int)(r - (int64_t)y * p.W));
    if (ob < 0) continue;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int c = c0 + ty + 16 * jj;
      if (c >= p.C) continue;
      const int64_t xi = nn * p.CHW + (int64_t)c * p.HW + r;
      dx[ob + (int64_t)c * dxo.HWu] = two_s * (acc[i][jj] - x[xi] * sgb[i]);
    }
  }
}

// ---------------------------------------------------------------- wgrad
constexpr int WJ = 32, WK = 64, WP = 16;

template <typename T>
__global__ void __launch_bounds__(kThreads)
simt_wgrad_kernel(const T *__restrict__ grad, const T *__restrict__ x, const T *__restrict__ hsum, Problem p,
                  int64_t pix_per_split, T *__restrict__ part, T *__restrict__ sums) {
  __shared__ T g1s[WP][WJ], g2s[WP][WJ];
  __shared__ T cs[WP][WK];
  __shared__ int64_t pin[WP], pout[WP];
  __shared__ int64_t koff[WK];

  const int tid = threadIdx.x;
  const int tk = tid % 16, tj = tid / 16;
  const int k0 = blockIdx.x * WK;
  const int j0 = blockIdx.y * WJ;
  const int z = blockIdx.z;
  const int m = p.m;
  const int d = (int)p.d;
  const int64_t gbeg = (int64_t)z * pix_per_split;
  const int64_t gend = std::min<int64_t>(p.NPQ, gbeg + pix_per_split);

  if (tid < WK) {
    const int k = k0 + tid;
    if (k < d) {
      const int c = k / p.T, tap = k - c * p.T;
      koff[tid] = (int64_t)c * p.HW + (int64_t)tap_row(p, tap) * p.W + tap_col(p, tap);
    } else {
      koff[tid] = -1;
    }
  }
  T acc1[2][4], acc2[2][4], s1[2], s2[2];
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    s1[jj] = s2[jj] = T(0);
#pragma unroll
    for (int i = 0; i < 4; ++i) acc1[jj][i] = acc2[jj][i] = T(0);
  }

  for (int64_t gc = gbeg; gc < gend; gc += WP) {
    __syncthreads();
    if (tid < WP) {
      const int64_t g = gc + tid;
      if (g < gend) {
        const int64_t nn = g / p.PQ;
        const int64_t r = g - nn * p.PQ;
        const int oy = (int)(r / p.Q), ox = (int)(r - (int64_t)oy * p.Q);
        pin[tid] = nn * p.CHW + (int64_t)oy * p.s0 * p.W + (int64_t)ox * p.s1;
        pout[tid] = nn * m * p.PQ + r;
      } else {
        pin[tid] = -1;
        pout[tid] = 0;
      }
    }
    __syncthreads();
    for (int e = tid; e < WP * WJ; e += kThreads) {
      const int jj = e / WP, px = e % WP;
      const int j = j0 + jj;
      T v1 = T(0), v2 = T(0);
      if (pin[px] >= 0 && j < m) {
        const int64_t idx = pout[px] + (int64_t)j * p.PQ;
        const T gv = grad[idx];
        v1 = gv * hsum[idx];
        v2 = gv;
      }
      g1s[px][jj] = v1;
      g2s[px][jj] = v2;
    }
    for (int e = tid; e < WP * WK; e += kThreads) {
      const int kk = e / WP, px = e % WP;
      T v = T(0);
      if (pin[px] >= 0 && koff[kk] >= 0) v = x[pin[px] + koff[kk]];
      cs[px][kk] = v;
    }
    __syncthreads();
#pragma unroll
    for (int px = 0; px < WP; ++px) {
      T a1[2], a2[2], b[4];
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        a1[jj] = g1s[px][tj + 16 * jj];
        a2[jj] = g2s[px][tj + 16 * jj];
        s1[jj] += a1[jj];
        s2[jj] += a2[jj];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) b[i] = cs[px][tk + 16 * i];
#pragma unroll
      for (int jj = 0; jj < 2; ++jj)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc1[jj][i] = fma(a1[jj], b[i], acc1[jj][i]);
          acc2[jj][i] = fma(a2[jj], b[i], acc2[jj][i]);
        }
    }
  }

#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    const int j = j0 + tj + 16 * jj;
    if (j >= m) continue;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = k0 + tk + 16 * i;
      if (k >= d) continue;
      part[((int64_t)(2 * z + 0) * m + j) * d + k] = acc1[jj][i];
      part[((int64_t)(2 * z + 1) * m + j) * d + k] = acc2[jj][i];
    }
    if (blockIdx.x == 0 && tk == 0) {
      sums[(int64_t)(2 * z + 0) * m + j] = s1[jj];
      sums[(int64_t)(2 * z + 1) * m + j] = s2[jj];
    }
  }
}

// Fixed-order reduction of the wgrad partials and the parameter-gradient
// epilogue (reference paraconv2d.cc:186-237):
//   dh0 = 2f sum g*hsum        dh = 2f sum g*hsum*win
//   dp  = 2f (sum g*win - p * sum g)     dp0 = 2f * (-p0) * sum g
template <typename T>
__global__ void __launch_bounds__(kThreads)
simt_wgrad_finalize_kernel(const T *__restrict__ part, const T *__restrict__ sums, int splits,
                           const T *__restrict__ pars, Problem p, double f2, T *__restrict__ dpars) {
  __shared__ double s_sums[2];
  const int m = p.m;
  const int d = (int)p.d;
  const int j = blockIdx.y;
  const int k = blockIdx.x * kThreads + threadIdx.x;
  if (threadIdx.x < 32) {
    double a = 0.0, b = 0.0;
    for (int z = threadIdx.x; z < splits; z += 32) {
      a += (double)sums[(int64_t)(2 * z + 0) * m + j];
      b += (double)sums[(int64_t)(2 * z + 1) * m + j];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      a += __shfl_down_sync(0xffffffffu, a, off);
      b += __shfl_down_sync(0xffffffffu, b, off);
    }
    if (threadIdx.x == 0) {
      s_sums[0] = a;
      s_sums[1] = b;
    }
  }
  __syncthreads();
  const double sg1 = s_sums[0], sg = s_sums[1];
  const T *pp = pars + m + (int64_t)m * d;
  const T *p0 = pp + (int64_t)m * d;
  T *dh0 = dpars, *dh = dpars + m, *dpp = dh + (int64_t)m * d, *dp0 = dpp + (int64_t)m * d;
  if (k < d) {
    double ah = 0.0, ap = 0.0;
    for (int z = 0; z < splits; ++z) {
      ah += (double)part[((int64_t)(2 * z + 0) * m + j) * d + k];
      ap += (double)part[((int64_t)(2 * z + 1) * m + j) * d + k];
    }
    const int64_t wi = (int64_t)j * d + k;
    dh[wi] = (T)(f2 * ah);
    dpp[wi] = (T)(f2 * (ap - (double)pp[wi] * sg));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    dh0[j] = (T)(f2 * sg1);
    dp0[j] = (T)(f2 * (-(double)p0[j]) * sg);
  }
}

// Number of pixel splits of the wgrad GEMM (K = n*P*Q split across CTAs).
inline int wgrad_splits(const Problem &p) {
  const int tiles = ceil_div(p.d, WK) * ceil_div(p.m, WJ);
  int splits = std::max(1, (148 * 4) / std::max(1, tiles));
  splits = std::min<int64_t>(splits, std::max<int64_t>(1, ceil_div(p.NPQ, WP * 4)));
  return std::max(1, splits);
}

}  // namespace

template <typename T>
int simt_forward(const Problem &p, const T *x, const T *pars, double factor, T *out, T *hsum,
                 cudaStream_t stream) {
  if (p.NPQ == 0 || p.m == 0) return PC2D_OK;
  const dim3 grid(ceil_div(p.NPQ, FM), ceil_div(p.m, FN));
  if (grid.y > 65535) {
    set_last_error("too many output channels for the CUDA-core forward (m=%d)", p.m);
    return PC2D_ERR_UNSUPPORTED;
  }
  timing_begin(K_SIMT_FORWARD, stream);
  simt_forward_kernel<T><<<grid, kThreads, 0, stream>>>(x, pars, (T)factor, p, out, hsum);
  timing_end(K_SIMT_FORWARD, stream);
  PC2D_LAUNCH_CHECK("simt_forward_kernel");
  return PC2D_OK;
}

template <typename T>
size_t simt_backward_workspace(const Problem &p, bool) {
  if (p.m == 0 || p.d == 0) return 0;
  const int splits = wgrad_splits(p);
  const size_t part = align_up((size_t)splits * 2 * p.m * p.d * sizeof(T), 256);
  const size_t sums = align_up((size_t)splits * 2 * p.m * sizeof(T), 256);
  return part + sums;
}

template <typename T>
int simt_backward(const Problem &p, const T *grad, const T *x, const T *pars, const T *hsum,
                  double factor, bool skip_input_grad, T *dx, T *dpars, void *ws, size_t ws_bytes,
                  cudaStream_t stream, const DxOut &dxo, bool leave_dx, bool skip_wgrad) {
  const size_t npars = (size_t)p.m * 2 * (p.d + 1);
  if (leave_dx) {
  } else if (skip_input_grad || p.NPQ == 0) {
    if (p.NHW > 0 && dx) PC2D_CUDA_CHECK(cudaMemsetAsync(dx, 0, sizeof(T) * (size_t)p.n * dxo.CHWu, stream));
  } else {
    const dim3 grid(ceil_div(p.NHW, DM), ceil_div(p.C, DC));
    timing_begin(K_SIMT_DGRAD, stream);
    simt_dgrad_kernel<T><<<grid, kThreads, 0, stream>>>(grad, x, pars, hsum, p, dxo, dx);
    timing_end(K_SIMT_DGRAD, stream);
    PC2D_LAUNCH_CHECK("simt_dgrad_kernel");
  }
  if (npars == 0 || skip_wgrad) return PC2D_OK;
  if (p.NPQ == 0) {
    PC2D_CUDA_CHECK(cudaMemsetAsync(dpars, 0, sizeof(T) * npars, stream));
    return PC2D_OK;
  }
  const int splits = wgrad_splits(p);
  const size_t part_bytes = align_up((size_t)splits * 2 * p.m * p.d * sizeof(T), 256);
  if (ws_bytes < simt_backward_workspace<T>(p, skip_input_grad) || ws == nullptr) {
    set_last_error("backward workspace too small: %zu < %zu", ws_bytes, simt_backward_workspace<T>(p, skip_input_grad));
    return PC2D_ERR_WORKSPACE;
  }
  T *part = reinterpret_cast<T *>(ws);
  T *sums = reinterpret_cast<T *>(reinterpret_cast<char *>(ws) + part_bytes);
  int64_t pix_per_split = (p.NPQ + splits - 1) / splits;
  pix_per_split = (pix_per_split + WP - 1) / WP * WP;
  const dim3 grid(ceil_div(p.d, WK), ceil_div(p.m, WJ), splits);
  timing_begin(K_SIMT_WGRAD, stream);
  simt_wgrad_kernel<T><<<grid, kThreads, 0, stream>>>(grad, x, hsum, p, pix_per_split, part, sums);
  timing_end(K_SIMT_WGRAD, stream);
  PC2D_LAUNCH_CHECK("simt_wgrad_kernel");
  const dim3 fgrid(ceil_div(p.d, kThreads), p.m);
  simt_wgrad_finalize_kernel<T><<<fgrid, kThreads, 0, stream>>>(part, sums, splits, pars, p, 2.0 * (double)(T)factor, dpars);
  PC2D_LAUNCH_CHECK("simt_wgrad_finalize_kernel");
  return PC2D_OK;
}

template int simt_forward<float>(const Problem &, const float *, const float *, double, float *, float *, cudaStream_t);
template int simt_forward<double>(const Problem &, const double *, const double *, double, double *, double *, cudaStream_t);
template size_t simt_backward_workspace<float>(const Problem &, bool);
template size_t simt_backward_workspace<double>(const Problem &, bool);
template int simt_backward<float>(const Problem &, const float *, const float *, const float *, const float *, double, bool,
                                  float *, float *, void *, size_t, cudaStream_t, const DxOut &, bool, bool);
template int simt_backward<double>(const Problem &, const double *, const double *, const double *, const double *, double,
                                   bool, double *, double *, void *, size_t, cudaStream_t, const DxOut &, bool, bool);

}  // namespace pc2d
