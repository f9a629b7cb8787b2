// The module's input preparation in one pass: out = F.pad(scale * x) with
// zeros (reference ptparaconv2d.py:216-217, `input_factor * input` then a
// constant F.pad), reading x once and writing the padded copy once instead of
// a scaled copy, a zero fill and a copy into the interior.
#include <algorithm>

#include "pc2d_common.cuh"

namespace pc2d {
namespace {

constexpr int kPadThreads = 256;

// One warp per padded row; lanes over its columns.  Rows of the padding and
// columns outside [pl, pl + W) are zeros; the rest are scale * x.
template <typename T>
__global__ void __launch_bounds__(kPadThreads) pad_scale_kernel(const T *__restrict__ in, int64_t rows, int Hp, int Wp,
                                                               int H, int W, int pt, int pl, T scale,
                                                               T *__restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t w0 = ((int64_t)blockIdx.x * kPadThreads + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * kPadThreads) >> 5;
  for (int64_t row = w0; row < rows; row += nw) {
    const int64_t plane = row / Hp;
    const int y = (int)(row - plane * Hp) - pt;
    const bool yin = (unsigned)y < (unsigned)H;
    const T *src = in + (plane * H + (yin ? y : 0)) * W;
    T *dst = out + row * Wp;
    for (int x = lane; x < Wp; x += 32) {
      const int xi = x - pl;
      T v = T(0);
      if (yin && (unsigned)xi < (unsigned)W) v = scale * __ldg(src + xi);
      dst[x] = v;
    }
  }
}

}  // namespace

int pad_scale(int dtype, const void *in, int n, int C, int H, int W, int pt, int pb, int pl, int pr, double scale,
              void *out, cudaStream_t stream) {
  const int Hp = H + pt + pb, Wp = W + pl + pr;
  const int64_t rows = (int64_t)n * C * Hp;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (rows + kPadThreads / 32 - 1) / (kPadThreads / 32);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sms * 8));
  if (dtype == PC2D_DTYPE_F32)
    pad_scale_kernel<float><<<grid, kPadThreads, 0, stream>>>((const float *)in, rows, Hp, Wp, H, W, pt, pl,
                                                              (float)scale, (float *)out);
  else
    pad_scale_kernel<double><<<grid, kPadThreads, 0, stream>>>((const double *)in, rows, Hp, Wp, H, W, pt, pl, scale,
                                                               (double *)out);
  PC2D_LAUNCH_CHECK("pad_scale_kernel");
  return PC2D_OK;
}

}  // namespace pc2d
