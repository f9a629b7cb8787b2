// The module's input preparation in one pass: out = F.pad(scale * x) with
// zeros (reference ptparaconv2d.py:216-217, `input_factor * input` then a
// constant F.pad), reading x once and writing the padded copy once instead of
// a scaled copy, a zero fill and a copy into the interior.
#include <algorithm>

#include "pc2d_common.cuh"

namespace pc2d {
namespace {

constexpr int kPadThreads = 256;
constexpr int kPadUnroll = 8;        // loads in flight per lane
constexpr int kPadSegment = 1024;    // output elements per warp segment (about)

// A warp writes a contiguous segment of the output: R whole padded rows
// (R * Wp ~ kPadSegment elements), lane l the elements l, l + 32, ...  Row,
// column, plane and input row of a lane's element are stepped, not divided,
// from one element to its next, and each lane issues kPadUnroll loads before
// its stores, so that enough reads are in flight to stream at HBM speed (one
// warp per row, loading and storing one 32-column piece at a time, kept a
// single load per warp in flight: about a third of the bandwidth).  Rows of
// the padding and columns outside [pl, pl + W) are zeros; the rest are
// scale * x.
template <typename T>
__global__ void __launch_bounds__(kPadThreads) pad_scale_kernel(const T *__restrict__ in, int64_t rows, int Hp, int Wp,
                                                               int H, int W, int pt, int pl, int R, T scale,
                                                               T *__restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t w0 = ((int64_t)blockIdx.x * kPadThreads + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * kPadThreads) >> 5;
  for (int64_t row0 = w0 * R; row0 < rows; row0 += nw * R) {
    const int S = (int)(rows - row0 < R ? rows - row0 : R) * Wp;
    // position of element `lane` of the segment
    int r = lane / Wp, x = lane - r * Wp;
    int64_t plane = (row0 + r) / Hp;
    int y = (int)(row0 + r - plane * Hp) - pt;
    T *dst = out + row0 * Wp;
    for (int e0 = 0; e0 < S; e0 += 32 * kPadUnroll) {
      T v[kPadUnroll];
#pragma unroll
      for (int u = 0; u < kPadUnroll; ++u) {
        const int xi = x - pl;
        v[u] = T(0);
        if (e0 + lane + 32 * u < S && (unsigned)y < (unsigned)H && (unsigned)xi < (unsigned)W)
          v[u] = scale * __ldg(in + (plane * H + y) * W + xi);
        // next element of this lane: 32 further on
        x += 32;
        while (x >= Wp) {
          x -= Wp;
          if (++y == Hp - pt) {
            y = -pt;
            ++plane;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kPadUnroll; ++u) {
        const int e = e0 + lane + 32 * u;
        if (e < S) dst[e] = v[u];
      }
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
  if (rows == 0 || Wp == 0) return PC2D_OK;
  const int R = std::max(1, kPadSegment / Wp);
  const int64_t segments = (rows + R - 1) / R;
  const int64_t want = (segments + kPadThreads / 32 - 1) / (kPadThreads / 32);
  // one resident wave: the warps loop over the segments, so a second,
  // partial wave of blocks would run as long as the first
  int per_sm = 0;
  if (dtype == PC2D_DTYPE_F32)
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pad_scale_kernel<float>, kPadThreads, 0);
  else
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pad_scale_kernel<double>, kPadThreads, 0);
  per_sm = std::max(1, per_sm);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sms * per_sm));
  if (dtype == PC2D_DTYPE_F32)
    pad_scale_kernel<float><<<grid, kPadThreads, 0, stream>>>((const float *)in, rows, Hp, Wp, H, W, pt, pl, R,
                                                              (float)scale, (float *)out);
  else
    pad_scale_kernel<double><<<grid, kPadThreads, 0, stream>>>((const double *)in, rows, Hp, Wp, H, W, pt, pl, R,
                                                               scale, (double *)out);
  PC2D_LAUNCH_CHECK("pad_scale_kernel");
  return PC2D_OK;
}

}  // namespace pc2d
