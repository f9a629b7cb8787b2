/*
 * ORACLE -- test infrastructure only.
 *
 * A plain-C restatement of the reference CPU implementation of the ParaConv2d
 * paraboloid convolution (GeoND-tech/ParaConv2d, paraconv2d.cc).  It is the
 * checker that the CUDA kernels of this repository are compared against; it
 * is never called by the product path.  Only tests/, __graft_entry__.smoke()
 * and the CPU-baseline leg of bench.py load it.
 *
 * The loops, their nesting order and the order of every floating-point
 * accumulation follow the reference line by line, so that the fp32 results
 * are bit-identical to the reference op compiled from its own source
 * (oracle/build_ref.sh).  That identity is what pins this restatement
 * (tests/test_oracle.py).
 *
 * Layouts (reference paraconv2d.cc:23-37):
 *   input  [n][channels][height][width]   (already padded by the caller)
 *   pars   [h0 (m) | h (m*d) | p (m*d) | p0 (m)],  d = channels*k0*k1,
 *          h and p row-major [m][channels][k0][k1]
 *   output, hsum [n][m][out_height][out_width]
 *   parsgrad packed like pars.
 */
#include <stdint.h>
#include <string.h>

/* Input offset of tap (ix2, iy2) of output pixel (x1, y1): the window is
 * flipped, row = x1*s0 + (2*(k0/2) - ix2)*dl0 (reference paraconv2d.cc:89-92). */
#define PC2D_IN_INDEX(i, k, x1, y1, ix2, iy2)                                   \
  ((int64_t)(i) * channels * height * width + (int64_t)(k) * height * width +  \
   (int64_t)((x1) * s0 + (((k0 / 2) - (ix2)) + (k0 / 2)) * dl0) * width +      \
   ((y1) * s1 + (((k1 / 2) - (iy2)) + (k1 / 2)) * dl1))
#define PC2D_W_INDEX(j, k, ix2, iy2) \
  ((int64_t)(j) * channels * k0 * k1 + (int64_t)(k) * k0 * k1 + (ix2) * k1 + (iy2))
#define PC2D_O_INDEX(i, j, x1, y1)                                              \
  ((int64_t)(i) * m * out_height * out_width + (int64_t)(j) * out_height * out_width + \
   (int64_t)(x1) * out_width + (y1))

/* Forward pass: reference paraconv2d.cc:70-124.  First pass hsum and hsum^2
 * (:82-101), second pass subtracts the squared focal distance and p0^2, then
 * scales by the output factor (:103-122). */
#define PC2D_DEFINE_FORWARD(T, NAME)                                                    \
  void NAME(const T *input, const T *pars, double doublefactor, int k0, int k1,        \
            int s0, int s1, int dl0, int dl1, int n, int channels, int height,          \
            int width, int m, int out_height, int out_width, T *output, T *hsum) {      \
    const int64_t d = (int64_t)channels * k0 * k1;                                      \
    const T *h0 = pars, *h = h0 + m, *p = h + m * d, *p0 = p + m * d;                   \
    const T factor = (T)doublefactor;                                                    \
    for (int i = 0; i < n; i++)                                                          \
      for (int x1 = 0; x1 < out_height; x1++)                                           \
        for (int y1 = 0; y1 < out_width; y1++)                                          \
          for (int j = 0; j < m; j++) {                                                  \
            T tmp = h0[j];                                                               \
            for (int k = 0; k < channels; k++)                                           \
              for (int ix2 = 0; ix2 < k0; ix2++)                                         \
                for (int iy2 = 0; iy2 < k1; iy2++)                                       \
                  tmp += h[PC2D_W_INDEX(j, k, ix2, iy2)] *                               \
                         input[PC2D_IN_INDEX(i, k, x1, y1, ix2, iy2)];                   \
            hsum[PC2D_O_INDEX(i, j, x1, y1)] = tmp;                                      \
            output[PC2D_O_INDEX(i, j, x1, y1)] = tmp * tmp;                              \
          }                                                                              \
    for (int i = 0; i < n; i++)                                                          \
      for (int x1 = 0; x1 < out_height; x1++)                                           \
        for (int y1 = 0; y1 < out_width; y1++)                                          \
          for (int j = 0; j < m; j++) {                                                  \
            T *o = &output[PC2D_O_INDEX(i, j, x1, y1)];                                  \
            for (int k = 0; k < channels; k++)                                           \
              for (int ix2 = 0; ix2 < k0; ix2++)                                         \
                for (int iy2 = 0; iy2 < k1; iy2++) {                                     \
                  T t = input[PC2D_IN_INDEX(i, k, x1, y1, ix2, iy2)] -                   \
                        p[PC2D_W_INDEX(j, k, ix2, iy2)];                                 \
                  *o -= t * t;                                                           \
                }                                                                        \
            *o -= p0[j] * p0[j];                                                         \
            *o *= factor;                                                                \
          }                                                                              \
  }

/* Backward pass: reference paraconv2d.cc:128-239.
 *   dx  (:153-184): 2 * scatter_j g*(hsum*h - x + p)   -- no output factor
 *   dh, dh0 (:186-205), dp, dp0 (:207-224), then *2f (:226-237).
 * When skip_input_grad is set, dx stays all zero (:147, :153). */
#define PC2D_DEFINE_BACKWARD(T, NAME)                                                   \
  void NAME(const T *grad, const T *input, const T *pars, const T *hsum,               \
            double doublefactor, int k0, int k1, int s0, int s1, int dl0, int dl1,      \
            int n, int channels, int height, int width, int m, int out_height,          \
            int out_width, T *inputgrad, T *parsgrad, int skip_input_grad) {            \
    const int64_t d = (int64_t)channels * k0 * k1;                                      \
    const T *h = pars + m, *p = h + m * d, *p0 = p + m * d;                             \
    T *h0grad = parsgrad, *hgrad = h0grad + m, *pgrad = hgrad + m * d,                  \
      *p0grad = pgrad + m * d;                                                          \
    const T factor = (T)doublefactor;                                                    \
    memset(inputgrad, 0, sizeof(T) * (size_t)n * channels * height * width);            \
    memset(parsgrad, 0, sizeof(T) * (size_t)m * 2 * (d + 1));                           \
    if (!skip_input_grad) {                                                              \
      for (int i = 0; i < n; i++)                                                        \
        for (int x1 = 0; x1 < out_height; x1++)                                         \
          for (int y1 = 0; y1 < out_width; y1++)                                        \
            for (int k = 0; k < channels; k++)                                           \
              for (int ix2 = 0; ix2 < k0; ix2++)                                         \
                for (int iy2 = 0; iy2 < k1; iy2++) {                                     \
                  const int64_t xi = PC2D_IN_INDEX(i, k, x1, y1, ix2, iy2);              \
                  T acc = 0;                                                             \
                  for (int j = 0; j < m; j++) {                                          \
                    const int64_t oi = PC2D_O_INDEX(i, j, x1, y1);                       \
                    const int64_t wi = PC2D_W_INDEX(j, k, ix2, iy2);                     \
                    acc += grad[oi] * ((hsum[oi] * h[wi]) - input[xi] + p[wi]);          \
                  }                                                                      \
                  inputgrad[xi] += acc;                                                  \
                }                                                                        \
      for (int64_t e = 0; e < (int64_t)n * channels * height * width; e++)               \
        inputgrad[e] *= 2;                                                               \
    }                                                                                    \
    for (int i = 0; i < n; i++)                                                          \
      for (int x1 = 0; x1 < out_height; x1++)                                           \
        for (int y1 = 0; y1 < out_width; y1++)                                          \
          for (int j = 0; j < m; j++) {                                                  \
            const int64_t oi = PC2D_O_INDEX(i, j, x1, y1);                               \
            for (int ix2 = 0; ix2 < k0; ix2++)                                           \
              for (int iy2 = 0; iy2 < k1; iy2++)                                         \
                for (int k = 0; k < channels; k++)                                       \
                  hgrad[PC2D_W_INDEX(j, k, ix2, iy2)] +=                                 \
                      grad[oi] * hsum[oi] * input[PC2D_IN_INDEX(i, k, x1, y1, ix2, iy2)]; \
            h0grad[j] += grad[oi] * hsum[oi];                                            \
          }                                                                              \
    for (int i = 0; i < n; i++)                                                          \
      for (int x1 = 0; x1 < out_height; x1++)                                           \
        for (int y1 = 0; y1 < out_width; y1++)                                          \
          for (int j = 0; j < m; j++) {                                                  \
            const int64_t oi = PC2D_O_INDEX(i, j, x1, y1);                               \
            for (int ix2 = 0; ix2 < k0; ix2++)                                           \
              for (int iy2 = 0; iy2 < k1; iy2++)                                         \
                for (int k = 0; k < channels; k++) {                                     \
                  const int64_t wi = PC2D_W_INDEX(j, k, ix2, iy2);                       \
                  pgrad[wi] += grad[oi] *                                                \
                      (input[PC2D_IN_INDEX(i, k, x1, y1, ix2, iy2)] - p[wi]);            \
                }                                                                        \
            p0grad[j] += grad[oi] * (-p0[j]);                                            \
          }                                                                              \
    for (int j = 0; j < m; j++) {                                                        \
      h0grad[j] *= 2 * factor;                                                           \
      p0grad[j] *= 2 * factor;                                                           \
      for (int64_t w = 0; w < d; w++) {                                                  \
        hgrad[(int64_t)j * d + w] *= 2 * factor;                                         \
        pgrad[(int64_t)j * d + w] *= 2 * factor;                                         \
      }                                                                                  \
    }                                                                                    \
  }

PC2D_DEFINE_FORWARD(float, pc2d_oracle_forward_f32)
PC2D_DEFINE_FORWARD(double, pc2d_oracle_forward_f64)
PC2D_DEFINE_BACKWARD(float, pc2d_oracle_backward_f32)
PC2D_DEFINE_BACKWARD(double, pc2d_oracle_backward_f64)

/* Output spatial size (reference paraconv2d.cc:268-269). */
int pc2d_oracle_out_size(int in, int k, int s, int dl) { return ((in - (dl * (k - 1)) - 1) / s) + 1; }
