// Host entry points of the tcgen05 (tensor-core, 3xTF32) kernels.
#pragma once

#include <cuda.h>  // CUtensorMap (types only; the encoder is resolved at run time)

#include "pc2d_common.cuh"

namespace pc2d {

// Forward pass (pc2d_tc_fwd.cu).
bool tc_forward_supported(const Problem &p);
size_t tc_forward_workspace(const Problem &p);
int tc_forward(const Problem &p, const float *x, const float *pars, double factor, float *out, float *hsum,
               void *ws, cudaStream_t stream);

// Backward pass (pc2d_tc_bwd.cu).
bool tc_backward_supported(const Problem &p);
size_t tc_backward_workspace(const Problem &p, bool skip_input_grad);
int tc_backward(const Problem &p, const float *grad, const float *x, const float *pars, const float *hsum,
                double factor, bool skip_input_grad, float *dx, float *dpars, void *ws, size_t ws_bytes,
                cudaStream_t stream, const DxOut &dxo);

// Input gradient of narrow inputs (C <= 8): GEMM over output pixels + col2im
// (pc2d_tc_dgcol.cu).
bool tc_dgcol_supported(const Problem &p);
size_t tc_dgcol_workspace(const Problem &p);
int tc_dgcol(const Problem &p, const float *grad, const float *x, const float *pars, const float *hsum,
             const DxOut &dxo, float *dx, void *ws, cudaStream_t stream);

// Parameter-gradient GEMM and its reduction (pc2d_tc_wgrad.cu).
bool tc_wgrad_supported(const Problem &p);
size_t tc_wgrad_workspace(const Problem &p);
int tc_wgrad(const Problem &p, const float *grad, const float *x, const float *pars, const float *hsum, double factor,
             float *dpars, void *ws, cudaStream_t stream);

// Fixed-order fp64 reduction of per-segment parameter-gradient partials and
// the epilogue dh = 2f dH, dp = 2f (dP - p SG), dh0 = 2f S1, dp0 = -2f p0 SG
// (pc2d_tc_wgrad.cu).  Layout: for segment s and window range nr, channel
// block mb (item = (s*nNR + nr)*nmb + mb), part[(item*128 + r)*NR + kl] holds
// sum_o A[r,o] win_o[nr*NR + kl] and sums[item*128 + r] the row sum of A,
// with rows r = [g*hsum of the block's JM channels; g of the same channels].
// Launched as a programmatic dependent of the kernel that writes the
// partials; it waits for that kernel before reading them.
int tc_wgrad_reduce(const Problem &p, const float *part, const float *sums, const float *pars, double factor,
                    float *dpars, int64_t nseg, int nNR, int nmb, int JM, int NR, cudaStream_t stream);

// Parameter gradients of narrow windows (d <= 31 window elements, m <= 32
// output channels) on the CUDA cores (pc2d_nw_wgrad.cu).
bool nw_wgrad_supported(const Problem &p);
size_t nw_wgrad_workspace(const Problem &p);
int nw_wgrad(const Problem &p, const float *grad, const float *x, const float *pars, const float *hsum, double factor,
             float *dpars, void *ws, cudaStream_t stream);

// A kernel that waits on an mbarrier nothing completes, bounded by timeout_us.
int tc_selftest_bounded_wait(unsigned int timeout_us, int *status, cudaStream_t stream);

// Number of SMs of the current device (cached per device).
int device_sm_count();

// Tensor map of the input planes for one 2-D TMA copy per stage: x viewed as
// rows = n*C channel planes of HW floats, boxes of box_rows planes x box_inner
// floats, zero fill outside.  False (map unusable) when the driver entry point
// is missing, x is not 16-byte aligned or HW*4 is not a multiple of 16.
bool encode_planes_map(const float *x, int64_t HW, int64_t rows, int box_inner, int box_rows, CUtensorMap *map);
// 2-D tensor map over a [rows][cols] fp32 tensor (cols % 4 == 0, 16-byte
// aligned base) with boxes of 32 floats x box_rows rows and the 128-byte
// swizzle: in shared memory, 16-byte chunk q of box row r lands at position
// q ^ (r % 8) of the row's 128 bytes (box base 1024-byte aligned).
bool encode_rows_map_sw128(const float *t, int64_t cols, int64_t rows, int box_rows, CUtensorMap *map);

}  // namespace pc2d
