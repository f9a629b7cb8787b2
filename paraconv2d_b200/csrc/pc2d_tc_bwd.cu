// tcgen05 backward kernels of the ParaConv2d paraboloid convolution.
// (The CUDA-core kernels in pc2d_simt.cu serve every backward problem until
// the tensor-core wgrad/dgrad kernels land here.)
#include "pc2d_tc.cuh"

namespace pc2d {

bool tc_backward_supported(const Problem &) { return false; }

size_t tc_backward_workspace(const Problem &, bool) { return 0; }

int tc_backward(const Problem &, const float *, const float *, const float *, const float *, double, bool, float *,
                float *, void *, size_t, cudaStream_t) {
  set_last_error("tensor-core backward not available");
  return PC2D_ERR_UNSUPPORTED;
}

}  // namespace pc2d
