/*
 * paraconv2d.h -- C ABI of the B200 (sm_100a) ParaConv2d paraboloid convolution.
 *
 * libpc2d_sm100.so exports these entry points.  The signatures use only plain
 * C types: device pointers, sizes, a CUDA stream passed as void*.  They do not
 * use torch types.  The torch op library libptparaconv2d.so (schema
 * ptparaconv2d::forward / ptparaconv2d::backward, identical to the reference)
 * is a thin client of this ABI.
 *
 * Semantics follow the reference op GeoND-tech/ParaConv2d:
 *   input   [n][channels][height][width], already padded by the caller
 *   pars    [h0 (m) | h (m*d) | p (m*d) | p0 (m)], d = channels*k0*k1,
 *           h and p row-major [m][channels][k0][k1]   (paraconv2d.cc:23-37)
 *   output, hsum  [n][m][out_height][out_width]
 *   out_height = (height - dl0*(k0-1) - 1)/s0 + 1     (paraconv2d.cc:268-269)
 *   hsum   = h0[j] + sum_k h[j,k] * win[k]
 *   output = f * (hsum^2 - sum_k (win[k] - p[j,k])^2 - p0[j]^2)
 * The window is flipped: tap (ix2, iy2) reads input row
 * oy*s0 + (k0-1-ix2)*dl0 and column ox*s1 + (k1-1-iy2)*dl1 (paraconv2d.cc:89-92).
 * The backward pass returns inputgrad [n][channels][height][width] (scaled by
 * 2, with no output factor, paraconv2d.cc:166-183) and parsgrad, packed like
 * pars (scaled by 2f, paraconv2d.cc:226-237).  When skip_input_grad is
 * nonzero, inputgrad is written as all zeros (paraconv2d.cc:147,153).
 *
 * Conventions of every compute entry point:
 *   - all tensor pointers are device pointers to contiguous arrays of the
 *     given dtype; inputs are read only; outputs are fully overwritten;
 *   - work is enqueued on `stream` (a cudaStream_t; NULL = legacy default);
 *     nothing synchronises the host, and nothing allocates device memory:
 *     scratch comes from the caller's `workspace` of at least the size
 *     reported by the matching *_workspace_size query (256-byte aligned);
 *   - the return value is a pc2d_status; on failure pc2d_last_error()
 *     gives a message (thread local).  Odd kernel sizes only: even sizes make
 *     the reference read outside the window and are rejected.
 *   - kernels that wait on on-chip barriers give up after a bounded time;
 *     they then record PC2D_ERR_TIMEOUT in a device-side status word that
 *     pc2d_device_status() reads (it synchronises the device), and in a
 *     mirror of it in pinned host memory.  Every later compute call in that
 *     CUDA context reads the mirror on entry (no synchronisation) and returns
 *     PC2D_ERR_TIMEOUT until pc2d_clear_device_status() is called.  The
 *     first compute call in a context allocates the mirror (cudaHostAlloc),
 *     so make it before any stream capture; pc2d_forward_noalloc never does.
 */
#ifndef PARACONV2D_B200_H_
#define PARACONV2D_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PC2D_ABI_VERSION 1

typedef enum {
  PC2D_OK = 0,
  PC2D_ERR_INVALID_ARGUMENT = 1, /* bad shape, dtype, null pointer, pars length ... */
  PC2D_ERR_UNSUPPORTED = 2,      /* valid for the reference but not supported here */
  PC2D_ERR_WORKSPACE = 3,        /* workspace missing, too small or misaligned */
  PC2D_ERR_CUDA = 4,             /* a CUDA runtime call or launch failed */
  PC2D_ERR_TIMEOUT = 5           /* a device-side barrier wait gave up */
} pc2d_status;

typedef enum { PC2D_DTYPE_F32 = 0, PC2D_DTYPE_F64 = 1 } pc2d_dtype;

/* Kernel families.  AUTO picks the tcgen05 tensor-core kernels (3xTF32 split
 * precision) for fp32 shapes they support and the CUDA-core kernels
 * otherwise; SIMT forces the CUDA-core kernels (fp32 or fp64 FMA). */
typedef enum { PC2D_ALGO_AUTO = 0, PC2D_ALGO_SIMT = 1, PC2D_ALGO_TC = 2 } pc2d_algo;

/* Library ABI version (PC2D_ABI_VERSION). */
int pc2d_abi_version(void);

/* Output extent along one axis (reference paraconv2d.cc:268-269); <= 0 means empty/invalid. */
int pc2d_out_size(int in, int kernel, int stride, int dilation);

/* Number of output channels implied by the flat parameter count
 * (reference paraconv2d.cc:266: m = npars / (2*(d+1))); -1 when npars is not
 * a positive multiple of 2*(d+1). */
int64_t pc2d_infer_m(int64_t npars, int channels, int k0, int k1);

/* Process-wide kernel family selection (default PC2D_ALGO_AUTO).  Returns the previous value. */
int pc2d_set_algo(int algo);
int pc2d_get_algo(void);

/* Scratch bytes pc2d_forward needs for this problem (0 is possible). */
size_t pc2d_forward_workspace_size(int dtype, int n, int channels, int height, int width, int m,
                                   int k0, int k1, int s0, int s1, int dl0, int dl1);

/* Forward pass.  Replaces the reference's paraconv2d_forward_cuda_main<T>
 * (paraconv2d.cu:81-123) and the kernels it launches
 * (paraconv2dkernels.cu:27-141); `factor` is the op's `doublefactor`
 * argument (paraconv2d.cc:292). */
int pc2d_forward(int dtype, const void *input, const void *pars, double factor,
                 int k0, int k1, int s0, int s1, int dl0, int dl1,
                 int n, int channels, int height, int width, int m,
                 void *output, void *hsum, void *workspace, size_t workspace_bytes, void *stream);

/* Forward pass that allocates nothing and takes no workspace.  It has no
 * counterpart in the reference.  It is meant for callers that may not
 * allocate device memory while the op runs, such as plugin interfaces that
 * pass an operator only its input and output buffers, or real-time code with
 * a fixed memory budget: cudaMalloc can synchronise the device or fail, and
 * those hosts forbid it.  The scratch lives in a static 8 MiB device array
 * that every GPU loading the library keeps until exit.  Problems needing more
 * scratch than that fail with PC2D_ERR_WORKSPACE.  The first call in each
 * CUDA context (with a device's primary context current: the first call on
 * that device) resolves the array's address with cudaGetSymbolAddress, so
 * make that first call before any stream capture.  All calls share the
 * array: calls that overlap on the GPU race and must be serialised by the
 * caller.  Arguments, results and the other errors are those of pc2d_forward. */
int pc2d_forward_noalloc(int dtype, const void *input, const void *pars, double factor,
                         int k0, int k1, int s0, int s1, int dl0, int dl1,
                         int n, int channels, int height, int width, int m,
                         void *output, void *hsum, void *stream);

/* Scratch bytes pc2d_backward needs for this problem. */
size_t pc2d_backward_workspace_size(int dtype, int n, int channels, int height, int width, int m,
                                    int k0, int k1, int s0, int s1, int dl0, int dl1,
                                    int skip_input_grad);

/* Backward pass.  Replaces the reference's paraconv2d_backward_cuda_main<T>
 * (paraconv2d.cu:131-223) and the kernels it launches
 * (paraconv2dgradkernels.cu:27-249). */
int pc2d_backward(int dtype, const void *grad, const void *input, const void *pars, const void *hsum,
                  double factor, int k0, int k1, int s0, int s1, int dl0, int dl1,
                  int n, int channels, int height, int width, int m, int skip_input_grad,
                  void *inputgrad, void *parsgrad, void *workspace, size_t workspace_bytes, void *stream);

/* The two steps of the reference module's forward before the op
 * (ptparaconv2d.py:216-217: `x = input_factor * input`, then a constant-zero
 * F.pad) as one pass: output[n][c][y][x] = scale * input[n][c][y - pad_top]
 * [x - pad_left] inside, 0 in the padding; output is
 * [n][channels][height+pad_top+pad_bottom][width+pad_left+pad_right].  fp32 or
 * fp64; pads must be >= 0 (F.pad's negative pads crop; use torch for those). */
int pc2d_pad_scale(int dtype, const void *input, int n, int channels, int height, int width,
                   int pad_top, int pad_bottom, int pad_left, int pad_right, double scale,
                   void *output, void *stream);

/* Backward pass of the reference module around the op
 * (ptparaconv2d.py:52-58 and the backward of its pad and input factor,
 * :216-217): as pc2d_backward on the padded input, but the input gradient is
 * written only for the unpadded input, rows pad_top .. height-pad_bottom-1
 * and columns pad_left .. width-pad_right-1, into an
 * [n][channels][height-pad_top-pad_bottom][width-pad_left-pad_right] array,
 * multiplied by dx_scale (the module's input_factor * grad_factor).  This
 * replaces the module's slice of the padded gradient and its two scalings
 * (three passes over the input gradient) with the kernels' own stores.  With
 * skip_input_grad nonzero, inputgrad is zero-filled, or left alone when it is
 * NULL (a caller that does not need it).  Workspace: as pc2d_backward. */
int pc2d_backward_interior(int dtype, const void *grad, const void *input, const void *pars, const void *hsum,
                           double factor, int k0, int k1, int s0, int s1, int dl0, int dl1,
                           int n, int channels, int height, int width, int m, int skip_input_grad,
                           int pad_top, int pad_bottom, int pad_left, int pad_right, double dx_scale,
                           void *inputgrad, void *parsgrad, void *workspace, size_t workspace_bytes,
                           void *stream);

/* ---------------------------------------------------------------------------
 * Data-parallel training: the backward pass with the parameter gradient
 * summed over the ranks (one process per GPU, up to 8 GPUs of one node with
 * peer access), over NVLink peer memory instead of a separate all-reduce.
 * The reference has no multi-GPU path; this replaces the all-reduce (SUM) of
 * pars.grad after the backward in a data-parallel loop.
 *
 * Setup, once per process group (allocates: do it before any stream capture):
 *   pc2d_comm_create   -> this rank's exchange buffer (cudaMalloc) and an IPC
 *                         handle of pc2d_comm_handle_bytes() bytes;
 *   (the caller gathers every rank's handle, in rank order, by any channel,
 *    e.g. torch.distributed.all_gather_object)
 *   pc2d_comm_connect  -> maps every peer's buffer;
 *   pc2d_comm_destroy  -> unmaps and frees (after every rank's last call has
 *                         completed: a barrier first).
 * pc2d_backward_sum: as pc2d_backward (fp32), with parsgrad receiving the sum
 * of all ranks' parameter gradients, the same bits on every rank (fixed rank
 * order).  Every rank must make the same sequence of pc2d_backward_sum calls
 * on its communicator (like a collective); the calls of one communicator go
 * on one stream.  A rank that waits longer than 2 s for its peers records
 * PC2D_ERR_TIMEOUT in the device status (see above) and returns its own
 * gradient.
 * pc2d_comm_allreduce: dst = the sum over the ranks of every rank's src
 * (count fp32 values, count <= max_params; dst may be src), the same bits on
 * every rank, through the same exchange buffer: e.g. one bucket of several
 * layers' parameter gradients after an autograd backward.  It shares the
 * call sequence of pc2d_backward_sum (every rank the same calls, in the same
 * order, on one stream) and its timeout behaviour (dst = own src). */
typedef struct pc2d_comm pc2d_comm;
size_t pc2d_comm_handle_bytes(void);
int pc2d_comm_create(int rank, int world, size_t max_params, pc2d_comm **comm, void *handle_out);
int pc2d_comm_connect(pc2d_comm *comm, const void *handles);
int pc2d_comm_destroy(pc2d_comm *comm);
int pc2d_backward_sum(pc2d_comm *comm, int dtype, const void *grad, const void *input, const void *pars,
                      const void *hsum, double factor, int k0, int k1, int s0, int s1, int dl0, int dl1,
                      int n, int channels, int height, int width, int m, int skip_input_grad,
                      void *inputgrad, void *parsgrad, void *workspace, size_t workspace_bytes, void *stream);
int pc2d_comm_allreduce(pc2d_comm *comm, const void *src, void *dst, size_t count, void *stream);

/* ---------------------------------------------------------------------------
 * Optimizer step on one layer's flat parameter vector [h0 | h | p | p0]
 * (m output channels, window of d = C*k0*k1 elements), using the multipliers
 * the module attaches to `pars` (reference ptparaconv2d.py:194-198):
 *   d_i   = grad_i + (weight_decay * wd_factor) * w_i
 *   buf_i = momentum * buf_i + d_i     (buf_i = d_i when first_step != 0;
 *                                       momentum_buf unused when momentum == 0)
 *   w_i  -= (lr * factor_i) * buf_i,   factor = h_lr_factor on [h0 | h] (the
 *                                       first m*(1+d) values), p_lr_factor on [p | p0]
 * i.e. torch.optim.SGD (no dampening, no Nesterov) with the learning rate and
 * weight decay scaled per parameter group, in one pass over HBM.  dtype F32 or
 * F64; pars, grad and momentum_buf hold 2*m*(1+d) values each. */
int pc2d_param_step(int dtype, void *pars, const void *grad, void *momentum_buf, int m, int d, double lr,
                    double h_lr_factor, double p_lr_factor, double weight_decay, double wd_factor,
                    double momentum, int first_step, void *stream);

/* Human-readable name of a pc2d_status. */
const char *pc2d_status_string(int status);

/* Message of the last failing call on this host thread ("" if none). */
const char *pc2d_last_error(void);

/* Synchronises the current device and returns PC2D_OK, or the first
 * device-side error (PC2D_ERR_TIMEOUT) recorded since the last call to
 * pc2d_clear_device_status(); also reports pending CUDA errors as PC2D_ERR_CUDA. */
int pc2d_device_status(void);
int pc2d_clear_device_status(void);

/* Kernel timing (profiling aid, off by default).  While enabled, every main
 * kernel the library launches is bracketed by two CUDA events recorded on its
 * stream; pc2d_timing_read synchronises those events and returns, for the
 * kernel family `kernel` ("forward", "dgrad", "wgrad", "simt_forward",
 * "simt_dgrad", "simt_wgrad"), the summed duration in milliseconds and the
 * launch count since the last reset.  Returns PC2D_OK, or
 * PC2D_ERR_INVALID_ARGUMENT for an unknown name. */
int pc2d_timing_enable(int on);
int pc2d_timing_reset(void);
int pc2d_timing_read(const char *kernel, double *total_ms, int *launches);

/* Test hook: a kernel that waits on an mbarrier that nothing completes, with
 * a wait limit of `timeout_us` microseconds; it must return by itself and
 * record PC2D_ERR_TIMEOUT.  Used to check the bounded-wait path without
 * faulting or hanging the GPU. */
int pc2d_selftest_bounded_wait(unsigned int timeout_us, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* PARACONV2D_B200_H_ */
