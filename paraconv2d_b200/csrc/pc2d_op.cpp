// torch.ops.ptparaconv2d: the reference op's schema (GeoND-tech/ParaConv2d
// paraconv2d.cc:63-66), registered from C++ for the CUDA dispatch key only,
// on top of the C ABI of libpc2d_sm100.so.
//
// Differences from the reference wrappers (paraconv2d.cc:243-425), all of
// them turning undefined behaviour into errors:
//   - inputs are checked (device, dtype, rank, pars length, odd kernel) and
//     every failure raises with the library's message;
//   - non-contiguous tensors (for example the expanded gradient of
//     y.sum().backward()) are made contiguous instead of being read raw;
//   - work runs on torch's current CUDA stream, scratch comes from torch's
//     caching allocator;
//   - there is no CPU kernel: calling the op on CPU tensors raises
//     NotImplementedError from the dispatcher.
// Two more ops, in their own namespace paraconv2d_b200, serve the module
// mirror: its input factor and constant pad in one pass (pad_scale), and a
// backward that writes the unpadded input's gradient directly
// (backward_interior).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <vector>

#include "paraconv2d.h"

namespace {

struct PairArg {
  int v0, v1;
};

PairArg read_pair(const at::Tensor &t, const char *name) {
  TORCH_CHECK(t.numel() == 2, "ptparaconv2d: ", name, " must have 2 elements, got ", t.numel());
  TORCH_CHECK(t.scalar_type() == at::kInt || t.scalar_type() == at::kLong, "ptparaconv2d: ", name,
              " must be an integer tensor");
  const at::Tensor c = t.to(at::kCPU, at::kLong).contiguous();
  const int64_t *p = c.data_ptr<int64_t>();
  return PairArg{(int)p[0], (int)p[1]};
}

int dtype_code(const at::Tensor &t) {
  if (t.scalar_type() == at::kFloat) return PC2D_DTYPE_F32;
  if (t.scalar_type() == at::kDouble) return PC2D_DTYPE_F64;
  TORCH_CHECK_NOT_IMPLEMENTED(false, "ptparaconv2d: not implemented for '", t.scalar_type(),
                              "' (float32 and float64 only, as the reference)");
  return -1;
}

void check_status(int st, const char *what) {
  TORCH_CHECK(st == PC2D_OK, "ptparaconv2d.", what, ": ", pc2d_status_string(st), ": ", pc2d_last_error());
}

struct Shape {
  int n, C, H, W, m, P, Q;
  PairArg k, s, dl;
};

Shape shape_of(const at::Tensor &input, const at::Tensor &parameters, const at::Tensor &kt, const at::Tensor &st,
               const at::Tensor &dt) {
  TORCH_CHECK(input.is_cuda(), "ptparaconv2d: input must be a CUDA tensor");
  TORCH_CHECK(input.dim() == 4, "ptparaconv2d: input must be [N, C, H, W], got ", input.sizes());
  TORCH_CHECK(parameters.device() == input.device(), "ptparaconv2d: parameters must be on ", input.device());
  TORCH_CHECK(parameters.scalar_type() == input.scalar_type(), "ptparaconv2d: parameters dtype ",
              parameters.scalar_type(), " differs from input dtype ", input.scalar_type());
  Shape s;
  s.k = read_pair(kt, "kernel_size_tensor");
  s.s = read_pair(st, "strides_tensor");
  s.dl = read_pair(dt, "dilation_rate_tensor");
  s.n = (int)input.size(0);
  s.C = (int)input.size(1);
  s.H = (int)input.size(2);
  s.W = (int)input.size(3);
  const int64_t m = pc2d_infer_m(parameters.numel(), s.C, s.k.v0, s.k.v1);
  TORCH_CHECK(m >= 1, "ptparaconv2d: parameters has ", parameters.numel(),
              " elements, not a positive multiple of 2*(C*k0*k1+1) = ",
              2 * ((int64_t)s.C * s.k.v0 * s.k.v1 + 1));
  s.m = (int)m;
  s.P = pc2d_out_size(s.H, s.k.v0, s.s.v0, s.dl.v0);
  s.Q = pc2d_out_size(s.W, s.k.v1, s.s.v1, s.dl.v1);
  TORCH_CHECK(s.P >= 1 && s.Q >= 1, "ptparaconv2d: input ", s.H, "x", s.W, " is smaller than the dilated kernel");
  return s;
}

std::vector<at::Tensor> pc2d_forward_cuda(const at::Tensor &input_, const at::Tensor &parameters_,
                                          double doublefactor, const at::Tensor &kernel_size_tensor,
                                          const at::Tensor &strides_tensor, const at::Tensor &dilation_rate_tensor) {
  const int dt = dtype_code(input_);
  const Shape s = shape_of(input_, parameters_, kernel_size_tensor, strides_tensor, dilation_rate_tensor);
  const c10::cuda::CUDAGuard guard(input_.device());
  const at::Tensor input = input_.contiguous();
  const at::Tensor parameters = parameters_.contiguous();
  auto opts = input.options();
  at::Tensor output = at::empty({s.n, s.m, s.P, s.Q}, opts);
  at::Tensor hsum = at::empty({s.n, s.m, s.P, s.Q}, opts);
  const size_t ws_bytes = pc2d_forward_workspace_size(dt, s.n, s.C, s.H, s.W, s.m, s.k.v0, s.k.v1, s.s.v0, s.s.v1,
                                                      s.dl.v0, s.dl.v1);
  at::Tensor ws;
  if (ws_bytes > 0) ws = at::empty({(int64_t)ws_bytes}, opts.dtype(at::kByte));
  auto stream = c10::cuda::getCurrentCUDAStream();
  const int st = pc2d_forward(dt, input.data_ptr(), parameters.data_ptr(), doublefactor, s.k.v0, s.k.v1, s.s.v0,
                              s.s.v1, s.dl.v0, s.dl.v1, s.n, s.C, s.H, s.W, s.m, output.data_ptr(), hsum.data_ptr(),
                              ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, (void *)stream.stream());
  check_status(st, "forward");
  return {output, hsum};
}

struct BackwardArgs {
  int dt;
  Shape s;
  at::Tensor grad, input, parameters, hsum;
};

BackwardArgs backward_args(const at::Tensor &grad_, const at::Tensor &input_, const at::Tensor &parameters_,
                           const at::Tensor &hsum_, const at::Tensor &kernel_size_tensor,
                           const at::Tensor &strides_tensor, const at::Tensor &dilation_rate_tensor) {
  BackwardArgs a;
  a.dt = dtype_code(input_);
  a.s = shape_of(input_, parameters_, kernel_size_tensor, strides_tensor, dilation_rate_tensor);
  const Shape &s = a.s;
  const std::vector<int64_t> oshape = {s.n, s.m, s.P, s.Q};
  TORCH_CHECK(grad_.sizes() == at::IntArrayRef(oshape), "ptparaconv2d.backward: grad must be ", oshape, ", got ",
              grad_.sizes());
  TORCH_CHECK(hsum_.sizes() == at::IntArrayRef(oshape), "ptparaconv2d.backward: hsum must be ", oshape, ", got ",
              hsum_.sizes());
  TORCH_CHECK(grad_.device() == input_.device() && hsum_.device() == input_.device(),
              "ptparaconv2d.backward: all tensors must be on ", input_.device());
  TORCH_CHECK(grad_.scalar_type() == input_.scalar_type() && hsum_.scalar_type() == input_.scalar_type(),
              "ptparaconv2d.backward: grad/hsum dtype must match input dtype ", input_.scalar_type());
  a.grad = grad_.contiguous();
  a.input = input_.contiguous();
  a.parameters = parameters_.contiguous();
  a.hsum = hsum_.contiguous();
  return a;
}

std::vector<at::Tensor> pc2d_backward_cuda(const at::Tensor &grad_, const at::Tensor &input_,
                                           const at::Tensor &parameters_, const at::Tensor &hsum_,
                                           double doublefactor, const at::Tensor &kernel_size_tensor,
                                           const at::Tensor &strides_tensor,
                                           const at::Tensor &dilation_rate_tensor, bool skip_input_grad) {
  const c10::cuda::CUDAGuard guard(input_.device());
  const BackwardArgs a = backward_args(grad_, input_, parameters_, hsum_, kernel_size_tensor, strides_tensor,
                                       dilation_rate_tensor);
  const Shape &s = a.s;
  auto opts = a.input.options();
  at::Tensor inputgrad = at::empty({s.n, s.C, s.H, s.W}, opts);
  at::Tensor parametersgrad = at::empty({a.parameters.numel()}, opts);
  const size_t ws_bytes = pc2d_backward_workspace_size(a.dt, s.n, s.C, s.H, s.W, s.m, s.k.v0, s.k.v1, s.s.v0,
                                                       s.s.v1, s.dl.v0, s.dl.v1, skip_input_grad ? 1 : 0);
  at::Tensor ws;
  if (ws_bytes > 0) ws = at::empty({(int64_t)ws_bytes}, opts.dtype(at::kByte));
  auto stream = c10::cuda::getCurrentCUDAStream();
  const int st = pc2d_backward(a.dt, a.grad.data_ptr(), a.input.data_ptr(), a.parameters.data_ptr(),
                               a.hsum.data_ptr(), doublefactor, s.k.v0, s.k.v1, s.s.v0, s.s.v1, s.dl.v0, s.dl.v1,
                               s.n, s.C, s.H, s.W, s.m, skip_input_grad ? 1 : 0, inputgrad.data_ptr(),
                               parametersgrad.data_ptr(), ws_bytes ? ws.data_ptr() : nullptr, ws_bytes,
                               (void *)stream.stream());
  check_status(st, "backward");
  return {inputgrad, parametersgrad};
}

// --------------------------------------------------------------------------
// Fused module steps (namespace paraconv2d_b200, beside the reference's two
// ops): the ParaConv2d module's input factor + constant pad as one pass, and
// a backward that writes the gradient of the unpadded input directly.
// `padding` is in F.pad order: (left, right) or (left, right, top, bottom).

struct Pad4 {
  int t, b, l, r;
};

Pad4 pad4(at::IntArrayRef padding) {
  TORCH_CHECK(padding.size() == 2 || padding.size() == 4, "paraconv2d_b200: padding must have 2 or 4 entries");
  Pad4 p{0, 0, (int)padding[0], (int)padding[1]};
  if (padding.size() == 4) {
    p.t = (int)padding[2];
    p.b = (int)padding[3];
  }
  TORCH_CHECK(p.t >= 0 && p.b >= 0 && p.l >= 0 && p.r >= 0, "paraconv2d_b200: padding must be non-negative");
  return p;
}

at::Tensor pad_scale_cuda(const at::Tensor &input_, at::IntArrayRef padding, double scale) {
  const int dt = dtype_code(input_);
  TORCH_CHECK(input_.is_cuda() && input_.dim() == 4, "paraconv2d_b200.pad_scale: input must be a CUDA [N, C, H, W]");
  const c10::cuda::CUDAGuard guard(input_.device());
  const Pad4 p = pad4(padding);
  const at::Tensor input = input_.contiguous();
  const int64_t n = input.size(0), C = input.size(1), H = input.size(2), W = input.size(3);
  at::Tensor out = at::empty({n, C, H + p.t + p.b, W + p.l + p.r}, input.options());
  auto stream = c10::cuda::getCurrentCUDAStream();
  const int st = pc2d_pad_scale(dt, input.data_ptr(), (int)n, (int)C, (int)H, (int)W, p.t, p.b, p.l, p.r, scale,
                                out.data_ptr(), (void *)stream.stream());
  check_status(st, "pad_scale");
  return out;
}

std::vector<at::Tensor> backward_interior_cuda(const at::Tensor &grad_, const at::Tensor &input_,
                                               const at::Tensor &parameters_, const at::Tensor &hsum_,
                                               double doublefactor, const at::Tensor &kernel_size_tensor,
                                               const at::Tensor &strides_tensor,
                                               const at::Tensor &dilation_rate_tensor, bool skip_input_grad,
                                               at::IntArrayRef padding, double dx_scale, bool need_input_grad) {
  const c10::cuda::CUDAGuard guard(input_.device());
  const BackwardArgs a = backward_args(grad_, input_, parameters_, hsum_, kernel_size_tensor, strides_tensor,
                                       dilation_rate_tensor);
  const Shape &s = a.s;
  const Pad4 p = pad4(padding);
  TORCH_CHECK(p.t + p.b <= s.H && p.l + p.r <= s.W, "paraconv2d_b200.backward_interior: padding exceeds the input");
  auto opts = a.input.options();
  // without need_input_grad the kernels skip the input gradient entirely
  at::Tensor inputgrad = need_input_grad ? at::empty({s.n, s.C, s.H - p.t - p.b, s.W - p.l - p.r}, opts)
                                         : at::empty({0}, opts);
  at::Tensor parametersgrad = at::empty({a.parameters.numel()}, opts);
  const bool skip = skip_input_grad || !need_input_grad;
  const size_t ws_bytes = pc2d_backward_workspace_size(a.dt, s.n, s.C, s.H, s.W, s.m, s.k.v0, s.k.v1, s.s.v0,
                                                       s.s.v1, s.dl.v0, s.dl.v1, skip ? 1 : 0);
  at::Tensor ws;
  if (ws_bytes > 0) ws = at::empty({(int64_t)ws_bytes}, opts.dtype(at::kByte));
  auto stream = c10::cuda::getCurrentCUDAStream();
  const int st = pc2d_backward_interior(
      a.dt, a.grad.data_ptr(), a.input.data_ptr(), a.parameters.data_ptr(), a.hsum.data_ptr(), doublefactor, s.k.v0,
      s.k.v1, s.s.v0, s.s.v1, s.dl.v0, s.dl.v1, s.n, s.C, s.H, s.W, s.m, skip ? 1 : 0, p.t, p.b, p.l, p.r, dx_scale,
      need_input_grad ? inputgrad.data_ptr() : nullptr, parametersgrad.data_ptr(), ws_bytes ? ws.data_ptr() : nullptr,
      ws_bytes, (void *)stream.stream());
  check_status(st, "backward_interior");
  return {inputgrad, parametersgrad};
}

}  // namespace

TORCH_LIBRARY(ptparaconv2d, m) {
  m.def(
      "forward(Tensor input, Tensor parameters, float doublefactor, Tensor kernel_size_tensor, Tensor "
      "strides_tensor, Tensor dilation_rate_tensor) -> (Tensor[])");
  m.def(
      "backward(Tensor grad, Tensor input, Tensor parameters, Tensor hsum, float doublefactor, Tensor "
      "kernel_size_tensor, Tensor strides_tensor, Tensor dilation_rate_tensor, bool skip_input_grad) -> (Tensor[])");
}

TORCH_LIBRARY_IMPL(ptparaconv2d, CUDA, m) {
  m.impl("forward", pc2d_forward_cuda);
  m.impl("backward", pc2d_backward_cuda);
}

TORCH_LIBRARY(paraconv2d_b200, m) {
  m.def("pad_scale(Tensor input, int[] padding, float scale) -> Tensor");
  m.def(
      "backward_interior(Tensor grad, Tensor input, Tensor parameters, Tensor hsum, float doublefactor, Tensor "
      "kernel_size_tensor, Tensor strides_tensor, Tensor dilation_rate_tensor, bool skip_input_grad, int[] padding, "
      "float dx_scale, bool need_input_grad) -> (Tensor[])");
}

TORCH_LIBRARY_IMPL(paraconv2d_b200, CUDA, m) {
  m.impl("pad_scale", pad_scale_cuda);
  m.impl("backward_interior", backward_interior_cuda);
}
