// Data-parallel sum of the parameter gradient over NVLink peer memory, fused
// into the backward pass (pc2d_backward_sum).
//
// In data-parallel training every rank computes the parameter gradient of its
// shard of the batch, and the ranks need the sum (the loss is a sum over
// images).  A collective library call after the backward (an NCCL all-reduce)
// costs a stream hand-off, its own launch and its protocol: 15-40 us for the
// 295 KB gradient of a 64->64-channel 3x3 layer on 2-8 B200s, which is 4-10 %
// of that layer's 0.41 ms step.  Here the backward's own fixed-order reduction
// writes the rank's gradient into an exchange buffer that every rank has
// mapped (CUDA IPC, one process per GPU), and one more small kernel sums it:
//   - it is a programmatic dependent of the reduction (its launch overlaps
//     the reduction; griddepcontrol.wait holds it until the gradient is
//     complete);
//   - block b of the sum kernel owns a slice of the gradient; it publishes
//     "slice b of epoch e is ready" by a posted store into every PEER's
//     buffer (flag[rank][b] there), then waits until flag[q][b] in its OWN
//     buffer has reached the epoch for every peer q (a bounded spin on local
//     memory, acquire at system scope: a flag arrives after one NVLink
//     crossing, no round trip per poll);
//   - then every thread loads one 16-byte vector of the slice from every rank
//     (all ranks' loads in flight together: one round trip) and adds them in
//     rank order (fp64), writing the caller's gradient array;
//   - the grid is no larger than what is resident at once, so every block of
//     every rank runs at the same time and no block waits on one that cannot
//     be scheduled;
//   - the exchange slot alternates with the epoch's parity: a rank can be at
//     most one call ahead of a peer (its next call waits on the peer's flags
//     of this call), so it never overwrites a slot a peer is still reading.
// Every rank adds the same values in the same order: the summed gradient is
// bitwise identical on all ranks.  Loads and stores only: no multicast, no
// NVLS.
#include <algorithm>
#include <cstring>

#include "pc2d_common.cuh"

namespace pc2d {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kSumThreads = 256;
constexpr uint64_t kPeerWaitNs = 2000000000ull;  // 2 s

struct PeerPtrs {
  float *data[kMaxRanks];      // [2 slots][stride] per rank
  unsigned *flags[kMaxRanks];  // [kMaxRanks sources][nblocks] per rank
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(unsigned *p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Grid: nblocks blocks of kSumThreads; block b sums vectors
// [b * kSumThreads * vpt, (b + 1) * kSumThreads * vpt) of the gradient, 4
// floats each (npars need not be a multiple of 4: the last vector is summed
// element by element).  stride (floats between the two slots) is a multiple
// of 4, so every vector is 16-byte aligned.  own_flags is
// peers.flags[rank], passed on its own: indexing the parameter array with the
// run-time rank would copy it to local memory.
__global__ void __launch_bounds__(kSumThreads) peer_sum_kernel(PeerPtrs peers, int world, int rank, unsigned epoch,
                                                               int slot, int64_t stride, int64_t npars, int vpt,
                                                               const unsigned *own_flags, const float *own_data,
                                                               float *__restrict__ out, int *status) {
  __shared__ int s_ok;
  // the rank's own slice is written by the reduction this grid depends on
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) {
    // publish: the slot is complete (fence: the reduction's writes before the
    // flag, at system scope), into every peer's buffer
    __threadfence_system();
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q)
      if (q < world && q != rank) st_relaxed_sys(peers.flags[q] + (size_t)rank * gridDim.x + blockIdx.x, epoch);
    int ok = 1;
    const uint64_t t0 = now_ns();
    for (int q = 0; q < world && ok; ++q) {
      if (q == rank) continue;
      while ((int)(ld_acquire_sys(own_flags + (size_t)q * gridDim.x + blockIdx.x) - epoch) < 0) {
        if (now_ns() - t0 > kPeerWaitNs) {
          ok = 0;
          break;
        }
      }
    }
    if (!ok) record_device_error(status, PC2D_ERR_TIMEOUT);
    s_ok = ok;
  }
  __syncthreads();
  const int64_t base = (int64_t)slot * stride;
  const int64_t nvec = (npars + 3) / 4;
  const int64_t v0 = (int64_t)blockIdx.x * kSumThreads * vpt;
  if (!s_ok) {
    // a peer did not arrive: the slice gets this rank's own values (the
    // status word carries the error)
    const float *own = own_data + base;
    for (int64_t e = v0 * 4 + threadIdx.x; e < min(npars, (v0 + (int64_t)kSumThreads * vpt) * 4); e += kSumThreads)
      out[e] = own[e];
    return;
  }
  for (int u = 0; u < vpt; ++u) {
    const int64_t v = v0 + (int64_t)u * kSumThreads + threadIdx.x;
    if (v >= nvec) break;
    // every rank's vector in flight at once, then the sum in rank order
    float4 x[kMaxRanks];
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q)
      x[q] = q < world ? __ldcv(reinterpret_cast<const float4 *>(peers.data[q] + base) + v) : make_float4(0, 0, 0, 0);
    double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q)
      if (q < world) {
        a0 += (double)x[q].x;
        a1 += (double)x[q].y;
        a2 += (double)x[q].z;
        a3 += (double)x[q].w;
      }
    const int64_t e = 4 * v;
    if (e + 4 <= npars && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
      reinterpret_cast<float4 *>(out)[v] = make_float4((float)a0, (float)a1, (float)a2, (float)a3);
    } else {
      out[e] = (float)a0;
      if (e + 1 < npars) out[e + 1] = (float)a1;
      if (e + 2 < npars) out[e + 2] = (float)a2;
      if (e + 3 < npars) out[e + 3] = (float)a3;
    }
  }
}

}  // namespace
}  // namespace pc2d

using namespace pc2d;

struct pc2d_comm {
  int rank = 0, world = 1, dev = -1;
  size_t max_params = 0;
  size_t stride = 0;  // floats per exchange slot: max_params rounded up to 4
  int nblocks = 0;    // sum kernel grid (fixed: the flags are per block)
  int vpt = 1;        // 4-float vectors per thread of the sum kernel
  unsigned epoch = 0;
  void *own = nullptr;  // cudaMalloc'd: [2][stride] floats, then [world][nblocks] flags
  void *peer_base[kMaxRanks] = {};
  PeerPtrs ptrs = {};
  bool connected = false;
};

namespace {
size_t flags_offset(size_t stride) { return align_up(2 * stride * sizeof(float), 256); }
}  // namespace

namespace {

// The sum kernel over the first npars floats of every rank's slot, as a
// programmatic dependent of whatever wrote this rank's slot last on the
// stream (a kernel: its launch overlaps that kernel; a copy: plain order).
int launch_peer_sum(pc2d_comm *c, unsigned epoch, int slot, int64_t npars, float *out, cudaStream_t s) {
  int *status = device_status_ptr();
  if (!status) {
    set_last_error("could not resolve the device status word");
    return PC2D_ERR_CUDA;
  }
  NvtxRange sum_range("peer_sum");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(c->nblocks);
  cfg.blockDim = dim3(kSumThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PC2D_CUDA_CHECK(cudaLaunchKernelEx(&cfg, peer_sum_kernel, c->ptrs, c->world, c->rank, epoch, slot,
                                     (int64_t)c->stride, npars, c->vpt, (const unsigned *)c->ptrs.flags[c->rank],
                                     (const float *)c->ptrs.data[c->rank], out, status));
  PC2D_LAUNCH_CHECK("peer_sum_kernel");
  c->epoch = epoch;
  return PC2D_OK;
}

}  // namespace

extern "C" {

int pc2d_comm_create(int rank, int world, size_t max_params, pc2d_comm **comm, void *handle_out) {
  if (!comm || !handle_out || world < 1 || world > kMaxRanks || rank < 0 || rank >= world || max_params == 0) {
    set_last_error("pc2d_comm_create: invalid arguments (rank %d, world %d, at most %d ranks)", rank, world,
                   kMaxRanks);
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  pc2d_comm *c = new pc2d_comm();
  c->rank = rank;
  c->world = world;
  c->max_params = max_params;
  c->stride = align_up(max_params, 4);
  if (cudaGetDevice(&c->dev) != cudaSuccess) {
    delete c;
    set_last_error("pc2d_comm_create: no current device");
    return PC2D_ERR_CUDA;
  }
  int sms = 148, per_sm = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c->dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, peer_sum_kernel, kSumThreads, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  // every block resident at once (see the file comment); one vector per
  // thread when the gradient fits such a grid
  const int64_t nvec = (int64_t)c->stride / 4;
  c->nblocks = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(nvec, kSumThreads), (int64_t)sms * per_sm));
  c->vpt = ceil_div(nvec, (int64_t)c->nblocks * kSumThreads);
  const size_t bytes = flags_offset(c->stride) + (size_t)world * c->nblocks * sizeof(unsigned);
  cudaError_t e = cudaMalloc(&c->own, bytes);
  if (e == cudaSuccess) e = cudaMemset(c->own, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->own);
  if (e != cudaSuccess) {
    if (c->own) cudaFree(c->own);
    delete c;
    set_last_error("pc2d_comm_create: %s", cudaGetErrorString(e));
    return PC2D_ERR_CUDA;
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *comm = c;
  return PC2D_OK;
}

size_t pc2d_comm_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int pc2d_comm_connect(pc2d_comm *c, const void *handles) {
  if (!c || !handles || c->connected) {
    set_last_error("pc2d_comm_connect: invalid communicator or already connected");
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  const char *hb = static_cast<const char *>(handles);
  const size_t fo = flags_offset(c->stride);
  for (int q = 0; q < c->world; ++q) {
    void *base = c->own;
    if (q != c->rank) {
      cudaIpcMemHandle_t h;
      std::memcpy(&h, hb + (size_t)q * sizeof(h), sizeof(h));
      const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        for (int r = 0; r < q; ++r)
          if (r != c->rank && c->peer_base[r]) cudaIpcCloseMemHandle(c->peer_base[r]);
        set_last_error("pc2d_comm_connect: opening rank %d's buffer failed: %s", q, cudaGetErrorString(e));
        return PC2D_ERR_CUDA;
      }
    }
    c->peer_base[q] = base;
    c->ptrs.data[q] = static_cast<float *>(base);
    c->ptrs.flags[q] = reinterpret_cast<unsigned *>(static_cast<char *>(base) + fo);
  }
  c->connected = true;
  return PC2D_OK;
}

int pc2d_comm_destroy(pc2d_comm *c) {
  if (!c) return PC2D_OK;
  for (int q = 0; q < c->world; ++q)
    if (q != c->rank && c->peer_base[q]) cudaIpcCloseMemHandle(c->peer_base[q]);
  if (c->own) cudaFree(c->own);
  delete c;
  return PC2D_OK;
}

int pc2d_backward_sum(pc2d_comm *c, int dtype, const void *grad, const void *input, const void *pars,
                      const void *hsum, double factor, int k0, int k1, int s0, int s1, int dl0, int dl1, int n,
                      int channels, int height, int width, int m, int skip_input_grad, void *inputgrad,
                      void *parsgrad, void *workspace, size_t workspace_bytes, void *stream) {
  NvtxRange range("pc2d_backward_sum");
  if (!c || !c->connected) {
    set_last_error("pc2d_backward_sum: communicator not connected");
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  if (dtype != PC2D_DTYPE_F32) {
    set_last_error("pc2d_backward_sum: float32 only");
    return PC2D_ERR_UNSUPPORTED;
  }
  const int64_t npars = (int64_t)m * 2 * ((int64_t)channels * k0 * k1 + 1);
  if (npars > (int64_t)c->max_params) {
    set_last_error("pc2d_backward_sum: %lld parameters, more than the communicator's %zu", (long long)npars,
                   c->max_params);
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  if (c->world == 1)
    return pc2d_backward(dtype, grad, input, pars, hsum, factor, k0, k1, s0, s1, dl0, dl1, n, channels, height, width,
                         m, skip_input_grad, inputgrad, parsgrad, workspace, workspace_bytes, stream);
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != c->dev) {
    set_last_error("pc2d_backward_sum: the current device is not the communicator's (%d)", c->dev);
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  const unsigned epoch = c->epoch + 1;
  const int slot = (int)(epoch & 1);
  float *mine = c->ptrs.data[c->rank] + (size_t)slot * c->stride;
  // this rank's gradient, into its exchange slot
  int st = pc2d_backward(dtype, grad, input, pars, hsum, factor, k0, k1, s0, s1, dl0, dl1, n, channels, height, width,
                         m, skip_input_grad, inputgrad, mine, workspace, workspace_bytes, stream);
  if (st != PC2D_OK) return st;
  if (npars == 0) return PC2D_OK;
  return launch_peer_sum(c, epoch, slot, npars, static_cast<float *>(parsgrad),
                         reinterpret_cast<cudaStream_t>(stream));
}

int pc2d_comm_allreduce(pc2d_comm *c, const void *src, void *dst, size_t count, void *stream) {
  NvtxRange range("pc2d_comm_allreduce");
  if (!c || !c->connected) {
    set_last_error("pc2d_comm_allreduce: communicator not connected");
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  if (count > c->max_params || (count > 0 && (!src || !dst))) {
    set_last_error("pc2d_comm_allreduce: %zu floats (the communicator holds %zu) or a null buffer", count,
                   c->max_params);
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != c->dev) {
    set_last_error("pc2d_comm_allreduce: the current device is not the communicator's (%d)", c->dev);
    return PC2D_ERR_INVALID_ARGUMENT;
  }
  const int pend = pending_device_error();
  if (pend != PC2D_OK) return pend;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (count == 0) return PC2D_OK;
  if (c->world == 1) {
    if (src != dst) PC2D_CUDA_CHECK(cudaMemcpyAsync(dst, src, count * sizeof(float), cudaMemcpyDeviceToDevice, s));
    return PC2D_OK;
  }
  const unsigned epoch = c->epoch + 1;
  const int slot = (int)(epoch & 1);
  float *mine = c->ptrs.data[c->rank] + (size_t)slot * c->stride;
  // this rank's values into its exchange slot, then the sum over the ranks
  // (dst may be src: the sum reads the slots only)
  PC2D_CUDA_CHECK(cudaMemcpyAsync(mine, src, count * sizeof(float), cudaMemcpyDeviceToDevice, s));
  return launch_peer_sum(c, epoch, slot, (int64_t)count, static_cast<float *>(dst), s);
}

}  // extern "C"
