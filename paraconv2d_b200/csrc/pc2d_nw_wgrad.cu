// Parameter gradients of narrow windows on the CUDA cores (fp32).
//
// Parameter gradients (reference paraconv2d.cc:186-237) as one contraction
// over the output pixels o:
//   D[r, k] = sum_o A[r, o] * B[k, o],
//   A = [g*hsum (rows 0..31); g (rows 32..63)] of up to 32 output channels,
//   B = [win_o (k < d); 1 (k = d); 0]      (window of d <= 31 elements)
// The ones column gives the row sums of A (dh0 and the sum of g of dp, dp0).
// With a window this short the tensor-core kernel's 32-pixel MMAs carry too
// little work for their hand-offs (and N = 32 wastes most of an MMA), while
// the contraction's arithmetic (2 * 64 * 32 FMA per pixel) is small enough
// for the CUDA cores: the kernel streams g, hsum and the windows from HBM
// once.
//
// Each warp works on its own: it owns the whole 64 x 32 tile of D (lane
// (rg, cg) = (lane / 4, lane % 4) holds rows {j, 32 + j : j = rg + 8i} and
// columns {cg + 4i}), and takes segments of consecutive 32-pixel chunks.  Per
// chunk it stages, with asynchronous copies into one of two buffers of its
// own, the chunk's g and hsum rows ([32 channels][32 pixels]) and its window
// matrix B ([32][32 pixels], gathered element by element from the input),
// then accumulates 4 pixels at a time with packed two-lane FMAs
// (fma.rn.f32x2): the two halves of each accumulator take the even and the
// odd pixels, so the operands come as loaded, without packing.  Shared-memory
// rows are 36 floats apart, so the 16-byte loads of a quarter-warp (two rows
// of A, or four of B) fall in distinct banks.
//
// At the end of a segment the warp writes its partial D (even + odd halves)
// to the segment's slice of the workspace, in the layout of the tensor-core
// kernel's partials, and the same fixed-order fp64 reduction
// (tc_wgrad_reduce) applies the epilogue.  No floating-point atomics; the
// result is deterministic.
#include <algorithm>

#include "pc2d_tc.cuh"
#include "pc2d_tc_common.cuh"

namespace pc2d {
namespace {
using namespace sm100;

constexpr int kWarps = 4;                    // warps per CTA (independent)
constexpr int kNwThreads = 32 * kWarps;
constexpr int kPitch = 36;                   // floats per shared row (32 pixels + 4)
constexpr int kTile = 32 * kPitch;           // floats of one [32][36] tile
constexpr int kStage = 3 * kTile;            // g, hsum and window tiles of one chunk
constexpr int kNwSmem = kWarps * 2 * kStage * 4;  // two stages per warp: 110,592 bytes
constexpr int kCols = 32;                    // columns of the partial layout (NR)
constexpr int kRowsJM = 32;                  // g rows start at row 32 (JM of the partial layout)
constexpr int kMaxSegNw = 128;               // chunks per segment at most

struct NwCfg {
  int cpi;          // 32-pixel chunks per image
  int64_t chunks;   // n * cpi
  int SEG;          // chunks per segment
  int64_t nseg;     // segments (= work items, one warp each)
  int vec;          // 1: g/hsum rows staged as 16-byte pieces (PQ % 4 == 0, 16-byte aligned)
};

NwCfg nw_cfg(const Problem &p, int sms) {
  NwCfg c;
  c.cpi = ceil_div(p.PQ, 32);
  c.chunks = (int64_t)p.n * c.cpi;
  const int64_t warps = (int64_t)std::max(1, sms) * 2 * kWarps;  // two CTAs per SM
  // the segment length whose critical path (rounds of segments per warp x
  // chunks per segment, plus about one chunk's time for the epilogue) is
  // shortest
  c.SEG = kMaxSegNw;
  int64_t best = -1;
  for (int seg = 8; seg <= kMaxSegNw; ++seg) {
    const int64_t items = (c.chunks + seg - 1) / seg;
    const int64_t cost = (items + warps - 1) / warps * (seg + 1);
    if (best < 0 || cost < best) {
      best = cost;
      c.SEG = seg;
    }
  }
  c.nseg = (c.chunks + c.SEG - 1) / c.SEG;
  c.vec = 0;
  return c;
}

inline size_t nw_part_bytes(const NwCfg &c) { return align_up((size_t)c.nseg * 128 * kCols * 4, 256); }
inline size_t nw_sums_bytes(const NwCfg &c) { return align_up((size_t)c.nseg * 128 * 4, 256); }

// 16-byte asynchronous copy global -> shared; with valid == false nothing is
// read and the destination is zero-filled.
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src),
               "r"(valid ? 16 : 0)
               : "memory");
}

__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ void fma2(uint64_t &acc, uint64_t a, uint64_t b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}

// Stages chunk gc: g and hsum rows of the m channels (rows >= m stay zero)
// and the chunk's window matrix (rows >= d keep their constant values).
__device__ __forceinline__ void nw_issue(const float *__restrict__ grad, const float *__restrict__ x,
                                         const float *__restrict__ hsum, const Problem &p, const NwCfg &c,
                                         int64_t gc, float *st, int lane, int koff) {
  const int64_t n = gc / c.cpi;
  const int pq0 = (int)(gc - n * c.cpi) * 32;
  const int64_t rbase = n * p.m * p.PQ + pq0;
  if (c.vec) {
    const int per_t = 8 * p.m;  // 16-byte pieces of one tensor's rows
    for (int e = lane; e < 2 * per_t; e += 32) {
      const int t = e >= per_t ? 1 : 0, rem = e - t * per_t;
      const int row = rem >> 3, pc = rem & 7;
      const bool ok = pq0 + 4 * pc < p.PQ;
      const float *src = (t ? hsum : grad) + rbase + (int64_t)row * p.PQ + 4 * pc;
      cp_async16(st + t * kTile + row * kPitch + 4 * pc, ok ? src : grad, ok);
    }
  } else {
    const bool ok = pq0 + lane < p.PQ;
    for (int row = 0; row < p.m; ++row) {
      const int64_t o = rbase + (int64_t)row * p.PQ + lane;
      cp_async4(st + row * kPitch + lane, ok ? grad + o : grad, ok);
      cp_async4(st + kTile + row * kPitch + lane, ok ? hsum + o : hsum, ok);
    }
  }
  const int pq = pq0 + lane;
  const bool pv = pq < p.PQ;
  int64_t pbase = 0;
  if (pv) {
    const int oy = pq / p.Q, ox = pq - oy * p.Q;
    pbase = n * p.CHW + (int64_t)oy * p.s0 * p.W + (int64_t)ox * p.s1;
  }
  float *bt = st + 2 * kTile;
  for (int k = 0; k < (int)p.d; ++k) {
    const int ko = __shfl_sync(0xffffffffu, koff, k);
    cp_async4(bt + k * kPitch + lane, pv ? x + pbase + ko : x, pv);
  }
}

__global__ void __launch_bounds__(kNwThreads, 2)
nw_wgrad_kernel(const float *__restrict__ grad, const float *__restrict__ x, const float *__restrict__ hsum,
                Problem p, NwCfg c, float *__restrict__ part, float *__restrict__ sums) {
  extern __shared__ __align__(16) float nw_smem[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float *wb = nw_smem + (size_t)warp * 2 * kStage;
  // the reduction launched after this grid waits for it to complete; let it
  // be scheduled as this grid's CTAs finish
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // constant parts of both stages: channel rows past m zero; window rows past
  // d: the ones row at d, zeros beyond
  for (int s = 0; s < 2; ++s) {
    float *st = wb + s * kStage;
    for (int e = lane; e < kTile; e += 32) {
      const int row = e / kPitch;
      if (row >= p.m) {
        st[e] = 0.f;
        st[kTile + e] = 0.f;
      }
      if (row >= p.d) st[2 * kTile + e] = row == p.d ? 1.f : 0.f;
    }
  }
  __syncwarp();
  // this lane's window element k = lane (< d): its offset in an image
  int koff = 0;
  if (lane < p.d) {
    const int ch = lane / p.T, tap = lane - ch * p.T;
    koff = ch * (int)p.HW + tap_row(p, tap) * p.W + tap_col(p, tap);
  }
  const int rg = lane >> 2, cg = lane & 3;
  const int64_t nwarps = (int64_t)gridDim.x * kWarps;
  for (int64_t item = (int64_t)blockIdx.x * kWarps + warp; item < c.nseg; item += nwarps) {
    const int64_t g0 = item * c.SEG, g1 = std::min<int64_t>(c.chunks, g0 + c.SEG);
    uint64_t acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0ull;
    nw_issue(grad, x, hsum, p, c, g0, wb, lane, koff);
    cp_async_commit();
    for (int64_t gc = g0; gc < g1; ++gc) {
      const int s = (int)((gc - g0) & 1);
      if (gc + 1 < g1) {
        nw_issue(grad, x, hsum, p, c, gc + 1, wb + (s ^ 1) * kStage, lane, koff);
        cp_async_commit();
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncwarp();
      const float *G = wb + s * kStage, *Hs = G + kTile, *B = Hs + kTile;
#pragma unroll 2
      for (int q = 0; q < 8; ++q) {
        const int o = 4 * q;
        ulonglong2 gv[4], hv[4], bv[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          gv[i] = *reinterpret_cast<const ulonglong2 *>(G + (rg + 8 * i) * kPitch + o);
          hv[i] = *reinterpret_cast<const ulonglong2 *>(Hs + (rg + 8 * i) * kPitch + o);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) bv[i] = *reinterpret_cast<const ulonglong2 *>(B + (cg + 4 * i) * kPitch + o);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint64_t ghx = mul2(gv[i].x, hv[i].x), ghy = mul2(gv[i].y, hv[i].y);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            fma2(acc[i][k], ghx, bv[k].x);
            fma2(acc[i][k], ghy, bv[k].y);
            fma2(acc[4 + i][k], gv[i].x, bv[k].x);
            fma2(acc[4 + i][k], gv[i].y, bv[k].y);
          }
        }
      }
      __syncwarp();
    }
    // partial of this segment: rows j (g*hsum) and 32 + j (g), columns k
    float *dst = part + (size_t)item * 128 * kCols;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = (i < 4 ? 0 : kRowsJM) + rg + 8 * (i & 3);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int col = cg + 4 * k;
        const float v = __uint_as_float((uint32_t)acc[i][k]) + __uint_as_float((uint32_t)(acc[i][k] >> 32));
        dst[r * kCols + col] = v;
        if (col == p.d) sums[item * 128 + r] = v;
      }
    }
  }
  // This grid may have started while the kernel before it was still running
  // (programmatic launch); it ends only after that kernel has completed, so
  // that work after it on the stream never overtakes that kernel.
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

PerContext<uint64_t> g_nw_attr;

}  // namespace

bool nw_wgrad_supported(const Problem &p) {
  return p.NPQ > 0 && p.m >= 1 && p.m <= 32 && p.d <= 31 && p.CHW < ((int64_t)1 << 31) &&
         (int64_t)p.n * p.m * p.PQ < ((int64_t)1 << 40);
}

size_t nw_wgrad_workspace(const Problem &p) {
  const NwCfg c = nw_cfg(p, device_sm_count());
  return nw_part_bytes(c) + nw_sums_bytes(c);
}

int nw_wgrad(const Problem &p, const float *grad, const float *x, const float *pars, const float *hsum, double factor,
             float *dpars, void *ws, cudaStream_t stream) {
  NwCfg c = nw_cfg(p, device_sm_count());
  c.vec = (p.PQ % 4 == 0 && ((reinterpret_cast<uintptr_t>(grad) | reinterpret_cast<uintptr_t>(hsum)) & 15) == 0) ? 1
                                                                                                                : 0;
  float *part = reinterpret_cast<float *>(ws);
  float *sums = reinterpret_cast<float *>(reinterpret_cast<char *>(ws) + nw_part_bytes(c));
  const int ast = once_per_context(g_nw_attr, 1, []() -> int {
    PC2D_CUDA_CHECK(cudaFuncSetAttribute(nw_wgrad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kNwSmem));
    return (int)PC2D_OK;
  });
  if (ast != PC2D_OK) return ast;
  const int grid = (int)std::min<int64_t>((c.nseg + kWarps - 1) / kWarps, (int64_t)device_sm_count() * 2);
  timing_begin(K_WGRAD, stream);
  {
    // programmatic dependent launch, as the tensor-core parameter-gradient
    // kernel: it reads none of the input-gradient kernel's outputs
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kNwThreads);
    cfg.dynamicSmemBytes = kNwSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    PC2D_CUDA_CHECK(cudaLaunchKernelEx(&cfg, nw_wgrad_kernel, grad, x, hsum, p, c, part, sums));
  }
  timing_end(K_WGRAD, stream);
  PC2D_LAUNCH_CHECK("nw_wgrad_kernel");
  return tc_wgrad_reduce(p, part, sums, pars, factor, dpars, c.nseg, 1, 1, kRowsJM, kCols, stream);
}

}  // namespace pc2d
