// tcgen05 forward kernel of the ParaConv2d paraboloid convolution (fp32 via
// 3xTF32 split precision).
//
// Decomposition of the reference forward (paraconv2d.cc:82-122): for output
// pixel i and output channel j, with win the flipped window of pixel i,
//   hsum = h0[j] + H[j].win
//   out  = f * (hsum^2 - S2[i] + 2 P[j].win - |P[j]|^2 - p0[j]^2),
//   S2[i] = sum_k win[k]^2
// so the two contractions H.win and P.win are one implicit GEMM
//   D[i][0:NB]   = win_i . H[j]^T,   D[i][NB:2NB] = win_i . P[j]^T
// with M = 128 output pixels per tile, N = 2*NB (NB <= 64 output channels
// per channel block) and K = the window (C*k0*k1), swept 32 at a time.
//
// Operands:
//   A (the im2col window, M x K) lives in Tensor Memory.  Producer warps
//     (one TMEM lane = one output pixel per thread) gather the window from
//     global memory (coalesced across the 32 pixels of a warp), split every
//     value into tf32 hi + lo, accumulate S2 on the way, and tcgen05.st the
//     hi and lo slices into a 4-stage ring of TMEM columns.  A never touches
//     shared memory.
//   B (weights [H;P], N x K) is split into hi/lo once per call by a prep
//     kernel, already in the 128-byte-swizzled K-major layout, and streamed
//     into a 4-stage shared-memory ring by 1-D bulk async copies.
//   D (N fp32 accumulator columns per tile) is double-buffered in TMEM, so
//     the epilogue of tile t overlaps the MMAs of tile t+1.
// Each 8-wide K step issues three MMAs: Ahi*Bhi + Alo*Bhi + Ahi*Blo.
//
// Warp roles (320 threads, one CTA per SM, persistent over work items):
//   warps 0-3 producers, warp 4 MMA issuer (and TMEM owner), warp 5 B
//   loader, warps 6-9 epilogue.  All barrier waits are bounded in time; a
//   wait that gives up records PC2D_ERR_TIMEOUT, raises a CTA-wide abort
//   flag, and the CTA drains its in-flight copies and MMAs and exits.
#include <algorithm>
#include <mutex>

#include "pc2d_sm100.cuh"
#include "pc2d_tc.cuh"

namespace pc2d {

namespace {
using namespace sm100;

constexpr int kTileM = 128;
constexpr int kKC = 32;
constexpr int kAStages = 4;
constexpr int kBStages = 4;
constexpr int kMaxNB = 64;
constexpr int kMaxD = 8192;
constexpr int kFwdThreads = 320;
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr int kMinSmem = 120 * 1024;  // keeps one CTA per SM (it owns all 512 TMEM columns)

struct FwdCfg {
  int ncb;         // channel blocks
  int NB;          // channels per block (multiple of 8, <= 64)
  int N;           // MMA N = 2*NB
  int nK;          // 32-wide K chunks
  int64_t tiles;   // 128-pixel tiles
  int64_t items;   // tiles * ncb
};

FwdCfg fwd_cfg(const Problem &p) {
  FwdCfg c;
  c.ncb = std::max(1, ceil_div(p.m, kMaxNB));
  const int nb = ceil_div(p.m, c.ncb);
  c.NB = (nb + 7) / 8 * 8;
  c.N = 2 * c.NB;
  c.nK = ceil_div(p.d, kKC);
  c.tiles = (p.NPQ + kTileM - 1) / kTileM;
  c.items = c.tiles * c.ncb;
  return c;
}

inline size_t fwd_bsplit_bytes(const FwdCfg &c) { return (size_t)c.ncb * c.nK * 2 * c.N * 128; }
__host__ __device__ inline uint32_t fwd_bstage_bytes(const FwdCfg &c) { return (uint32_t)(2 * c.N * 128); }
inline size_t fwd_smem_bytes(const FwdCfg &c) {
  size_t s = 1024 + (size_t)kBStages * fwd_bstage_bytes(c) + (size_t)c.nK * kKC * 4 + 2 * kTileM * 4 + 32 * 8 + 64;
  return std::max<size_t>(s, kMinSmem);
}

// Splits [H;P] of channel block cb into hi/lo tf32 halves in the swizzled
// K-major layout the MMA reads: block (cb, kc) = [hi: N rows][lo: N rows],
// each row 32 floats of K with 16-byte chunk c stored at c ^ (row % 8).
// Rows 0..NB-1 are H of channels cb*NB.., rows NB..2NB-1 are P; channels >= m
// and K >= d are zero.
__global__ void tc_fwd_prep_weights(const float *__restrict__ pars, Problem p, FwdCfg c, float *__restrict__ wsB) {
  const int kc = blockIdx.x, cb = blockIdx.y;
  float *blk = wsB + ((int64_t)cb * c.nK + kc) * 2 * c.N * 32;
  const float *h = pars + p.m;
  const float *pp = h + (int64_t)p.m * p.d;
  for (int e = threadIdx.x; e < c.N * 32; e += blockDim.x) {
    const int r = e / 32, kk = e % 32;
    const int half = r / c.NB;
    const int j = cb * c.NB + (r - half * c.NB);
    const int64_t k = (int64_t)kc * 32 + kk;
    float v = 0.f;
    if (j < p.m && k < p.d) v = (half == 0 ? h : pp)[(int64_t)j * p.d + k];
    const float hi = __uint_as_float(tf32_hi_bits(v));
    const int pos = r * 32 + (((kk >> 2) ^ (r & 7)) << 2) + (kk & 3);
    blk[pos] = hi;
    blk[c.N * 32 + pos] = v - hi;
  }
}

// cj[cb*NB + jn] = |P[j]|^2 + p0[j]^2 (fp64 accumulation), 0 for padded channels.
__global__ void tc_fwd_prep_consts(const float *__restrict__ pars, Problem p, FwdCfg c, float *__restrict__ cj) {
  const int slot = blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (slot >= c.ncb * c.NB) return;
  const int cb = slot / c.NB;
  const int j = cb * c.NB + (slot - cb * c.NB);
  double acc = 0.0;
  if (j < p.m) {
    const float *pj = pars + p.m + (int64_t)p.m * p.d + (int64_t)j * p.d;
    for (int64_t k = lane; k < p.d; k += 32) {
      const double v = pj[k];
      acc += v * v;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    float r = 0.f;
    if (j < p.m) {
      const double p0 = pars[p.m + 2 * (int64_t)p.m * p.d + j];
      r = (float)(acc + p0 * p0);
    }
    cj[slot] = r;
  }
}

// Warp-uniform bounded wait: every lane polls, the warp agrees on the result.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  const bool ok = mbar_wait(bar, parity, kWaitNs, abort_flag);
  return __all_sync(0xffffffffu, ok);
}

__global__ void __launch_bounds__(kFwdThreads, 1)
tc_forward_kernel(const float *__restrict__ x, const float *__restrict__ pars, const float *__restrict__ wsB,
                  const float *__restrict__ cj, float factor, Problem p, FwdCfg c, float *__restrict__ out,
                  float *__restrict__ hsum, int *status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t bstage = fwd_bstage_bytes(c);
  uint8_t *sB = smem;
  const int dpad = c.nK * kKC;
  int *koff = reinterpret_cast<int *>(smem + kBStages * bstage);
  float *s2buf = reinterpret_cast<float *>(koff + dpad);
  uint64_t *bars = reinterpret_cast<uint64_t *>(s2buf + 2 * kTileM);
  uint64_t *a_full = bars, *a_empty = bars + 4, *b_full = bars + 8, *b_empty = bars + 12;
  uint64_t *d_full = bars + 16, *d_empty = bars + 18, *s2_full = bars + 20, *s2_empty = bars + 22;
  uint64_t *final_bar = bars + 24;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 25);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

  // Per-K input offset of the flipped window relative to the window origin;
  // -1 marks the zero padding of the last K chunk.
  for (int k = threadIdx.x; k < dpad; k += blockDim.x) {
    int v = -1;
    if (k < p.d) {
      const int ch = k / p.T, tap = k - ch * p.T;
      v = (int)((int64_t)ch * p.HW + (int64_t)tap_row(p, tap) * p.W + tap_col(p, tap));
    }
    koff[k] = v;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) {
      mbar_init(&a_full[i], 128);
      mbar_init(&a_empty[i], 1);
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&d_full[i], 1);
      mbar_init(&d_empty[i], 128);
      mbar_init(&s2_full[i], 128);
      mbar_init(&s2_empty[i], 128);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int m = p.m;

  if (warp < 4) {
    // ---------------------------------------------------------- producers
    const int r = threadIdx.x;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    uint32_t it = 0, tcount = 0;
    bool ok = true;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
      const int64_t t = item / c.ncb;
      const int64_t g = t * kTileM + r;
      const bool valid = g < p.NPQ;
      int64_t base = 0;
      if (valid) {
        const int64_t nn = g / p.PQ;
        const int64_t rr = g - nn * p.PQ;
        const int oy = (int)(rr / p.Q), ox = (int)(rr - (int64_t)oy * p.Q);
        base = nn * p.CHW + (int64_t)oy * p.s0 * p.W + (int64_t)ox * p.s1;
      }
      const float *xb = x + base;
      float s2 = 0.f;
      for (int kc = 0; kc < c.nK; ++kc) {
        const uint32_t st = it % kAStages, ph = (it / kAStages) & 1;
        if (!warp_wait(&a_empty[st], ph ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int kk = 0; kk < 32; ++kk) {
          const int o = koff[kc * kKC + kk];
          const float v = (valid && o >= 0) ? __ldg(xb + o) : 0.f;
          s2 = fmaf(v, v, s2);
          hi[kk] = tf32_hi_bits(v);
          lo[kk] = __float_as_uint(v - __uint_as_float(hi[kk]));
        }
        const uint32_t acol = tmem + lane_off + 256 + st * 64;
        tmem_st16(acol, *reinterpret_cast<const uint32_t(*)[16]>(&hi[0]));
        tmem_st16(acol + 16, *reinterpret_cast<const uint32_t(*)[16]>(&hi[16]));
        tmem_st16(acol + 32, *reinterpret_cast<const uint32_t(*)[16]>(&lo[0]));
        tmem_st16(acol + 48, *reinterpret_cast<const uint32_t(*)[16]>(&lo[16]));
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&a_full[st]);
        ++it;
      }
      if (!ok) break;
      const uint32_t b = tcount & 1, ph = (tcount >> 1) & 1;
      if (!warp_wait(&s2_empty[b], ph ^ 1, abort_flag)) {
        ok = false;
        break;
      }
      s2buf[b * kTileM + r] = s2;
      mbar_arrive(&s2_full[b]);
      ++tcount;
    }
    if (!ok) {
      if (lane == 0) record_device_error(status, PC2D_ERR_TIMEOUT);
      *abort_flag = 1;
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------- MMA
    const uint32_t idesc = idesc_tf32(kTileM, c.N);
    const uint32_t sB_addr = smem_u32(sB);
    uint32_t it = 0, tcount = 0;
    bool ok = true;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
      const uint32_t b = tcount & 1, ph = (tcount >> 1) & 1;
      if (!warp_wait(&d_empty[b], ph ^ 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t dcol = tmem + b * 128;
      for (int kc = 0; kc < c.nK; ++kc) {
        const uint32_t sa = it % kAStages, pa = (it / kAStages) & 1;
        const uint32_t sb = it % kBStages, pb = (it / kBStages) & 1;
        if (!warp_wait(&a_full[sa], pa, abort_flag) || !warp_wait(&b_full[sb], pb, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t ahi = tmem + 256 + sa * 64, alo = ahi + 32;
          const uint32_t bhi = sB_addr + sb * bstage, blo = bhi + c.N * 128;
#pragma unroll
          for (int ks = 0; ks < kKC / 8; ++ks) {
            const uint64_t dhi = sdesc_kmajor_sw128(bhi + ks * 32);
            const uint64_t dlo = sdesc_kmajor_sw128(blo + ks * 32);
            const uint32_t acc = (kc > 0 || ks > 0) ? 1u : 0u;
            mma_tf32_ts(dcol, ahi + ks * 8, dhi, idesc, acc);
            mma_tf32_ts(dcol, alo + ks * 8, dhi, idesc, 1u);
            mma_tf32_ts(dcol, ahi + ks * 8, dlo, idesc, 1u);
          }
          tc_commit(&a_empty[sa]);
          tc_commit(&b_empty[sb]);
        }
        __syncwarp();
        ++it;
      }
      if (!ok) break;
      if (lane == 0) tc_commit(&d_full[b]);
      __syncwarp();
      ++tcount;
    }
    if (!ok) {
      if (lane == 0) record_device_error(status, PC2D_ERR_TIMEOUT);
      *abort_flag = 1;
    }
    // Drain: every MMA issued by this warp completes before TMEM is freed.
    if (lane == 0) tc_commit(final_bar);
    __syncwarp();
    mbar_wait(final_bar, 0, kWaitNs, nullptr);
  } else if (warp == 5) {
    // ---------------------------------------------------------- B loader
    uint32_t it = 0;
    bool ok = true;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
      const int cb = (int)(item % c.ncb);
      for (int kc = 0; kc < c.nK; ++kc) {
        const uint32_t sb = it % kBStages, pb = (it / kBStages) & 1;
        if (!warp_wait(&b_empty[sb], pb ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&b_full[sb], bstage);
          bulk_g2s(sB + sb * bstage, wsB + ((int64_t)cb * c.nK + kc) * 2 * c.N * 32, bstage, &b_full[sb]);
        }
        __syncwarp();
        ++it;
      }
    }
    if (!ok) {
      if (lane == 0) record_device_error(status, PC2D_ERR_TIMEOUT);
      *abort_flag = 1;
    }
    // Drain: the copies issued last have landed before the CTA exits.
    const uint32_t last = std::min<uint32_t>(it, kBStages);
    for (uint32_t i = 0; i < last; ++i) {
      const uint32_t idx = it - 1 - i;
      mbar_wait(&b_full[idx % kBStages], (idx / kBStages) & 1, kWaitNs, nullptr);
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const int q = warp % 4;
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const float *h0 = pars;
    uint32_t tcount = 0;
    bool ok = true;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
      const int64_t t = item / c.ncb;
      const int cb = (int)(item - t * c.ncb);
      const uint32_t b = tcount & 1, ph = (tcount >> 1) & 1;
      if (!warp_wait(&d_full[b], ph, abort_flag) || !warp_wait(&s2_full[b], ph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float s2 = s2buf[b * kTileM + r];
      mbar_arrive(&s2_empty[b]);
      const int64_t g = t * kTileM + r;
      const bool valid = g < p.NPQ;
      int64_t obase = 0;
      if (valid) {
        const int64_t nn = g / p.PQ;
        obase = nn * (int64_t)m * p.PQ + (g - nn * p.PQ);
      }
      const uint32_t dcol = tmem + lane_off + b * 128;
      for (int jc = 0; jc < c.NB; jc += 8) {
        float hv[8], pv[8];
        tmem_ld8(dcol + jc, hv);
        tmem_ld8(dcol + c.NB + jc, pv);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const int j = cb * c.NB + jc + jj;
          if (valid && j < m) {
            const float hs = hv[jj] + __ldg(h0 + j);
            const float o = factor * (fmaf(hs, hs, -s2) + 2.f * pv[jj] - __ldg(cj + cb * c.NB + jc + jj));
            const int64_t oi = obase + (int64_t)j * p.PQ;
            out[oi] = o;
            hsum[oi] = hs;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&d_empty[b]);
      ++tcount;
    }
    if (!ok) {
      if (lane == 0) record_device_error(status, PC2D_ERR_TIMEOUT);
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

__global__ void selftest_wait_kernel(unsigned int timeout_us, int *status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait(&bar, 0, (uint64_t)timeout_us * 1000ull, nullptr))
    record_device_error(status, PC2D_ERR_TIMEOUT);
}

std::mutex g_attr_mutex;
bool g_attr_set[64] = {false};
int g_sm_count[64] = {0};

}  // namespace

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  if (g_sm_count[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    g_sm_count[dev] = v;
  }
  return g_sm_count[dev];
}

bool tc_forward_supported(const Problem &p) {
  return p.m >= 1 && p.d <= kMaxD && p.CHW < ((int64_t)1 << 31) && p.NPQ > 0;
}

size_t tc_forward_workspace(const Problem &p) {
  const FwdCfg c = fwd_cfg(p);
  return align_up(fwd_bsplit_bytes(c), 256) + align_up((size_t)c.ncb * c.NB * sizeof(float), 256);
}

int tc_forward(const Problem &p, const float *x, const float *pars, double factor, float *out, float *hsum, void *ws,
               cudaStream_t stream) {
  const FwdCfg c = fwd_cfg(p);
  int *status = device_status_ptr();
  if (!status) {
    set_last_error("could not resolve the device status word");
    return PC2D_ERR_CUDA;
  }
  float *wsB = reinterpret_cast<float *>(ws);
  float *cj = reinterpret_cast<float *>(reinterpret_cast<char *>(ws) + align_up(fwd_bsplit_bytes(c), 256));
  tc_fwd_prep_weights<<<dim3(c.nK, c.ncb), 256, 0, stream>>>(pars, p, c, wsB);
  PC2D_LAUNCH_CHECK("tc_fwd_prep_weights");
  tc_fwd_prep_consts<<<ceil_div(c.ncb * c.NB, 8), 256, 0, stream>>>(pars, p, c, cj);
  PC2D_LAUNCH_CHECK("tc_fwd_prep_consts");
  const size_t smem = fwd_smem_bytes(c);
  {
    int dev = 0;
    PC2D_CUDA_CHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    if (dev >= 0 && dev < 64 && !g_attr_set[dev]) {
      PC2D_CUDA_CHECK(cudaFuncSetAttribute(tc_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
      g_attr_set[dev] = true;
    }
  }
  const int grid = (int)std::min<int64_t>(c.items, device_sm_count());
  tc_forward_kernel<<<grid, kFwdThreads, smem, stream>>>(x, pars, wsB, cj, (float)factor, p, c, out, hsum, status);
  PC2D_LAUNCH_CHECK("tc_forward_kernel");
  return PC2D_OK;
}

int tc_selftest_bounded_wait(unsigned int timeout_us, int *status, cudaStream_t stream) {
  selftest_wait_kernel<<<1, 32, 0, stream>>>(timeout_us, status);
  PC2D_LAUNCH_CHECK("selftest_wait_kernel");
  return PC2D_OK;
}

}  // namespace pc2d
