// Input gradient of the ParaConv2d paraboloid convolution for narrow inputs
// (few input channels), as a dense tcgen05 GEMM over the output pixels
// followed by a col2im gather (fp32 via 3xTF32 split precision).
//
// The input-gradient (reference paraconv2d.cc:153-183)
//   dx[c,y,x] = 2 * (sum_{tap, o: window(o,tap) = (y,x)}
//                      sum_j (g*hsum)[j,o] h[j,c,tap] + g[j,o] p[j,c,tap]
//                    - x[c,y,x] * SG[y,x]),   SG = sum_{tap,o} sum_j g[j,o]
// splits into
//   Y[o, (c,tap)] = sum_j (g*hsum)[j,o] h[j,c,tap] + g[j,o] p[j,c,tap]
//   Y[o, SG]      = sum_j g[j,o]
// a GEMM with M = 128 output pixels of one image per tile, N = C*T + 1
// window columns (<= 192) and K = (j, {g*hsum, g}) = 2m, and
//   dx[c,y,x] = 2 * (sum_{tap} Y[o(y,x,tap), (c,tap)] - x[c,y,x] * sum_{tap} Y[o(y,x,tap), SG])
// over the taps whose output pixel o exists (col2im).  For C input channels
// the implicit GEMM of pc2d_tc_bwd.cu runs its channel dimension as an MMA N
// of 16 per block; this form puts C*T + 1 window columns there instead.
//
// GEMM kernel roles (448 threads, one CTA per SM, persistent over tiles):
//   - warps 0-3, producers (one TMEM lane = one output pixel): per 32-K
//     stage read g and hsum of 16 output channels at their pixel (from the
//     [16 x 128] tiles the loader staged, or straight from global memory
//     with an L2 prefetch of the next stage), form g*hsum and g, split into
//     tf32 hi + lo and tcgen05.st them (A operand);
//   - warps 4-7 and 10-13, epilogue (two warps per TMEM lane quarter, half
//     of the columns each): drain the tile's accumulator (one of two TMEM
//     slots) and write Y[n][col][o] (coalesced across pixels);
//   - warp 8, MMA: one elected lane issues Ahi*Bhi + Alo*Bhi + Ahi*Blo
//     (N = NP) per 8-wide K step, straight-line;
//   - warp 9, loader: per stage the g and hsum tiles (two 2-D tensor copies)
//     and one bulk copy of the pre-split weights.
// Every wait is bounded; on a timeout the kernel records the error, stops,
// drains its copies and MMAs and frees TMEM.
#include <algorithm>
#include <climits>
#include <cstring>
#include <mutex>

#include "pc2d_tc.cuh"
#include "pc2d_tc_common.cuh"

namespace pc2d {

namespace {
using namespace sm100;
using tc::kWaitNs;
using tc::warp_wait;

constexpr int kTileM = 128;
constexpr int kKS = 32;
constexpr int kStages = 2;        // A stages in TMEM
constexpr int kSlots = 2;         // accumulator slots
constexpr int kMaxNP = 192;       // GEMM N (window columns + SG, multiple of 16)
constexpr uint32_t kColSlot = 192;  // slot s at s * 192
constexpr uint32_t kColA = 384;     // A stage st at 384 + 64 * st
constexpr int kThreads = 448;
constexpr int kMinSmem = 120 * 1024;
constexpr int kSmemLimit = 227 * 1024;

struct DcCfg {
  int NY;           // Y columns: C*T + 1 (the last one is SG)
  int NP;           // GEMM N: NY rounded up to 16
  int nK;           // 32-K stages: K = 2m rounded up to 32
  int tpi;          // 128-pixel tiles per image
  int64_t tiles;    // n * tpi
  uint32_t bstage;  // bytes of one stage's B: [hi: NP rows][lo: NP rows] x 128 B
  int tma;          // 1: a stage's g and hsum tiles [16 channels][128 pixels] are 2-D tensor copies
};

DcCfg dc_cfg(const Problem &p) {
  DcCfg c;
  c.NY = p.C * p.T + 1;
  c.NP = (c.NY + 15) / 16 * 16;
  c.nK = ceil_div(2 * p.m, kKS);
  c.tpi = (int)((p.PQ + kTileM - 1) / kTileM);
  c.tiles = (int64_t)p.n * c.tpi;
  c.bstage = (uint32_t)(2 * c.NP * 128);
  c.tma = (p.PQ % 4 == 0 && (int64_t)p.n * p.m < ((int64_t)1 << 31)) ? 1 : 0;
  return c;
}

inline size_t dc_bsplit_bytes(const DcCfg &c) { return (size_t)c.nK * c.bstage; }
inline size_t dc_y_bytes(const Problem &p, const DcCfg &c) { return (size_t)p.n * c.NY * p.PQ * sizeof(float); }
constexpr uint32_t kTileBytes = 16 * kTileM * 4;  // one [16 channels][128 pixels] tile
inline size_t dc_smem_bytes(const DcCfg &c) {
  const size_t s = 1024 + (size_t)kStages * (c.bstage + 2 * kTileBytes) + 16 * 8 + 64;
  return std::max<size_t>(s, kMinSmem);
}

// B (weights) in the swizzled K-major layout the MMA reads: block kq =
// [hi: NP rows][lo: NP rows], row n = window column, 32 K per row with 16-byte
// chunk c stored at c ^ (n % 8).  K element k = 2j + w: w = 0 multiplies
// g*hsum (h[j][n]), w = 1 multiplies g (p[j][n]; 1 in the SG column).
// Grid (nK, NP / 16).
__global__ void __launch_bounds__(256) tc_dc_prep_weights(const float *__restrict__ pars, Problem p, DcCfg c,
                                                          float *__restrict__ wsB) {
  const int kq = blockIdx.x;
  float *blk = wsB + (int64_t)kq * 2 * c.NP * 32;
  const float *h = pars + p.m;
  const float *pp = h + (int64_t)p.m * p.d;
  for (int e = threadIdx.x; e < 16 * 32; e += blockDim.x) {
    const int n = blockIdx.y * 16 + e / 32, kk = e % 32;
    const int k = kq * kKS + kk, j = k / 2, w = k & 1;
    float v = 0.f;
    if (j < p.m) {
      if (n < c.NY - 1) v = (w == 0 ? h : pp)[(int64_t)j * p.d + n];
      else if (n == c.NY - 1) v = w == 1 ? 1.f : 0.f;
    }
    float hi, lo;
    tf32_split_rn(v, hi, lo);
    const int pos = n * 32 + (((kk >> 2) ^ (n & 7)) << 2) + (kk & 3);
    blk[pos] = hi;
    blk[c.NP * 32 + pos] = lo;
  }
}

// Epilogue of one warp: 16-column blocks C0 .. C1-1 of its 32 lanes' rows of
// the accumulator, two blocks per wait, written to Y (column stride PQ).
template <int C0, int C1>
__device__ __forceinline__ void dc_drain(uint32_t dcol, float *yb, bool valid, int NY, int64_t PQ) {
#pragma unroll
  for (int ch = C0; ch < C1; ch += 2) {
    const int cc = ch * 16;
    uint32_t v[16], w[16];
    if (ch + 1 < C1) {
      tmem_ld16_nowait(dcol + cc, v);
      tmem_ld16_nowait(dcol + cc + 16, w);
      tmem_ld_wait_tie(v, w);
    } else {
      tmem_ld16_nowait(dcol + cc, v);
      tmem_ld_wait_tie(v);
    }
    if (valid) {
#pragma unroll
      for (int q = 0; q < 16; ++q)
        if (cc + q < NY) yb[(int64_t)(cc + q) * PQ] = __uint_as_float(v[q]);
      if (ch + 1 < C1) {
#pragma unroll
        for (int q = 0; q < 16; ++q)
          if (cc + 16 + q < NY) yb[(int64_t)(cc + 16 + q) * PQ] = __uint_as_float(w[q]);
      }
    }
  }
}

template <int NP>
__global__ void __launch_bounds__(kThreads, 1)
tc_dc_gemm_kernel(const float *__restrict__ grad, const float *__restrict__ hsum, const float *__restrict__ wsB,
                  Problem p, DcCfg c, const __grid_constant__ CUtensorMap gmap,
                  const __grid_constant__ CUtensorMap hmap, float *__restrict__ Y, int *status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  uint8_t *sB = base;                                          // kStages x bstage
  float *sT = reinterpret_cast<float *>(sB + (size_t)kStages * c.bstage);  // kStages x [g tile | hsum tile]
  uint64_t *bars = reinterpret_cast<uint64_t *>(sT + kStages * 2 * 16 * kTileM);
  uint64_t *a_full = bars, *s_empty = bars + 2, *d_full = bars + 4, *d_empty = bars + 6, *final_bar = bars + 8;
  uint64_t *t_full = bars + 9, *t_empty = bars + 11;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 13);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      // 128 producer arrivals + the loader's arrival with the bytes of its copy
      mbar_init(&a_full[i], 129);
      mbar_init(&s_empty[i], 1);
    }
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&d_full[i], 1);
      mbar_init(&d_empty[i], 256);
    }
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&t_full[i], 1);
      mbar_init(&t_empty[i], 128);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  bool ok = true;

  if (warp < 4) {
    // ---------------------------------------------------------- producers
    const int r = warp * 32 + lane;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    uint32_t it = 0;
    for (int64_t t = blockIdx.x; t < c.tiles && ok; t += gridDim.x) {
      const int64_t n = t / c.tpi;
      const int o = (int)(t - n * c.tpi) * kTileM + r;
      const bool valid = o < p.PQ;
      const float *g0 = grad + n * p.m * p.PQ + o;
      const float *h0 = hsum + n * p.m * p.PQ + o;
      for (int kq = 0; kq < c.nK; ++kq, ++it) {
        const uint32_t st = it % kStages, ph = (it / kStages) & 1;
        float gv[kKS / 2], hv[kKS / 2];
        if (c.tma) {
          if (!warp_wait(&t_full[st], ph, abort_flag)) {
            ok = false;
            break;
          }
          const float *tg = sT + st * 2 * 16 * kTileM;
#pragma unroll
          for (int jl = 0; jl < kKS / 2; ++jl) {
            const bool in = valid && kq * (kKS / 2) + jl < p.m;
            gv[jl] = in ? tg[jl * kTileM + r] : 0.f;
            hv[jl] = in ? tg[(16 + jl) * kTileM + r] : 0.f;
          }
          mbar_arrive(&t_empty[st]);
        } else {
          // next stage's rows of this pixel into L2
          if (valid && kq + 1 < c.nK) {
#pragma unroll
            for (int jl = 0; jl < kKS / 2; ++jl) {
              const int j = (kq + 1) * (kKS / 2) + jl;
              if (j < p.m) {
                prefetch_l2(g0 + (int64_t)j * p.PQ);
                prefetch_l2(h0 + (int64_t)j * p.PQ);
              }
            }
          }
#pragma unroll
          for (int jl = 0; jl < kKS / 2; ++jl) {
            const int j = kq * (kKS / 2) + jl;
            const bool in = valid && j < p.m;
            gv[jl] = in ? __ldg(g0 + (int64_t)j * p.PQ) : 0.f;
            hv[jl] = in ? __ldg(h0 + (int64_t)j * p.PQ) : 0.f;
          }
        }
        uint32_t hi[kKS], lo[kKS];
#pragma unroll
        for (int jl = 0; jl < kKS / 2; ++jl) {
          const float a0 = gv[jl] * hv[jl], a1 = gv[jl];
          hi[2 * jl] = tf32_hi_bits(a0);
          lo[2 * jl] = __float_as_uint(a0 - __uint_as_float(hi[2 * jl]));
          hi[2 * jl + 1] = tf32_hi_bits(a1);
          lo[2 * jl + 1] = __float_as_uint(a1 - __uint_as_float(hi[2 * jl + 1]));
        }
        // the MMAs that read this A stage last have completed
        if (!warp_wait(&s_empty[st], ph ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acol = tmem + lane_off + kColA + st * 64;
        tmem_st16(acol, *reinterpret_cast<const uint32_t(*)[16]>(&hi[0]));
        tmem_st16(acol + 16, *reinterpret_cast<const uint32_t(*)[16]>(&hi[16]));
        tmem_st16(acol + 32, *reinterpret_cast<const uint32_t(*)[16]>(&lo[0]));
        tmem_st16(acol + 48, *reinterpret_cast<const uint32_t(*)[16]>(&lo[16]));
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&a_full[st]);
      }
    }
  } else if (warp < 8 || warp >= 10) {
    // ---------------------------------------------------------- epilogue
    // Two warps per TMEM lane quarter (warps 4-7 and 10-13; warp w reaches
    // lanes 32*(w%4) .. +31), each draining and writing half of the
    // 16-column blocks.
    constexpr int kCh = NP / 16, kCh0 = (kCh + 1) / 2;
    const int qq = warp % 4, half = warp >= 10 ? 1 : 0;
    const int r = qq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qq * 32) << 16;
    uint32_t ti = 0;
    for (int64_t t = blockIdx.x; t < c.tiles && ok; t += gridDim.x, ++ti) {
      const uint32_t slot = ti % kSlots, ph = (ti / kSlots) & 1;
      if (!warp_wait(&d_full[slot], ph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int64_t n = t / c.tpi;
      const int o = (int)(t - n * c.tpi) * kTileM + r;
      float *yb = Y + n * (int64_t)c.NY * p.PQ + o;
      const uint32_t dcol = tmem + lane_off + slot * kColSlot;
      if (half == 0)
        dc_drain<0, kCh0>(dcol, yb, o < p.PQ, c.NY, p.PQ);
      else
        dc_drain<kCh0, kCh>(dcol, yb, o < p.PQ, c.NY, p.PQ);
      tc_fence_before();
      mbar_arrive(&d_empty[slot]);
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------- MMA
    const uint32_t idesc = idesc_tf32(kTileM, NP);
    constexpr uint32_t kBlo = NP * 128;  // bytes of the hi rows of a stage
    const uint32_t sB_addr = smem_u32(sB);
    uint32_t it = 0, ti = 0;
    for (int64_t t = blockIdx.x; t < c.tiles && ok; t += gridDim.x, ++ti) {
      const uint32_t slot = ti % kSlots;
      if (!warp_wait(&d_empty[slot], ((ti / kSlots) & 1) ^ 1, abort_flag)) {
        ok = false;
        break;
      }
      const uint32_t dcol = tmem + slot * kColSlot;
      for (int kq = 0; kq < c.nK; ++kq, ++it) {
        const uint32_t st = it % kStages, ph = (it / kStages) & 1;
        if (!warp_wait(&a_full[st], ph, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // straight-line issue from one elected lane, operands formed outside
        const uint32_t ahi = tmem + kColA + st * 64, alo = ahi + 32;
        const uint32_t bhi0 = sB_addr + st * c.bstage;
        const uint32_t acc0 = kq == 0 ? 0u : 1u;
        const bool last = kq == c.nK - 1;
        if (elect_one()) {
#pragma unroll
          for (int ks = 0; ks < kKS / 8; ++ks) {
            const uint32_t bhi = bhi0 + ks * 32, blo = bhi + kBlo;
            mma_tf32_ts(dcol, ahi + ks * 8, sdesc_kmajor_sw128(bhi), idesc, ks == 0 ? acc0 : 1u);
            mma_tf32_ts(dcol, alo + ks * 8, sdesc_kmajor_sw128(bhi), idesc, 1u);
            mma_tf32_ts(dcol, ahi + ks * 8, sdesc_kmajor_sw128(blo), idesc, 1u);
          }
          tc_commit(&s_empty[st]);
          if (last) tc_commit(&d_full[slot]);
        }
        __syncwarp();
      }
    }
    if (elect_one()) tc_commit(final_bar);
    __syncwarp();
    mbar_wait(final_bar, 0, kWaitNs, nullptr);
  } else {
    // ------------------------------------------------------------- loader
    uint32_t it = 0;
    for (int64_t t = blockIdx.x; t < c.tiles && ok; t += gridDim.x) {
      const int64_t n = t / c.tpi;
      const int o0 = (int)(t - n * c.tpi) * kTileM;
      for (int kq = 0; kq < c.nK; ++kq, ++it) {
        const uint32_t st = it % kStages, ph = (it / kStages) & 1;
        if (c.tma) {
          // g and hsum of channels kq*16 .. +15 at the tile's pixels (channels
          // past m are never read; pixels past the image are zero)
          if (!warp_wait(&t_empty[st], ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            float *tg = sT + st * 2 * 16 * kTileM;
            const int yc = (int)(n * p.m + kq * (kKS / 2));
            mbar_arrive_expect_tx(&t_full[st], 2 * kTileBytes);
            tma_load_2d(tg, &gmap, o0, yc, &t_full[st]);
            tma_load_2d(tg + 16 * kTileM, &hmap, o0, yc, &t_full[st]);
          }
          __syncwarp();
        }
        if (!warp_wait(&s_empty[st], ph ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&a_full[st], c.bstage);
          bulk_g2s(sB + (size_t)st * c.bstage, wsB + (int64_t)kq * 2 * c.NP * 32, c.bstage, &a_full[st]);
        }
        __syncwarp();
      }
    }
    if (c.tma) {
      const uint32_t tl = it < (uint32_t)kStages ? it : (uint32_t)kStages;
      for (uint32_t i = 0; i < tl; ++i) {
        const uint32_t idx = it - 1 - i;
        mbar_wait(&t_full[idx % kStages], (idx / kStages) & 1, kWaitNs, nullptr);
      }
    }
    // Drain: the copies issued last have landed before the CTA exits (the
    // phase also needs the producers' arrivals, which come on every path
    // that issued the copies without an abort).
    const uint32_t last = it < (uint32_t)kStages ? it : (uint32_t)kStages;
    for (uint32_t i = 0; i < last; ++i) {
      const uint32_t idx = it - 1 - i;
      mbar_wait(&a_full[idx % kStages], (idx / kStages) & 1, kWaitNs, nullptr);
    }
  }

  if (!ok) {
    if (lane == 0) record_device_error(status, PC2D_ERR_TIMEOUT);
    *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// col2im over stride phases: block (bx, n * s0 * s1 + ph) handles input
// pixels (y, x) = (py + s0*a, px + s1*b) of phase ph = (py, px), one thread per
// phase-grid position (a, b), consecutive b across a warp.  Only the taps
// whose row/column offsets have the residues (py, px) reach these pixels, from
// output pixel (a - dy, b - dx) with the tap's offsets (k0-1-ix2)*dl0 =
// py + s0*dy, (k1-1-iy2)*dl1 = px + s1*dx; the block lists them in shared
// memory in tap order (so the sums are deterministic) and every tap's loads
// of Y are 32 consecutive output pixels per warp.
//   dx = 2 * (sum_tap Y[o, (c,tap)] - x * sum_tap Y[o, SG]).
// Each listed tap carries its Y offset relative to the thread's own position
// a*Q + b (tap*PQ - dy*Q - dx, and dy*Q + dx for the SG column), so a thread
// whose taps all land inside the output (the interior of the phase grid)
// loads without any per-tap arithmetic beyond one add; border threads check
// each tap's output pixel.  An image's Y is below 2^31 floats.
constexpr int kColThreads = 256;
constexpr int kMaxT = 256;

template <int CC, bool CHECK>
__device__ __forceinline__ void col2im_taps(const float *__restrict__ yb, const float *__restrict__ ysg, int ntaps,
                                            const int2 *s_tp, const int2 *s_d, int cstride, int a, int b, int P, int Q,
                                            float (&acc)[CC], float &sg) {
  // groups of 4 taps: all loads of a group first (latency overlap), then the
  // adds in tap order
  for (int i0 = 0; i0 < ntaps; i0 += 4) {
    float ys[4], yv[4][CC];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u;
      bool v = i < ntaps;
      int2 tp = make_int2(0, 0);
      if (v) {
        tp = s_tp[i];
        if (CHECK) {
          const int2 d = s_d[i];
          const int oy = a - d.x, ox = b - d.y;
          v = oy >= 0 && ox >= 0 && oy < P && ox < Q;
        }
      }
      ys[u] = v ? __ldg(ysg - tp.y) : 0.f;
#pragma unroll
      for (int ci = 0; ci < CC; ++ci) yv[u][ci] = v ? __ldg(yb + tp.x + ci * cstride) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (i0 + u < ntaps) {
        sg += ys[u];
#pragma unroll
        for (int ci = 0; ci < CC; ++ci) acc[ci] += yv[u][ci];
      }
    }
  }
}

template <int CC>
__global__ void __launch_bounds__(kColThreads) tc_dc_col2im(const float *__restrict__ Y, const float *__restrict__ x,
                                                            Problem p, DcCfg c, DxOut dout, float *__restrict__ dx) {
  __shared__ int2 s_tp[kMaxT];  // (tap*PQ - (dy*Q + dx), dy*Q + dx) of the phase's taps, tap order
  __shared__ int2 s_d[kMaxT];   // (dy, dx)
  __shared__ int s_wcnt[kColThreads / 32];
  __shared__ int s_ext[4];      // max dy, max dx, -min dy, -min dx
  const int nph = p.s0 * p.s1;
  const int64_t n = blockIdx.y / nph;
  const int ph = (int)(blockIdx.y - n * nph);
  const int py = ph / p.s1, px = ph - py * p.s1;
  const int rows = p.H > py ? (p.H - py + p.s0 - 1) / p.s0 : 0;
  const int cols = p.W > px ? (p.W - px + p.s1 - 1) / p.s1 : 0;
  const int PQ = (int)p.PQ, Q = p.Q;
  if (threadIdx.x < 4) s_ext[threadIdx.x] = INT_MIN;
  __syncthreads();
  // this phase's taps, in tap order: ballot compaction per warp of 32 taps
  int ntaps = 0;
  for (int t0 = 0; t0 < p.T; t0 += kColThreads) {
    const int t = t0 + (int)threadIdx.x;
    bool v = false;
    int dy = 0, dxo = 0;
    if (t < p.T) {
      const int rr = tap_row(p, t), cc = tap_col(p, t);
      v = (rr % p.s0) == py && (cc % p.s1) == px;
      dy = (rr - py) / p.s0;
      dxo = (cc - px) / p.s1;
    }
    const unsigned bal = __ballot_sync(0xffffffffu, v);
    const int lane = threadIdx.x % 32, w = threadIdx.x / 32;
    if (lane == 0) s_wcnt[w] = __popc(bal);
    if (v) {
      atomicMax(&s_ext[0], dy);
      atomicMax(&s_ext[1], dxo);
      atomicMax(&s_ext[2], -dy);
      atomicMax(&s_ext[3], -dxo);
    }
    __syncthreads();
    int base = ntaps;
    for (int i = 0; i < w; ++i) base += s_wcnt[i];
    if (v) {
      const int pos = base + __popc(bal & ((1u << lane) - 1u));
      const int dd = dy * Q + dxo;
      s_tp[pos] = make_int2(t * PQ - dd, dd);
      s_d[pos] = make_int2(dy, dxo);
    }
    for (int i = 0; i < kColThreads / 32; ++i) ntaps += s_wcnt[i];
    __syncthreads();
  }
  const int64_t q = (int64_t)blockIdx.x * kColThreads + threadIdx.x;
  if (q >= (int64_t)rows * cols) return;
  const int a = (int)(q / cols), b = (int)(q - (int64_t)(q / cols) * cols);
  const int own = a * Q + b;  // may exceed the output grid; only offsets from it are loaded
  const float *yb = Y + n * (int64_t)c.NY * p.PQ + own;
  const float *ysg = yb + (int64_t)(c.NY - 1) * p.PQ;
  float acc[CC];
#pragma unroll
  for (int ci = 0; ci < CC; ++ci) acc[ci] = 0.f;
  float sg = 0.f;
  const bool interior = ntaps > 0 && a - s_ext[0] >= 0 && b - s_ext[1] >= 0 && a + s_ext[2] < p.P && b + s_ext[3] < Q;
  if (interior)
    col2im_taps<CC, false>(yb, ysg, ntaps, s_tp, s_d, p.T * PQ, a, b, p.P, Q, acc, sg);
  else
    col2im_taps<CC, true>(yb, ysg, ntaps, s_tp, s_d, p.T * PQ, a, b, p.P, Q, acc, sg);
  const int y = py + p.s0 * a, xc = px + p.s1 * b;
  const int64_t ob = dx_index(dout, n, y, xc);
  if (ob < 0) return;  // a pixel of the padding
  const float two_s = 2.f * (float)dout.scale;
#pragma unroll
  for (int ci = 0; ci < CC; ++ci) {
    const int64_t xi = n * p.CHW + (int64_t)ci * p.HW + (int64_t)y * p.W + xc;
    dx[ob + (int64_t)ci * dout.HWu] = two_s * (acc[ci] - __ldg(x + xi) * sg);
  }
}

PerContext<uint64_t> g_attr;

template <int NP>
int launch_dc_gemm(const Problem &p, DcCfg c, const float *grad, const float *hsum, const float *wsB, float *Y,
                   int *status, cudaStream_t stream) {
  // g and hsum viewed as [n*m rows][PQ floats], boxes of 16 rows x 128 floats
  CUtensorMap gmap, hmap;
  std::memset(&gmap, 0, sizeof(gmap));
  std::memset(&hmap, 0, sizeof(hmap));
  if (c.tma && !(encode_planes_map(grad, p.PQ, (int64_t)p.n * p.m, kTileM, 16, &gmap) &&
                 encode_planes_map(hsum, p.PQ, (int64_t)p.n * p.m, kTileM, 16, &hmap)))
    c.tma = 0;  // direct global loads instead
  const int ast = once_per_context(g_attr, 1ull << (NP / 16 - 1), []() -> int {
    PC2D_CUDA_CHECK(cudaFuncSetAttribute(tc_dc_gemm_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemLimit));
    return (int)PC2D_OK;
  });
  if (ast != PC2D_OK) return ast;
  const int grid = (int)std::min<int64_t>(c.tiles, device_sm_count());
  tc_dc_gemm_kernel<NP><<<grid, kThreads, dc_smem_bytes(c), stream>>>(grad, hsum, wsB, p, c, gmap, hmap, Y, status);
  PC2D_LAUNCH_CHECK("tc_dc_gemm_kernel");
  return PC2D_OK;
}

}  // namespace

bool tc_dgcol_supported(const Problem &p) {
  // at least one 128-pixel tile per SM: below that the three launches of this
  // path cost more than the implicit GEMM's one
  if (p.NPQ < (int64_t)148 * kTileM || p.m < 1 || p.C > 8 || p.HW >= ((int64_t)1 << 30) ||
      p.PQ >= ((int64_t)1 << 30))
    return false;
  const DcCfg c = dc_cfg(p);
  return c.NP <= kMaxNP && p.T <= kMaxT && (int64_t)p.n * p.s0 * p.s1 < 65536 && (int64_t)c.NY * p.PQ < ((int64_t)1 << 31) &&
         dc_smem_bytes(c) <= (size_t)kSmemLimit;
}

size_t tc_dgcol_workspace(const Problem &p) {
  const DcCfg c = dc_cfg(p);
  return align_up(dc_bsplit_bytes(c), 256) + align_up(dc_y_bytes(p, c), 256);
}

int tc_dgcol(const Problem &p, const float *grad, const float *x, const float *pars, const float *hsum,
             const DxOut &dxo, float *dx, void *ws, cudaStream_t stream) {
  const DcCfg c = dc_cfg(p);
  int *status = device_status_ptr();
  if (!status) {
    set_last_error("could not resolve the device status word");
    return PC2D_ERR_CUDA;
  }
  float *wsB = reinterpret_cast<float *>(ws);
  float *Y = reinterpret_cast<float *>(reinterpret_cast<char *>(ws) + align_up(dc_bsplit_bytes(c), 256));
  timing_begin(K_DGRAD, stream);
  tc_dc_prep_weights<<<dim3(c.nK, c.NP / 16), 256, 0, stream>>>(pars, p, c, wsB);
  PC2D_LAUNCH_CHECK("tc_dc_prep_weights");
  int st = PC2D_OK;
  switch (c.NP / 16) {
#define PC2D_DC_CASE(k) \
  case k: st = launch_dc_gemm<16 * k>(p, c, grad, hsum, wsB, Y, status, stream); break;
    PC2D_DC_CASE(1) PC2D_DC_CASE(2) PC2D_DC_CASE(3) PC2D_DC_CASE(4) PC2D_DC_CASE(5) PC2D_DC_CASE(6)
    PC2D_DC_CASE(7) PC2D_DC_CASE(8) PC2D_DC_CASE(9) PC2D_DC_CASE(10) PC2D_DC_CASE(11) PC2D_DC_CASE(12)
#undef PC2D_DC_CASE
    default:
      set_last_error("internal: unsupported GEMM width %d", c.NP);
      return PC2D_ERR_UNSUPPORTED;
  }
  if (st != PC2D_OK) return st;
  {
    // phase grids: at most ceil(H/s0) x ceil(W/s1) pixels each
    const int64_t ppg = (int64_t)((p.H + p.s0 - 1) / p.s0) * ((p.W + p.s1 - 1) / p.s1);
    const dim3 cgrid((unsigned)((ppg + kColThreads - 1) / kColThreads), (unsigned)(p.n * p.s0 * p.s1));
    switch (p.C) {
#define PC2D_COL_CASE(k) \
  case k: tc_dc_col2im<k><<<cgrid, kColThreads, 0, stream>>>(Y, x, p, c, dxo, dx); break;
      PC2D_COL_CASE(1) PC2D_COL_CASE(2) PC2D_COL_CASE(3) PC2D_COL_CASE(4)
      PC2D_COL_CASE(5) PC2D_COL_CASE(6) PC2D_COL_CASE(7) PC2D_COL_CASE(8)
#undef PC2D_COL_CASE
      default:
        set_last_error("internal: unsupported channel count %d", p.C);
        return PC2D_ERR_UNSUPPORTED;
    }
  }
  PC2D_LAUNCH_CHECK("tc_dc_col2im");
  timing_end(K_DGRAD, stream);
  return PC2D_OK;
}

}  // namespace pc2d
