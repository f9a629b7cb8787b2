// tcgen05 forward kernel of the ParaConv2d paraboloid convolution (fp32 via
// 3xTF32 split precision).
//
// Decomposition of the reference forward (paraconv2d.cc:82-122): for output
// pixel i and output channel j, with win the flipped window of pixel i,
//   hsum = h0[j] + H[j].win
//   out  = f * (hsum^2 - S2[i] + 2 P[j].win - |P[j]|^2 - p0[j]^2),
//   S2[i] = sum_k win[k]^2
// so H.win and P.win form one implicit GEMM with M = 128 output pixels per
// tile, N = NB output channels per channel block (NB <= 64) for each of H and
// P, and K = the window (C*k0*k1), swept 16 at a time.
//
// Operands:
//   A (the im2col window, M x K) lives in Tensor Memory.  Four producer
//     warps (one TMEM lane = one output pixel per thread) gather the window
//     with 4-byte cp.async copies (coalesced across the 32 pixels of a warp)
//     into a per-thread shared-memory ring that keeps 5 stages of 16 K in
//     flight, then split every value into tf32 hi + lo, accumulate S2, and
//     tcgen05.st the hi and lo slices into a 4-stage ring of TMEM columns.
//   B ([H;P], 2NB x K) is split into hi/lo once per call by a prep kernel,
//     already in the 128-byte-swizzled K-major layout, and streamed into a
//     4-stage shared-memory ring (32 K per stage) by 1-D bulk async copies.
//
// Accumulation (3xTF32 = Ahi*Bhi + Alo*Bhi + Ahi*Blo per 8-wide K step,
// each one MMA of N = 2NB over [H;P]):
//   The tensor core's fp32 accumulation loses up to one unit in the last
//   place of the accumulator per instruction, so a long K sweep into one
//   accumulator drifts by O(K/8) ulps of the running sum.  Instead, every 32
//   K of the sweep accumulate into a fresh partial sum (enable_input_d = 0)
//   in one of three [H | P] slots of TMEM, and the epilogue warps drain each
//   partial into fp32 registers (round-to-nearest adds) while the MMAs fill
//   the next slot.  TMEM columns: slots [0,128) [128,256) [256,384); A
//   stages [384,512) as 4 x (hi 16 | lo 16).
//
// Warp roles (320 threads, one CTA per SM, persistent over work items):
//   warps 0-3 producers, warps 4-7 epilogue, warp 8 MMA issuer (and TMEM
//   owner), warp 9 B loader.  Every barrier wait is bounded in
//   time; a wait that gives up records PC2D_ERR_TIMEOUT, raises a CTA-wide
//   abort flag, and the CTA drains its in-flight copies and MMAs and exits.
#include <algorithm>
#include <mutex>

#include "pc2d_sm100.cuh"
#include "pc2d_tc.cuh"

namespace pc2d {

namespace {
using namespace sm100;

constexpr int kTileM = 128;
constexpr int kKB = 32;          // K per B stage (one 128-byte swizzle row of tf32)
constexpr int kKA = 32;          // K per A stage (= one B stage)
constexpr int kAStages = 2;
constexpr int kBStages = 4;
constexpr int kMaxNB = 64;
constexpr int kMaxD = 8192;
constexpr int kGroupStages = 1;  // A stages per partial sum (32 K)
constexpr int kSlots = 3;        // partial-sum slots in TMEM
constexpr int kDepth = 2;        // A stages whose window gathers are in flight (cp.async)
constexpr int kRing = kDepth + 1;
constexpr int kFwdThreads = 320;
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr int kMinSmem = 120 * 1024;  // keeps one CTA per SM (it owns all 512 TMEM columns)

// TMEM column map: partial-sum slots [H | P] at 128 * slot (slots 0-2),
// A stages at 384 + 64 * stage (hi 32 columns, then lo 32 columns).
constexpr uint32_t kColA = 384;

struct FwdCfg {
  int ncb;         // channel blocks
  int NB;          // channels per block (multiple of 16, <= 64)
  int N;           // rows of a B stage = 2*NB ([H;P])
  int nKB;         // 32-wide K chunks (B stages per tile)
  int nKA;         // A stages per tile (= nKB)
  int nGroups;     // H partial sums per tile
  int64_t tiles;   // 128-pixel tiles
  int64_t items;   // tiles * ncb
};

FwdCfg fwd_cfg(const Problem &p) {
  FwdCfg c;
  c.ncb = std::max(1, ceil_div(p.m, kMaxNB));
  const int nb = ceil_div(p.m, c.ncb);
  c.NB = (nb + 15) / 16 * 16;
  c.N = 2 * c.NB;
  c.nKB = ceil_div(p.d, kKB);
  c.nKA = c.nKB;
  c.nGroups = ceil_div(c.nKA, kGroupStages);
  c.tiles = (p.NPQ + kTileM - 1) / kTileM;
  c.items = c.tiles * c.ncb;
  return c;
}

inline size_t fwd_bsplit_bytes(const FwdCfg &c) { return (size_t)c.ncb * c.nKB * 2 * c.N * 128; }
__host__ __device__ inline uint32_t fwd_bstage_bytes(const FwdCfg &c) { return (uint32_t)(2 * c.N * 128); }
inline size_t fwd_smem_bytes(const FwdCfg &c) {
  size_t s = 1024 + (size_t)kBStages * fwd_bstage_bytes(c) + (size_t)kRing * kKA * kTileM * 4 +
             (size_t)c.nKB * kKB * 4 + 2 * kTileM * 4 + 32 * 8 + 64;
  return std::max<size_t>(s, kMinSmem);
}

// Splits [H;P] of channel block cb into hi/lo tf32 halves in the swizzled
// K-major layout the MMA reads: block (cb, kc) = [hi: N rows][lo: N rows],
// each row 32 floats of K with 16-byte chunk c stored at c ^ (row % 8).
// Rows 0..NB-1 are H of channels cb*NB.., rows NB..2NB-1 are P; channels >= m
// and K >= d are zero.
__global__ void tc_fwd_prep_weights(const float *__restrict__ pars, Problem p, FwdCfg c, float *__restrict__ wsB) {
  const int kc = blockIdx.x, cb = blockIdx.y;
  float *blk = wsB + ((int64_t)cb * c.nKB + kc) * 2 * c.N * 32;
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

// Input offset of the window origin of output pixel g (or -1 past the end).
__device__ __forceinline__ int64_t pixel_base(const Problem &p, int64_t g) {
  if (g >= p.NPQ) return -1;
  const int64_t nn = g / p.PQ;
  const int64_t rr = g - nn * p.PQ;
  const int oy = (int)(rr / p.Q), ox = (int)(rr - (int64_t)oy * p.Q);
  return nn * p.CHW + (int64_t)oy * p.s0 * p.W + (int64_t)ox * p.s1;
}

struct Smem {
  uint8_t *sB;
  float *ring;   // [kRing][kKA][128] gathered window values of A stages in flight
  int *koff;
  float *s2buf;  // [tile buffer 2][128]
  uint64_t *a_full, *a_empty, *b_full, *b_empty, *gr_full, *gr_empty, *s2_full, *s2_empty, *final_bar;
  uint32_t *tmem_holder;
  volatile int *abort_flag;
};

template <int NB>
__global__ void __launch_bounds__(kFwdThreads, 1)
tc_forward_kernel(const float *__restrict__ x, const float *__restrict__ pars, const float *__restrict__ wsB,
                  const float *__restrict__ cj, float factor, Problem p, FwdCfg c, float *__restrict__ out,
                  float *__restrict__ hsum, int *status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t bstage = fwd_bstage_bytes(c);
  const int dpad = c.nKB * kKB;
  Smem S;
  S.sB = base;
  S.ring = reinterpret_cast<float *>(base + kBStages * bstage);
  S.koff = reinterpret_cast<int *>(S.ring + kRing * kKA * kTileM);
  S.s2buf = reinterpret_cast<float *>(S.koff + dpad);
  uint64_t *bars = reinterpret_cast<uint64_t *>(S.s2buf + 2 * kTileM);
  S.a_full = bars;
  S.a_empty = bars + 4;
  S.b_full = bars + 8;
  S.b_empty = bars + 12;
  S.gr_full = bars + 16;
  S.gr_empty = bars + 20;
  S.s2_full = bars + 24;
  S.s2_empty = bars + 26;
  S.final_bar = bars + 28;
  S.tmem_holder = reinterpret_cast<uint32_t *>(bars + 29);
  S.abort_flag = reinterpret_cast<volatile int *>(S.tmem_holder + 1);

  // Per-K input offset of the flipped window relative to the window origin;
  // -1 marks the zero padding of the last K chunk.
  for (int k = threadIdx.x; k < dpad; k += blockDim.x) {
    int v = -1;
    if (k < p.d) {
      const int ch = k / p.T, tap = k - ch * p.T;
      v = (int)((int64_t)ch * p.HW + (int64_t)tap_row(p, tap) * p.W + tap_col(p, tap));
    }
    S.koff[k] = v;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) {
      mbar_init(&S.a_full[i], 128);
      mbar_init(&S.a_empty[i], 1);
      mbar_init(&S.b_full[i], 1);
      mbar_init(&S.b_empty[i], 1);
    }
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&S.gr_full[i], 1);
      mbar_init(&S.gr_empty[i], 128);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.s2_full[i], 128);
      mbar_init(&S.s2_empty[i], 128);
    }
    mbar_init(S.final_bar, 1);
    *S.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc(S.tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *S.tmem_holder;
  bool ok = true;

  if (warp < 4) {
    // ---------------------------------------------------------- producers
    const int r = warp * 32 + lane;      // pixel row of the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    // Issue cursor: the next A stage whose window values are copied
    // (cp.async, zero-filled outside the window) into ring slot s % kRing.
    // Each thread copies and later reads only its own pixel's values.
    int64_t i_item = blockIdx.x;
    int i_kq = 0;
    int64_t i_base = (i_item < c.items) ? pixel_base(p, (i_item / c.ncb) * kTileM + r) : -1;
    auto issue = [&](uint32_t s_index) {
      if (i_item < c.items) {
        float *dst = S.ring + (s_index % kRing) * (kKA * kTileM) + r;
#pragma unroll
        for (int kk = 0; kk < kKA; ++kk) {
          const int o = S.koff[i_kq * kKA + kk];
          const bool v = (i_base >= 0 && o >= 0);
          cp_async4(dst + kk * kTileM, x + (v ? i_base + o : 0), v);
        }
        if (++i_kq == c.nKA) {
          i_kq = 0;
          i_item += gridDim.x;
          i_base = (i_item < c.items) ? pixel_base(p, (i_item / c.ncb) * kTileM + r) : -1;
        }
      }
      cp_async_commit();
    };
#pragma unroll 1
    for (int d0 = 0; d0 < kDepth; ++d0) issue(d0);
    uint32_t s = 0;
    int64_t li = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x, ++li) {
      float s2 = 0.f;
      for (int kq = 0; kq < c.nKA; ++kq, ++s) {
        cp_async_wait<kDepth - 1>();
        float cur[kKA];
        const float *src = S.ring + (s % kRing) * (kKA * kTileM) + r;
#pragma unroll
        for (int kk = 0; kk < kKA; ++kk) cur[kk] = src[kk * kTileM];
        uint32_t hi[kKA], lo[kKA];
#pragma unroll
        for (int kk = 0; kk < kKA; ++kk) {
          s2 = fmaf(cur[kk], cur[kk], s2);
          hi[kk] = tf32_hi_bits(cur[kk]);
          lo[kk] = __float_as_uint(cur[kk] - __uint_as_float(hi[kk]));
        }
        issue(s + kDepth);
        const uint32_t sa = s % kAStages, ph = (s / kAStages) & 1;
        if (!warp_wait(&S.a_empty[sa], ph ^ 1, S.abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acol = tmem + lane_off + kColA + sa * 64;
        tmem_st16(acol, *reinterpret_cast<const uint32_t(*)[16]>(&hi[0]));
        tmem_st16(acol + 16, *reinterpret_cast<const uint32_t(*)[16]>(&hi[16]));
        tmem_st16(acol + 32, *reinterpret_cast<const uint32_t(*)[16]>(&lo[0]));
        tmem_st16(acol + 48, *reinterpret_cast<const uint32_t(*)[16]>(&lo[16]));
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&S.a_full[sa]);
      }
      if (!ok) break;
      // hand S2 of this tile to the epilogue
      const uint32_t tb = (uint32_t)(li & 1), tph = (uint32_t)((li >> 1) & 1);
      if (!warp_wait(&S.s2_empty[tb], tph ^ 1, S.abort_flag)) {
        ok = false;
        break;
      }
      S.s2buf[tb * kTileM + r] = s2;
      mbar_arrive(&S.s2_full[tb]);
    }
    cp_async_wait<0>();
  } else if (warp < 8) {
    // ---------------------------------------------------------- epilogue
    const int q = warp % 4;
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const float *h0 = pars;
    uint32_t grp = 0;
    int64_t li = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x, ++li) {
      const int64_t t = item / c.ncb;
      const int cb = (int)(item - t * c.ncb);
      float hacc[NB], pacc[NB];
#pragma unroll
      for (int j = 0; j < NB; ++j) hacc[j] = pacc[j] = 0.f;
      for (int gi = 0; gi < c.nGroups; ++gi, ++grp) {
        const uint32_t slot = grp % kSlots, ph = (grp / kSlots) & 1;
        if (!warp_wait(&S.gr_full[slot], ph, S.abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dcol = tmem + lane_off + slot * 128;
        // 32 columns of H and of P per round, one wait per round
#pragma unroll
        for (int jc = 0; jc < NB; jc += 32) {
          uint32_t hv[32], pv[32];
          tmem_ld32_nowait(dcol + jc, hv);
          tmem_ld32_nowait(dcol + NB + jc, pv);
          tmem_ld_wait_tie(hv);
          tmem_ld_wait_tie(pv);
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            if (jc + jj < NB) {
              hacc[jc + jj] += __uint_as_float(hv[jj]);
              pacc[jc + jj] += __uint_as_float(pv[jj]);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&S.gr_empty[slot]);
      }
      if (!ok) break;
      const uint32_t tb = (uint32_t)(li & 1), tph = (uint32_t)((li >> 1) & 1);
      if (!warp_wait(&S.s2_full[tb], tph, S.abort_flag)) {
        ok = false;
        break;
      }
      const float s2 = S.s2buf[tb * kTileM + r];
      mbar_arrive(&S.s2_empty[tb]);
      const int64_t g = t * kTileM + r;
      const bool valid = g < p.NPQ;
      int64_t obase = 0;
      if (valid) {
        const int64_t nn = g / p.PQ;
        obase = nn * (int64_t)p.m * p.PQ + (g - nn * p.PQ);
      }
#pragma unroll
      for (int jj = 0; jj < NB; ++jj) {
        const int j = cb * NB + jj;
        if (valid && j < p.m) {
          const float hs = __ldg(h0 + j) + hacc[jj];
          const float o = factor * (fmaf(hs, hs, -s2) + 2.f * pacc[jj] - __ldg(cj + cb * NB + jj));
          const int64_t oi = obase + (int64_t)j * p.PQ;
          out[oi] = o;
          hsum[oi] = hs;
        }
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------- MMA
    const uint32_t idesc = idesc_tf32(kTileM, 2 * NB);
    const uint32_t sB_addr = smem_u32(S.sB);
    uint32_t ita = 0, grp = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
      uint32_t dcol = 0, slot = 0;
      for (int kq = 0; kq < c.nKA; ++kq, ++ita) {
        const bool gstart = (kq % kGroupStages) == 0;
        const bool gend = (kq % kGroupStages) == kGroupStages - 1 || kq == c.nKA - 1;
        if (gstart) {
          slot = grp % kSlots;
          if (!warp_wait(&S.gr_empty[slot], ((grp / kSlots) & 1) ^ 1, S.abort_flag)) {
            ok = false;
            break;
          }
          dcol = tmem + slot * 128;
        }
        const uint32_t sa = ita % kAStages, pa = (ita / kAStages) & 1;
        const uint32_t sb = ita % kBStages, pb = (ita / kBStages) & 1;
        if (!warp_wait(&S.a_full[sa], pa, S.abort_flag) || !warp_wait(&S.b_full[sb], pb, S.abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t ahi = tmem + kColA + sa * 64, alo = ahi + 32;
          const uint32_t bhi = sB_addr + sb * bstage;                  // [H;P] rows, hi
          const uint32_t blo = bhi + c.N * 128;                        // lo
#pragma unroll
          for (int ks = 0; ks < kKA / 8; ++ks) {
            const uint32_t ko = ks * 32;
            const uint32_t acc = (gstart && ks == 0) ? 0u : 1u;
            mma_tf32_ts(dcol, ahi + ks * 8, sdesc_kmajor_sw128(bhi + ko), idesc, acc);
            mma_tf32_ts(dcol, alo + ks * 8, sdesc_kmajor_sw128(bhi + ko), idesc, 1u);
            mma_tf32_ts(dcol, ahi + ks * 8, sdesc_kmajor_sw128(blo + ko), idesc, 1u);
          }
          tc_commit(&S.a_empty[sa]);
          tc_commit(&S.b_empty[sb]);
          if (gend) tc_commit(&S.gr_full[slot]);
        }
        __syncwarp();
        if (gend) ++grp;
      }
    }
    // Drain: every MMA issued by this warp completes before TMEM is freed.
    if (lane == 0) tc_commit(S.final_bar);
    __syncwarp();
    mbar_wait(S.final_bar, 0, kWaitNs, nullptr);
  } else {
    // ---------------------------------------------------------- B loader
    uint32_t itb = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
      const int cb = (int)(item % c.ncb);
      for (int kc = 0; kc < c.nKB; ++kc, ++itb) {
        const uint32_t sb = itb % kBStages, pb = (itb / kBStages) & 1;
        if (!warp_wait(&S.b_empty[sb], pb ^ 1, S.abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&S.b_full[sb], bstage);
          bulk_g2s(S.sB + sb * bstage, wsB + ((int64_t)cb * c.nKB + kc) * 2 * c.N * 32, bstage, &S.b_full[sb]);
        }
        __syncwarp();
      }
    }
    // Drain: the copies issued last have landed before the CTA exits.
    const uint32_t last = std::min<uint32_t>(itb, kBStages);
    for (uint32_t i = 0; i < last; ++i) {
      const uint32_t idx = itb - 1 - i;
      mbar_wait(&S.b_full[idx % kBStages], (idx / kBStages) & 1, kWaitNs, nullptr);
    }
  }

  if (!ok) {
    if (lane == 0) record_device_error(status, PC2D_ERR_TIMEOUT);
    *S.abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
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
bool g_attr_set[64][4] = {};
int g_sm_count[64] = {0};

template <int NB>
int launch_forward(const Problem &p, const FwdCfg &c, const float *x, const float *pars, const float *wsB,
                   const float *cj, float factor, float *out, float *hsum, int *status, cudaStream_t stream) {
  int dev = 0;
  PC2D_CUDA_CHECK(cudaGetDevice(&dev));
  {
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    if (dev >= 0 && dev < 64 && !g_attr_set[dev][NB / 16 - 1]) {
      PC2D_CUDA_CHECK(
          cudaFuncSetAttribute(tc_forward_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
      g_attr_set[dev][NB / 16 - 1] = true;
    }
  }
  const int grid = (int)std::min<int64_t>(c.items, device_sm_count());
  tc_forward_kernel<NB><<<grid, kFwdThreads, fwd_smem_bytes(c), stream>>>(x, pars, wsB, cj, factor, p, c, out, hsum,
                                                                          status);
  PC2D_LAUNCH_CHECK("tc_forward_kernel");
  return PC2D_OK;
}

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
  tc_fwd_prep_weights<<<dim3(c.nKB, c.ncb), 256, 0, stream>>>(pars, p, c, wsB);
  PC2D_LAUNCH_CHECK("tc_fwd_prep_weights");
  tc_fwd_prep_consts<<<ceil_div(c.ncb * c.NB, 8), 256, 0, stream>>>(pars, p, c, cj);
  PC2D_LAUNCH_CHECK("tc_fwd_prep_consts");
  const float f = (float)factor;
  switch (c.NB) {
    case 16: return launch_forward<16>(p, c, x, pars, wsB, cj, f, out, hsum, status, stream);
    case 32: return launch_forward<32>(p, c, x, pars, wsB, cj, f, out, hsum, status, stream);
    case 48: return launch_forward<48>(p, c, x, pars, wsB, cj, f, out, hsum, status, stream);
    case 64: return launch_forward<64>(p, c, x, pars, wsB, cj, f, out, hsum, status, stream);
    default:
      set_last_error("internal: unsupported channel block %d", c.NB);
      return PC2D_ERR_UNSUPPORTED;
  }
}

int tc_selftest_bounded_wait(unsigned int timeout_us, int *status, cudaStream_t stream) {
  selftest_wait_kernel<<<1, 32, 0, stream>>>(timeout_us, status);
  PC2D_LAUNCH_CHECK("selftest_wait_kernel");
  return PC2D_OK;
}

}  // namespace pc2d
