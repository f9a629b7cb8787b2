// tcgen05 forward kernel of the ParaConv2d paraboloid convolution (fp32 via
// 3xTF32 split precision).
//
// Decomposition of the reference forward (paraconv2d.cc:82-122): for output
// pixel i and output channel j, with win the flipped window of pixel i,
//   hsum = h0[j] + H[j].win
//   out  = f * (hsum^2 - S2[i] + 2 P[j].win - |P[j]|^2 - p0[j]^2),
//   S2[i] = sum_k win[k]^2
// so H.win and P.win form one implicit GEMM: M = 128 consecutive output
// pixels of one image per tile, N = [H;P] rows of a channel block (2*NB,
// NB <= 64) and K = the window (C*k0*k1), swept 32 at a time.
//
// Data movement per stage (64 K = two 32-K sub-stages with 2 stages in flight
// when the halo is one tensor copy, else 32 K with 4 in flight):
//   - the loader warp copies (a) the pre-split weights of the stage ([H;P] hi
//     and lo of two 32-K blocks, 128-byte-swizzled K-major, written once per
//     call by a prep kernel; one bulk copy) and (b) the input "halo" of the
//     stage: for each channel the stage's window touches, the run of input
//     rows the tile reads (one 2-D tensor copy, or 16-byte-rounded bulk
//     copies per channel), all completing on one barrier;
//   - four producer warps (one TMEM lane = one output pixel per thread)
//     gather the 64 window values of their pixel from the halo in shared
//     memory, split them into tf32 hi + lo, accumulate S2, and tcgen05.st
//     the hi and lo slices into the stage's TMEM columns (A operand);
//   - one elected thread of the MMA warp issues, per 8-wide K step, the
//     three products Ahi*Bhi + Alo*Bhi + Ahi*Blo as MMAs with N = 2NB.
//
// Accumulation: the tensor core's fp32 accumulation loses up to one unit in
// the last place per instruction, so a long K sweep into one accumulator
// drifts by O(K/8) ulps of the running sum.  Every 64 K therefore start a
// fresh partial sum (enable_input_d = 0) in one of two [H | P] slots of TMEM,
// and the epilogue warps drain each partial into fp32 registers
// (round-to-nearest adds) while the MMAs fill the other slot.
//   TMEM columns: slots [0,128) [128,256); A stages [256,512): 2 x (hi 32 |
//   lo 32 | hi 32 | lo 32) with 64-K stages, 4 x (hi 32 | lo 32) with 32-K
//   stages.
//
// Warp roles (448 threads, one CTA per SM, persistent over work items):
//   warps 0-3 producers, 4-7 and 10-13 epilogue (two warps per TMEM lane
//   quarter, half of the channels each), 8 MMA issuer (and TMEM owner),
//   9 loader.  Every barrier wait is bounded in time; a wait that gives up
//   records PC2D_ERR_TIMEOUT, raises a CTA-wide abort flag, and the CTA
//   drains its in-flight copies and MMAs and exits.
#include <algorithm>
#include <cstring>
#include <mutex>

#include "pc2d_tc.cuh"
#include "pc2d_tc_common.cuh"

namespace pc2d {

namespace {
using namespace sm100;
using tc::warp_wait;
using tc::kWaitNs;

constexpr int kTileM = 128;
constexpr int kKS = 32;          // K per sub-stage (one 128-byte swizzle row of tf32)
constexpr int kMaxStages = 4;    // barrier sets; SUB-K stages in flight = 4 / SUB
constexpr int kMaxCh = 64;       // channel planes a stage may touch
constexpr int kSlots = 2;        // partial-sum slots in TMEM
constexpr int kMaxNB = 64;
constexpr int kMaxD = 8192;
constexpr int kFwdThreads = 448;
constexpr int kMinSmem = 120 * 1024;  // keeps one CTA per SM (it owns all 512 TMEM columns)
constexpr int kSmemLimit = 227 * 1024;
constexpr uint32_t kColA = 256;       // A stages at 256 + 64 * SUB * stage: (hi 32, lo 32) per sub-stage

struct FwdCfg {
  int ncb;          // channel blocks
  int NB;           // channels per block (multiple of 16, <= 64)
  int N;            // rows of a B stage = 2*NB ([H;P])
  int sub;          // 32-K sub-stages per stage (2 with a single-copy halo, else 1)
  int nK;           // stages per tile (= partial sums per tile)
  int nKB;          // 32-wide K blocks of the weight layout (= sub * nK)
  int nst;          // stages in flight (4 / sub)
  int nGroups;      // partial sums (64 K each) per tile
  int tpi;          // tiles per image
  int64_t tiles;    // 128-pixel tiles (never crossing an image)
  int64_t items;    // tiles * ncb
  int PS;           // halo plane stride in floats (multiple of 4)
  int nchs;         // channels a stage touches at most
  uint32_t bstage;  // B bytes of one 32-K block (hi + lo); a stage holds SUB blocks
  uint32_t sstage;  // shared bytes per stage (B + halo, multiple of 1024)
  int tma;          // 1: a stage's halo is one 2-D tensor copy [nchs planes][PS floats]
};

FwdCfg fwd_cfg(const Problem &p) {
  FwdCfg c;
  c.ncb = std::max(1, ceil_div(p.m, kMaxNB));
  const int nb = ceil_div(p.m, c.ncb);
  c.NB = (nb + 15) / 16 * 16;
  c.N = 2 * c.NB;
  // output rows a run of 128 consecutive pixels of one image can touch
  {
    const int orow = std::min<int64_t>(p.P, (p.Q + kTileM - 2) / p.Q + 1);
    const int R = (orow - 1) * p.s0 + (p.k0 - 1) * p.dl0 + 1;
    c.PS = (int)(((int64_t)R * p.W + 8 + 3) / 4 * 4);
  }
  // one tensor copy per stage: channel planes 16-byte strided, the plane
  // stride PS (from the 16-byte boundary at or below the tile's first input
  // element) at most 256 floats
  c.tma = (p.HW % 4 == 0 && c.PS <= 256 && (int64_t)p.n * p.C < ((int64_t)1 << 31)) ? 1 : 0;
  // 64-K stages halve the hand-offs per K when a tile has many of them; with
  // a short window (few stages per tile) four 32-K stages in flight hide the
  // copies better
  c.sub = p.d >= 256 ? 2 : 1;
  c.nst = kMaxStages / c.sub;
  c.nK = ceil_div(p.d, kKS * c.sub);
  c.nKB = c.nK * c.sub;
  c.nGroups = ceil_div(c.nK, 2 / c.sub);
  c.tpi = ceil_div(p.PQ, kTileM);
  c.tiles = (int64_t)p.n * c.tpi;
  c.items = c.tiles * c.ncb;
  c.nchs = 0;
  const int kst = kKS * c.sub;
  for (int kq = 0; kq < c.nK; ++kq) {
    const int clo = (int)(((int64_t)kq * kst) / p.T);
    const int chi = (int)(std::min<int64_t>((int64_t)kq * kst + kst - 1, p.d - 1) / p.T);
    c.nchs = std::max(c.nchs, chi - clo + 1);
  }
  c.bstage = (uint32_t)(2 * c.N * 128);
  const size_t hb = align_up((size_t)c.nchs * c.PS * 4, 1024);
  c.sstage = (uint32_t)(c.sub * c.bstage + hb);
  return c;
}

inline size_t fwd_bsplit_bytes(const FwdCfg &c) { return (size_t)c.ncb * c.nKB * c.bstage; }
inline size_t fwd_smem_bytes(const Problem &p, const FwdCfg &c) {
  size_t s = 1024 + (size_t)c.nst * c.sstage + (size_t)c.nKB * kKS * 8 + (size_t)kMaxStages * kKS * 4 +
             (size_t)kMaxStages * kMaxCh * 4 + 2 * kTileM * 4 + 8 * 2 * 64 * 4 + (size_t)c.PS * 4 + 16 + 28 * 8 + 64;
  (void)p;
  return std::max<size_t>(s, kMinSmem);
}

inline FwdCfg fwd_cfg_fit(const Problem &p) { return fwd_cfg(p); }

// Per-call preparation of the forward's constant operands, one launch:
//  - blocks [0, ncb * nKB * kPrepSplit): split [H;P] of channel block cb into
//    hi/lo tf32 halves in the swizzled K-major layout the MMA reads: block
//    (cb, kc) = [hi: N rows][lo: N rows], each row 32 floats of K with 16-byte
//    chunk c stored at c ^ (row % 8).  Rows 0..NB-1 are H of channels
//    cb*NB.., rows NB..2NB-1 are P; channels >= m and K >= d are zero.  Each
//    thread block writes N / kPrepSplit rows of one (cb, kc) block.
//  - the remaining blocks: cj[cb*NB + jn] = |P[j]|^2 + p0[j]^2 (fp64
//    accumulation, one warp per channel), 0 for padded channels.
constexpr int kPrepSplit = 8;
__global__ void __launch_bounds__(256) tc_fwd_prep(const float *__restrict__ pars, Problem p, FwdCfg c,
                                                   float *__restrict__ wsB, float *__restrict__ cj) {
  const int nwb = c.ncb * c.nKB * kPrepSplit;
  if ((int)blockIdx.x < nwb) {
    const int sp = blockIdx.x % kPrepSplit, kc = (blockIdx.x / kPrepSplit) % c.nKB;
    const int cb = blockIdx.x / (kPrepSplit * c.nKB);
    float *blk = wsB + ((int64_t)cb * c.nKB + kc) * 2 * c.N * 32;
    const float *h = pars + p.m;
    const float *pp = h + (int64_t)p.m * p.d;
    const int rows = c.N / kPrepSplit;  // N = 2 NB is a multiple of 32
    for (int e = threadIdx.x; e < rows * 32; e += blockDim.x) {
      const int r = sp * rows + e / 32, kk = e % 32;
      const int half = r / c.NB;
      const int j = cb * c.NB + (r - half * c.NB);
      const int64_t k = (int64_t)kc * 32 + kk;
      float v = 0.f;
      if (j < p.m && k < p.d) v = (half == 0 ? h : pp)[(int64_t)j * p.d + k];
      float hi, lo;
      tf32_split_rn(v, hi, lo);
      const int pos = r * 32 + (((kk >> 2) ^ (r & 7)) << 2) + (kk & 3);
      blk[pos] = hi;
      blk[c.N * 32 + pos] = lo;
    }
    return;
  }
  const int slot = ((int)blockIdx.x - nwb) * 8 + threadIdx.x / 32;
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

// Geometry of a tile: image, first pixel, first input row and rows of its halo.
struct TileGeo {
  int64_t n;
  int p0, ir0, rows;
};

__device__ __forceinline__ TileGeo tile_geo(const Problem &p, const FwdCfg &c, int64_t t) {
  TileGeo g;
  g.n = t / c.tpi;
  g.p0 = (int)(t - g.n * c.tpi) * kTileM;
  const int plast = min(g.p0 + kTileM - 1, (int)p.PQ - 1);
  const int oya = g.p0 / p.Q, oyb = plast / p.Q;
  g.ir0 = oya * p.s0;
  g.rows = (oyb - oya) * p.s0 + (p.k0 - 1) * p.dl0 + 1;
  return g;
}

struct Smem {
  uint8_t *stage;   // nst x [SUB x (B hi | B lo) | halo planes]
  int2 *koff;       // per K: (channel, tap offset row*W + col), channel -1 past d
  int *offs;        // [stage][32 SUB] halo offset of each K of the stage (past the window: zbuf)
  int *lead;        // [stage][64] floats before each halo plane's first element
  float *s2buf;     // [tile buffer 2][128]
  float *hcbuf;     // [epilogue warp 8][h0 | cj of its channels, 64 each]
  float *zbuf;      // PS zeros: window entries past the window point here
  uint64_t *full, *b_full, *a_full, *s_empty, *gr_full, *gr_empty, *s2_full, *s2_empty, *final_bar;
  uint32_t *tmem_holder;
  volatile int *abort_flag;
};

template <int NB, int SUB>
__global__ void __launch_bounds__(kFwdThreads, 1)
tc_forward_kernel(const float *__restrict__ x, const float *__restrict__ pars, const float *__restrict__ wsB,
                  const float *__restrict__ cj, float factor, Problem p, FwdCfg c,
                  const __grid_constant__ CUtensorMap xmap, float *__restrict__ out, float *__restrict__ hsum,
                  int *status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  Smem S;
  const int nst = c.nst;
  S.stage = base;
  S.koff = reinterpret_cast<int2 *>(base + (size_t)nst * c.sstage);
  constexpr int kKStage = kKS * SUB;  // K per stage = one partial sum
  S.offs = reinterpret_cast<int *>(S.koff + c.nK * kKStage);
  S.lead = S.offs + kMaxStages * kKS;
  S.s2buf = reinterpret_cast<float *>(S.lead + kMaxStages * kMaxCh);
  S.hcbuf = S.s2buf + 2 * kTileM;
  S.zbuf = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(S.hcbuf + 8 * 2 * 64) + 15) & ~(uintptr_t)15);
  uint64_t *bars = reinterpret_cast<uint64_t *>(
      (reinterpret_cast<uintptr_t>(S.hcbuf + 8 * 2 * 64 + c.PS + 4) + 7) & ~(uintptr_t)7);
  S.full = bars;            // [4] halo + offsets landed (loader expect_tx)
  S.a_full = bars + 4;      // [4] A stage in TMEM (128 producer arrivals)
  S.s_empty = bars + 8;     // [4] stage consumed by the MMAs (commit)
  S.gr_full = bars + 12;    // [2] partial sum ready (commit)
  S.gr_empty = bars + 14;   // [2] partial sum drained (256 epilogue arrivals)
  S.s2_full = bars + 16;    // [2]
  S.s2_empty = bars + 18;   // [2]
  S.final_bar = bars + 20;
  S.b_full = bars + 21;     // [4] B landed (loader expect_tx); only the MMA waits for it
  S.tmem_holder = reinterpret_cast<uint32_t *>(bars + 25);
  S.abort_flag = reinterpret_cast<volatile int *>(S.tmem_holder + 1);

  for (int k = threadIdx.x; k < c.nK * kKStage; k += blockDim.x) {
    int2 v = make_int2(-1, 0);
    if (k < p.d) {
      const int ch = k / p.T, tap = k - ch * p.T;
      v = make_int2(ch, tap_row(p, tap) * p.W + tap_col(p, tap));
    }
    S.koff[k] = v;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < kMaxStages; ++i) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.b_full[i], 1);
      mbar_init(&S.a_full[i], 128);
      mbar_init(&S.s_empty[i], 1);
    }
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&S.gr_full[i], 1);
      mbar_init(&S.gr_empty[i], 256);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.s2_full[i], 128);
      mbar_init(&S.s2_empty[i], 256);
    }
    mbar_init(S.final_bar, 1);
    *S.abort_flag = 0;
    fence_mbar_init();
  }
  for (int e = threadIdx.x; e < c.PS; e += blockDim.x) S.zbuf[e] = 0.f;
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
    const int r = warp * 32 + lane;  // pixel of the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    uint32_t it = 0;
    int64_t li = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x, ++li) {
      const TileGeo tg = tile_geo(p, c, item / c.ncb);
      const int pix = tg.p0 + r;
      const bool valid = pix < p.PQ;
      int poff = 0;
      if (valid) {
        const int oy = pix / p.Q, ox = pix - (pix / p.Q) * p.Q;
        poff = (oy * p.s0 - tg.ir0) * p.W + ox * p.s1;
      }
      float s2 = 0.f;
      for (int kq = 0; kq < c.nK; ++kq, ++it) {
        const uint32_t st = it % nst, ph = (it / nst) & 1;
        if (!warp_wait(&S.full[st], ph, S.abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float *halo = reinterpret_cast<const float *>(S.stage + (size_t)st * c.sstage + SUB * c.bstage);
#pragma unroll
        for (int sub = 0; sub < SUB; ++sub) {
          const int4 *offs = reinterpret_cast<const int4 *>(S.offs + st * kKStage + sub * kKS);
          int o[32];
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const int4 t4 = offs[q4];
            o[4 * q4 + 0] = t4.x;
            o[4 * q4 + 1] = t4.y;
            o[4 * q4 + 2] = t4.z;
            o[4 * q4 + 3] = t4.w;
          }
          float v[32];
#pragma unroll
          for (int kk = 0; kk < 32; ++kk) v[kk] = valid ? halo[o[kk] + poff] : 0.f;
          uint32_t hi[32], lo[32];
#pragma unroll
          for (int kk = 0; kk < 32; ++kk) {
            s2 = fmaf(v[kk], v[kk], s2);
            hi[kk] = tf32_hi_bits(v[kk]);
            lo[kk] = __float_as_uint(v[kk] - __uint_as_float(hi[kk]));
          }
          const uint32_t acol = tmem + lane_off + kColA + st * (SUB * 64) + sub * 64;
          tmem_st16(acol, *reinterpret_cast<const uint32_t(*)[16]>(&hi[0]));
          tmem_st16(acol + 16, *reinterpret_cast<const uint32_t(*)[16]>(&hi[16]));
          tmem_st16(acol + 32, *reinterpret_cast<const uint32_t(*)[16]>(&lo[0]));
          tmem_st16(acol + 48, *reinterpret_cast<const uint32_t(*)[16]>(&lo[16]));
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&S.a_full[st]);
      }
      if (!ok) break;
      const uint32_t tb = (uint32_t)(li & 1), tph = (uint32_t)((li >> 1) & 1);
      if (!warp_wait(&S.s2_empty[tb], tph ^ 1, S.abort_flag)) {
        ok = false;
        break;
      }
      S.s2buf[tb * kTileM + r] = s2;
      mbar_arrive(&S.s2_full[tb]);
    }
  } else if (warp < 8 || warp >= 10) {
    // ---------------------------------------------------------- epilogue
    // Two warps per TMEM lane quarter (warps 4-7 and 10-13; warp w reaches
    // lanes 32*(w%4) .. +31), each draining and writing half of the block's
    // channels.
    constexpr int NBH = NB / 2;
    const int q = warp % 4, half = warp >= 10 ? 1 : 0;
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const int c0 = half * NBH;  // this warp's first channel within the block
    const float *h0 = pars;
    uint32_t grp = 0;
    int64_t li = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x, ++li) {
      const int64_t t = item / c.ncb;
      const int cb = (int)(item - t * c.ncb);
      float hacc[NBH], pacc[NBH];
#pragma unroll
      for (int j = 0; j < NBH; ++j) hacc[j] = pacc[j] = 0.f;
      for (int gi = 0; gi < c.nGroups; ++gi, ++grp) {
        const uint32_t slot = grp % kSlots, ph = (grp / kSlots) & 1;
        if (!warp_wait(&S.gr_full[slot], ph, S.abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dcol = tmem + lane_off + slot * 128 + c0;
#pragma unroll
        for (int jc = 0; jc + 16 <= NBH; jc += 16) {
          uint32_t hv[16], pv[16];
          tmem_ld16_nowait(dcol + jc, hv);
          tmem_ld16_nowait(dcol + NB + jc, pv);
          tmem_ld_wait_tie(hv, pv);
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            hacc[jc + jj] += __uint_as_float(hv[jj]);
            pacc[jc + jj] += __uint_as_float(pv[jj]);
          }
        }
        if constexpr (NBH % 16 == 8) {
          constexpr int jc = NBH - 8;
          float hv[8], pv[8];
          tmem_ld8(dcol + jc, hv);
          tmem_ld8(dcol + NB + jc, pv);
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            hacc[jc + jj] += hv[jj];
            pacc[jc + jj] += pv[jj];
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
      const int64_t nimg = t / c.tpi;
      const int pix = (int)(t - nimg * c.tpi) * kTileM + r;
      const bool valid = pix < p.PQ;
      const int64_t obase = nimg * (int64_t)p.m * p.PQ + pix;
      // h0 and |P|^2 + p0^2 of this warp's channels: its copy in shared
      // memory, then all outputs in registers, then the stores
      float *hc = S.hcbuf + (q + 4 * half) * 2 * 64;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int jj = lane + 32 * e;
        if (jj < NBH) {
          const int j = cb * NB + c0 + jj;
          hc[jj] = j < p.m ? __ldg(h0 + j) : 0.f;
          hc[64 + jj] = __ldg(cj + cb * NB + c0 + jj);
        }
      }
      __syncwarp();
#pragma unroll
      for (int jj = 0; jj < NBH; ++jj) {
        const float hs = hc[jj] + hacc[jj];
        pacc[jj] = factor * (fmaf(hs, hs, -s2) + 2.f * pacc[jj] - hc[64 + jj]);
        hacc[jj] = hs;
      }
      __syncwarp();
      if (valid) {
#pragma unroll
        for (int jj = 0; jj < NBH; ++jj) {
          const int j = cb * NB + c0 + jj;
          if (j < p.m) {
            const int64_t oi = obase + (int64_t)j * p.PQ;
            out[oi] = pacc[jj];
            hsum[oi] = hacc[jj];
          }
        }
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------- MMA
    const uint32_t idesc = idesc_tf32(kTileM, 2 * NB);
    constexpr uint32_t kBlo = 2 * NB * 128;  // bytes of the hi rows of a B stage
    const uint32_t stage_addr = smem_u32(S.stage);
    constexpr int kGS = 2 / SUB;  // stages per partial sum (64 K)
    uint32_t it = 0, grp = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
      uint32_t slot = 0;
      for (int kq = 0; kq < c.nK; ++kq, ++it) {
        const bool gstart = (kq % kGS) == 0;
        const bool gend = (kq % kGS) == kGS - 1 || kq == c.nK - 1;
        if (gstart) {
          slot = grp % kSlots;
          if (!warp_wait(&S.gr_empty[slot], ((grp / kSlots) & 1) ^ 1, S.abort_flag)) {
            ok = false;
            break;
          }
        }
        const uint32_t st = it % nst, ph = (it / nst) & 1;
        if (!warp_wait(&S.b_full[st], ph, S.abort_flag) || !warp_wait(&S.a_full[st], ph, S.abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // straight-line issue from one elected lane, operands formed outside
        const uint32_t dcol = tmem + slot * 128;
        const uint32_t acol = tmem + kColA + st * (SUB * 64);
        const uint32_t bst = stage_addr + st * c.sstage;  // per sub-stage: [H;P] hi rows, then lo rows
        const uint32_t bsub = c.bstage;
        const uint32_t acc0 = gstart ? 0u : 1u;
        if (elect_one()) {
#pragma unroll
          for (int sub = 0; sub < SUB; ++sub) {
#pragma unroll
            for (int ks = 0; ks < kKS / 8; ++ks) {
              const uint32_t ahi = acol + sub * 64 + ks * 8, alo = ahi + 32;
              const uint32_t bhi = bst + sub * bsub + ks * 32;
              const uint32_t blo = bhi + kBlo;
              mma_tf32_ts(dcol, ahi, sdesc_kmajor_sw128(bhi), idesc, (sub == 0 && ks == 0) ? acc0 : 1u);
              mma_tf32_ts(dcol, alo, sdesc_kmajor_sw128(bhi), idesc, 1u);
              mma_tf32_ts(dcol, ahi, sdesc_kmajor_sw128(blo), idesc, 1u);
            }
          }
          tc_commit(&S.s_empty[st]);
          if (gend) tc_commit(&S.gr_full[slot]);
        }
        __syncwarp();
        if (gend) ++grp;
      }
    }
    // Drain: every MMA issued by this warp completes before TMEM is freed.
    if (elect_one()) tc_commit(S.final_bar);
    __syncwarp();
    mbar_wait(S.final_bar, 0, kWaitNs, nullptr);
  } else {
    // ------------------------------------------------------------- loader
    uint32_t it = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
      const int64_t t = item / c.ncb;
      const int cb = (int)(item - t * c.ncb);
      const TileGeo tg = tile_geo(p, c, t);
      const float *ximg = x + tg.n * p.CHW + (int64_t)tg.ir0 * p.W;
      const int64_t run = (int64_t)tg.rows * p.W;
      for (int kq = 0; kq < c.nK; ++kq, ++it) {
        const uint32_t st = it % nst, ph = (it / nst) & 1;
        if (!warp_wait(&S.s_empty[st], ph ^ 1, S.abort_flag)) {
          ok = false;
          break;
        }
        const int clo = S.koff[kq * kKStage].x;
        uint8_t *sbase = S.stage + (size_t)st * c.sstage;
        uint8_t *hbase = sbase + SUB * c.bstage;
        // entries past the window read the zero buffer (relative to this
        // stage's halo, where the producers add the pixel's offset)
        const int zoff = (int)(S.zbuf - reinterpret_cast<const float *>(hbase));
        const float *bsrc = wsB + ((int64_t)cb * c.nKB + (int64_t)kq * SUB) * 2 * c.N * 32;
        if (c.tma) {
          // one tensor copy: planes clo .. clo+nchs-1 of image n, PS floats
          // each from the 16-byte boundary at or below the tile's first input
          // element (zero past the end of the tensor)
          const int xo = tg.ir0 * p.W, x0 = xo & ~3, ld = xo - x0;
#pragma unroll
          for (int e = 0; e < kKStage / 32; ++e) {
            const int2 ko = S.koff[kq * kKStage + lane + 32 * e];
            S.offs[st * kKStage + lane + 32 * e] = ko.x >= 0 ? (ko.x - clo) * c.PS + ld + ko.y : zoff;
          }
          __syncwarp();
          if (lane == 0) {
            mbar_arrive_expect_tx(&S.full[st], (uint32_t)(c.nchs * c.PS * 4));
            tma_load_2d(hbase, &xmap, x0, (int)(tg.n * p.C + clo), &S.full[st]);
            mbar_arrive_expect_tx(&S.b_full[st], SUB * c.bstage);
            bulk_g2s(sbase, bsrc, SUB * c.bstage, &S.b_full[st]);
          }
          __syncwarp();
          continue;
        }
        // Channel planes of the stage (lanes, two rounds): 16-byte-rounded
        // spans, their leads and the total byte count.
        int chi = clo;
#pragma unroll 1
        for (int kk = kKStage - 1; kk >= 0; --kk) {
          const int ch = S.koff[kq * kKStage + kk].x;
          if (ch >= 0) {
            chi = ch;
            break;
          }
        }
        const int nch = chi - clo + 1;
        uint32_t bytes = 0;
        for (int ci = lane; ci < nch; ci += 32) {
          const tc::BulkSpan sp = tc::bulk_span(ximg + (int64_t)(clo + ci) * p.HW, run);
          S.lead[st * kMaxCh + ci] = sp.lead;
          bytes += sp.bytes;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, off);
        __syncwarp();
        // Offset of every K of the stage inside the halo: plane, lead, tap.
#pragma unroll
        for (int e = 0; e < kKStage / 32; ++e) {
          const int2 ko = S.koff[kq * kKStage + lane + 32 * e];
          S.offs[st * kKStage + lane + 32 * e] =
              ko.x >= 0 ? (ko.x - clo) * c.PS + S.lead[st * kMaxCh + (ko.x - clo)] + ko.y : zoff;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(&S.full[st], bytes);
        __syncwarp();
        for (int ci = lane; ci < nch; ci += 32) {
          const tc::BulkSpan sp = tc::bulk_span(ximg + (int64_t)(clo + ci) * p.HW, run);
          bulk_g2s(hbase + (size_t)ci * c.PS * 4, sp.src, sp.bytes, &S.full[st]);
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&S.b_full[st], SUB * c.bstage);
          bulk_g2s(sbase, bsrc, SUB * c.bstage, &S.b_full[st]);
        }
        __syncwarp();
      }
    }
    // Drain: the copies issued last have landed before the CTA exits.
    const uint32_t last = it < (uint32_t)nst ? it : (uint32_t)nst;
    for (uint32_t i = 0; i < last; ++i) {
      const uint32_t idx = it - 1 - i;
      mbar_wait(&S.full[idx % nst], (idx / nst) & 1, kWaitNs, nullptr);
      mbar_wait(&S.b_full[idx % nst], (idx / nst) & 1, kWaitNs, nullptr);
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

PerContext<uint64_t> g_attr;
std::mutex g_sm_mutex;
int g_sm_count[64] = {0};

template <int NB, int SUB>
int launch_forward_sub(const Problem &p, const FwdCfg &c, const CUtensorMap &xmap, const float *x, const float *pars,
                       const float *wsB, const float *cj, float factor, float *out, float *hsum, int *status,
                       cudaStream_t stream) {
  const int ast = once_per_context(g_attr, 1ull << ((NB / 16 - 1) * 2 + (SUB - 1)), []() -> int {
    PC2D_CUDA_CHECK(cudaFuncSetAttribute(tc_forward_kernel<NB, SUB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024));
    return (int)PC2D_OK;
  });
  if (ast != PC2D_OK) return ast;
  const int grid = (int)std::min<int64_t>(c.items, device_sm_count());
  timing_begin(K_FORWARD, stream);
  tc_forward_kernel<NB, SUB><<<grid, kFwdThreads, fwd_smem_bytes(p, c), stream>>>(x, pars, wsB, cj, factor, p, c, xmap,
                                                                               out, hsum, status);
  timing_end(K_FORWARD, stream);
  PC2D_LAUNCH_CHECK("tc_forward_kernel");
  return PC2D_OK;
}

template <int NB>
int launch_forward(const Problem &p, FwdCfg c, const float *x, const float *pars, const float *wsB,
                   const float *cj, float factor, float *out, float *hsum, int *status, cudaStream_t stream) {
  CUtensorMap xmap;
  std::memset(&xmap, 0, sizeof(xmap));
  if (c.tma && !encode_planes_map(x, p.HW, (int64_t)p.n * p.C, c.PS, c.nchs, &xmap))
    c.tma = 0;  // per-channel bulk copies instead (same layout)
  if (c.sub == 2) return launch_forward_sub<NB, 2>(p, c, xmap, x, pars, wsB, cj, factor, out, hsum, status, stream);
  return launch_forward_sub<NB, 1>(p, c, xmap, x, pars, wsB, cj, factor, out, hsum, status, stream);
}

}  // namespace

namespace {
// cuTensorMapEncodeTiled, resolved once through the runtime (no link-time
// dependency on the driver library).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}
}  // namespace

bool encode_planes_map(const float *x, int64_t HW, int64_t rows, int box_inner, int box_rows, CUtensorMap *map) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn || (reinterpret_cast<uintptr_t>(x) & 15) != 0 || HW % 4 != 0 || box_inner % 4 != 0 || box_inner < 4 ||
      box_inner > 256 || box_rows < 1 || box_rows > 256 || rows < 1)
    return false;
  const cuuint64_t dims[2] = {(cuuint64_t)HW, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)HW * 4};
  const cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_rows_map_sw128(const float *t, int64_t cols, int64_t rows, int box_rows, CUtensorMap *map) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn || (reinterpret_cast<uintptr_t>(t) & 15) != 0 || cols % 4 != 0 || cols < 32 || box_rows < 1 ||
      box_rows > 256 || rows < 1)
    return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
  const cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(t), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(g_sm_mutex);
  if (g_sm_count[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    g_sm_count[dev] = v;
  }
  return g_sm_count[dev];
}

bool tc_forward_supported(const Problem &p) {
  if (p.m < 1 || p.d > kMaxD || p.CHW >= ((int64_t)1 << 31) || p.NPQ <= 0 || p.PQ >= ((int64_t)1 << 30)) return false;
  const FwdCfg c = fwd_cfg_fit(p);
  return c.nchs <= kMaxCh && fwd_smem_bytes(p, c) <= (size_t)kSmemLimit;
}

size_t tc_forward_workspace(const Problem &p) {
  const FwdCfg c = fwd_cfg_fit(p);
  return align_up(fwd_bsplit_bytes(c), 256) + align_up((size_t)c.ncb * c.NB * sizeof(float), 256);
}

int tc_forward(const Problem &p, const float *x, const float *pars, double factor, float *out, float *hsum, void *ws,
               cudaStream_t stream) {
  const FwdCfg c = fwd_cfg_fit(p);
  int *status = device_status_ptr();
  if (!status) {
    set_last_error("could not resolve the device status word");
    return PC2D_ERR_CUDA;
  }
  float *wsB = reinterpret_cast<float *>(ws);
  float *cj = reinterpret_cast<float *>(reinterpret_cast<char *>(ws) + align_up(fwd_bsplit_bytes(c), 256));
  tc_fwd_prep<<<c.ncb * c.nKB * kPrepSplit + ceil_div(c.ncb * c.NB, 8), 256, 0, stream>>>(pars, p, c, wsB, cj);
  PC2D_LAUNCH_CHECK("tc_fwd_prep");
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
