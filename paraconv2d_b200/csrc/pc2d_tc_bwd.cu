// tcgen05 backward kernels of the ParaConv2d paraboloid convolution (fp32 via
// 3xTF32 split precision).
//
// Input gradient (reference paraconv2d.cc:153-183):
//   dx[c,y,x] = 2 * sum_{tap, o: window(o,tap) = (y,x)} sum_j
//                 g[j,o] * (hsum[j,o] * h[j,c,tap] - x[c,y,x] + p[j,c,tap])
//             = 2 * (sum_{tap,j} (g*hsum)[j,o] h[j,c,tap] + g[j,o] p[j,c,tap]
//                    - x[c,y,x] * SG[y,x]),   SG = sum_{tap,j} g[j,o(tap)]
// is an implicit GEMM with M = 128 input pixels of one image per tile,
// N = input channels of a block (NC <= 64) and K = (j-block of 16 output
// channels, tap, j, {g*hsum, g}) swept 32 at a time.  With stride s > 1 only
// the taps whose row/column offset has the residue of (y, x) mod s reach an
// input pixel, so the tiles group pixels by stride phase (y mod s0, x mod s1)
// and K runs over that phase's taps only (a quarter of them for stride 2).
// The windows are flipped exactly as in the forward pass: tap (ix2, iy2) of output pixel (oy, ox)
// reads input (oy*s0 + (k0-1-ix2)*dl0, ox*s1 + (k1-1-iy2)*dl1).
//
// Warp roles (480 threads):
//   - warps 0-3, producers (one TMEM lane = one input pixel): per tap, locate
//     the output pixel whose window covers the pixel, form g*hsum and g for
//     the 16 channels of the stage from the staged planes, accumulate SG,
//     split into tf32 hi + lo and tcgen05.st them into TMEM (A operand).  A
//     producer reuses an A slot as soon as the MMAs that read it complete;
//   - warps 4-7 and 11-14, epilogue (two warps per TMEM lane quarter, half
//     of the channels each): drain the partial sums (a fresh one per j-block
//     of 16 output channels, in one of two TMEM slots) into fp32 registers,
//     and write
//     dx = 2 * (acc - x * SG), with x copied to shared memory (cp.async) at
//     the start of the tile;
//   - warp 8, MMA (one thread): per 8-wide K step two MMAs
//       [main | corr] = Ahi * [W hi; W lo]   (N = 2 NC)
//       corr         += Alo * W hi            (N = NC)
//     so main + corr = Ahi*Bhi + Ahi*Blo + Alo*Bhi (3xTF32);
//   - warp 9, weight loader: per 32-K stage the pre-split weights
//     [W hi; W lo] (written once per call by a prep kernel), one bulk copy;
//   - warp 10, plane loader: per j-block the rows of g and hsum that the
//     tile's windows reach, one 1-D bulk copy per output-channel plane,
//     shared by the taps of the j-block, two j-blocks in flight.
// Every wait is bounded; on a timeout the kernel records the error, stops
// its loops, drains its own copies and frees TMEM, as the forward kernel
// (pc2d_tc_fwd.cu) does.
#include <algorithm>
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
constexpr int kJB = 16;          // output channels per j-block (32 K per tap)
constexpr int kStages = 2;       // A/B stages of kTapsPS taps (64 K) each
constexpr int kTapsPS = 2;       // taps per stage
constexpr int kSlots = 2;        // accumulator slots (one partial sum per j-block)
constexpr int kMaxNC = 64;
constexpr int kThreads = 480;
constexpr int kMinSmem = 120 * 1024;
constexpr int kSmemLimit = 227 * 1024;
constexpr uint32_t kColA = 256;

constexpr int kMaxPh = 16;  // stride phases s0*s1
constexpr int kMaxKs = 32;  // kernel extent per axis

struct DgCfg {
  int ncb;          // input-channel blocks
  int NC;           // channels per block (multiple of 16, <= 64)
  int nJB;          // j-blocks
  int nK;           // weight stages of the prep layout = nJB * T
  int nph;          // stride phases (y mod s0, x mod s1)
  int ph_rows[kMaxPh], ph_cols[kMaxPh];   // phase grid of an image's pixel window
  int ph_a0[kMaxPh], ph_b0[kMaxPh];       // its first row and column within the phase's full grid
  int ph_ntaps[kMaxPh];                   // taps that reach the phase
  int ph_first[kMaxPh + 1];               // first tile of each phase within an image
  int ph_tap0[kMaxPh + 1];                // first entry of each phase in the tap table
  int tpi;          // tiles per image (all phases)
  int64_t tiles, items;
  int PSo;          // g/hsum plane stride (floats, multiple of 4)
  uint32_t bstage;  // B bytes per stage (hi + lo)
  uint32_t jslot;   // bytes of a j-block slot (32 planes), multiple of 1024
  int tma;          // 1: a j-block's planes are two 2-D tensor copies (g planes, then hsum planes)
};

// Per-phase tables copied from DgCfg into shared memory at kernel start
// (indexing a kernel parameter with a run-time index makes the compiler read
// every field of it through generic loads).
struct DgPhases {
  int first[kMaxPh + 1];
  int tap0[kMaxPh + 1];
  int rows[kMaxPh];
  int cols[kMaxPh];
  int a0[kMaxPh];
  int b0[kMaxPh];
  int ntaps[kMaxPh];
};

// The input pixels whose gradient is computed: rows [y0, y1) and columns
// [x0, x1) of the padded input.  The op needs all of them; a module that pads
// its input needs only the unpadded interior, and tiling just that saves the
// tiles of the border (on a 34x34 padded plane 8 tiles of 128 pixels instead
// of 10; on a stride-2 layer's 17x17 phase grids 2 instead of 3).
struct DgWindow {
  int y0, y1, x0, x1;
};

inline DgWindow dg_full_window(const Problem &p) { return DgWindow{0, p.H, 0, p.W}; }

// Taps that reach input rows y with y % s0 == py: tap row (k0-1-ix2)*dl0 must
// have the same residue (the output pixel is then (y - row)/s0 exactly).
inline int phase_rows(int k, int dl, int s, int py, int *list) {
  int n = 0;
  for (int i = 0; i < k; ++i)
    if (((k - 1 - i) * dl) % s == py) {
      if (list) list[n] = i;
      ++n;
    }
  return n;
}

// First index i >= 0 of the progression r + s*i that is >= v.
inline int first_at_or_after(int v, int r, int s) { return v > r ? (v - r + s - 1) / s : 0; }

DgCfg dg_cfg(const Problem &p, const DgWindow &w) {
  DgCfg c;
  c.ncb = std::max(1, ceil_div(p.C, kMaxNC));
  const int nc = ceil_div(p.C, c.ncb);
  c.NC = (nc + 15) / 16 * 16;
  c.nJB = ceil_div(p.m, kJB);
  c.nK = c.nJB * p.T;
  c.nph = p.s0 * p.s1;
  int orows = 1;
  c.tpi = 0;
  for (int ph = 0; ph < kMaxPh; ++ph) {
    c.ph_rows[ph] = c.ph_cols[ph] = c.ph_ntaps[ph] = 0;
    c.ph_a0[ph] = c.ph_b0[ph] = 0;
    c.ph_first[ph] = 0;
    c.ph_tap0[ph] = 0;
  }
  int taps = 0;
  for (int ph = 0; ph < c.nph && ph < kMaxPh; ++ph) {
    const int py = ph / p.s1, px = ph % p.s1;
    c.ph_a0[ph] = first_at_or_after(w.y0, py, p.s0);
    c.ph_b0[ph] = first_at_or_after(w.x0, px, p.s1);
    c.ph_rows[ph] = std::max(0, first_at_or_after(w.y1, py, p.s0) - c.ph_a0[ph]);
    c.ph_cols[ph] = std::max(0, first_at_or_after(w.x1, px, p.s1) - c.ph_b0[ph]);
    c.ph_ntaps[ph] = phase_rows(p.k0, p.dl0, p.s0, py, nullptr) * phase_rows(p.k1, p.dl1, p.s1, px, nullptr);
    c.ph_first[ph] = c.tpi;
    c.ph_tap0[ph] = taps;
    taps += c.ph_ntaps[ph];
    const int64_t npix = (int64_t)c.ph_rows[ph] * c.ph_cols[ph];
    c.tpi += (int)((npix + kTileM - 1) / kTileM);
    if (c.ph_cols[ph] > 0) {
      const int span = (int)std::min<int64_t>(c.ph_rows[ph], (c.ph_cols[ph] + kTileM - 2) / c.ph_cols[ph] + 1);
      const int yspan = (span - 1) * p.s0 + 1;
      orows = std::max(orows, std::min<int>(p.P, (yspan - 1 + (p.k0 - 1) * p.dl0) / p.s0 + 2));
    }
  }
  c.ph_first[std::min(c.nph, kMaxPh)] = c.tpi;
  c.ph_tap0[std::min(c.nph, kMaxPh)] = taps;
  c.tiles = (int64_t)p.n * c.tpi;
  c.items = c.tiles * c.ncb;
  c.PSo = (int)(((int64_t)orows * p.Q + 8 + 3) / 4 * 4);
  c.bstage = (uint32_t)(2 * c.NC * 128);  // one tap
  // 32 planes, then one plane of zeros that missing channels point at
  c.jslot = (uint32_t)align_up((size_t)(2 * kJB + 1) * c.PSo * 4, 1024);
  // the 16 g (and 16 hsum) planes of a j-block as one tensor copy each: rows
  // of PQ floats 16-byte strided, the staged run (from the 16-byte boundary
  // at or below its first element) at most 256 floats
  c.tma = (p.PQ % 4 == 0 && c.PSo <= 256 && (int64_t)p.n * p.m < ((int64_t)1 << 31)) ? 1 : 0;
  return c;
}

inline size_t dg_bsplit_bytes(const DgCfg &c) { return (size_t)c.ncb * c.nK * c.bstage; }
inline size_t dg_smem_bytes(const DgCfg &c) {
  size_t s = 1024 + (size_t)kStages * kTapsPS * c.bstage + 2 * (size_t)c.jslot + (size_t)c.NC * kTileM * 4 +
             2 * 2 * kJB * 4 + 2 * kTileM * 4 + 24 * 8 + 64 +
             sizeof(DgPhases) + (size_t)(c.nK / c.nJB) * 8;
  return std::max<size_t>(s, kMinSmem);
}

// Weights of input-channel block cb for stage kq = (jb, tap), split into
// tf32 hi/lo, 128-byte-swizzled K-major: rows = channels (hi block then lo
// block), K element kk = (j_local = kk/2, w = kk%2) holds h[j][c][tap]
// (w = 0, multiplies g*hsum) or p[j][c][tap] (w = 1, multiplies g).
// Grid (nK, ncb, NC / 8): each thread block writes 8 channel rows of one
// (j-block, tap) block.
__global__ void __launch_bounds__(256) tc_dg_prep_weights(const float *__restrict__ pars, Problem p, DgCfg c,
                                                          float *__restrict__ wsB) {
  const int kq = blockIdx.x, cb = blockIdx.y;
  const int jb = kq / p.T, tap = kq - (kq / p.T) * p.T;
  float *blk = wsB + ((int64_t)cb * c.nK + kq) * 2 * c.NC * 32;
  const float *h = pars + p.m;
  const float *pp = h + (int64_t)p.m * p.d;
  for (int e = threadIdx.x; e < 8 * 32; e += blockDim.x) {
    const int r = blockIdx.z * 8 + e / 32, kk = e % 32;
    const int ch = cb * c.NC + r;
    const int j = jb * kJB + kk / 2;
    float v = 0.f;
    if (ch < p.C && j < p.m) v = ((kk & 1) ? pp : h)[(int64_t)j * p.d + (int64_t)ch * p.T + tap];
    float hi, lo;
    tf32_split_rn(v, hi, lo);
    const int pos = r * 32 + (((kk >> 2) ^ (r & 7)) << 2) + (kk & 3);
    blk[pos] = hi;
    blk[c.NC * 32 + pos] = lo;
  }
}

struct DgGeo {
  int64_t n;
  int ph, py, px;  // stride phase
  int q0;          // first phase-grid pixel of the tile
  int cols, npix;  // phase grid width and size
  int a0, b0;      // first row and column of the phase grid (within the phase's full grid)
  int oylo;        // first output row staged
  int orows;       // output rows staged (may be 0)
  int ntaps;       // taps reaching this phase
  int tap0;        // the phase's first entry in the tap table
};

__device__ __forceinline__ DgGeo dg_geo(const Problem &p, const DgCfg &c, const DgPhases &ps, int64_t t) {
  DgGeo g;
  g.n = t / c.tpi;
  const int r = (int)(t - g.n * c.tpi);
  int ph = 0;
  while (ph + 1 < c.nph && ps.first[ph + 1] <= r) ++ph;
  g.ph = ph;
  g.py = ph / p.s1;
  g.px = ph - g.py * p.s1;
  g.q0 = (r - ps.first[ph]) * kTileM;
  g.cols = ps.cols[ph];
  g.npix = ps.rows[ph] * g.cols;
  g.a0 = ps.a0[ph];
  g.b0 = ps.b0[ph];
  g.ntaps = ps.ntaps[ph];
  g.tap0 = ps.tap0[ph];
  const int qlast = min(g.q0 + kTileM - 1, g.npix - 1);
  const int ya = g.py + p.s0 * (g.a0 + g.q0 / g.cols), yb = g.py + p.s0 * (g.a0 + qlast / g.cols);
  const int lo = ya - (p.k0 - 1) * p.dl0;
  const int oylo = lo <= 0 ? 0 : (lo + p.s0 - 1) / p.s0;
  const int oyhi = min(p.P - 1, yb / p.s0);
  g.oylo = oylo;
  g.orows = oyhi >= oylo ? oyhi - oylo + 1 : 0;
  return g;
}

// Entry e of the tap table, phase by phase in K order: the tap index
// (ix2*k1 + iy2) and, packed as (dy << 16) | dx, the output-pixel offsets of
// the tap within the phase grid.  An input pixel at phase-grid position
// (a, b) of phase (py, px), i.e. (y, x) = (py + s0*a, px + s1*b), receives
// that tap from output pixel (a - dy, b - dx), because the tap's row offset
// (k0-1-ix2)*dl0 is py + s0*dy (columns likewise).
__device__ __forceinline__ int2 dg_tap_entry(const Problem &p, const DgCfg &c, const DgPhases &ps, int e) {
  int ph = 0;
  while (ph + 1 < c.nph && ps.tap0[ph + 1] <= e) ++ph;
  const int py = ph / p.s1, px = ph - py * p.s1;
  int ncl = 0;
  for (int i = 0; i < p.k1; ++i) ncl += (((p.k1 - 1 - i) * p.dl1) % p.s1 == px);
  const int ti = e - ps.tap0[ph];
  const int ri = ti / ncl, ci = ti - ri * ncl;
  int ix2 = 0, iy2 = 0;
  for (int i = 0, n = 0; i < p.k0; ++i)
    if (((p.k0 - 1 - i) * p.dl0) % p.s0 == py && n++ == ri) ix2 = i;
  for (int i = 0, n = 0; i < p.k1; ++i)
    if (((p.k1 - 1 - i) * p.dl1) % p.s1 == px && n++ == ci) iy2 = i;
  const int dy = ((p.k0 - 1 - ix2) * p.dl0 - py) / p.s0, dxo = ((p.k1 - 1 - iy2) * p.dl1 - px) / p.s1;
  return make_int2(ix2 * p.k1 + iy2, (dy << 16) | dxo);
}

// 32 A values of one tap for this pixel: {g*hsum, g} of the j-block's 16
// channels at the output pixel ooff of the staged planes (a channel past m
// reads the slot's zero plane), split into tf32 hi + lo; accumulates SG.
__device__ __forceinline__ void dg_gather(const float *planes, const int (&to)[2 * kJB], bool valid, int ooff,
                                          float &sg, uint32_t (&hi)[kKS], uint32_t (&lo)[kKS]) {
#pragma unroll
  for (int jl = 0; jl < kJB; ++jl) {
    const int og = to[2 * jl], oh = to[2 * jl + 1];
    const float gv = valid ? planes[og + ooff] : 0.f;
    const float hv = valid ? planes[oh + ooff] : 0.f;
    sg += gv;
    const float a0 = gv * hv, a1 = gv;
    hi[2 * jl] = tf32_hi_bits(a0);
    lo[2 * jl] = __float_as_uint(a0 - __uint_as_float(hi[2 * jl]));
    hi[2 * jl + 1] = tf32_hi_bits(a1);
    lo[2 * jl + 1] = __float_as_uint(a1 - __uint_as_float(hi[2 * jl + 1]));
  }
}

template <int NC>
__global__ void __launch_bounds__(kThreads, 1)
tc_dgrad_kernel(const float *__restrict__ grad, const float *__restrict__ x, const float *__restrict__ hsum,
                const float *__restrict__ wsB, Problem p, DgCfg c, const __grid_constant__ CUtensorMap gmap,
                const __grid_constant__ CUtensorMap hmap, DxOut dxo, float *__restrict__ dx, int *status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  uint8_t *sB = base;                                                 // [kStages][kTapsPS] x bstage
  uint8_t *sJ = base + (size_t)kStages * kTapsPS * c.bstage;          // 2 x jslot
  float *sx = reinterpret_cast<float *>(sJ + 2 * (size_t)c.jslot);    // [NC][128] input values of the tile
  int *jtab = reinterpret_cast<int *>(sx + NC * kTileM);              // [2][32] plane offsets (missing planes: the zero plane)
  float *sgbuf = reinterpret_cast<float *>(jtab + 2 * 2 * kJB);       // [2][128]
  uint64_t *bars = reinterpret_cast<uint64_t *>((reinterpret_cast<uintptr_t>(sgbuf + 2 * kTileM) + 7) & ~(uintptr_t)7);
  uint64_t *a_full = bars, *s_empty = bars + 2, *jfull = bars + 4, *jempty = bars + 6;
  uint64_t *gr_full = bars + 8, *gr_empty = bars + 10, *sg_full = bars + 12, *sg_empty = bars + 14;
  uint64_t *final_bar = bars + 16;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 17);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  DgPhases &ps = *reinterpret_cast<DgPhases *>(tmem_holder + 2);
  int2 *ptab = reinterpret_cast<int2 *>(&ps + 1);  // [T] tap table

  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i <= kMaxPh; ++i) {
      ps.first[i] = c.ph_first[i];
      ps.tap0[i] = c.ph_tap0[i];
    }
#pragma unroll
    for (int i = 0; i < kMaxPh; ++i) {
      ps.rows[i] = c.ph_rows[i];
      ps.cols[i] = c.ph_cols[i];
      ps.a0[i] = c.ph_a0[i];
      ps.b0[i] = c.ph_b0[i];
      ps.ntaps[i] = c.ph_ntaps[i];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < p.T; e += blockDim.x) ptab[e] = dg_tap_entry(p, c, ps, e);
  // the zero plane after the 32 planes of each j-block slot (no copy writes it)
  for (int e = threadIdx.x; e < 2 * c.PSo; e += blockDim.x)
    reinterpret_cast<float *>(sJ + (size_t)(e / c.PSo) * c.jslot)[2 * kJB * c.PSo + e % c.PSo] = 0.f;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      // 128 producer arrivals + the weight loader's arrival with the bytes of
      // its copies
      mbar_init(&a_full[i], 129);
      mbar_init(&s_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&jfull[i], 1);
      mbar_init(&jempty[i], 128);
      mbar_init(&gr_full[i], 1);
      mbar_init(&gr_empty[i], 256);
      mbar_init(&sg_full[i], 128);
      mbar_init(&sg_empty[i], 256);
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
  // The parameter-gradient kernel launched after this one reads nothing it
  // writes: let it start on SMs this grid has left.
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp < 4) {
    // ---------------------------------------------------------- producers
    const int r = warp * 32 + lane;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    uint32_t it = 0, jit = 0;
    int64_t li = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x, ++li) {
      const DgGeo tg = dg_geo(p, c, ps, item / c.ncb);
      const int q = tg.q0 + r;
      const bool pvalid = q < tg.npix;
      const int qa = q / tg.cols;
      const int ay = tg.a0 + qa, bx = tg.b0 + (q - qa * tg.cols);  // phase-grid position
      float sg = 0.f;
      for (int jb = 0; jb < c.nJB && ok; ++jb, ++jit) {
        const uint32_t js = jit & 1, jph = (jit >> 1) & 1;
        if (!warp_wait(&jfull[js], jph, abort_flag)) {
          ok = false;
          break;
        }
        const float *planes = reinterpret_cast<const float *>(sJ + (size_t)js * c.jslot);
        int to[2 * kJB];
#pragma unroll
        for (int q4 = 0; q4 < 2 * kJB / 4; ++q4) {
          const int4 t4 = reinterpret_cast<const int4 *>(jtab + js * 2 * kJB)[q4];
          to[4 * q4 + 0] = t4.x;
          to[4 * q4 + 1] = t4.y;
          to[4 * q4 + 2] = t4.z;
          to[4 * q4 + 3] = t4.w;
        }
        for (int ti = 0; ti < tg.ntaps; ti += kTapsPS, ++it) {
          const uint32_t st = it % kStages, ph = (it / kStages) & 1;
          const uint32_t acol = tmem + lane_off + kColA + st * (kTapsPS * 64);
#pragma unroll
          for (int h = 0; h < kTapsPS; ++h) {
            if (ti + h >= tg.ntaps) break;
            // output pixel whose window puts this tap on the input pixel
            const int dyx = ptab[tg.tap0 + ti + h].y;
            const int oy = ay - (dyx >> 16), ox = bx - (dyx & 0xffff);
            const bool valid = pvalid && oy >= 0 && ox >= 0 && oy < p.P && ox < p.Q;
            uint32_t hi[kKS], lo[kKS];
            dg_gather(planes, to, valid, (oy - tg.oylo) * p.Q + ox, sg, hi, lo);
            if (h == 0) {
              // the MMAs that read this A stage last have completed (the
              // gather above needs only the staged planes, so it overlaps
              // that wait)
              if (!warp_wait(&s_empty[st], ph ^ 1, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
            tmem_st16(acol + h * 64, *reinterpret_cast<const uint32_t(*)[16]>(&hi[0]));
            tmem_st16(acol + h * 64 + 16, *reinterpret_cast<const uint32_t(*)[16]>(&hi[16]));
            tmem_st16(acol + h * 64 + 32, *reinterpret_cast<const uint32_t(*)[16]>(&lo[0]));
            tmem_st16(acol + h * 64 + 48, *reinterpret_cast<const uint32_t(*)[16]>(&lo[16]));
          }
          if (!ok) break;
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(&a_full[st]);
        }
        mbar_arrive(&jempty[js]);
      }
      if (!ok) break;
      const uint32_t tb = (uint32_t)(li & 1), tph = (uint32_t)((li >> 1) & 1);
      if (!warp_wait(&sg_empty[tb], tph ^ 1, abort_flag)) {
        ok = false;
        break;
      }
      sgbuf[tb * kTileM + r] = sg;
      mbar_arrive(&sg_full[tb]);
    }
  } else if (warp < 8 || warp >= 11) {
    // ---------------------------------------------------------- epilogue
    // Two warps per TMEM lane quarter (warps 4-7 and 11-14; warp w reaches
    // lanes 32*(w%4) .. +31), each draining and writing half of the block's
    // channels.
    constexpr int NH = NC / 2;
    const float two_s = 2.f * (float)dxo.scale;  // 2 (x input factor x grad factor, for a padding module)
    const int qq = warp % 4, half = warp >= 11 ? 1 : 0;
    const int c0 = half * NH;  // this warp's first channel within the block
    const int r = qq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qq * 32) << 16;
    uint32_t grp = 0;
    int64_t li = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x, ++li) {
      const int64_t t = item / c.ncb;
      const int cb = (int)(item - t * c.ncb);
      const DgGeo tg = dg_geo(p, c, ps, t);
      const int ngroups = tg.ntaps > 0 ? c.nJB : 0;  // one partial sum per j-block
      // this pixel's input values are needed at the end of the item: copy
      // them to shared memory now, behind the item's MMAs (each thread reads
      // back only what it copied, so the cp.async wait alone orders them)
      const int q = tg.q0 + r;
      const bool pv = q < tg.npix;
      int64_t xb = 0, ob = -1;
      if (pv) {
        const int qa = q / tg.cols;
        const int yy = tg.py + p.s0 * (tg.a0 + qa), xx = tg.px + p.s1 * (tg.b0 + q - qa * tg.cols);
        xb = tg.n * p.CHW + (int64_t)yy * p.W + xx;
        ob = dx_index(dxo, tg.n, yy, xx);
#pragma unroll 8
        for (int cc = c0; cc < c0 + NH; ++cc) {
          const bool have = cb * NC + cc < p.C;
          cp_async4(sx + cc * kTileM + r, have ? x + xb + (int64_t)(cb * NC + cc) * p.HW : x, have);
        }
      }
      cp_async_commit();
      float acc[NH];
#pragma unroll
      for (int j = 0; j < NH; ++j) acc[j] = 0.f;
      for (int gi = 0; gi < ngroups; ++gi, ++grp) {
        const uint32_t slot = grp % kSlots, ph = (grp / kSlots) & 1;
        if (!warp_wait(&gr_full[slot], ph, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dcol = tmem + lane_off + slot * 128 + c0;
#pragma unroll
        for (int jc = 0; jc + 16 <= NH; jc += 16) {
          uint32_t mv[16], cv[16];
          tmem_ld16_nowait(dcol + jc, mv);
          tmem_ld16_nowait(dcol + NC + jc, cv);
          tmem_ld_wait_tie(mv, cv);
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) acc[jc + jj] += __uint_as_float(mv[jj]) + __uint_as_float(cv[jj]);
        }
        if constexpr (NH % 16 == 8) {
          constexpr int jc = NH - 8;
          float mv[8], cv[8];
          tmem_ld8(dcol + jc, mv);
          tmem_ld8(dcol + NC + jc, cv);
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) acc[jc + jj] += mv[jj] + cv[jj];
        }
        tc_fence_before();
        mbar_arrive(&gr_empty[slot]);
      }
      if (!ok) break;
      const uint32_t tb = (uint32_t)(li & 1), tph = (uint32_t)((li >> 1) & 1);
      if (!warp_wait(&sg_full[tb], tph, abort_flag)) {
        ok = false;
        break;
      }
      const float sg = sgbuf[tb * kTileM + r];
      mbar_arrive(&sg_empty[tb]);
      cp_async_wait<0>();
      if (ob >= 0) {
#pragma unroll
        for (int cc = 0; cc < NH; ++cc)
          if (cb * NC + c0 + cc < p.C)
            dx[ob + (int64_t)(cb * NC + c0 + cc) * dxo.HWu] = two_s * (acc[cc] - sx[(c0 + cc) * kTileM + r] * sg);
      }
    }
    cp_async_wait<0>();  // copies of an item left on an error path
  } else if (warp == 8) {
    // ------------------------------------------------------------- MMA
    // One partial sum per j-block (2 x 16 x taps K, e.g. 288 for a 3x3
    // window): a fresh accumulator slot at the j-block's first stage,
    // drained by the epilogue after its last.  Within a stage the main MMAs
    // go back to back, then the corrections.
    constexpr uint32_t kBTap = 2 * NC * 128;  // bytes of one tap's [W hi; W lo] tile
    const uint32_t id_main = idesc_tf32(kTileM, 2 * NC);
    const uint32_t id_corr = idesc_tf32(kTileM, NC);
    const uint32_t sB_addr = smem_u32(sB);
    uint32_t it = 0, grp = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
      const DgGeo tg = dg_geo(p, c, ps, item / c.ncb);
      if (tg.ntaps == 0) continue;
      for (int jb = 0; jb < c.nJB && ok; ++jb, ++grp) {
        const uint32_t slot = grp % kSlots;
        if (!warp_wait(&gr_empty[slot], ((grp / kSlots) & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t dcol = tmem + slot * 128;
        for (int ti = 0; ti < tg.ntaps; ti += kTapsPS, ++it) {
          const int nh = min(kTapsPS, tg.ntaps - ti);
          const uint32_t st = it % kStages, ph = (it / kStages) & 1;
          if (!warp_wait(&a_full[st], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // straight-line issue from one elected lane (no branch between the
          // MMAs of a stage)
          const uint32_t acol = tmem + kColA + st * (kTapsPS * 64);
          const uint32_t bst = sB_addr + st * (kTapsPS * kBTap);  // per tap: rows W hi then W lo
          const uint32_t acc0 = ti == 0 ? 0u : 1u;
          const bool last = ti + kTapsPS >= tg.ntaps;
          if (elect_one()) {
            if (nh == 2) {
#pragma unroll
              for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int ks = 0; ks < kKS / 8; ++ks)
                  mma_tf32_ts(dcol, acol + h * 64 + ks * 8, sdesc_kmajor_sw128(bst + h * kBTap + ks * 32), id_main,
                              (h == 0 && ks == 0) ? acc0 : 1u);
#pragma unroll
              for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int ks = 0; ks < kKS / 8; ++ks)
                  mma_tf32_ts(dcol + NC, acol + h * 64 + 32 + ks * 8, sdesc_kmajor_sw128(bst + h * kBTap + ks * 32),
                              id_corr, 1u);
            } else {
#pragma unroll
              for (int ks = 0; ks < kKS / 8; ++ks)
                mma_tf32_ts(dcol, acol + ks * 8, sdesc_kmajor_sw128(bst + ks * 32), id_main, ks == 0 ? acc0 : 1u);
#pragma unroll
              for (int ks = 0; ks < kKS / 8; ++ks)
                mma_tf32_ts(dcol + NC, acol + 32 + ks * 8, sdesc_kmajor_sw128(bst + ks * 32), id_corr, 1u);
            }
            tc_commit(&s_empty[st]);
            if (last) tc_commit(&gr_full[slot]);
          }
          __syncwarp();
        }
      }
    }
    if (elect_one()) tc_commit(final_bar);
    __syncwarp();
    mbar_wait(final_bar, 0, kWaitNs, nullptr);
  } else if (warp == 9) {
    // ---------------------------------------------------- weight loader
    uint32_t it = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
      const int64_t t = item / c.ncb;
      const int cb = (int)(item - t * c.ncb);
      const DgGeo tg = dg_geo(p, c, ps, t);
      for (int jb = 0; jb < c.nJB && ok; ++jb) {
        for (int ti = 0; ti < tg.ntaps; ti += kTapsPS, ++it) {
          const uint32_t st = it % kStages, ph = (it / kStages) & 1;
          if (!warp_wait(&s_empty[st], ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            const int nh = min(kTapsPS, tg.ntaps - ti);
            mbar_arrive_expect_tx(&a_full[st], (uint32_t)nh * c.bstage);
            for (int h = 0; h < nh; ++h) {
              const int tap = ptab[tg.tap0 + ti + h].x;
              bulk_g2s(sB + ((size_t)st * kTapsPS + h) * c.bstage,
                       wsB + ((int64_t)cb * c.nK + jb * p.T + tap) * 2 * c.NC * 32, c.bstage, &a_full[st]);
            }
          }
          __syncwarp();
        }
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
  } else {
    // ------------------------------------------- g / hsum plane loader
    // Runs up to two j-blocks ahead of the producers, independently of the
    // weight stages.
    uint32_t jit = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
      const DgGeo tg = dg_geo(p, c, ps, item / c.ncb);
      const int64_t run = (int64_t)tg.orows * p.Q;
      for (int jb = 0; jb < c.nJB; ++jb, ++jit) {
        const uint32_t js = jit & 1, jph = (jit >> 1) & 1;
        if (!warp_wait(&jempty[js], jph ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        if (c.tma) {
          // g planes of channels jb*16 .. +15 to slots 0..15, hsum planes to
          // slots 16..31, PSo floats each from the 16-byte boundary at or
          // below the first staged element (rows past the image's channels
          // are never read: their table entries are -1)
          const int xo = tg.oylo * p.Q, x0 = xo & ~3, ld = xo - x0;
          const int jl = lane % kJB, isH = lane / kJB;
          const int j = jb * kJB + jl;
          jtab[js * 2 * kJB + 2 * jl + isH] = (j < p.m && run > 0) ? (isH * kJB + jl) * c.PSo + ld : 2 * kJB * c.PSo;
          __syncwarp();
          if (lane == 0) {
            if (run > 0) {
              uint8_t *slot = sJ + (size_t)js * c.jslot;
              mbar_arrive_expect_tx(&jfull[js], (uint32_t)(2 * kJB * c.PSo * 4));
              tma_load_2d(slot, &gmap, x0, (int)(tg.n * p.m + jb * kJB), &jfull[js]);
              tma_load_2d(slot + (size_t)kJB * c.PSo * 4, &hmap, x0, (int)(tg.n * p.m + jb * kJB), &jfull[js]);
            } else {
              mbar_arrive(&jfull[js]);
            }
          }
          __syncwarp();
          continue;
        }
        // lane l: plane l of the j-block = channel jb*16 + l/2, g (l even) or hsum (l odd)
        const int j = jb * kJB + lane / 2;
        const bool have = (j < p.m) && run > 0;
        tc::BulkSpan sp{};
        uint32_t bytes = 0;
        if (have) {
          const float *src = ((lane & 1) ? hsum : grad) + (tg.n * p.m + j) * p.PQ + (int64_t)tg.oylo * p.Q;
          sp = tc::bulk_span(src, run);
          bytes = sp.bytes;
        }
        jtab[js * 2 * kJB + lane] = have ? lane * c.PSo + sp.lead : 2 * kJB * c.PSo;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, off);
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(&jfull[js], bytes);
        __syncwarp();
        if (have) bulk_g2s(sJ + (size_t)js * c.jslot + (size_t)lane * c.PSo * 4, sp.src, sp.bytes, &jfull[js]);
        __syncwarp();
      }
    }
    const uint32_t jlast = jit < 2u ? jit : 2u;
    for (uint32_t i = 0; i < jlast; ++i) {
      const uint32_t idx = jit - 1 - i;
      mbar_wait(&jfull[idx & 1], (idx >> 1) & 1, kWaitNs, nullptr);
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

PerContext<uint64_t> g_attr;

template <int NC>
int launch_dgrad(const Problem &p, DgCfg c, const float *grad, const float *x, const float *hsum,
                 const float *wsB, const DxOut &dxo, float *dx, int *status, cudaStream_t stream) {
  const int ast = once_per_context(g_attr, 1ull << (NC / 16 - 1), []() -> int {
    PC2D_CUDA_CHECK(cudaFuncSetAttribute(tc_dgrad_kernel<NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit));
    return (int)PC2D_OK;
  });
  if (ast != PC2D_OK) return ast;
  CUtensorMap gmap, hmap;
  std::memset(&gmap, 0, sizeof(gmap));
  std::memset(&hmap, 0, sizeof(hmap));
  if (c.tma && !(encode_planes_map(grad, p.PQ, (int64_t)p.n * p.m, c.PSo, kJB, &gmap) &&
                 encode_planes_map(hsum, p.PQ, (int64_t)p.n * p.m, c.PSo, kJB, &hmap)))
    c.tma = 0;  // per-plane bulk copies instead (same slot size)
  const int grid = (int)std::min<int64_t>(c.items, device_sm_count());
  timing_begin(K_DGRAD, stream);
  tc_dgrad_kernel<NC><<<grid, kThreads, dg_smem_bytes(c), stream>>>(grad, x, hsum, wsB, p, c, gmap, hmap, dxo, dx,
                                                                      status);
  timing_end(K_DGRAD, stream);
  PC2D_LAUNCH_CHECK("tc_dgrad_kernel");
  return PC2D_OK;
}

bool dg_cfg_fits(const DgCfg &c) { return dg_smem_bytes(c) <= (size_t)kSmemLimit && c.PSo * 2 * kJB < (1 << 30); }

bool dg_supported(const Problem &p) {
  if (p.NPQ <= 0 || p.m < 1 || p.HW >= ((int64_t)1 << 30) || p.PQ >= ((int64_t)1 << 30)) return false;
  if (p.s0 * p.s1 > kMaxPh || p.k0 > kMaxKs || p.k1 > kMaxKs) return false;
  return dg_cfg_fits(dg_cfg(p, dg_full_window(p)));
}

}  // namespace

bool tc_backward_supported(const Problem &p) {
  return dg_supported(p) || tc_wgrad_supported(p) || nw_wgrad_supported(p);
}

namespace {
// Workspace layout: [parameter-gradient scratch | dgrad weights]
size_t wgrad_scratch(const Problem &p, bool skip_input_grad) {
  if (nw_wgrad_supported(p)) return align_up(nw_wgrad_workspace(p), 256);
  return align_up(tc_wgrad_supported(p) ? tc_wgrad_workspace(p) : simt_backward_workspace<float>(p, skip_input_grad),
                  256);
}
}  // namespace

size_t tc_backward_workspace(const Problem &p, bool skip_input_grad) {
  size_t ws = wgrad_scratch(p, skip_input_grad);
  if (!skip_input_grad) {
    if (tc_dgcol_supported(p)) ws += align_up(tc_dgcol_workspace(p), 256);
    else if (dg_supported(p)) ws += align_up(dg_bsplit_bytes(dg_cfg(p, dg_full_window(p))), 256);
  }
  return ws;
}

int tc_backward(const Problem &p, const float *grad, const float *x, const float *pars, const float *hsum,
                double factor, bool skip_input_grad, float *dx, float *dpars, void *ws, size_t ws_bytes,
                cudaStream_t stream, const DxOut &dxo) {
  const size_t wscr = wgrad_scratch(p, skip_input_grad);
  bool dx_done = false;
  if (skip_input_grad || p.NPQ == 0) {
    if (p.NHW > 0 && dx) PC2D_CUDA_CHECK(cudaMemsetAsync(dx, 0, sizeof(float) * (size_t)p.n * dxo.CHWu, stream));
    dx_done = true;
  } else if (tc_dgcol_supported(p)) {
    // few input channels: dense GEMM over the output pixels + col2im
    NvtxRange range("dgrad");
    const int st = tc_dgcol(p, grad, x, pars, hsum, dxo, dx, reinterpret_cast<char *>(ws) + wscr, stream);
    if (st != PC2D_OK) return st;
    dx_done = true;
  } else if (dg_supported(p)) {
    NvtxRange range("dgrad");
    int *status = device_status_ptr();
    if (!status) {
      set_last_error("could not resolve the device status word");
      return PC2D_ERR_CUDA;
    }
    // only the pixels whose gradient is written are tiled (the interior, for
    // a module that pads its input), unless that geometry needs more shared
    // memory than the whole plane's
    DgCfg c = dg_cfg(p, dg_full_window(p));
    if (dxo.Hu < p.H || dxo.Wu < p.W) {
      const DgCfg ci = dg_cfg(p, DgWindow{dxo.pt, dxo.pt + dxo.Hu, dxo.pl, dxo.pl + dxo.Wu});
      if (dg_cfg_fits(ci)) c = ci;
    }
    float *wsB = reinterpret_cast<float *>(reinterpret_cast<char *>(ws) + wscr);
    tc_dg_prep_weights<<<dim3(c.nK, c.ncb, c.NC / 8), 256, 0, stream>>>(pars, p, c, wsB);
    PC2D_LAUNCH_CHECK("tc_dg_prep_weights");
    int st = PC2D_OK;
    if (c.items == 0) c.NC = 0;  // an empty interior: nothing to launch
    switch (c.NC) {
      case 0: break;
      case 16: st = launch_dgrad<16>(p, c, grad, x, hsum, wsB, dxo, dx, status, stream); break;
      case 32: st = launch_dgrad<32>(p, c, grad, x, hsum, wsB, dxo, dx, status, stream); break;
      case 48: st = launch_dgrad<48>(p, c, grad, x, hsum, wsB, dxo, dx, status, stream); break;
      case 64: st = launch_dgrad<64>(p, c, grad, x, hsum, wsB, dxo, dx, status, stream); break;
      default: set_last_error("internal: unsupported channel block %d", c.NC); return PC2D_ERR_UNSUPPORTED;
    }
    if (st != PC2D_OK) return st;
    dx_done = true;
  }
  // parameter gradients: narrow windows on the CUDA cores, else the
  // tensor-core GEMM
  const bool nw = nw_wgrad_supported(p);
  if (p.NPQ > 0 && (nw || tc_wgrad_supported(p))) {
    if (!dx_done) {
      // input gradient on the CUDA cores, then the parameter gradients
      const int st = simt_backward<float>(p, grad, x, pars, hsum, factor, false, dx, dpars, nullptr, 0, stream, dxo,
                                          /*leave_dx=*/false, /*skip_wgrad=*/true);
      if (st != PC2D_OK) return st;
    }
    NvtxRange range("wgrad");
    if (nw) return nw_wgrad(p, grad, x, pars, hsum, factor, dpars, ws, stream);
    return tc_wgrad(p, grad, x, pars, hsum, factor, dpars, ws, stream);
  }
  return simt_backward<float>(p, grad, x, pars, hsum, factor, skip_input_grad, dx, dpars, ws, wscr, stream, dxo,
                              /*leave_dx=*/dx_done);
}

}  // namespace pc2d
