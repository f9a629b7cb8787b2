// tcgen05 parameter-gradient kernel of the ParaConv2d paraboloid convolution
// (fp32 via 3xTF32 split precision) and its fixed-order reduction.
//
// Parameter gradients (reference paraconv2d.cc:186-237):
//   dh[j,k]  = 2f sum_o (g*hsum)[j,o] win_o[k]     dh0[j] = 2f sum_o (g*hsum)[j,o]
//   dp[j,k]  = 2f (sum_o g[j,o] win_o[k] - p[j,k] sum_o g[j,o])
//   dp0[j]   = 2f (-p0[j]) sum_o g[j,o]
// The two contractions are one GEMM over the output pixels o:
//   D[r, k] = sum_o A[r, o] * win_o[k],  A = [g*hsum (JM rows); g (JM rows)]
// with M = 128 rows (a block of JM <= 64 output channels), N = a range of
// NR <= 256 window elements k = (c, tap) and K = output pixels, swept in
// 32-pixel chunks of one image; the pixels are split into segments across
// CTAs.
//
// Per 32-pixel chunk:
//   - four A-producer warps (one TMEM lane = one row r) load the 32 values
//     of their row with vector loads, form g*hsum or g, accumulate the row
//     sum, split into tf32 hi + lo and tcgen05.st them into TMEM;
//   - a loader warp stages the input rows the chunk's windows read (one
//     16-byte-rounded bulk copy per channel of the window range);
//   - eight B-producer warps (one lane = one pixel of the chunk) gather the
//     flipped windows of the chunk's pixels from those rows, split them and
//     store rows k of the 128-byte-swizzled K-major B operand in shared
//     memory;
//   - the MMA thread issues Ahi*Bhi + Alo*Bhi + Ahi*Blo (N = NR) per 8
//     pixels.
// At the end of a segment the epilogue warps drain the fp32 accumulator to a
// per-segment slice of the workspace (a partial over at most 2048 pixels, so
// the tensor core's per-instruction accumulation error stays small; a longer
// segment also halves the slices the reduction reads); a second
// kernel sums the slices in a fixed order in fp64 and applies the epilogue
// above.  No floating-point atomics: the result is deterministic.
//
// Warp roles (608 threads, one CTA per SM): warps 0-3 A producers, 4-11 B
// producers, 12-15 epilogue, 16 MMA issuer and TMEM owner, 17 loader of the
// input rows the B producers gather from, 18 loader of the A rows' g and
// hsum tiles (when they are staged by tensor copies).  All waits are bounded
// as in the forward kernel.
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

constexpr int kChunk = 32;        // pixels per K chunk
constexpr int kAhead = 8;         // chunks an A producer prefetches ahead (L2)
constexpr int kStages = 3;
constexpr int kMaxSeg = 64;       // chunks per segment
constexpr int kThreads = 608;
constexpr int kBWarps = 8;
constexpr int kMinSmem = 120 * 1024;
constexpr int kSmemLimit = 227 * 1024;
constexpr uint32_t kColA = 256;   // A stages at 256 + 64 * stage

struct WgCfg {
  int nmb, JM;      // output-channel blocks, channels per block
  int nNR, NR;      // window-row ranges, rows per range (multiple of 16, <= 256)
  int cpi;          // 32-pixel chunks per image
  int64_t chunks;   // n * cpi
  int SEG;          // chunks per segment
  int64_t nseg;
  int64_t items;    // nseg * nNR * nmb
  uint32_t bstage;  // B bytes per stage (hi + lo)
  int halo;         // 1: B rows gathered from input rows staged in shared memory
  int nchm;         // channels a window-row range touches at most
  int PSw;          // staged plane stride (floats, multiple of 4)
  uint32_t hstage;  // halo bytes per stage (multiple of 1024)
  int tma;          // 1: the halo of a chunk is one 2-D tensor copy [nchm][PSw] (see tc_wgrad)
  int atma;         // 1: a chunk's g and hsum rows are two 2-D tensor copies [JM][32] (128-byte swizzled)
  int kst;          // B / halo stages in flight (3, or 2 to make room for the A tiles)
  uint32_t tbytes;  // shared bytes of those tiles: 2 stages x (g, hsum) x 8 KB, or 0
  int dqy, dqx;     // a chunk's 32 pixels as output rows and columns: 32 = dqy * Q + dqx
};

WgCfg wg_cfg(const Problem &p, int sms) {
  WgCfg c;
  c.nmb = std::max(1, ceil_div(p.m, 64));
  c.JM = ceil_div(p.m, c.nmb);
  c.nNR = std::max(1, ceil_div(p.d, 256));
  c.NR = (ceil_div(p.d, c.nNR) + 15) / 16 * 16;
  c.cpi = ceil_div(p.PQ, kChunk);
  c.chunks = (int64_t)p.n * c.cpi;
  c.dqy = kChunk / (int)std::max<int64_t>(1, p.Q);
  c.dqx = kChunk - c.dqy * (int)std::max<int64_t>(1, p.Q);
  const int64_t per = (int64_t)c.nNR * c.nmb;
  // Segment length: the one whose critical path (rounds of items per SM x
  // chunks per item, plus a per-item cost of ~2 chunks for the drain and
  // the hand-over) is shortest.
  c.SEG = kMaxSeg;
  int64_t best = -1;
  for (int seg = 4; seg <= kMaxSeg; ++seg) {
    const int64_t items = (c.chunks + seg - 1) / seg * per;
    const int64_t rounds = (items + std::max(1, sms) - 1) / std::max(1, sms);
    const int64_t cost = rounds * (seg + 2);
    if (best < 0 || cost < best) {
      best = cost;
      c.SEG = seg;
    }
  }
  c.nseg = (c.chunks + c.SEG - 1) / c.SEG;
  c.items = c.nseg * per;
  c.bstage = (uint32_t)(2 * c.NR * 128);
  c.nchm = 0;
  for (int nr = 0; nr < c.nNR; ++nr) {
    const int64_t k0 = (int64_t)nr * c.NR, k1 = std::min<int64_t>(k0 + c.NR, p.d) - 1;
    c.nchm = std::max(c.nchm, (int)(k1 / p.T - k0 / p.T + 1));
  }
  const int orow = std::min<int64_t>(p.P, (p.Q + kChunk - 2) / p.Q + 1);
  const int rows = (orow - 1) * p.s0 + (p.k0 - 1) * p.dl0 + 1;
  c.PSw = (int)(((int64_t)rows * p.W + 8 + 3) / 4 * 4);
  c.hstage = (uint32_t)align_up((size_t)c.nchm * c.PSw * 4, 1024);
  c.halo = c.nchm <= 64 ? 1 : 0;
  // One 2-D tensor copy per chunk needs the channel plane stride to be a
  // multiple of 16 bytes; its box is the staged plane (PSw floats from the
  // 16-byte boundary at or below the chunk's first element), at most 256.
  c.tma = (p.HW % 4 == 0 && c.PSw <= 256 && (int64_t)p.n * p.C < ((int64_t)1 << 31)) ? 1 : 0;
  c.kst = kStages;
  const size_t need = 1024 + (size_t)kStages * (c.bstage + c.hstage) + (size_t)kStages * (64 + 256 + 32) * 4 + 28 * 8 + 64;
  if (need > (size_t)kSmemLimit) c.halo = 0;  // gather from global memory instead
  if (!c.halo) {
    c.hstage = 0;
    c.tma = 0;
  }
  // A rows as tensor copies when the rows of g and hsum are 16-byte strided
  // and the tiles fit next to the B and halo stages; else each A producer
  // loads its own row
  c.atma = 0;
  c.tbytes = 0;
  // (with the halo path, two B and halo stages when three leave no room)
  if (p.PQ % 4 == 0 && p.PQ >= kChunk && (int64_t)p.n * p.m < ((int64_t)1 << 31)) {
    for (int kst = kStages; kst >= (c.halo ? 2 : kStages); --kst) {
      const size_t need2 = 1024 + (size_t)kst * (c.bstage + c.hstage) + (size_t)kst * (64 + 256 + 32) * 4 + 28 * 8 + 64;
      if (need2 + 2 * 2 * 8192 <= (size_t)kSmemLimit) {
        c.atma = 1;
        c.tbytes = 2 * 2 * 8192;
        c.kst = kst;
        break;
      }
    }
  }
  return c;
}

inline size_t wg_smem_bytes(const WgCfg &c) {
  size_t s = 1024 + (size_t)c.kst * (c.bstage + c.hstage) + c.tbytes + (size_t)c.kst * 64 * 4 +
             (size_t)c.kst * (256 + 32) * 4 + 28 * 8 + 64;
  return std::max<size_t>(s, kMinSmem);
}

// Halo geometry of one 32-pixel chunk: image, first input row, input rows.
struct ChunkGeo {
  int64_t n;
  int pq0, npx, ir0, rows;
};

// Chunk gc = image n, chunk ci of that image.  The roles walk the chunks of
// a segment in order and step (n, ci) instead of dividing gc per chunk.
struct ChunkPos {
  int64_t n;
  int ci;
};
__device__ __forceinline__ ChunkPos chunk_pos(const WgCfg &c, int64_t gc) {
  ChunkPos t;
  t.n = gc / c.cpi;
  t.ci = (int)(gc - t.n * c.cpi);
  return t;
}
__device__ __forceinline__ void chunk_next(const WgCfg &c, ChunkPos &t) {
  if (++t.ci == c.cpi) {
    t.ci = 0;
    ++t.n;
  }
}

// Output pixel pq0 + lane of the chunk at t as (row qy, column qx); stepped
// with the chunk: +32 pixels = +dqy rows, +dqx columns (one carry at most,
// as dqx < Q), or back to pixel lane of the next image.
struct LanePix {
  int qy, qx;
};
__device__ __forceinline__ LanePix lane_pix(const Problem &p, const ChunkPos &t, int lane) {
  LanePix v;
  const int q = t.ci * kChunk + lane;
  v.qy = q / (int)p.Q;
  v.qx = q - v.qy * (int)p.Q;
  return v;
}
__device__ __forceinline__ void chunk_next(const Problem &p, const WgCfg &c, ChunkPos &t, LanePix &v, int lane) {
  chunk_next(c, t);
  if (t.ci == 0) {
    v = lane_pix(p, t, lane);
  } else {
    v.qy += c.dqy;
    v.qx += c.dqx;
    if (v.qx >= (int)p.Q) {
      v.qx -= (int)p.Q;
      ++v.qy;
    }
  }
}

__device__ __forceinline__ ChunkGeo chunk_geo(const Problem &p, const ChunkPos &t) {
  ChunkGeo g;
  g.n = t.n;
  g.pq0 = t.ci * kChunk;
  g.npx = min(kChunk, (int)p.PQ - g.pq0);
  const int oya = g.pq0 / p.Q, oyb = (g.pq0 + g.npx - 1) / p.Q;
  g.ir0 = oya * p.s0;
  g.rows = (oyb - oya) * p.s0 + (p.k0 - 1) * p.dl0 + 1;
  return g;
}
inline size_t wg_part_bytes(const WgCfg &c) { return align_up((size_t)c.items * 128 * c.NR * 4, 256); }
inline size_t wg_sums_bytes(const WgCfg &c) { return align_up((size_t)c.items * 128 * 4, 256); }

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <bool ATMA, int KST>
__global__ void __launch_bounds__(kThreads, 1)
tc_wgrad_kernel(const float *__restrict__ grad, const float *__restrict__ x, const float *__restrict__ hsum,
                Problem p, WgCfg c, const __grid_constant__ CUtensorMap xmap,
                const __grid_constant__ CUtensorMap gmap, const __grid_constant__ CUtensorMap hmap,
                float *__restrict__ part, float *__restrict__ sums, int *status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  uint8_t *sB = base;                                                  // KST x bstage
  uint8_t *sH = base + (size_t)KST * c.bstage;                     // KST x hstage
  uint8_t *sT = sH + (size_t)KST * c.hstage;                      // 2 x [g tile 8 KB | hsum tile 8 KB]
  int *lead = reinterpret_cast<int *>(sT + c.tbytes);                 // [KST][64]
  int *roffs = lead + KST * 64;                                    // [KST][8 warps][32 slots]
  int *pofs = roffs + KST * 256;  // [KST][32]: pixel offsets in the staged rows (-1: past the chunk)
  uint64_t *bars = reinterpret_cast<uint64_t *>(pofs + KST * 32);
  uint64_t *a_full = bars, *a_empty = bars + 3, *b_full = bars + 6, *b_empty = bars + 9;
  uint64_t *d_full = bars + 12, *d_empty = bars + 13, *final_bar = bars + 14;
  uint64_t *h_full = bars + 15, *h_empty = bars + 18;
  uint64_t *t_full = bars + 21, *t_empty = bars + 23;  // A tiles landed / read (128 A threads)
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 25);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

  if (threadIdx.x == 0) {
    for (int i = 0; i < KST; ++i) {
      mbar_init(&a_full[i], 128);
      mbar_init(&a_empty[i], 1);
      mbar_init(&b_full[i], kBWarps);
      mbar_init(&b_empty[i], 1);
      mbar_init(&h_full[i], 1);
      mbar_init(&h_empty[i], kBWarps);
    }
    mbar_init(d_full, 1);
    mbar_init(d_empty, 128);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&t_full[i], 1);
      mbar_init(&t_empty[i], 128);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 16) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int per = c.nNR * c.nmb;
  bool ok = true;
  // the reduction launched after this grid waits for it to complete; let it
  // be scheduled as this grid's CTAs finish
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp < 4) {
    // -------------------------------------------------------- A producers
    const int r = warp * 32 + lane;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t sT_addr = smem_u32(sT);
    const bool vec_ok = ((reinterpret_cast<uintptr_t>(grad) | reinterpret_cast<uintptr_t>(hsum)) & 15) == 0 &&
                        (p.PQ % 4) == 0;
    uint32_t it = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
      const int64_t seg = item / per;
      const int mb = (int)((item - seg * per) % c.nmb);
      const int w = r < c.JM ? 0 : 1;
      const int j = mb * c.JM + (r - w * c.JM);
      const bool rvalid = r < 2 * c.JM && j < p.m;
      float rowsum = 0.f;
      const int64_t g0 = seg * c.SEG, g1 = std::min<int64_t>(c.chunks, g0 + c.SEG);
      ChunkPos cp = chunk_pos(c, g0), ca = chunk_pos(c, g0 + kAhead);
      for (int64_t gc = g0; gc < g1; ++gc, ++it, chunk_next(c, cp), chunk_next(c, ca)) {
        const int64_t n = cp.n;
        const int pq0 = cp.ci * kChunk;
        const int npx = min(kChunk, (int)p.PQ - pq0);
        // this row kAhead chunks ahead: start bringing it into L2 now (one
        // thread holds one 128-byte row of a chunk)
        if (rvalid && gc + kAhead < g1) {
          const int64_t offa = (ca.n * p.m + j) * p.PQ + ca.ci * kChunk;
          prefetch_l2(grad + offa);
          if (w == 0) prefetch_l2(hsum + offa);
        }
        float v[kChunk];
        if (ATMA) {
          // this row of the chunk's g (and hsum) tile: tile row j - mb*JM,
          // 16-byte chunk q at position q ^ (row % 8)
          const uint32_t ts = it & 1, tph = (it >> 1) & 1;
          if (!warp_wait(&t_full[ts], tph, abort_flag)) {
            ok = false;
            break;
          }
          const int tr = rvalid ? r - w * c.JM : 0;
          const uint32_t gt = sT_addr + ts * 16384u + (uint32_t)tr * 128u;
#pragma unroll
          for (int q = 0; q < kChunk / 4; ++q) {
            const uint32_t cq = (uint32_t)((q ^ (tr & 7)) << 4);
            const int4 g4 = lds_v4s32(gt + cq);
            float4 a4 = make_float4(__int_as_float(g4.x), __int_as_float(g4.y), __int_as_float(g4.z),
                                    __int_as_float(g4.w));
            if (w == 0) {
              const int4 h4 = lds_v4s32(gt + 8192u + cq);
              a4.x *= __int_as_float(h4.x);
              a4.y *= __int_as_float(h4.y);
              a4.z *= __int_as_float(h4.z);
              a4.w *= __int_as_float(h4.w);
            }
            v[4 * q] = rvalid ? a4.x : 0.f;
            v[4 * q + 1] = rvalid ? a4.y : 0.f;
            v[4 * q + 2] = rvalid ? a4.z : 0.f;
            v[4 * q + 3] = rvalid ? a4.w : 0.f;
          }
        } else if (rvalid) {
          const int64_t off = (n * p.m + j) * p.PQ + pq0;
          if (vec_ok && npx == kChunk) {
            const float4 *gp = reinterpret_cast<const float4 *>(grad + off);
#pragma unroll
            for (int q = 0; q < kChunk / 4; ++q) {
              const float4 t4 = __ldg(gp + q);
              v[4 * q] = t4.x;
              v[4 * q + 1] = t4.y;
              v[4 * q + 2] = t4.z;
              v[4 * q + 3] = t4.w;
            }
            if (w == 0) {
              const float4 *hp = reinterpret_cast<const float4 *>(hsum + off);
#pragma unroll
              for (int q = 0; q < kChunk / 4; ++q) {
                const float4 t4 = __ldg(hp + q);
                v[4 * q] *= t4.x;
                v[4 * q + 1] *= t4.y;
                v[4 * q + 2] *= t4.z;
                v[4 * q + 3] *= t4.w;
              }
            }
          } else {
#pragma unroll
            for (int q = 0; q < kChunk; ++q) {
              float a = 0.f;
              if (q < npx) {
                a = __ldg(grad + off + q);
                if (w == 0) a *= __ldg(hsum + off + q);
              }
              v[q] = a;
            }
          }
        } else {
#pragma unroll
          for (int q = 0; q < kChunk; ++q) v[q] = 0.f;
        }
        uint32_t hi[kChunk], lo[kChunk];
#pragma unroll
        for (int q = 0; q < kChunk; ++q) {
          rowsum += v[q];
          hi[q] = tf32_hi_bits(v[q]);
          lo[q] = __float_as_uint(v[q] - __uint_as_float(hi[q]));
        }
        const uint32_t st = it % KST, ph = (it / KST) & 1;
        if (!warp_wait(&a_empty[st], ph ^ 1, abort_flag)) {
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
        // the tile slot is free once the values read from it have been
        // stored (an arrive right after the shared loads could overtake them)
        if (ATMA) mbar_arrive(&t_empty[it & 1]);
      }
      sums[item * 128 + r] = rowsum;
    }
  } else if (warp < 4 + kBWarps) {
    // -------------------------------------------------------- B producers
    // Warp bw builds rows kl = bw + 8*i of each chunk's B tile.  With c.halo
    // the window values come from the input rows the loader warp staged in
    // shared memory (this warp's row offsets in roffs[stage][bw][i]);
    // otherwise they are gathered from global memory.
    const int bw = warp - 4;
    const int nrows = (c.NR - bw + kBWarps - 1) / kBWarps;  // <= 32
    const uint32_t cpos = (uint32_t)(lane & 3) * 4;
    uint32_t it = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
      const int64_t seg = item / per;
      const int nr = (int)((item - seg * per) / c.nmb);
      int myoff = -1;
      if (!c.halo) {
        const int kl = bw + kBWarps * lane;
        const int64_t k = (int64_t)nr * c.NR + kl;
        if (kl < c.NR && k < p.d) {
          const int ch = (int)(k / p.T), tap = (int)(k - (int64_t)ch * p.T);
          myoff = ch * (int)p.HW + tap_row(p, tap) * p.W + tap_col(p, tap);
        }
      }
      const int64_t g0 = seg * c.SEG, g1 = std::min<int64_t>(c.chunks, g0 + c.SEG);
      ChunkPos cp = chunk_pos(c, g0);
      for (int64_t gc = g0; gc < g1; ++gc, ++it, chunk_next(c, cp)) {
        const uint32_t st = it % KST, ph = (it / KST) & 1;
        if (c.halo && !warp_wait(&h_full[st], ph, abort_flag)) {
          ok = false;
          break;
        }
        if (!warp_wait(&b_empty[st], ph ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t stg_a = smem_u32(sB + (size_t)st * c.bstage), lo_off = (uint32_t)c.NR * 128;
        if (c.halo) {
          // Lane = (row slot rr = lane / 8, 4-pixel group g = lane % 8): it
          // writes the 16-byte chunk g of rows kl = bw + 8*(4*i + rr) (hi and
          // lo), i.e. pixels 4g .. 4g+3 of the chunk, gathered from the input
          // rows the loader staged.  kl % 8 == bw, so the swizzled position
          // of chunk g is g ^ bw for every row of this warp.
          const int g = lane & 7, rr = lane >> 3;
          const uint32_t halo = smem_u32(sH + (size_t)st * c.hstage);
          const int *ro = roffs + st * 256 + bw * 32;
          // offsets of pixels 4g .. 4g+3 in the staged rows (the loader's)
          const int4 po4 = lds_v4s32(smem_u32(pofs + st * 32 + 4 * g));
          const int poff[4] = {po4.x, po4.y, po4.z, po4.w};
          bool pv[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) pv[j] = poff[j] >= 0;
          const uint32_t cbyte = (uint32_t)((g ^ bw) << 4);
          int o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = (4 * i + rr < nrows) ? ro[4 * i + rr] : -1;
          float v[8][4];
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j)
              v[i][j] = (pv[j] && o[i] >= 0) ? lds_f32(halo + 4u * (uint32_t)(o[i] + poff[j])) : 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (4 * i + rr < nrows) {
              const uint32_t kl = (uint32_t)(bw + kBWarps * (4 * i + rr));
              uint32_t h[4], l[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                h[j] = tf32_hi_bits(v[i][j]);
                l[j] = __float_as_uint(v[i][j] - __uint_as_float(h[j]));
              }
              const uint32_t a = stg_a + kl * 128 + cbyte;
              sts_v4u32(a, h[0], h[1], h[2], h[3]);
              sts_v4u32(a + lo_off, l[0], l[1], l[2], l[3]);
            }
          }
        } else {
          // lane = pixel; row kl = bw + 8*i gathered from global memory (lane
          // i holds the input offset of row bw + 8*i of the window range)
          const ChunkGeo cg = chunk_geo(p, cp);
          const int pq = cg.pq0 + lane;
          const bool pvalid = lane < cg.npx;
          const int oy = pq / p.Q, ox = pq - oy * p.Q;
          const int64_t pbase = cg.n * p.CHW + (int64_t)oy * p.s0 * p.W + (int64_t)ox * p.s1;
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int o = __shfl_sync(0xffffffffu, myoff, i);
            v[i] = (i < nrows && pvalid && o >= 0) ? __ldg(x + pbase + o) : 0.f;
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (i < nrows) {
              const uint32_t kl = (uint32_t)(bw + kBWarps * i);
              const uint32_t hb = tf32_hi_bits(v[i]);
              const uint32_t off = kl * 128 + ((((uint32_t)lane >> 2) ^ (kl & 7)) << 4) + cpos;
              sts_u32(stg_a + off, hb);
              sts_u32(stg_a + lo_off + off, __float_as_uint(v[i] - __uint_as_float(hb)));
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&b_full[st]);
          if (c.halo) mbar_arrive(&h_empty[st]);
        }
      }
    }
  } else if (warp < 16) {
    // ----------------------------------------------------------- epilogue
    const int q = warp % 4;
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    uint32_t di = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x, ++di) {
      if (!warp_wait(d_full, di & 1, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float *dst = part + ((size_t)item * 128 + r) * c.NR;
      for (int cc = 0; cc < c.NR; cc += 32) {
        uint32_t vv[32];
        tmem_ld32_nowait(tmem + lane_off + cc, vv);
        tmem_ld_wait_tie(vv);
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4)
          if (cc + 4 * q4 < c.NR)
            reinterpret_cast<float4 *>(dst + cc)[q4] =
                make_float4(__uint_as_float(vv[4 * q4]), __uint_as_float(vv[4 * q4 + 1]),
                            __uint_as_float(vv[4 * q4 + 2]), __uint_as_float(vv[4 * q4 + 3]));
      }
      tc_fence_before();
      mbar_arrive(d_empty);
    }
  } else if (warp == 17) {
    // -------------------------------------------------------------- loader
    // Stages, per chunk, the input rows its windows read for the channels of
    // the item's window range (one 16-byte-rounded bulk copy per channel, or
    // one tensor copy), and the offset of every window row of the range
    // inside that stage.
    if (c.halo) {
      uint32_t it = 0;
      for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
        const int64_t seg = item / per;
        const int nr = (int)((item - seg * per) / c.nmb);
        const int64_t kbase = (int64_t)nr * c.NR;
        const int clo = (int)(kbase / p.T);
        // (channel - clo, tap offset) of the window rows this lane writes:
        // table entry e*32 + lane = slot `lane` of B-producer warp e = row
        // e + 8*lane (consecutive lanes store consecutive words)
        int rc[8], rt[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int kl = e + kBWarps * lane;
          const int64_t k = kbase + kl;
          rc[e] = -1;
          rt[e] = 0;
          if (kl < c.NR && k < p.d) {
            const int ch = (int)(k / p.T), tap = (int)(k - (int64_t)ch * p.T);
            rc[e] = ch - clo;
            rt[e] = tap_row(p, tap) * p.W + tap_col(p, tap);
          }
        }
        // row offsets in a stage without the chunk's lead (a row past the
        // range stays negative whatever the lead)
        int rb[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) rb[e] = rc[e] >= 0 ? rc[e] * c.PSw + rt[e] : -(1 << 30);
        const int nch = (int)(std::min<int64_t>(kbase + c.NR, p.d) - 1) / p.T - clo + 1;
        const int64_t g0 = seg * c.SEG, g1 = std::min<int64_t>(c.chunks, g0 + c.SEG);
        ChunkPos cp = chunk_pos(c, g0);
        LanePix lp = lane_pix(p, cp, lane);
        for (int64_t gc = g0; gc < g1; ++gc, ++it, chunk_next(p, c, cp, lp, lane)) {
          ChunkGeo cg;
          cg.n = cp.n;
          cg.pq0 = cp.ci * kChunk;
          cg.npx = min(kChunk, (int)p.PQ - cg.pq0);
          const int oya = __shfl_sync(0xffffffffu, lp.qy, 0), oyb = __shfl_sync(0xffffffffu, lp.qy, cg.npx - 1);
          cg.ir0 = oya * p.s0;
          cg.rows = (oyb - oya) * p.s0 + (p.k0 - 1) * p.dl0 + 1;
          const uint32_t st = it % KST, ph = (it / KST) & 1;
          if (!warp_wait(&h_empty[st], ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          // lane = pixel of the chunk: its offset from the first staged input
          // row (published with the row offsets below)
          pofs[st * 32 + lane] = lane < cg.npx ? (lp.qy * p.s0 - cg.ir0) * p.W + lp.qx * p.s1 : -1;
          uint8_t *hb = sH + (size_t)st * c.hstage;
          if (c.tma) {
            // one tensor copy: channels clo .. clo+nchm-1 of image n, each
            // from the 16-byte boundary at or below the chunk's first input
            // element (zero past the end of the tensor)
            const int xo = cg.ir0 * p.W, x0 = xo & ~3, ld = xo - x0;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int v = rb[e] + ld;
              roffs[st * 256 + 32 * e + lane] = v >= 0 ? v : -1;
            }
            __syncwarp();
            if (lane == 0) {
              mbar_arrive_expect_tx(&h_full[st], (uint32_t)(c.nchm * c.PSw * 4));
              tma_load_2d(hb, &xmap, x0, (int)(cg.n * p.C + clo), &h_full[st]);
            }
            __syncwarp();
            continue;
          }
          const float *xrow = x + cg.n * p.CHW + (int64_t)cg.ir0 * p.W;
          const int64_t run = (int64_t)cg.rows * p.W;
          uint32_t bytes = 0;
          for (int ci = lane; ci < nch; ci += 32) {
            const tc::BulkSpan sp = tc::bulk_span(xrow + (int64_t)(clo + ci) * p.HW, run);
            lead[st * 64 + ci] = sp.lead;
            bytes += sp.bytes;
          }
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, off);
          __syncwarp();
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            // (entries past NR stay -1, read as zero rows)
            roffs[st * 256 + 32 * e + lane] = rc[e] >= 0 ? rc[e] * c.PSw + lead[st * 64 + rc[e]] + rt[e] : -1;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive_expect_tx(&h_full[st], bytes);
          __syncwarp();
          for (int ci = lane; ci < nch; ci += 32) {
            const tc::BulkSpan sp = tc::bulk_span(xrow + (int64_t)(clo + ci) * p.HW, run);
            bulk_g2s(hb + (size_t)ci * c.PSw * 4, sp.src, sp.bytes, &h_full[st]);
          }
          __syncwarp();
        }
      }
      // Drain: the copies issued last have landed before the CTA exits.
      const uint32_t last = it < (uint32_t)KST ? it : (uint32_t)KST;
      for (uint32_t i = 0; i < last; ++i) {
        const uint32_t idx = it - 1 - i;
        mbar_wait(&h_full[idx % KST], (idx / KST) & 1, kWaitNs, nullptr);
      }
    }
  } else if (warp == 18) {
    // ------------------------------------------------------- A tile loader
    // Per chunk, rows mb*JM .. +JM-1 of image n's g and hsum, pixels
    // pq0 .. +31 (zero past the end of a row), into one of two tile slots.
    // A warp of its own, so that these copies and the halo copies are
    // issued side by side.
    if (ATMA) {
      uint32_t it = 0;
      for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x) {
        const int64_t seg = item / per;
        const int mb = (int)((item - seg * per) % c.nmb);
        const int64_t g0 = seg * c.SEG, g1 = std::min<int64_t>(c.chunks, g0 + c.SEG);
        ChunkPos cp = chunk_pos(c, g0);
        for (int64_t gc = g0; gc < g1; ++gc, ++it, chunk_next(c, cp)) {
          const uint32_t ts = it & 1, tph = (it >> 1) & 1;
          if (!warp_wait(&t_empty[ts], tph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            const int64_t n = cp.n;
            const int pq0 = cp.ci * kChunk;
            uint8_t *tb = sT + (size_t)ts * 16384;
            const int ty = (int)(n * p.m + mb * c.JM);
            mbar_arrive_expect_tx(&t_full[ts], (uint32_t)(2 * c.JM * 128));
            tma_load_2d(tb, &gmap, pq0, ty, &t_full[ts]);
            tma_load_2d(tb + 8192, &hmap, pq0, ty, &t_full[ts]);
          }
          __syncwarp();
        }
      }
      // Drain: the copies issued last have landed before the CTA exits.
      const uint32_t tlast = it < 2u ? it : 2u;
      for (uint32_t i = 0; i < tlast; ++i) {
        const uint32_t idx = it - 1 - i;
        mbar_wait(&t_full[idx & 1], (idx >> 1) & 1, kWaitNs, nullptr);
      }
    }
  } else {
    // ---------------------------------------------------------------- MMA
    const uint32_t idesc = idesc_tf32(128, c.NR);
    const uint32_t sB_addr = smem_u32(sB);
    uint32_t it = 0, di = 0;
    for (int64_t item = blockIdx.x; item < c.items && ok; item += gridDim.x, ++di) {
      if (!warp_wait(d_empty, (di & 1) ^ 1, abort_flag)) {
        ok = false;
        break;
      }
      const int64_t seg = item / per;
      const int64_t g0 = seg * c.SEG, g1 = std::min<int64_t>(c.chunks, g0 + c.SEG);
      for (int64_t gc = g0; gc < g1; ++gc, ++it) {
        const uint32_t st = it % KST, ph = (it / KST) & 1;
        if (!warp_wait(&a_full[st], ph, abort_flag) || !warp_wait(&b_full[st], ph, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // straight-line issue from one elected lane, operands formed outside
        const uint32_t ahi = tmem + kColA + st * 64, alo = ahi + 32;
        const uint32_t bhi0 = sB_addr + st * c.bstage, blo_off = c.NR * 128;
        const uint32_t acc0 = gc == g0 ? 0u : 1u;
        if (elect_one()) {
#pragma unroll
          for (int ks = 0; ks < kChunk / 8; ++ks) {
            const uint32_t bhi = bhi0 + ks * 32;
            const uint32_t blo = bhi + blo_off;
            mma_tf32_ts(tmem, ahi + ks * 8, sdesc_kmajor_sw128(bhi), idesc, ks == 0 ? acc0 : 1u);
            mma_tf32_ts(tmem, alo + ks * 8, sdesc_kmajor_sw128(bhi), idesc, 1u);
            mma_tf32_ts(tmem, ahi + ks * 8, sdesc_kmajor_sw128(blo), idesc, 1u);
          }
          tc_commit(&a_empty[st]);
          tc_commit(&b_empty[st]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (elect_one()) tc_commit(d_full);
      __syncwarp();
    }
    if (elect_one()) tc_commit(final_bar);
    __syncwarp();
    mbar_wait(final_bar, 0, kWaitNs, nullptr);
  }

  if (!ok) {
    if (lane == 0) record_device_error(status, PC2D_ERR_TIMEOUT);
    *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 16) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  // This grid may have started while the input-gradient kernel before it
  // was still running (programmatic launch).  It ends only after that kernel
  // has completed and its writes are visible, so that the work after this
  // one on the stream (the reduction, then the caller's use of dx) never
  // overtakes it.  A no-op after an ordinary launch.
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Fixed-order fp64 reduction of the per-segment partials and the parameter
// gradient epilogue:  dh = 2f dH, dp = 2f (dP - p SG), dh0 = 2f S1,
// dp0 = -2f p0 SG.  Grid (ceil(d/32), m), 32 * fq threads: thread (q, kx)
// sums the segments s = q, q+fq, ... of window element 32*blockIdx.x + kx
// (eight segments' loads in flight, added in segment order), and the fq
// partials are added in the order q = 0..fq-1, so the result does not depend
// on timing.  The host picks the largest fq (<= 16) whose grid is resident in
// one wave: the sum is a chain of dependent loads per thread, so its length
// (segments / fq / 8 load latencies) sets the time.
constexpr int kFinK = 32, kFinQ = 16;
__global__ void __launch_bounds__(kFinK * kFinQ, 2)
tc_wgrad_finalize(const float *__restrict__ part, const float *__restrict__ sums, const float *__restrict__ pars,
                  Problem p, WgCfg c, int fq, double f2, float *__restrict__ dpars) {
  __shared__ double s_sums[2];
  __shared__ double s_part[2][kFinQ][kFinK];
  // launched as a programmatic dependent of the parameter-gradient kernel:
  // its partials are complete and visible only after this wait
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // a programmatic dependent of this grid (the data-parallel peer sum) may
  // start now: it waits for this grid's completion before it reads anything
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int j = blockIdx.y;
  const int kx = threadIdx.x % kFinK, q = threadIdx.x / kFinK;
  const int64_t k = (int64_t)blockIdx.x * kFinK + kx;
  const int mb = j / c.JM, jl = j - mb * c.JM;
  const int r1 = jl, r2 = c.JM + jl;
  const int per = c.nNR * c.nmb;
  if (threadIdx.x < 32) {
    double a = 0.0, b = 0.0;
    // loads of four segments first, then the adds in segment order
    for (int64_t s0 = threadIdx.x; s0 < c.nseg; s0 += 4 * 32) {
      float va[4], vb[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t s = s0 + 32 * u;
        const int64_t item = s * per + mb;  // nr = 0 slice carries the row sums
        va[u] = s < c.nseg ? sums[item * 128 + r1] : 0.f;
        vb[u] = s < c.nseg ? sums[item * 128 + r2] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (s0 + 32 * u < c.nseg) {
          a += (double)va[u];
          b += (double)vb[u];
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      a += __shfl_down_sync(0xffffffffu, a, off);
      b += __shfl_down_sync(0xffffffffu, b, off);
    }
    if (threadIdx.x == 0) {
      s_sums[0] = a;
      s_sums[1] = b;
    }
  }
  const int64_t d = p.d;
  double ah = 0.0, ap = 0.0;
  if (k < d) {
    const int nr = (int)(k / c.NR);
    const int kl = (int)(k - (int64_t)nr * c.NR);
    // consecutive segments of one element are this far apart (floats)
    const int64_t sstride = (int64_t)c.nNR * c.nmb * 128 * c.NR;
    const float *sh = part + ((int64_t)nr * c.nmb + mb) * 128 * c.NR + (int64_t)r1 * c.NR + kl;
    const float *sp = sh + (int64_t)(r2 - r1) * c.NR;
    for (int64_t s0 = q; s0 < c.nseg; s0 += 8 * fq) {
      float vh[8], vp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t s = s0 + (int64_t)fq * u;
        vh[u] = s < c.nseg ? sh[s * sstride] : 0.f;
        vp[u] = s < c.nseg ? sp[s * sstride] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (s0 + (int64_t)fq * u < c.nseg) {
          ah += (double)vh[u];
          ap += (double)vp[u];
        }
      }
    }
  }
  s_part[0][q][kx] = ah;
  s_part[1][q][kx] = ap;
  __syncthreads();
  const double s1 = s_sums[0], sg = s_sums[1];
  const int m = p.m;
  const float *pp = pars + m + (int64_t)m * d;
  const float *p0 = pp + (int64_t)m * d;
  float *dh0 = dpars, *dh = dpars + m, *dpp = dh + (int64_t)m * d, *dp0 = dpp + (int64_t)m * d;
  if (q == 0 && k < d) {
    double th = s_part[0][0][kx], tp = s_part[1][0][kx];
    for (int qq = 1; qq < fq; ++qq) {
      th += s_part[0][qq][kx];
      tp += s_part[1][qq][kx];
    }
    const int64_t wi = (int64_t)j * d + k;
    dh[wi] = (float)(f2 * th);
    dpp[wi] = (float)(f2 * (tp - (double)pp[wi] * sg));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    dh0[j] = (float)(f2 * s1);
    dp0[j] = (float)(f2 * (-(double)p0[j]) * sg);
  }
}

PerContext<uint64_t> g_attr;

}  // namespace

bool tc_wgrad_supported(const Problem &p) {
  if (p.NPQ <= 0 || p.m < 1 || p.CHW >= ((int64_t)1 << 31) || p.PQ >= ((int64_t)1 << 30)) return false;
  const WgCfg c = wg_cfg(p, device_sm_count());
  return wg_smem_bytes(c) <= (size_t)kSmemLimit && c.NR <= 256 && 2 * c.JM <= 128;
}

size_t tc_wgrad_workspace(const Problem &p) {
  const WgCfg c = wg_cfg(p, device_sm_count());
  return wg_part_bytes(c) + wg_sums_bytes(c);
}

int tc_wgrad(const Problem &p, const float *grad, const float *x, const float *pars, const float *hsum, double factor,
             float *dpars, void *ws, cudaStream_t stream) {
  WgCfg c = wg_cfg(p, device_sm_count());
  CUtensorMap xmap;
  std::memset(&xmap, 0, sizeof(xmap));
  if (c.tma && !encode_planes_map(x, p.HW, (int64_t)p.n * p.C, c.PSw, c.nchm, &xmap))
    c.tma = 0;  // per-channel bulk copies instead (same layout)
  CUtensorMap gmap, hmap;
  std::memset(&gmap, 0, sizeof(gmap));
  std::memset(&hmap, 0, sizeof(hmap));
  if (c.atma && !(encode_rows_map_sw128(grad, p.PQ, (int64_t)p.n * p.m, c.JM, &gmap) &&
                  encode_rows_map_sw128(hsum, p.PQ, (int64_t)p.n * p.m, c.JM, &hmap))) {
    c.atma = 0;  // each A producer loads its own row instead
    c.tbytes = 0;
    c.kst = kStages;
  }
  int *status = device_status_ptr();
  if (!status) {
    set_last_error("could not resolve the device status word");
    return PC2D_ERR_CUDA;
  }
  float *part = reinterpret_cast<float *>(ws);
  float *sums = reinterpret_cast<float *>(reinterpret_cast<char *>(ws) + wg_part_bytes(c));
  const int ast = once_per_context(g_attr, 1, []() -> int {
    PC2D_CUDA_CHECK(
        cudaFuncSetAttribute(tc_wgrad_kernel<false, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit));
    PC2D_CUDA_CHECK(
        cudaFuncSetAttribute(tc_wgrad_kernel<true, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit));
    PC2D_CUDA_CHECK(
        cudaFuncSetAttribute(tc_wgrad_kernel<true, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit));
    return (int)PC2D_OK;
  });
  if (ast != PC2D_OK) return ast;
  const int grid = (int)std::min<int64_t>(c.items, device_sm_count());
  timing_begin(K_WGRAD, stream);
  // Programmatic dependent launch: when the input-gradient kernel precedes
  // this one on the stream, this grid may start on the SMs it has left (it
  // reads none of that kernel's outputs, and their workspace regions are
  // disjoint; everything earlier on the stream has completed before that
  // kernel's own launch), and waits for it to complete before it ends
  // (griddepcontrol.wait at the end of the kernel).  After any other kernel
  // it starts as usual.
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = wg_smem_bytes(c);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (c.atma && c.kst == 2)
      PC2D_CUDA_CHECK(
          cudaLaunchKernelEx(&cfg, tc_wgrad_kernel<true, 2>, grad, x, hsum, p, c, xmap, gmap, hmap, part, sums, status));
    else if (c.atma)
      PC2D_CUDA_CHECK(
          cudaLaunchKernelEx(&cfg, tc_wgrad_kernel<true, 3>, grad, x, hsum, p, c, xmap, gmap, hmap, part, sums, status));
    else
      PC2D_CUDA_CHECK(cudaLaunchKernelEx(&cfg, tc_wgrad_kernel<false, 3>, grad, x, hsum, p, c, xmap, gmap, hmap, part,
                                         sums, status));
  }
  timing_end(K_WGRAD, stream);
  PC2D_LAUNCH_CHECK("tc_wgrad_kernel");
  return tc_wgrad_reduce(p, part, sums, pars, factor, dpars, c.nseg, c.nNR, c.nmb, c.JM, c.NR, stream);
}

int tc_wgrad_reduce(const Problem &p, const float *part, const float *sums, const float *pars, double factor,
                    float *dpars, int64_t nseg, int nNR, int nmb, int JM, int NR, cudaStream_t stream) {
  WgCfg c;
  std::memset(&c, 0, sizeof(c));
  c.nseg = nseg;
  c.nNR = nNR;
  c.nmb = nmb;
  c.JM = JM;
  c.NR = NR;
  const dim3 fgrid(ceil_div(p.d, kFinK), p.m);
  int fq = kFinQ;
  while (fq > 2 && (int64_t)fgrid.x * fgrid.y * kFinK * fq > (int64_t)device_sm_count() * 1792) fq /= 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = fgrid;
  cfg.blockDim = dim3(kFinK * fq);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PC2D_CUDA_CHECK(cudaLaunchKernelEx(&cfg, tc_wgrad_finalize, part, sums, pars, p, c, fq, 2.0 * (double)(float)factor,
                                     dpars));
  PC2D_LAUNCH_CHECK("tc_wgrad_finalize");
  return PC2D_OK;
}

}  // namespace pc2d
