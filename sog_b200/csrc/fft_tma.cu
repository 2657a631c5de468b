// Column FFT passes of fp64 spectra along 256- and 512-point axes with TMA
// tile movement (the y passes of the mesh pipeline, forward and inverse).
//
// The spectrum is viewed as a 2-D array of doubles, rows = [outer][n] and
// 2*inner doubles per row.  A tile is 8 consecutive columns (128 bytes of a
// row) by n rows; CTA = 8 consumer warps (warp w transforms column w of the
// tile) + 1 producer warp whose first lane issues the tile loads and stores.
// Two tile buffers: while the consumers transform tile i in one buffer, the
// producer stores tile i-1 from the other and loads tile i+1 into it.
//
//   full[b]  : the TMA load of buffer b completed (expect_tx, 1 arrival)
//   ready[b] : the 8 consumer warps wrote their columns back (8 arrivals)
//
// Same transform as k_cols_pipe (same radix sequence and twiddle table), so
// the results are the same numbers.
#include <cudaTypedefs.h>

#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "fft_tma.cuh"
#include "fft_tma.hpp"

namespace sogb {

template <int L>
struct ColsTmaLayout {
  static constexpr int N = 1 << L;
  static constexpr int TILE = N * 8;                        // complex elements per tile
  static constexpr unsigned TBYTES = TILE * 16;
  static constexpr int BOX = N < 256 ? N : 256;             // rows per TMA box (box dims <= 256)
  static constexpr size_t bytes = 2 * (size_t)TILE * 16 + 8 * (size_t)WarpFft<L>::XROW * 16 +
                                  (size_t)StageTw<L>::size * 16 + 2 * 2 * sizeof(uint64_t) + 1024;
};

template <int DIR, int L>
__global__ void __launch_bounds__(288, 1) k_cols_tma(const __grid_constant__ CUtensorMap tmap, int64_t nchunks,
                                                     int64_t ntiles, const double2 *__restrict__ tw,
                                                     unsigned *status) {
  using LY = ColsTmaLayout<L>;
  constexpr int N = LY::N, EPT = WarpFft<L>::EPT, TILE = LY::TILE, BOX = LY::BOX;
  extern __shared__ __align__(1024) unsigned char smem_tma[];
  // tile buffers 1024-byte aligned (the swizzle pattern repeats every 8 rows)
  unsigned char *base = smem_tma + ((1024u - (smem_u32(smem_tma) & 1023u)) & 1023u);
  double2 *buf = reinterpret_cast<double2 *>(base);
  double2 *xrow = buf + 2 * TILE;
  double2 *stg = xrow + 8 * WarpFft<L>::XROW;
  uint64_t *full = reinterpret_cast<uint64_t *>(stg + StageTw<L>::size);
  uint64_t *ready = full + 2;
  const int w = threadIdx.x >> 5, t = threadIdx.x & 31;
  if (threadIdx.x == 256) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(&ready[0], 8);
    mbar_init(&ready[1], 8);
    mbar_init_fence();
  }
  load_stage_twiddles<double, L, 0>(stg, tw);
  __syncthreads();
  // tiles of this CTA: blockIdx.x, + gridDim.x, ...
  const int64_t my = ntiles > blockIdx.x ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  if (w == 8) {
    if (t != 0) return;
    auto coords = [&](int64_t it, int &x, int &y) {
      const int64_t tile = blockIdx.x + it * gridDim.x;
      const int64_t o = tile / nchunks;
      x = (int)((tile - o * nchunks) * 16);
      y = (int)(o * N);
    };
    bool pending[2] = {false, false};   // a load into the buffer not yet known to have landed
    unsigned pend_par[2] = {0u, 0u};
    bool ok = true;
    for (int64_t it = 0; it < my + 2 && ok; ++it) {
      const int b = (int)(it & 1);
      if (it >= 2) {
        // tile it-2 was transformed in buffer b: store it, then reuse b
        ok = mbar_wait(&ready[b], (unsigned)(((it - 2) >> 1) & 1), status);
        if (!ok) break;
        pending[b] = false;
        int x, y;
        coords(it - 2, x, y);
        for (int h = 0; h < N / BOX; ++h) tma_store_2d(&tmap, x, y + h * BOX, buf + b * TILE + h * BOX * 8);
        bulk_commit();
        bulk_wait_read_all();
      }
      if (it < my) {
        int x, y;
        coords(it, x, y);
        mbar_expect_tx(&full[b], LY::TBYTES);
        for (int h = 0; h < N / BOX; ++h) tma_load_2d(buf + b * TILE + h * BOX * 8, &tmap, x, y + h * BOX, &full[b]);
        pending[b] = true;
        pend_par[b] = (unsigned)((it >> 1) & 1);
      }
    }
    if (!ok) {
      // a consumer stopped: let the loads in flight land before the CTA exits
      for (int b = 0; b < 2; ++b)
        if (pending[b]) mbar_wait(&full[b], pend_par[b], status);
    }
    bulk_wait_all();
    return;
  }
  double2 *row = xrow + w * WarpFft<L>::XROW;
  for (int64_t it = 0; it < my; ++it) {
    const int b = (int)(it & 1);
    if (!mbar_wait(&full[b], (unsigned)((it >> 1) & 1), status)) break;
    double2 *cur = buf + b * TILE;
    double2 v[EPT];
#pragma unroll
    for (int e = 0; e < EPT; ++e) v[e] = cur[tile_slot(t + 32 * e, w)];
    warp_fft<DIR, L>(v, t, stg, row);
#pragma unroll
    for (int e = 0; e < EPT; ++e) cur[tile_slot(t + 32 * e, w)] = v[e];
    fence_proxy_async_smem();
    __syncwarp();
    if (t == 0) mbar_arrive(&ready[b]);
  }
}

// Inverse y pass of the field spectra [nf][F][nz][n][inner] that forms the
// fields of two-slot frames (the TMA form of k_cols_fields, same results).
// Work is a sequence of jobs, one inverse transform each; a tile (plane o,
// 8 columns) gives:
//   slot 0 of an orthorhombic two-slot frame (Y1): job FY (field y =
//     ky IFFT(i my Y1) -> slot 1), job POT (IFFT(Y1) -> slot 3, when the
//     potential is wanted and the frame has no alias-summed potential), job FX
//     (field x = i kx mx IFFT(Y1), in place) -- in this order, so the in-place
//     store comes after every read of the tile;
//   slot 2 of such a frame (Y2): job FZ (field z = kz IFFT(Y2), in place);
//   every plane of other frames (and slot 3 of alias frames): job PLAIN;
//   slot 1 (and slot 3 when not stored) of two-slot frames: nothing.
// The jobs of one tile run back to back on one CTA: the repeated loads of a
// slot-0 tile come from L2.
enum : int { kJobFY = 0, kJobPot = 1, kJobFX = 2, kJobFZ = 3, kJobPlain = 4 };

struct FieldJobs {
  const FrameGeom *geom;
  int F, nz, two_slot, want_pot;
  int64_t nchunks;
  // jobs of the tile starting at plane o: their count, and their kinds packed
  // four bits each (job j: (kinds >> 4j) & 15), so no local array is needed
  __device__ __forceinline__ int jobs(int64_t o, int &kinds) const {
    const int64_t fs = o / nz;
    const int f = (int)(fs / F), sl = (int)(fs - (int64_t)f * F);
    const FrameGeom &g = geom[f];
    if (!(two_slot && g.ortho)) { kinds = kJobPlain; return 1; }
    if (sl == 0) {
      if (want_pot && !g.pad) { kinds = kJobFY | (kJobPot << 4) | (kJobFX << 8); return 3; }
      kinds = kJobFY | (kJobFX << 4);
      return 2;
    }
    if (sl == 2) { kinds = kJobFZ; return 1; }
    if (sl == 3 && g.pad) { kinds = kJobPlain; return 1; }
    return 0;
  }
  // plane the job's output goes to
  __device__ __forceinline__ int64_t dst_plane(int64_t o, int kind) const {
    const int64_t sl = (o / nz) % F;
    const int64_t o0 = o - sl * nz;
    if (kind == kJobFY) return o0 + nz;
    if (kind == kJobPot) return o0 + 3 * (int64_t)nz;
    return o;
  }
};

template <int L>
__global__ void __launch_bounds__(288, 1) k_cols_fields_tma(const __grid_constant__ CUtensorMap tmap, FieldJobs jb,
                                                            int64_t ntiles, const double2 *__restrict__ tw,
                                                            unsigned *status) {
  using LY = ColsTmaLayout<L>;
  constexpr int N = LY::N, EPT = WarpFft<L>::EPT, TILE = LY::TILE, BOX = LY::BOX;
  extern __shared__ __align__(1024) unsigned char smem_tma[];
  unsigned char *base = smem_tma + ((1024u - (smem_u32(smem_tma) & 1023u)) & 1023u);
  double2 *buf = reinterpret_cast<double2 *>(base);
  double2 *xrow = buf + 2 * TILE;
  double2 *stg = xrow + 8 * WarpFft<L>::XROW;
  uint64_t *full = reinterpret_cast<uint64_t *>(stg + StageTw<L>::size);
  uint64_t *ready = full + 2;
  const int w = threadIdx.x >> 5, t = threadIdx.x & 31;
  if (threadIdx.x == 256) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(&ready[0], 8);
    mbar_init(&ready[1], 8);
    mbar_init_fence();
  }
  load_stage_twiddles<double, L, 0>(stg, tw);
  __syncthreads();
  if (w == 8) {
    if (t != 0) return;
    int tx[2] = {0, 0}, ty[2] = {0, 0};   // store target of the job in each buffer
    bool pending[2] = {false, false};
    unsigned pend_par[2] = {0u, 0u};
    bool ok = true;
    int64_t it = 0;
    // store the job that used buffer b (job index jt)
    auto retire = [&](int64_t jt) -> bool {
      const int b = (int)(jt & 1);
      if (!mbar_wait(&ready[b], (unsigned)((jt >> 1) & 1), status)) return false;
      pending[b] = false;
      for (int h = 0; h < N / BOX; ++h) tma_store_2d(&tmap, tx[b], ty[b] + h * BOX, buf + b * TILE + h * BOX * 8);
      bulk_commit();
      bulk_wait_read_all();
      return true;
    };
    for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      const int64_t o = tile / jb.nchunks;
      const int x = (int)((tile - o * jb.nchunks) * 16);
      int kinds = 0;
      const int nj = jb.jobs(o, kinds);
      for (int j = 0; j < nj; ++j, ++it) {
        const int b = (int)(it & 1);
        if (it >= 2 && !(ok = retire(it - 2))) break;
        tx[b] = x;
        ty[b] = (int)(jb.dst_plane(o, (kinds >> (4 * j)) & 15) * N);
        mbar_expect_tx(&full[b], LY::TBYTES);
        for (int h = 0; h < N / BOX; ++h)
          tma_load_2d(buf + b * TILE + h * BOX * 8, &tmap, x, (int)(o * N) + h * BOX, &full[b]);
        pending[b] = true;
        pend_par[b] = (unsigned)((it >> 1) & 1);
      }
    }
    for (int64_t jt = it >= 2 ? it - 2 : 0; jt < it && ok; ++jt) ok = retire(jt);
    if (!ok) {
      for (int b = 0; b < 2; ++b)
        if (pending[b]) mbar_wait(&full[b], pend_par[b], status);
    }
    bulk_wait_all();
    return;
  }
  double2 *row = xrow + w * WarpFft<L>::XROW;
  int64_t it = 0;
  bool ok = true;
  for (int64_t tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
    const int64_t o = tile / jb.nchunks;
    const int mx = (int)((tile - o * jb.nchunks) * 8) + w;
    const int f = (int)(o / jb.nz / jb.F);
    int kinds = 0;
    const int nj = jb.jobs(o, kinds);
    for (int j = 0; j < nj; ++j, ++it) {
      const int b = (int)(it & 1);
      if (!(ok = mbar_wait(&full[b], (unsigned)((it >> 1) & 1), status))) break;
      double2 *cur = buf + b * TILE;
      const int kd = (kinds >> (4 * j)) & 15;
      double2 v[EPT];
#pragma unroll
      for (int e = 0; e < EPT; ++e) {
        v[e] = cur[tile_slot(t + 32 * e, w)];
        if (kd == kJobFY) {   // i my Y1
          const double my = (double)signed_mode(t + 32 * e, N);
          v[e] = make_double2(-my * v[e].y, my * v[e].x);
        }
      }
      warp_fft<+1, L>(v, t, stg, row);
      const FrameGeom &g = jb.geom[f];
      if (kd == kJobFY || kd == kJobFZ) {
        const double k = kd == kJobFY ? g.kmat[4] : g.kmat[8];
#pragma unroll
        for (int e = 0; e < EPT; ++e) v[e] = make_double2(k * v[e].x, k * v[e].y);
      } else if (kd == kJobFX) {   // i kx mx
        const double kxm = g.kmat[0] * mx;
#pragma unroll
        for (int e = 0; e < EPT; ++e) v[e] = make_double2(-kxm * v[e].y, kxm * v[e].x);
      }
#pragma unroll
      for (int e = 0; e < EPT; ++e) cur[tile_slot(t + 32 * e, w)] = v[e];
      fence_proxy_async_smem();
      __syncwarp();
      if (t == 0) mbar_arrive(&ready[b]);
    }
  }
}

// Inverse C2R x pass of F fields with interleaved real output (the bulk-copy
// form of k_c2r_pipe, same arithmetic and results), n = 512 reals per row as
// a 256-point complex transform.  A tile is RPT = 8/F rows x F fields; one
// consumer warp per (row, field): the pre-twiddle Z[k] = A + i conj(W^k) B
// from X[k] and X[h-k] of its input row, the warp-local transform with its
// exchanges in its own row slot, then -- after a named barrier of the row's
// F warps, which frees the row's slots -- its values written interleaved
// into the row's region.  The producer warp's first lane moves the rows:
// a 1-D bulk copy per input row (4112 bytes) on the buffer's full barrier,
// a 1-D bulk store per output row (n*F doubles) once the consumers arrive on
// the buffer's ready barrier.
template <int L>
struct C2rTmaLayout {
  static constexpr int N = 1 << L, H = N / 2, NXH = H + 1;
  static constexpr int HP = H + H / 8;                       // padded exchange row
  static constexpr int ROWSZ = HP > NXH ? HP : NXH;          // complex slots per (row, field)
  // shared memory with nw = RPT * F consumer warps (one row-field slot each, two buffers)
  static constexpr size_t bytes(int nw) {
    return (2 * (size_t)nw * ROWSZ + N + StageTw<L - 1>::size) * 16 + 4 * sizeof(uint64_t) + 16;
  }
};

// NW consumer warps (RPT * F: 6 for three fields, else 8) + 1 producer warp;
// three CTAs per SM with six consumer warps, two with eight.
template <int L, int NW>
__global__ void __launch_bounds__(32 * (NW + 1), NW == 6 ? 3 : 2)
    k_c2r_tma(const double2 *__restrict__ in, double *__restrict__ out, int F, int rpt, int64_t nzy, int64_t nrows,
              int64_t ntiles, const double2 *__restrict__ tw, unsigned *status) {
  using LY = C2rTmaLayout<L>;
  constexpr int N = LY::N, H = LY::H, NXH = LY::NXH, ROWSZ = LY::ROWSZ, SLOTS = NW * ROWSZ;
  constexpr int TPT = H / kEPT;
  static_assert(TPT == 32, "one warp per row-field transform");
  extern __shared__ __align__(16) unsigned char smem_c2r[];
  double2 *bufs = reinterpret_cast<double2 *>(smem_c2r);
  double2 *stw = bufs + 2 * SLOTS;        // n-th roots of unity (pre-twiddle)
  double2 *stg = stw + N;                 // stage table of the length n/2 transform
  uint64_t *full = reinterpret_cast<uint64_t *>(stg + StageTw<L - 1>::size);
  uint64_t *ready = full + 2;
  constexpr int nw = NW;                  // consumer warps (= rpt * F)
  const int w = threadIdx.x >> 5, t = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(&ready[0], nw);
    mbar_init(&ready[1], nw);
    mbar_init_fence();
  }
  load_twiddles<double>(stw, tw, N);
  load_stage_twiddles<double, L - 1, 1>(stg, tw);
  __syncthreads();
  const int64_t my = ntiles > blockIdx.x ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  if (w == nw) {
    if (t != 0) return;
    bool pending[2] = {false, false};
    unsigned pend_par[2] = {0u, 0u};
    bool ok = true;
    for (int64_t it = 0; it < my + 2 && ok; ++it) {
      const int b = (int)(it & 1);
      double2 *buf = bufs + b * SLOTS;
      if (it >= 2) {
        ok = mbar_wait(&ready[b], (unsigned)(((it - 2) >> 1) & 1), status);
        if (!ok) break;
        pending[b] = false;
        const int64_t row0 = (blockIdx.x + (it - 2) * gridDim.x) * rpt;
        const int nv = (int)min((int64_t)rpt, nrows - row0);
        for (int r = 0; r < nv; ++r)
          bulk_store_1d(out + (row0 + r) * N * F, buf + (size_t)r * F * ROWSZ, (unsigned)(N * F * sizeof(double)));
        bulk_commit();
        bulk_wait_read_all();
      }
      if (it < my) {
        const int64_t row0 = (blockIdx.x + it * gridDim.x) * rpt;
        const int nv = (int)min((int64_t)rpt, nrows - row0);
        mbar_expect_tx(&full[b], (unsigned)(nv * F * NXH * 16));
        for (int r = 0; r < nv; ++r) {
          const int64_t row = row0 + r, frame = row / nzy, zy = row - frame * nzy;
          for (int f = 0; f < F; ++f)
            bulk_load_1d(buf + (size_t)(r * F + f) * ROWSZ, in + ((frame * F + f) * nzy + zy) * NXH, NXH * 16,
                         &full[b]);
        }
        pending[b] = true;
        pend_par[b] = (unsigned)((it >> 1) & 1);
      }
    }
    if (!ok) {
      for (int b = 0; b < 2; ++b)
        if (pending[b]) mbar_wait(&full[b], pend_par[b], status);
    }
    bulk_wait_all();
    return;
  }
  if (w > nw) return;
  const int rr = w / F, f = w - rr * F;
  for (int64_t it = 0; it < my; ++it) {
    const int b = (int)(it & 1);
    if (!mbar_wait(&full[b], (unsigned)((it >> 1) & 1), status)) break;
    const int64_t row0 = (blockIdx.x + it * gridDim.x) * rpt;
    const bool valid = row0 + rr < nrows;   // warp-uniform, and uniform over the row's F warps
    double2 *cur = bufs + b * SLOTS;
    if (valid) {
      double2 *X = cur + (size_t)(rr * F + f) * ROWSZ;
      double2 v[kEPT];
#pragma unroll
      for (int e = 0; e < kEPT; ++e) {
        const int k = t + e * TPT;
        if (k == 0) {
          const double x0 = X[0].x, xh = X[H].x;
          v[e] = make_double2(x0 + xh, x0 - xh);
        } else {
          const double2 a = X[k], bb = X[H - k];
          const double Ar = a.x + bb.x, Ai = a.y - bb.y;
          const double Br = a.x - bb.x, Bi = a.y + bb.y;
          const double2 wk = stw[k];
          const double cr = wk.x * Br + wk.y * Bi, ci = wk.x * Bi - wk.y * Br;
          v[e] = make_double2(Ar - ci, Ai + cr);
        }
      }
      __syncwarp();   // the row slot's inputs are in registers: it becomes exchange space
      ct_fft<double, +1, L - 1, true, 1, true>(v, t, stg, X, 1);
      named_sync(1 + rr, F * 32);   // the row's F transforms are done with their slots
      double *so = reinterpret_cast<double *>(cur + (size_t)rr * F * ROWSZ);
#pragma unroll
      for (int e = 0; e < kEPT; ++e) {
        const int m = t + e * TPT;
        so[(2 * m) * F + f] = v[e].x;
        so[(2 * m + 1) * F + f] = v[e].y;
      }
      fence_proxy_async_smem();
    }
    __syncwarp();
    if (t == 0) mbar_arrive(&ready[b]);
  }
}

// Forward R2C x pass, n = 512 reals per row as a 256-point complex transform
// (the bulk-copy form of k_r2c_pipe, same arithmetic and results): a tile is
// 8 rows, one consumer warp per row packs z[m] = x[2m] + i x[2m+1] from its
// row slot, transforms it with warp-local exchanges in the slot, leaves Z in
// the slot (padded layout) for the post-processing
//   X[k] = (Z[k] + conj Z[h-k]) / 2 - i W_n^k (Z[k] - conj Z[h-k]) / 2,
// and writes X[0 .. h] back to the slot's start for the bulk store.
template <int L>
struct R2cTmaLayout {
  static constexpr int N = 1 << L, H = N / 2, NXH = H + 1;
  static constexpr int ROWSZ = H + H / 8;                    // padded exchange row (>= NXH and >= N/2)
  static constexpr size_t bytes = (2 * 8 * (size_t)ROWSZ + N + StageTw<L - 1>::size) * 16 + 4 * sizeof(uint64_t);
};

template <int L>
__global__ void __launch_bounds__(288, 2)
    k_r2c_tma(const double *__restrict__ in, double2 *__restrict__ out, int64_t nrows, int64_t ntiles,
              const double2 *__restrict__ tw, unsigned *status) {
  using LY = R2cTmaLayout<L>;
  constexpr int N = LY::N, H = LY::H, NXH = LY::NXH, ROWSZ = LY::ROWSZ, SLOTS = 8 * ROWSZ;
  constexpr int TPT = H / kEPT;
  static_assert(TPT == 32, "one warp per row transform");
  static_assert(ROWSZ >= NXH, "the output row fits its slot");
  extern __shared__ __align__(16) unsigned char smem_r2c[];
  double2 *bufs = reinterpret_cast<double2 *>(smem_r2c);
  double2 *stw = bufs + 2 * SLOTS;        // n-th roots of unity (post-processing)
  double2 *stg = stw + N;                 // stage table of the length n/2 transform
  uint64_t *full = reinterpret_cast<uint64_t *>(stg + StageTw<L - 1>::size);
  uint64_t *ready = full + 2;
  const int w = threadIdx.x >> 5, t = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(&ready[0], 8);
    mbar_init(&ready[1], 8);
    mbar_init_fence();
  }
  load_twiddles<double>(stw, tw, N);
  load_stage_twiddles<double, L - 1, 1>(stg, tw);
  __syncthreads();
  const int64_t my = ntiles > blockIdx.x ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  if (w == 8) {
    if (t != 0) return;
    bool pending[2] = {false, false};
    unsigned pend_par[2] = {0u, 0u};
    bool ok = true;
    for (int64_t it = 0; it < my + 2 && ok; ++it) {
      const int b = (int)(it & 1);
      double2 *buf = bufs + b * SLOTS;
      if (it >= 2) {
        ok = mbar_wait(&ready[b], (unsigned)(((it - 2) >> 1) & 1), status);
        if (!ok) break;
        pending[b] = false;
        const int64_t row0 = (blockIdx.x + (it - 2) * gridDim.x) * 8;
        const int nv = (int)min((int64_t)8, nrows - row0);
        for (int r = 0; r < nv; ++r) bulk_store_1d(out + (row0 + r) * NXH, buf + (size_t)r * ROWSZ, NXH * 16);
        bulk_commit();
        bulk_wait_read_all();
      }
      if (it < my) {
        const int64_t row0 = (blockIdx.x + it * gridDim.x) * 8;
        const int nv = (int)min((int64_t)8, nrows - row0);
        mbar_expect_tx(&full[b], (unsigned)(nv * N * 8));
        for (int r = 0; r < nv; ++r)
          bulk_load_1d(buf + (size_t)r * ROWSZ, in + (row0 + r) * N, N * 8, &full[b]);
        pending[b] = true;
        pend_par[b] = (unsigned)((it >> 1) & 1);
      }
    }
    if (!ok) {
      for (int b = 0; b < 2; ++b)
        if (pending[b]) mbar_wait(&full[b], pend_par[b], status);
    }
    bulk_wait_all();
    return;
  }
  for (int64_t it = 0; it < my; ++it) {
    const int b = (int)(it & 1);
    if (!mbar_wait(&full[b], (unsigned)((it >> 1) & 1), status)) break;
    const int64_t row0 = (blockIdx.x + it * gridDim.x) * 8;
    double2 *zrow = bufs + b * SLOTS + (size_t)w * ROWSZ;
    if (row0 + w < nrows) {
      double2 v[kEPT];
#pragma unroll
      for (int e = 0; e < kEPT; ++e) v[e] = zrow[t + e * TPT];   // (x[2m], x[2m+1]), m = t + e TPT
      __syncwarp();   // the inputs are in registers: the slot becomes exchange space
      ct_fft<double, -1, L - 1, true, 1, true, true>(v, t, stg, zrow, 1);
#pragma unroll
      for (int e = 0; e < kEPT; ++e) zrow[sidx<true>(t + e * TPT, 1)] = v[e];
      __syncwarp();
      double2 o[kEPT], oh = make_double2(0.0, 0.0);
#pragma unroll
      for (int e = 0; e < kEPT; ++e) {
        const int k = t + e * TPT;
        const double2 a = v[e];
        const double2 bb = zrow[sidx<true>((H - k) & (H - 1), 1)];
        const double er = 0.5 * (a.x + bb.x), ei = 0.5 * (a.y - bb.y);
        const double dr = 0.5 * (a.x - bb.x), di = 0.5 * (a.y + bb.y);
        const double2 wk = stw[k];
        const double pr = wk.x * dr - wk.y * di, pi = wk.x * di + wk.y * dr;
        o[e] = make_double2(er + pi, ei - pr);
        if (k == 0) oh = make_double2(er - pi, ei + pr);
      }
      __syncwarp();   // every lane has read Z: the slot takes the output row
#pragma unroll
      for (int e = 0; e < kEPT; ++e) zrow[t + e * TPT] = o[e];
      if (t == 0) zrow[H] = oh;
      fence_proxy_async_smem();
    }
    __syncwarp();
    if (t == 0) mbar_arrive(&ready[b]);
  }
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::atomic<void *> fn{nullptr};
  void *f = fn.load(std::memory_order_acquire);
  if (!f) {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    cudaGetLastError();
    if (f) fn.store(f, std::memory_order_release);
  }
  return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
}

// one wave of resident CTAs of `kernel` on the current device (cached)
template <typename K>
int tiles_grid(K kernel, size_t smem, int64_t ntiles, int threads = 288) {
  static std::mutex mu;
  static std::map<std::pair<const void *, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_pair(reinterpret_cast<const void *>(kernel), dev);
  std::lock_guard<std::mutex> lock(mu);
  auto itc = cache.find(key);
  int total;
  if (itc != cache.end()) {
    total = itc->second;
  } else {
    int nsm = 1, per = 1;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, threads, smem) != cudaSuccess || per < 1) per = 0;
    cudaGetLastError();
    total = per > 0 ? nsm * per : 0;
    cache[key] = total;
  }
  if (total <= 0) return 0;
  return (int)std::min<int64_t>(ntiles, total);
}

template <int DIR, int L>
bool launch_one(double2 *data, int64_t inner, int64_t outer, const double2 *tw, unsigned *status, cudaStream_t st) {
  using LY = ColsTmaLayout<L>;
  constexpr int N = 1 << L;
  auto encode = encode_fn();
  if (!encode) return false;
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)(2 * inner), (cuuint64_t)(outer * N)};
  cuuint64_t strides[1] = {(cuuint64_t)(inner * 16)};
  cuuint32_t box[2] = {16, (cuuint32_t)LY::BOX};
  cuuint32_t es[2] = {1, 1};
  if (encode(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, data, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  const int64_t nchunks = (inner + 7) / 8;
  const int64_t ntiles = outer * nchunks;
  const int grid = tiles_grid(k_cols_tma<DIR, L>, LY::bytes, ntiles);
  if (grid <= 0) return false;
  k_cols_tma<DIR, L><<<grid, 288, LY::bytes, st>>>(m, nchunks, ntiles, tw, status);
  return true;
}

template <int L>
bool launch_fields(double2 *data, const FrameGeom *geom, int nf, int F, int nz, int64_t inner, const double2 *tw,
                   int two_slot, int want_pot, unsigned *status, cudaStream_t st) {
  using LY = ColsTmaLayout<L>;
  constexpr int N = 1 << L;
  auto encode = encode_fn();
  if (!encode) return false;
  const int64_t planes = (int64_t)nf * F * nz;
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)(2 * inner), (cuuint64_t)(planes * N)};
  cuuint64_t strides[1] = {(cuuint64_t)(inner * 16)};
  cuuint32_t box[2] = {16, (cuuint32_t)LY::BOX};
  cuuint32_t es[2] = {1, 1};
  if (encode(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, data, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  FieldJobs jb;
  jb.geom = geom;
  jb.F = F;
  jb.nz = nz;
  jb.two_slot = two_slot;
  jb.want_pot = want_pot;
  jb.nchunks = (inner + 7) / 8;
  const int64_t ntiles = planes * jb.nchunks;
  const int grid = tiles_grid(k_cols_fields_tma<L>, LY::bytes, ntiles);
  if (grid <= 0) return false;
  k_cols_fields_tma<L><<<grid, 288, LY::bytes, st>>>(m, jb, ntiles, tw, status);
  return true;
}

}  // namespace

bool launch_cols_tma(double2 *data, int n, int64_t inner, int64_t outer, int dir, const double2 *tw,
                     unsigned *status, cudaStream_t st) {
  // TMA constraints: 16-byte aligned base and row pitch (a complex<double>
  // row always is), int32 tile coordinates
  if ((reinterpret_cast<uintptr_t>(data) & 15) || inner < 1 || outer < 1) return false;
  if (outer * (int64_t)n >= ((int64_t)1 << 31) || 2 * inner + 16 >= ((int64_t)1 << 31)) return false;
  if (n == 512) return dir < 0 ? launch_one<-1, 9>(data, inner, outer, tw, status, st)
                               : launch_one<+1, 9>(data, inner, outer, tw, status, st);
  if (n == 256) return dir < 0 ? launch_one<-1, 8>(data, inner, outer, tw, status, st)
                               : launch_one<+1, 8>(data, inner, outer, tw, status, st);
  return false;
}

bool launch_cols_fields_tma(double2 *data, const FrameGeom *geom, int nf, int F, int nz, int n, int64_t inner,
                            const double2 *tw, int two_slot, int want_pot, unsigned *status, cudaStream_t st) {
  if ((reinterpret_cast<uintptr_t>(data) & 15) || inner < 1 || nf < 1 || F < 1 || nz < 1) return false;
  if ((int64_t)nf * F * nz * n >= ((int64_t)1 << 31) || 2 * inner + 16 >= ((int64_t)1 << 31)) return false;
  if (n == 512) return launch_fields<9>(data, geom, nf, F, nz, inner, tw, two_slot, want_pot, status, st);
  if (n == 256) return launch_fields<8>(data, geom, nf, F, nz, inner, tw, two_slot, want_pot, status, st);
  return false;
}

bool launch_c2r_tma(const double2 *in, double *out, int F, int64_t nzy, int64_t nrows, int n, const double2 *tw,
                    unsigned *status, cudaStream_t st) {
  if (n != 512 || F < 1 || F > 8 || nrows < 1) return false;
  if ((reinterpret_cast<uintptr_t>(in) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return false;
  using LY = C2rTmaLayout<9>;
  const int rpt = 8 / F, nw = rpt * F;
  if (nw != 6 && nw != 8) return false;
  const int64_t ntiles = (nrows + rpt - 1) / rpt;
  const size_t smem = LY::bytes(nw);
  const int grid = nw == 6 ? tiles_grid(k_c2r_tma<9, 6>, smem, ntiles, 32 * 7)
                           : tiles_grid(k_c2r_tma<9, 8>, smem, ntiles, 32 * 9);
  if (grid <= 0) return false;
  if (nw == 6)
    k_c2r_tma<9, 6><<<grid, 32 * 7, smem, st>>>(in, out, F, rpt, nzy, nrows, ntiles, tw, status);
  else
    k_c2r_tma<9, 8><<<grid, 32 * 9, smem, st>>>(in, out, F, rpt, nzy, nrows, ntiles, tw, status);
  return true;
}

bool launch_r2c_tma(const double *in, double2 *out, int64_t nrows, int n, const double2 *tw, unsigned *status,
                    cudaStream_t st) {
  if (n != 512 || nrows < 1) return false;
  if ((reinterpret_cast<uintptr_t>(in) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return false;
  using LY = R2cTmaLayout<9>;
  const int64_t ntiles = (nrows + 7) / 8;
  const int grid = tiles_grid(k_r2c_tma<9>, LY::bytes, ntiles);
  if (grid <= 0) return false;
  k_r2c_tma<9><<<grid, 288, LY::bytes, st>>>(in, out, nrows, ntiles, tw, status);
  return true;
}

}  // namespace sogb
