// Particle-mesh SOG solver on B200: cell-sorted deterministic spread, 3-D
// R2C/C2R FFT, fused Green / energy / ik-field k-space pass, gather.
//
// Pipeline of one call (all frames share the plan's mesh):
//   k_frame_setup   cells -> inverse, wave-vector matrix, volume, k=0 data
//   k_atom_bin      fractional coords -> stencil anchor, sort bin     (a6/a7)
//   radix sort      (bin, slot) pairs, stable -> fixed spread order
//   k_atom_sorted   sorted SoA: anchors, fractional offsets, charges
//   per channel:
//     k_spread      output-stationary tiles, smem candidate lists   (a7)
//     FFT  x R2C, y, z                                              (a8)
//     k_kspace      Green on the fly, energy/self partials, ik fields (a9/a10)
//     k_kspace_extra  dE/d(amp,bw2) and virial partials (optional)  (a11/a13)
//     FFT^-1 z, y, x C2R (fields batched)                          (a10)
//     k_gather      forces and potential at the atoms               (a10/a11)
//   k_reduce / k_finalize_frames / k_finalize_atoms
#include <algorithm>
#include <atomic>
#include <mutex>
#include <map>
#include <set>
#include <tuple>
#include <utility>
#include <cfloat>
#include <climits>
#include <functional>
#include <string>
#include <type_traits>
#include <cmath>
#include <cstring>
#include <vector>

#include "host_math.hpp"
#include "plan.hpp"
#include "sort.cuh"
#include "fft_pipe.cuh"
#include "fft_tma.hpp"
#include "frames.cuh"

namespace sogb {

struct QuadsCoef {
  double c[36];
};

// ------------------------------------------------------------------------
// atoms: stencil anchor + bin key
// ------------------------------------------------------------------------
struct AtomGrid {
  int nx, ny, nz, first, nbx, nby, nbz;
  int zb;             // z bin layers per block of the bin order (1: plain z-major)
  uint32_t bins_per_frame;
};

// Bin order: blocks of zb bin layers along z; inside a block the (y, z) rows
// run y-major, and the x bins of a row are consecutive (the spread's segment
// table relies on that).  A stencil's z neighbours inside a block are one row
// apart, so the gather (atoms in bin order) finds them in L2.
__host__ __device__ __forceinline__ uint32_t bin_row(const AtomGrid &ag, int bz, int by) {
  const int B = bz / ag.zb, zl = bz - B * ag.zb;
  const int zbe = min(ag.zb, ag.nbz - B * ag.zb);
  return ((uint32_t)B * ag.zb * ag.nby + (uint32_t)by * zbe + zl) * ag.nbx;
}

#ifndef SOG_BIN_ZB
#define SOG_BIN_ZB 1
#endif
// resident blocks per SM the register allocation of these kernels aims at
#ifndef SOG_GATHER_MINB
#define SOG_GATHER_MINB 1
#endif
#ifndef SOG_ZFUSED_MINB
#define SOG_ZFUSED_MINB 2
#endif
#ifndef SOG_GATHER_VEC
#define SOG_GATHER_VEC 1
#endif
// 1: forces-only fp64 gathers load their stencil rows cooperatively per warp
// (k_gather_f3c); 0: one thread's 16-byte row loads (k_gather_f3v)
#ifndef SOG_GATHER_COOP
#define SOG_GATHER_COOP 1
#endif
#ifndef SOG_SPREAD_MINB
#define SOG_SPREAD_MINB 4
#endif
// 1: separable splines spread with one warp per 8^3 block (k_spread_blk)
#ifndef SOG_SPREAD_BLK
#define SOG_SPREAD_BLK 1
#endif
#ifndef SOG_SPREAD_BLK_MINB
#define SOG_SPREAD_BLK_MINB 6
#endif
// threads per CTA of the fp64 column (y) passes: 256 (4 columns of a
// 512-point axis per tile, 64-byte rows) or 512 (8 columns, 128-byte rows)
#ifndef SOG_COLS_THR64
#define SOG_COLS_THR64 256
#endif
// the same for the z-slab's row-mapped y passes, and the fused z tile of the
// slab (256 threads: 4-column tiles, 64-byte peer-store runs; 512: 8 columns,
// 128-byte runs, which measured slower over 8 ranks: 2.44 against 2.27 ms a
// step for the 512^3 mesh)
#ifndef SOG_SLAB_COLS_THR64
#define SOG_SLAB_COLS_THR64 256
#endif
#ifndef SOG_SLAB_ZTHR
#define SOG_SLAB_ZTHR 256
#endif
// fused z tile of the single-device path for 512 and 1024 points: 256
// threads (4 columns, two CTAs per SM) or 512 (8 columns, 128-byte field
// rows, one CTA per SM).  With the two-slot output the 256-thread tile is
// faster at 512^3 (1.90 against 2.06 ms).
#ifndef SOG_ZTHR
#define SOG_ZTHR 256
#endif
// fp64 column passes of 256- and 512-point axes through TMA tiles and
// warp-resident transforms (fft_tma.cu)
#ifndef SOG_COLS_TMA
#define SOG_COLS_TMA 1
#endif
#ifndef SOG_SLAB_TWO_SLOT
#define SOG_SLAB_TWO_SLOT 1
#endif

// Fractional coordinate along axis a (r @ cell^-1, then remainder 1.0) and the
// anchor (first stencil node, wrapped) with the in-cell offset t
// (quads_fft.py:243, 45-53; lmp/sog.cpp:1977-2006).
template <typename T>
__device__ __forceinline__ void frac_anchor(const T *r, const double *ci, int a, int n, int first,
                                            int &anchor, T &t, bool &ok) {
  const double s = (double)r[0] * ci[0 * 3 + a] + (double)r[1] * ci[1 * 3 + a] + (double)r[2] * ci[2 * 3 + a];
  T sT = (T)s;
  T f = sT - floor(sT);
  T fx = f * (T)n;
  if (!isfinite(fx)) { ok = false; fx = T(0); }
  const T fl = floor(fx);
  t = fx - fl;
  int b = (int)fl + first;
  b %= n;
  if (b < 0) b += n;
  anchor = b;
}

template <typename T>
__global__ void k_atom_bin(const T *__restrict__ pos, const T *__restrict__ q, int nch,
                           const FrameGeom *__restrict__ geom, AtomGrid ag,
                           uint32_t *__restrict__ keys, int32_t *__restrict__ vals, unsigned *status) {
  const int f = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const FrameGeom &g = geom[f];
  if (i >= g.natoms) return;
  const int64_t atom = g.atom_begin + i;
  const T *r = pos + atom * 3;
  bool ok = true;
  int ax, ay, az;
  T t;
  frac_anchor(r, g.cinv, 0, ag.nx, ag.first, ax, t, ok);
  frac_anchor(r, g.cinv, 1, ag.ny, ag.first, ay, t, ok);
  frac_anchor(r, g.cinv, 2, ag.nz, ag.first, az, t, ok);
  for (int c = 0; c < nch; ++c)
    if (!isfinite((double)q[atom * nch + c])) ok = false;
  if (!ok) raise_status(status, kStatusNonFinite);
  const uint32_t key = (uint32_t)f * ag.bins_per_frame + bin_row(ag, az / kBin, ay / kBin) + (uint32_t)(ax / kBin);
  const int64_t slot = g.slot_base + i;
  keys[slot] = key;
  vals[slot] = (int32_t)slot;
}

// sorted SoA: anchor (ax, ay, az, frame), offsets t, charges [C][n], atom index
template <typename T>
__global__ void k_atom_sorted(const T *__restrict__ pos, const T *__restrict__ q, int nch,
                              const FrameGeom *__restrict__ geom, AtomGrid ag,
                              const uint32_t *__restrict__ skeys, const int32_t *__restrict__ svals,
                              int64_t nslots, int4 *__restrict__ s_anchor, T *__restrict__ s_t,
                              T *__restrict__ s_q, int32_t *__restrict__ s_atom) {
  const int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= nslots) return;
  const int f = (int)(skeys[s] / ag.bins_per_frame);
  const FrameGeom &g = geom[f];
  const int64_t atom = g.atom_begin + (svals[s] - g.slot_base);
  const T *r = pos + atom * 3;
  bool ok = true;
  int ax, ay, az;
  T tx, ty, tz;
  frac_anchor(r, g.cinv, 0, ag.nx, ag.first, ax, tx, ok);
  frac_anchor(r, g.cinv, 1, ag.ny, ag.first, ay, ty, ok);
  frac_anchor(r, g.cinv, 2, ag.nz, ag.first, az, tz, ok);
  s_anchor[s] = make_int4(ax, ay, az, f);
  s_t[s * 3 + 0] = tx;
  s_t[s * 3 + 1] = ty;
  s_t[s * 3 + 2] = tz;
  for (int c = 0; c < nch; ++c) {
    T v = q[atom * nch + c];
    if (!isfinite((double)v)) v = T(0);
    s_q[(int64_t)c * nslots + s] = v;
  }
  s_atom[s] = (int32_t)atom;
}

// ------------------------------------------------------------------------
// 1-D spline weights (device)
// ------------------------------------------------------------------------
// Cardinal B-spline, Cox-de Boor (lmp/sog.cpp:89-110); w[a] weights node
// anchor + a.
template <typename T, int P>
__device__ __forceinline__ void bspline_w(T t, T *w) {
  T prev[P];
#pragma unroll
  for (int a = 0; a < P; ++a) w[a] = T(0);
  w[0] = T(1) - t;
  w[1] = t;
#pragma unroll
  for (int k = 3; k <= P; ++k) {
    const T inv = T(1) / T(k - 1);
#pragma unroll
    for (int a = 0; a < P; ++a) prev[a] = w[a];
    w[k - 1] = t * prev[k - 2] * inv;
#pragma unroll
    for (int j = 1; j <= k - 2; ++j)
      w[k - 1 - j] = ((t + T(j)) * prev[k - 2 - j] + (T(k - j) - t) * prev[k - 1 - j]) * inv;
    w[0] = (T(1) - t) * prev[0] * inv;
  }
}

template <typename T, int P>
__device__ __forceinline__ void spline_w(int spline, T t, T *w, const QuadsCoef &qc) {
  if (spline == SOG_SPLINE_QUADS) {
#pragma unroll
    for (int k = 0; k < P; ++k) {
      T v = T(0), tp = T(1);
#pragma unroll
      for (int p = 0; p < P; ++p) { v += (T)qc.c[k * P + p] * tp; tp *= t; }
      w[k] = v;
    }
  } else {
    bspline_w<T, P>(t, w);
  }
}

// d w[k] / dt of the separable splines at offset t: the B-spline's
// M_p' = M_{p-1}(x) - M_{p-1}(x - 1), i.e. w_p'[a] = w_{p-1}[a-1] - w_{p-1}[a],
// and the QuadS polynomials' derivatives (quads_spline.py:69-158).
template <int P>
__device__ __forceinline__ void spline_dw(int spline, double t, double *dw, const QuadsCoef &qc) {
  if (spline == SOG_SPLINE_QUADS) {
#pragma unroll
    for (int k = 0; k < P; ++k) {
      double v = 0.0, tp = 1.0;
#pragma unroll
      for (int p = 1; p < P; ++p) { v += (double)p * qc.c[k * P + p] * tp; tp *= t; }
      dw[k] = v;
    }
  } else {
    double w1[P - 1];
    bspline_w<double, P - 1>(t, w1);
#pragma unroll
    for (int a = 0; a < P; ++a) dw[a] = (a >= 1 ? w1[a - 1] : 0.0) - (a < P - 1 ? w1[a] : 0.0);
  }
}

// d^2 w[k] / dt^2: the second difference of the order P-2 B-spline,
// w_p''[a] = w_{p-2}[a-2] - 2 w_{p-2}[a-1] + w_{p-2}[a], and the QuadS
// polynomials' second derivatives.
template <int P>
__device__ __forceinline__ void spline_d2w(int spline, double t, double *d2, const QuadsCoef &qc) {
  if (spline == SOG_SPLINE_QUADS) {
#pragma unroll
    for (int k = 0; k < P; ++k) {
      double v = 0.0, tp = 1.0;
#pragma unroll
      for (int p = 2; p < P; ++p) { v += (double)(p * (p - 1)) * qc.c[k * P + p] * tp; tp *= t; }
      d2[k] = v;
    }
  } else {
    double w2[P - 2];
    bspline_w<double, P - 2>(t, w2);
#pragma unroll
    for (int a = 0; a < P; ++a)
      d2[a] = (a >= 2 ? w2[a - 2] : 0.0) - 2.0 * (a >= 1 && a - 1 < P - 2 ? w2[a - 1] : 0.0) +
              (a < P - 2 ? w2[a] : 0.0);
  }
}

// CubeS2 (cubes2_spline.py): every node weight is a sum of products of 1-D
// polynomials of the three offsets, and summing the classes node by node
// gives a sum of separable stencils over the P = order window
// (offsets 1 - P/2 .. P/2):
//   order 4:  W = A_x e_y e_z + e_x A_y e_z + e_x e_y A_z
//   order 6:  W = A_x e_y e_z + e_x A_y e_z + e_x e_y A_z + B_x B_y B_z
// with, per axis and offset d (eta = t at d = 1, 2, 3 and 1 - t at d = 0,
// -1, -2):  e = eta on {0,1};  A = L (order 4) / L111 (order 6) on {0,1},
// R (order 4) / L211 (order 6) on {-1,2}, L311 on {-2,3};  B = S on {0,1},
// R on {-1,2}.  The node tables and class formulas this reproduces are
// cubes2_spline.py:60-97, 170-228 (nodes) and 231-380 (weights).
constexpr double kCubeS2Xi4 = 0.57735026918962576451;   // 1/sqrt(3), cubes2_spline.py:18
constexpr double kCubeS2Xi6 = 0.6503998764035732;       // cubes2_spline.py:19

__host__ __device__ constexpr double cubes2_xi(int order) { return order == 6 ? kCubeS2Xi6 : kCubeS2Xi4; }

// kinds[k][j] for offset d = j + 1 - P/2: kind 0 = e, 1 = A, 2 = B (kinds has
// three rows; B is zero for order 4)
template <typename T, int P>
__device__ __forceinline__ void cubes2_axis(T t, T (*kinds)[P]) {
  constexpr double xi = cubes2_xi(P);
  const T x2 = (T)(xi * xi), x4 = x2 * x2;
  auto L4 = [&](T u) { return -T(0.5) * u * u * u + T(0.5) * u * u - (T(9) * x2 - T(2)) / T(6) * u + T(0.5) * x2; };
  auto R = [&](T u) { return u * u * u / T(6) + (T(3) * x2 - T(1)) / T(6) * u; };
  auto L111 = [&](T u) {
    const T u2 = u * u, u3 = u2 * u;
    return u3 * u2 / T(12) - u2 * u2 / T(6) + (T(10) * x2 - T(1)) / T(12) * u3 - (T(6) * x2 - T(1)) / T(6) * u2 +
           (T(5) * x4 - x2) / T(4) * u - (T(3) * x4 - x2) / T(6);
  };
  auto L311 = [&](T u) {
    const T u3 = u * u * u;
    return u3 * u * u / T(120) + (T(2) * x2 - T(1)) / T(24) * u3 + (T(15) * x4 - T(15) * x2 + T(4)) / T(120) * u;
  };
  auto S6 = [&](T u) { return -T(0.5) * u * u * u + T(0.5) * u * u - (T(3) * x2 - T(2)) / T(2) * u + T(0.5) * x2; };
  constexpr int first = 1 - P / 2;
#pragma unroll
  for (int j = 0; j < P; ++j) {
    const int d = j + first;
    T e = T(0), A = T(0), B = T(0);
    if (d == 0 || d == 1) {
      const T eta = d == 1 ? t : T(1) - t;
      e = eta;
      A = P == 4 ? L4(eta) : L111(eta);
      B = P == 4 ? T(0) : S6(eta);
    } else if (d == -1 || d == 2) {
      const T eta = d == 2 ? t : T(1) - t;
      A = P == 4 ? R(eta) : (-T(0.25) * L111(eta) - T(2.5) * L311(eta));
      B = P == 4 ? T(0) : R(eta);
    } else {
      const T eta = d == 3 ? t : T(1) - t;
      A = L311(eta);
    }
    kinds[0][j] = e;
    kinds[1][j] = A;
    kinds[2][j] = B;
  }
}

// Term tables of the stencils: term i is kind TX[i] along x times TY[i]
// along y times TZ[i] along z (NT = 1: the separable splines, one kind).
template <int NT>
struct StencilTerms;
template <>
struct StencilTerms<1> {
  static constexpr int K = 1;
  __device__ static constexpr int x(int) { return 0; }
  __device__ static constexpr int y(int) { return 0; }
  __device__ static constexpr int z(int) { return 0; }
};
template <>
struct StencilTerms<3> {
  static constexpr int K = 2;
  __device__ static constexpr int x(int i) { return i == 0 ? 1 : 0; }
  __device__ static constexpr int y(int i) { return i == 1 ? 1 : 0; }
  __device__ static constexpr int z(int i) { return i == 2 ? 1 : 0; }
};
template <>
struct StencilTerms<4> {
  static constexpr int K = 3;
  __device__ static constexpr int x(int i) { return i == 3 ? 2 : (i == 0 ? 1 : 0); }
  __device__ static constexpr int y(int i) { return i == 3 ? 2 : (i == 1 ? 1 : 0); }
  __device__ static constexpr int z(int i) { return i == 3 ? 2 : (i == 2 ? 1 : 0); }
};

// Per-axis kinds of one coordinate: the spline weights (NT = 1) or the
// CubeS2 kinds.
// The weights are evaluated in fp64 and rounded once to T.  Evaluated in fp32,
// the recurrences' own roundings (of 1/3 and 1/5, say) bias every weight the
// same way, which scales each atom's charge cloud by about 1 + 1e-7 and so its
// mesh self-energy, while the subtracted self term stays exact: 2.9e-5 of the
// total energy of the 131,072-atom 256^3 system.  One rounding is unbiased.
template <typename T, int P, int NT>
__device__ __forceinline__ void axis_kinds(int spline, T t, T (*kinds)[P], const QuadsCoef &qc) {
  if constexpr (NT == 1) {
    double w[P];
    spline_w<double, P>(spline, (double)t, w, qc);
#pragma unroll
    for (int j = 0; j < P; ++j) kinds[0][j] = (T)w[j];
  } else {
    double tmp[3][P];
    cubes2_axis<double, P>((double)t, tmp);
#pragma unroll
    for (int k = 0; k < StencilTerms<NT>::K; ++k)
#pragma unroll
      for (int j = 0; j < P; ++j) kinds[k][j] = (T)tmp[k][j];
  }
}

// ------------------------------------------------------------------------
// spread: output-stationary tiles, deterministic, no global atomics
// ------------------------------------------------------------------------
template <typename T>
struct SpreadArgs {
  const int4 *s_anchor;
  const T *s_t;
  const T *s_q;        // channel slice [nslots]
  const uint32_t *bin_start;
  const FrameGeom *geom;
  void *rho;           // [nf][ng] of the grid type TG of the kernel (fp64 for every plan)
  AtomGrid ag;
  int spline;
  int ntx, nty, ntz;
  QuadsCoef qc;
  // z planes written: [zlo, zlo + zcnt) of nz, stored as rho[f][zcnt][ny][nx]
  int zlo, zcnt;
  // direction density of a Hessian-vector product (k_spread_dip): the
  // direction on the charges [N][nch] (channel `channel`) and positions [N][3]
  const void *dir_q, *dir_r;
  const int32_t *s_atom;
  int nch, channel;
};

constexpr int kSpreadThreads = kTileX * kTileY;
constexpr int kMaxSeg = 48;

__device__ __forceinline__ int imod(int a, int n) {
  a %= n;
  return a < 0 ? a + n : a;
}

// ascending, de-duplicated bins of anchors in [lo, lo+len) (mod n)
__device__ int axis_bins(int lo, int len, int n, int nb, int *out) {
  int cnt = 0;
  if (len >= n) {
    for (int b = 0; b < nb; ++b) out[cnt++] = b;
    return cnt;
  }
  const int s = imod(lo, n), e = imod(lo + len - 1, n);
  const int bs = s / kBin, be = e / kBin;
  if (s <= e) {
    for (int b = bs; b <= be; ++b) out[cnt++] = b;
  } else if (be >= bs) {
    for (int b = 0; b < nb; ++b) out[cnt++] = b;
  } else {
    for (int b = 0; b <= be; ++b) out[cnt++] = b;
    for (int b = bs; b < nb; ++b) out[cnt++] = b;
  }
  return cnt;
}

// Per chunk of candidates the relevant ones are bucketed by their x anchor
// relative to the tile (key = (ax - x0 + P - 1) mod nx, at most kTileX + P - 1
// keys); a thread at tile column lx then visits only the P buckets whose
// anchors reach it, with the x offset fixed per bucket.  Bucket positions come
// from warp match ranks and a warp-ordered prefix, so the summation order at
// every mesh point is fixed (bucket, then candidate order) and the result is
// bitwise reproducible.
// NT stencil terms (StencilTerms): 1 for the separable splines, 3 / 4 for
// CubeS2 order 4 / 6.  CH candidates per chunk (fewer with three kinds, to
// keep the staged weights at two CTAs per SM).
// TG: grid type; the mesh values are accumulated and stored in it (an fp32
// plan's atom data spread into an fp64 mesh).
template <typename T, int P, int NT = 1, typename TG = T>
__global__ void __launch_bounds__(kSpreadThreads, NT == 1 ? SOG_SPREAD_MINB : 2) k_spread(SpreadArgs<T> a) {
  using ST = StencilTerms<NT>;
  constexpr int KK = ST::K;
  constexpr int CH = KK == 3 ? kSpreadThreads / 2 : kSpreadThreads;
  constexpr int NW = kSpreadThreads / 32;
  constexpr int NK = kTileX + P - 1;       // x-anchor buckets of a tile
  static_assert(NK <= 64, "bucket scan covers two keys per lane");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // candidate arrays, component-major so that lanes reading neighbouring
  // buckets hit different banks
  T *c_wz = reinterpret_cast<T *>(smem_raw);            // [KK][kTileZ][CH]
  T *c_wx = c_wz + KK * CH * kTileZ;                    // [KK][P][CH]
  T *c_wy = c_wx + KK * CH * P;                         // [KK][P][CH]
  T *c_q = c_wy + KK * CH * P;                          // [CH]
  int *c_ay = reinterpret_cast<int *>(c_q + CH);        // [CH]
  __shared__ uint32_t seg_lo[kMaxSeg], seg_pre[kMaxSeg + 1];
  __shared__ int nseg_s;
  __shared__ int kcnt[NW][NK];      // per-warp bucket counts, then bases
  __shared__ int kstart[NK + 1];

  const AtomGrid &ag = a.ag;
  const int tiles_pf = a.ntx * a.nty * a.ntz;
  const int f = blockIdx.x / tiles_pf;
  int rem = blockIdx.x - f * tiles_pf;
  const int tz = rem / (a.ntx * a.nty);
  rem -= tz * a.ntx * a.nty;
  const int ty = rem / a.ntx, tx = rem - ty * a.ntx;
  const int x0 = tx * kTileX, y0 = ty * kTileY, z0 = a.zlo + tz * kTileZ;
  const int txv = min(kTileX, ag.nx - x0), tyv = min(kTileY, ag.ny - y0);
  const int tzv = min(kTileZ, a.zlo + a.zcnt - z0);
  const FrameGeom &g = a.geom[f];

  for (int i = threadIdx.x; i < NW * NK; i += blockDim.x) (&kcnt[0][0])[i] = 0;
  if (threadIdx.x < 32) {
    // Segments of the cell-sorted atom array: one lane per (z, y) bin row;
    // a row gives at most two runs of consecutive x bins (two when the tile
    // halo wraps).  Runs are numbered in lane order by a warp scan.
    constexpr int kRows = ((kTileY + P - 2) / kBin + 2) * ((kTileZ + P - 2) / kBin + 2);
    static_assert(kRows <= 32 && 2 * kRows <= kMaxSeg, "segment table too small for the tile");
    __shared__ int bl[3][16];
    __shared__ int nbl[3];
    const int lane = threadIdx.x;
    if (lane < 3) {
      const int lo = (lane == 0 ? x0 : lane == 1 ? y0 : z0) - P + 1;
      const int len = (lane == 0 ? txv : lane == 1 ? tyv : tzv) + P - 1;
      const int n = lane == 0 ? ag.nx : lane == 1 ? ag.ny : ag.nz;
      const int nb = lane == 0 ? ag.nbx : lane == 1 ? ag.nby : ag.nbz;
      nbl[lane] = axis_bins(lo, len, n, nb, bl[lane]);
    }
    __syncwarp();
    const int nxl = nbl[0], nyl = nbl[1], nzl = nbl[2];
    uint32_t lo2[2] = {0, 0}, cnt2[2] = {0, 0};
    if (lane < nzl * nyl) {
      const int iz = lane / nyl, iy = lane - iz * nyl;
      const uint32_t row = (uint32_t)f * ag.bins_per_frame + bin_row(ag, bl[2][iz], bl[1][iy]);
      // x bins are ascending with at most one break
      int brk = nxl;
      for (int i = 1; i < nxl; ++i)
        if (brk == nxl && bl[0][i] != bl[0][i - 1] + 1) brk = i;
      lo2[0] = a.bin_start[row + bl[0][0]];
      cnt2[0] = a.bin_start[row + bl[0][brk - 1] + 1] - lo2[0];
      if (brk < nxl) {
        lo2[1] = a.bin_start[row + bl[0][brk]];
        cnt2[1] = a.bin_start[row + bl[0][nxl - 1] + 1] - lo2[1];
      }
    }
    const int ne = (cnt2[0] > 0) + (cnt2[1] > 0);
    int eo = ne;
    uint32_t co = cnt2[0] + cnt2[1];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ue = __shfl_up_sync(0xffffffffu, eo, o);
      const uint32_t uc = __shfl_up_sync(0xffffffffu, co, o);
      if (lane >= o) { eo += ue; co += uc; }
    }
    int sg = eo - ne;
    uint32_t pre = co - (cnt2[0] + cnt2[1]);
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (cnt2[h] > 0) {
        seg_lo[sg] = lo2[h];
        seg_pre[sg] = pre;
        pre += cnt2[h];
        ++sg;
      }
    if (lane == 31) {
      nseg_s = eo;
      seg_pre[eo] = co;
    }
  }
  __syncthreads();
  const int nseg = nseg_s;
  const uint32_t ncand = seg_pre[nseg];

  const int lx = threadIdx.x % kTileX, ly = threadIdx.x / kTileX;
  const int gy = y0 + ly;
  const bool own = lx < txv && ly < tyv;
  TG acc[kTileZ];
#pragma unroll
  for (int z = 0; z < kTileZ; ++z) acc[z] = TG(0);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  for (uint32_t c0 = 0; c0 < ncand; c0 += CH) {
    // ---- load and filter one chunk of candidates ----
    const uint32_t ci = c0 + threadIdx.x;
    bool rel = false;
    int4 an = make_int4(0, 0, 0, 0);
    int key = 0;
    T tf[3] = {T(0), T(0), T(0)}, qv = T(0);
    if (threadIdx.x < CH && ci < ncand) {
      int lo = 0, hi = nseg - 1;
      while (lo < hi) {  // last segment with seg_pre <= ci
        const int mid = (lo + hi + 1) >> 1;
        if (seg_pre[mid] <= ci) lo = mid; else hi = mid - 1;
      }
      const uint32_t sidx = seg_lo[lo] + (ci - seg_pre[lo]);
      an = a.s_anchor[sidx];
      // issued with the anchor so that one memory latency covers all four
      tf[0] = a.s_t[(int64_t)sidx * 3 + 0];
      tf[1] = a.s_t[(int64_t)sidx * 3 + 1];
      tf[2] = a.s_t[(int64_t)sidx * 3 + 2];
      qv = a.s_q[sidx];
      key = imod(an.x - x0 + P - 1, ag.nx);
      const bool rx = key < txv + P - 1;
      const bool ry = imod(y0 - an.y, ag.ny) < P || imod(an.y - y0, ag.ny) < tyv;
      const bool rz = imod(z0 - an.z, ag.nz) < P || imod(an.z - z0, ag.nz) < tzv;
      rel = rx && ry && rz;
    }
    // ---- bucket positions: warp match ranks + warp-ordered prefix ----
    const unsigned peers = __match_any_sync(0xffffffffu, rel ? key : NK + lane);
    const int rank = __popc(peers & lt);
    if (rel && rank == 0) kcnt[warp][key] = __popc(peers);
    __syncthreads();
    if (warp == 0) {
      int tot[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int k = lane + 32 * h;
        int run = 0;
        if (k < NK) {
#pragma unroll
          for (int w = 0; w < NW; ++w) {
            const int c = kcnt[w][k];
            kcnt[w][k] = run;
            run += c;
          }
        }
        tot[h] = run;
      }
      // exclusive scan of the bucket totals over keys 0..63
      int inc0 = tot[0], inc1 = tot[1];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u0 = __shfl_up_sync(0xffffffffu, inc0, o), u1 = __shfl_up_sync(0xffffffffu, inc1, o);
        if (lane >= o) { inc0 += u0; inc1 += u1; }
      }
      const int all0 = __shfl_sync(0xffffffffu, inc0, 31);
      const int st0 = inc0 - tot[0], st1 = all0 + inc1 - tot[1];
      if (lane < NK) kstart[lane] = st0;
      if (lane + 32 < NK) kstart[lane + 32] = st1;
      if (lane == 31) kstart[NK] = all0 + inc1;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int k = lane + 32 * h;
        if (k < NK) {
          const int s = h ? st1 : st0;
#pragma unroll
          for (int w = 0; w < NW; ++w) kcnt[w][k] += s;
        }
      }
    }
    __syncthreads();
    if (rel) {
      const int slot = kcnt[warp][key] + rank;
      T w1[KK][P];
      axis_kinds<T, P, NT>(a.spline, tf[0], w1, a.qc);
#pragma unroll
      for (int kk = 0; kk < KK; ++kk)
#pragma unroll
        for (int k = 0; k < P; ++k) c_wx[(kk * P + k) * CH + slot] = w1[kk][k];
      axis_kinds<T, P, NT>(a.spline, tf[1], w1, a.qc);
#pragma unroll
      for (int kk = 0; kk < KK; ++kk)
#pragma unroll
        for (int k = 0; k < P; ++k) c_wy[(kk * P + k) * CH + slot] = w1[kk][k];
      axis_kinds<T, P, NT>(a.spline, tf[2], w1, a.qc);
      const int dz0 = imod(z0 - an.z, ag.nz);
#pragma unroll
      for (int z = 0; z < kTileZ; ++z) {
        int d = dz0 + z;
        if (d >= ag.nz) d -= ag.nz;
#pragma unroll
        for (int kk = 0; kk < KK; ++kk) {
          T wz = T(0);
          if (z < tzv) {
#pragma unroll
            for (int k = 0; k < P; ++k) wz = (d == k) ? w1[kk][k] : wz;
          }
          c_wz[(kk * kTileZ + z) * CH + slot] = wz;
        }
      }
      c_q[slot] = qv;
      c_ay[slot] = an.y;
    }
    __syncthreads();
    // counts for the next chunk; kcnt is not read again in this one
    for (int i = threadIdx.x; i < NW * NK; i += blockDim.x) (&kcnt[0][0])[i] = 0;
    // ---- accumulate: bucket of x offset dx holds the anchors gx - dx ----
    if (own) {
#pragma unroll
      for (int dx = 0; dx < P; ++dx) {
        int k = lx + P - 1 - dx;
        if (k >= ag.nx) k -= ag.nx;
        const int jb = kstart[k], je = kstart[k + 1];
        for (int j = jb; j < je; ++j) {
          int dy = gy - c_ay[j];
          if (dy < 0) dy += ag.ny;
          if (dy >= P) continue;
          const T qj = c_q[j];
#pragma unroll
          for (int tt = 0; tt < NT; ++tt) {
            const T wxy = c_wx[(ST::x(tt) * P + dx) * CH + j] * c_wy[(ST::y(tt) * P + dy) * CH + j] * qj;
            const T *wz = c_wz + ST::z(tt) * kTileZ * CH + j;
#pragma unroll
            for (int z = 0; z < kTileZ; ++z) acc[z] += (TG)wxy * (TG)wz[z * CH];
          }
        }
      }
    }
    __syncthreads();
  }
  if (own) {
    const int gx = x0 + lx;
    const int64_t plane = (int64_t)ag.nx * ag.ny;
    TG *out = static_cast<TG *>(a.rho) + (int64_t)f * plane * a.zcnt + (int64_t)gy * ag.nx + gx;
    // the charge scale N_g / V (quads_fft.py:287) applied once, in the grid
    // type: an fp32 copy of it would scale the whole mesh energy by its
    // rounding (1e-4 of the total energy of the 1,048,576-atom system, whose
    // mesh and self terms are a thousand times the total)
    const TG scale = (TG)g.scale;
#pragma unroll
    for (int z = 0; z < kTileZ; ++z)
      if (z < tzv) out[(int64_t)(z0 - a.zlo + z) * plane] = acc[z] * scale;
  }
}

// ------------------------------------------------------------------------
// spread, separable splines: one warp per 8 x 8 x 8 block of mesh points
// ------------------------------------------------------------------------
// A warp owns one block and writes each of its points once.  Its candidates
// are the cell-sorted atoms of the (at most 3 x 3 x 3) bins that hold the
// anchors able to reach the block; lanes test 32 candidates at a time from
// their anchors alone and append the relevant ones (stencil reaching the
// block on every axis, about a third of them) to a list in candidate order.
// For each 32 listed candidates, lane j evaluates candidate j's spline
// weights (fp64) at the block's 8 x, 8 y and 8 z points (zero where the
// stencil does not reach), and every lane then adds them, in list order, to
// its 2 x 8 points (x = lane % 8, y = lane / 8 and lane / 8 + 4, all z).  So
// the summation order at every point is the fixed candidate order: bitwise
// reproducible, no atomics, and no block-wide barriers (the warps of a CTA
// are independent blocks).
constexpr int kWarpsPerSpreadCta = 4;

// Candidate segments of one 8 x 8 x 8 block, built by its warp: the runs of
// the cell-sorted atom array whose bins hold anchors able to reach the block
// (at most 3 x 3 x 3 bins; a (z, y) bin row gives at most two runs of x bins,
// two when the halo wraps), numbered in lane order.  Returns the number of
// runs; s_pre[nsg] is the candidate count.
template <typename T, int P>
__device__ __forceinline__ int blk_segments(const SpreadArgs<T> &a, int f, int x0, int y0, int z0, int xv, int yv,
                                            int zv, int lane, uint32_t *s_lo, uint32_t *s_pre, int (*s_bl)[4],
                                            int *s_nb) {
  const AtomGrid &ag = a.ag;
  if (lane < 3) {
    const int lo = (lane == 0 ? x0 : lane == 1 ? y0 : z0) - P + 1;
    const int len = (lane == 0 ? xv : lane == 1 ? yv : zv) + P - 1;
    const int n = lane == 0 ? ag.nx : lane == 1 ? ag.ny : ag.nz;
    const int nb = lane == 0 ? ag.nbx : lane == 1 ? ag.nby : ag.nbz;
    s_nb[lane] = axis_bins(lo, len, n, nb, s_bl[lane]);
  }
  __syncwarp();
  const int nxl = s_nb[0], nyl = s_nb[1], nzl = s_nb[2];
  uint32_t lo2[2] = {0, 0}, cnt2[2] = {0, 0};
  if (lane < nzl * nyl) {
    const int iz = lane / nyl, iy = lane - iz * nyl;
    const uint32_t row = (uint32_t)f * ag.bins_per_frame + bin_row(ag, s_bl[2][iz], s_bl[1][iy]);
    int brk = nxl;   // x bins are ascending with at most one break
    for (int i = 1; i < nxl; ++i)
      if (brk == nxl && s_bl[0][i] != s_bl[0][i - 1] + 1) brk = i;
    lo2[0] = a.bin_start[row + s_bl[0][0]];
    cnt2[0] = a.bin_start[row + s_bl[0][brk - 1] + 1] - lo2[0];
    if (brk < nxl) {
      lo2[1] = a.bin_start[row + s_bl[0][brk]];
      cnt2[1] = a.bin_start[row + s_bl[0][nxl - 1] + 1] - lo2[1];
    }
  }
  const int ne = (cnt2[0] > 0) + (cnt2[1] > 0);
  int eo = ne;
  uint32_t co = cnt2[0] + cnt2[1];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ue = __shfl_up_sync(0xffffffffu, eo, o);
    const uint32_t uc = __shfl_up_sync(0xffffffffu, co, o);
    if (lane >= o) { eo += ue; co += uc; }
  }
  int sg = eo - ne;
  uint32_t pre = co - (cnt2[0] + cnt2[1]);
#pragma unroll
  for (int h = 0; h < 2; ++h)
    if (cnt2[h] > 0) {
      s_lo[sg] = lo2[h];
      s_pre[sg] = pre;
      pre += cnt2[h];
      ++sg;
    }
  if (lane == 31) s_pre[eo] = co;
  const int nsg = __shfl_sync(0xffffffffu, eo, 31);   // segments in all
  __syncwarp();
  return nsg;
}

// the sorted-atom index of candidate ci (last segment with s_pre <= ci)
__device__ __forceinline__ uint32_t blk_candidate(const uint32_t *s_lo, const uint32_t *s_pre, int nsg, uint32_t ci) {
  int lo = 0, hi = nsg - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_pre[mid] <= ci) lo = mid; else hi = mid - 1;
  }
  return s_lo[lo] + (ci - s_pre[lo]);
}


template <typename T, int P, typename TG>
__global__ void __launch_bounds__(32 * kWarpsPerSpreadCta, SOG_SPREAD_BLK_MINB) k_spread_blk(SpreadArgs<T> a, int nbx, int nby,
                                                                          int nbz, int64_t nblk) {
  constexpr int kSeg = 18;
  // per warp and lane: a candidate's x (times q), y, z weights; rows of 25
  // (odd) words so that the lanes' rows start in different banks
  __shared__ TG s_w[kWarpsPerSpreadCta][32][25];
  __shared__ uint32_t s_rel[kWarpsPerSpreadCta][64];
  __shared__ uint32_t s_lo[kWarpsPerSpreadCta][kSeg], s_pre[kWarpsPerSpreadCta][kSeg + 1];
  __shared__ int s_bl[kWarpsPerSpreadCta][3][4];
  __shared__ int s_nb[kWarpsPerSpreadCta][3];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t blk = (int64_t)blockIdx.x * kWarpsPerSpreadCta + warp;
  if (blk >= nblk) return;   // the whole warp
  const AtomGrid &ag = a.ag;
  const int64_t per_f = (int64_t)nbx * nby * nbz;
  const int f = (int)(blk / per_f);
  int64_t rem = blk - (int64_t)f * per_f;
  const int bz = (int)(rem / ((int64_t)nbx * nby));
  rem -= (int64_t)bz * nbx * nby;
  const int by = (int)(rem / nbx), bx = (int)(rem - (int64_t)by * nbx);
  const int x0 = bx * 8, y0 = by * 8, z0 = a.zlo + bz * 8;
  const int xv = min(8, ag.nx - x0), yv = min(8, ag.ny - y0), zv = min(8, a.zlo + a.zcnt - z0);
  // ---- segments of the sorted atom array holding the candidates ----
  const int nsg = blk_segments<T, P>(a, f, x0, y0, z0, xv, yv, zv, lane, s_lo[warp], s_pre[warp], s_bl[warp],
                                     s_nb[warp]);
  const uint32_t ncand = s_pre[warp][nsg];
  const int xl = lane & 7, yl0 = lane >> 3, yl1 = yl0 + 4;
  const int base[3] = {x0, y0, z0}, lim[3] = {xv, yv, zv}, nn[3] = {ag.nx, ag.ny, ag.nz};
  TG acc0[8], acc1[8];
#pragma unroll
  for (int z = 0; z < 8; ++z) { acc0[z] = TG(0); acc1[z] = TG(0); }
  // Weights of the first cnt relevant candidates (lane j: candidate j), then
  // their sums into this lane's points in list order.
  auto flush = [&](int cnt) {
    if (lane < cnt) {
      const uint32_t sidx = s_rel[warp][lane];
      const int4 an = a.s_anchor[sidx];
      const int anc[3] = {an.x, an.y, an.z};
      const double qv = (double)a.s_q[sidx];
      TG *w = s_w[warp][lane];   // x weights (times q), y, z
#pragma unroll
      for (int ax = 0; ax < 3; ++ax) {
        double w1[P];
        spline_w<double, P>(a.spline, (double)a.s_t[(int64_t)sidx * 3 + ax], w1, a.qc);
        if (ax == 0) {
#pragma unroll
          for (int jj = 0; jj < P; ++jj) w1[jj] *= qv;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) w[ax * 8 + i] = TG(0);
        // stencil node jj sits at block point (jj - k) mod n
        int k = base[ax] - anc[ax];
        if (k < 0) k += nn[ax];
#pragma unroll
        for (int jj = 0; jj < P; ++jj) {
          int i = jj - k;
          if (i < 0) i += nn[ax];
          if (i < lim[ax]) w[ax * 8 + i] = (TG)w1[jj];
        }
      }
    }
    __syncwarp();
    for (int j = 0; j < cnt; ++j) {
      const TG *wj = s_w[warp][j];
      const TG a0 = wj[xl] * wj[8 + yl0], a1 = wj[xl] * wj[8 + yl1];
#pragma unroll
      for (int z = 0; z < 8; ++z) {
        const TG wzz = wj[16 + z];
        acc0[z] += a0 * wzz;
        acc1[z] += a1 * wzz;
      }
    }
    __syncwarp();
  };
  // Relevant candidates (stencil reaches the block on every axis: the offset
  // k of block point 0 is below P, or the block wraps onto node 0), decided
  // from the anchors alone and listed in candidate order; weights are
  // computed for listed candidates only, 32 at a time.
  const unsigned lt = (1u << lane) - 1u;
  int nrel = 0;
  for (uint32_t c0 = 0; c0 < ncand; c0 += 32) {
    const uint32_t ci = c0 + lane;
    bool rel = false;
    uint32_t sidx = 0;
    if (ci < ncand) {
      sidx = blk_candidate(s_lo[warp], s_pre[warp], nsg, ci);
      const int4 an = a.s_anchor[sidx];
      const int anc[3] = {an.x, an.y, an.z};
      rel = true;
#pragma unroll
      for (int ax = 0; ax < 3; ++ax) {
        int k = base[ax] - anc[ax];
        if (k < 0) k += nn[ax];
        rel = rel && (k < P || k > nn[ax] - lim[ax]);
      }
    }
    const unsigned mask = __ballot_sync(0xffffffffu, rel);
    if (rel) s_rel[warp][nrel + __popc(mask & lt)] = sidx;
    nrel += __popc(mask);
    __syncwarp();
    if (nrel >= 32) {
      flush(32);
      if (lane < nrel - 32) s_rel[warp][lane] = s_rel[warp][32 + lane];   // disjoint halves
      nrel -= 32;
      __syncwarp();
    }
  }
  if (nrel > 0) flush(nrel);
  const int64_t plane = (int64_t)ag.nx * ag.ny;
  TG *out = static_cast<TG *>(a.rho) + (int64_t)f * plane * a.zcnt;
  const TG scale = (TG)a.geom[f].scale;
  if (xl < xv) {
#pragma unroll
    for (int z = 0; z < 8; ++z) {
      if (z >= zv) break;
      const int64_t zo = (int64_t)(z0 - a.zlo + z) * plane + x0 + xl;
      if (yl0 < yv) out[zo + (int64_t)(y0 + yl0) * ag.nx] = acc0[z] * scale;
      if (yl1 < yv) out[zo + (int64_t)(y0 + yl1) * ag.nx] = acc1[z] * scale;
    }
  }
}

// ------------------------------------------------------------------------
// Hessian-vector products: the direction density
// ------------------------------------------------------------------------
// The derivative of the charge mesh along a direction (a on the charges of
// channel `channel`, b on the positions):
//   drho(g) = (N_g / V) sum_j [a_j W_j(g) + q_j sum_x bt_jx dW_j/du_x(g)],
//   bt_jx = n_x sum_c b_jc (cell^-1)_cx   (the direction in mesh units),
// with the warp-per-block candidate walk and fixed summation order of
// k_spread_blk.  A candidate's weight is the sum of three separable terms,
//   (a w_x + q bt_x w_x') w_y w_z + w_x (q bt_y w_y') w_z + w_x w_y (q bt_z w_z'),
// so a lane stages six rows of eight (rows of 49 words: odd, bank-spread).
constexpr int kWarpsPerDipCta = 2;

template <typename T, int P>
__global__ void __launch_bounds__(32 * kWarpsPerDipCta) k_spread_dip(SpreadArgs<T> a, int nbx, int nby, int nbz,
                                                                     int64_t nblk) {
  __shared__ double s_w[kWarpsPerDipCta][32][49];
  __shared__ uint32_t s_lo[kWarpsPerDipCta][18], s_pre[kWarpsPerDipCta][19];
  __shared__ int s_bl[kWarpsPerDipCta][3][4];
  __shared__ int s_nb[kWarpsPerDipCta][3];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t blk = (int64_t)blockIdx.x * kWarpsPerDipCta + warp;
  if (blk >= nblk) return;   // the whole warp
  const AtomGrid &ag = a.ag;
  const int64_t per_f = (int64_t)nbx * nby * nbz;
  const int f = (int)(blk / per_f);
  int64_t rem = blk - (int64_t)f * per_f;
  const int bz = (int)(rem / ((int64_t)nbx * nby));
  rem -= (int64_t)bz * nbx * nby;
  const int by = (int)(rem / nbx), bx = (int)(rem - (int64_t)by * nbx);
  const int x0 = bx * 8, y0 = by * 8, z0 = a.zlo + bz * 8;
  const int xv = min(8, ag.nx - x0), yv = min(8, ag.ny - y0), zv = min(8, a.zlo + a.zcnt - z0);
  const int nsg = blk_segments<T, P>(a, f, x0, y0, z0, xv, yv, zv, lane, s_lo[warp], s_pre[warp], s_bl[warp],
                                     s_nb[warp]);
  const uint32_t ncand = s_pre[warp][nsg];
  const FrameGeom &g = a.geom[f];
  const double n3[3] = {(double)ag.nx, (double)ag.ny, (double)ag.nz};
  const int xl = lane & 7, yl0 = lane >> 3, yl1 = yl0 + 4;
  double acc0[8], acc1[8];
#pragma unroll
  for (int z = 0; z < 8; ++z) { acc0[z] = 0.0; acc1[z] = 0.0; }
  for (uint32_t c0 = 0; c0 < ncand; c0 += 32) {
    const uint32_t ci = c0 + lane;
    bool rel = false;
    double *w = s_w[warp][lane];   // rows: w_x, X, w_y, Y, w_z, Z
    if (ci < ncand) {
      const uint32_t sidx = blk_candidate(s_lo[warp], s_pre[warp], nsg, ci);
      const int4 an = a.s_anchor[sidx];
      const int anc[3] = {an.x, an.y, an.z};
      const int base[3] = {x0, y0, z0}, lim[3] = {xv, yv, zv}, nn[3] = {ag.nx, ag.ny, ag.nz};
      const int64_t atom = a.s_atom[sidx];
      const double qv = (double)a.s_q[sidx];
      const double av = ldir<T>(a.dir_q, atom * a.nch + a.channel);
      double br[3], bt[3];
#pragma unroll
      for (int c = 0; c < 3; ++c) br[c] = ldir<T>(a.dir_r, atom * 3 + c);
#pragma unroll
      for (int ax = 0; ax < 3; ++ax)
        bt[ax] = n3[ax] * (br[0] * g.cinv[0 * 3 + ax] + br[1] * g.cinv[1 * 3 + ax] + br[2] * g.cinv[2 * 3 + ax]);
      bool has = true;
#pragma unroll
      for (int ax = 0; ax < 3; ++ax) {
        double w1[P], d1[P];
        const double t = (double)a.s_t[(int64_t)sidx * 3 + ax];
        spline_w<double, P>(a.spline, t, w1, a.qc);
        spline_dw<P>(a.spline, t, d1, a.qc);
        const double cd = qv * bt[ax], cw = ax == 0 ? av : 0.0;
        int k = base[ax] - anc[ax];
        if (k < 0) k += nn[ax];
        bool h = false;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          double vw = 0.0, vd = 0.0;
#pragma unroll
          for (int jj = 0; jj < P; ++jj) {
            vw = (k == jj) ? w1[jj] : vw;
            vd = (k == jj) ? d1[jj] : vd;
          }
          const bool in = i < lim[ax];
          h |= (k < P && in);
          w[ax * 16 + i] = in ? vw : 0.0;
          w[ax * 16 + 8 + i] = in ? cw * vw + cd * vd : 0.0;
          if (++k == nn[ax]) k = 0;
        }
        has = has && h;
      }
      rel = has;
    }
    unsigned mask = __ballot_sync(0xffffffffu, rel);
    __syncwarp();
    while (mask) {   // the relevant candidates in lane order
      const int j = __ffs(mask) - 1;
      mask &= mask - 1u;
      const double *wj = s_w[warp][j];
      const double wx = wj[xl], X = wj[8 + xl];
      const double a0 = X * wj[16 + yl0] + wx * wj[24 + yl0], b0 = wx * wj[16 + yl0];
      const double a1 = X * wj[16 + yl1] + wx * wj[24 + yl1], b1 = wx * wj[16 + yl1];
#pragma unroll
      for (int z = 0; z < 8; ++z) {
        const double wzz = wj[32 + z], Zz = wj[40 + z];
        acc0[z] += a0 * wzz + b0 * Zz;
        acc1[z] += a1 * wzz + b1 * Zz;
      }
    }
    __syncwarp();
  }
  const int64_t plane = (int64_t)ag.nx * ag.ny;
  double *out = static_cast<double *>(a.rho) + (int64_t)f * plane * a.zcnt;
  const double scale = g.scale;
  if (xl < xv) {
#pragma unroll
    for (int z = 0; z < 8; ++z) {
      if (z >= zv) break;
      const int64_t zo = (int64_t)(z0 - a.zlo + z) * plane + x0 + xl;
      if (yl0 < yv) out[zo + (int64_t)(y0 + yl0) * ag.nx] = acc0[z] * scale;
      if (yl1 < yv) out[zo + (int64_t)(y0 + yl1) * ag.nx] = acc1[z] * scale;
    }
  }
}

// ------------------------------------------------------------------------
// k-space
// ------------------------------------------------------------------------
template <typename T>
struct KsArgs {
  const cplx_t<T> *spec;   // [nf][nh]
  // [nf][F][nh] field spectra; complex of the field type the writing kernel
  // is instantiated with (its TO: T itself, or float for the fp32 field path
  // of an fp32 plan whose spectrum is fp64)
  void *fspec;
  const FrameGeom *geom;
  const double *tx, *ty, *tz;  // per-axis Green factors
  const double *sx, *sy, *sz;  // B-spline alias sums
  const void *amp, *bw2;   // [M] kernel parameters: float when p32, else double
  int p32;
  int M, spline, order, alias_extent;
  int nx, ny, nz, nxh;
  int64_t nh;
  int nfield;              // 0, 3 or 4
  int want_force;
  double *part;            // [nf][gridDim.x][2]
  double *partx;           // [nf][gridDim.x][NX] extras
  int nx_acc;
  // separable kernel factors exp(-bw2_m k_a^2 / 2) per axis for orthorhombic
  // frames: per frame [M][nxh] (x), [M][ny] (y), [M][nz] (z)
  const double *btab;
  int64_t btab_stride;
  // Green tables [nf][nh]: gE (energy / potential) and, for frames whose
  // B-spline aliases fall inside the cutoff, gF (ik forces)
  double *gtab, *gtabF;
  double *partD;           // [nf][gridDim.z * gridDim.x] self-sum partials of k_green
  // y slab of the half spectrum held by this call (k_green, k_zfused_g): rows
  // y0 .. y0+nyl-1 of ny; the spectrum, tables and fields are [nz][nyl][nxh]
  int y0, nyl;
  // k_zfused_g writes the fields of z planes [b*zblk, (b+1)*zblk) as block b
  // of [nz/zblk][nfield][zblk][nyl][nxh] (zblk = nz: plain [nfield][nz][..]);
  // with zdst[0] set, block b goes to zdst[b] + [nfield][zblk][nyl][nxh]
  // instead (the receive buffer of rank b, possibly on another GPU)
  int zblk;
  void *zdst[kMaxSlabRanks];
  // column layout of the spectrum rows held by this call: 0 = plain
  // (col = y*nxh + mx); cw > 0 = chunked (col = (xc*nyl + y)*cw + xw,
  // mx = xc*cw + xw), the receive layout of the peer slab transport in which
  // one tile of cw columns is contiguous for every z; with cw > 0 the fields
  // of z block b go to zdst[b] as [nfield][xc*nyl + y][zblk][cw]
  int cw;
  // Radial kernel tables [nf][krad_stride] of cubic frames (green_radial),
  // or null: K(k) = sum_m amp_m exp(-bw2_m k^2 / 2) with k^2 = kappa^2 s, s =
  // mx^2 + my^2 + mz^2, so one fp64 value per integer s serves every mode.
  // The fused z pass then evaluates those frames' Green function from it
  // (times the per-axis deconvolution) and sums their self term itself;
  // k_green builds the tables of the other frames only.
  const double *krad;
  int64_t krad_stride;
  // 1: the fused z pass stores Y1 / Y2 of orthorhombic frames in field slots
  // 0 / 2 for k_cols_fields (single-device calls with forces)
  int two_slot;
};

// kernel parameter m as a double
__device__ __forceinline__ double kpar(const void *p, int p32, int m) {
  return p32 ? (double)static_cast<const float *>(p)[m] : static_cast<const double *>(p)[m];
}

// complex value converted to the field type TO
template <typename TO, typename C>
__device__ __forceinline__ cplx_t<TO> to_field(const C &v) {
  return cmk<cplx_t<TO>, TO>((TO)v.x, (TO)v.y);
}

// Frames whose Green function is separable: orthorhombic, no B-spline alias
// inside the cutoff, at most 16 Gaussians, not CubeS2 (its variance
// subtraction is not a per-axis product over the Cartesian components it uses)
template <typename T>
__device__ __forceinline__ bool green_separable(const KsArgs<T> &a, const FrameGeom &g) {
  return g.ortho && a.btab && !g.pad && a.M <= 16 && a.spline != SOG_SPLINE_CUBES2;
}

// Cubic frames (one wave-vector scale on all three axes, no alias inside the
// cutoff, not CubeS2) whose kernel comes from the radial table.
template <typename T>
__device__ __forceinline__ bool green_radial(const KsArgs<T> &a, const FrameGeom &g) {
  return a.krad && g.ortho && !g.pad && a.spline != SOG_SPLINE_CUBES2 && g.kmat[0] == g.kmat[4] &&
         g.kmat[4] == g.kmat[8];
}

// Radial kernel table of every cubic frame: entry s = sum_m amp_m exp(-bw2_m
// kappa^2 s / 2), s = 0 .. krad_stride - 1.
template <typename T>
__global__ void k_radial_table(KsArgs<T> a) {
  const int f = blockIdx.y;
  const FrameGeom &g = a.geom[f];
  if (!green_radial(a, g)) return;
  const double k2 = g.kmat[0] * g.kmat[0];
  double *out = const_cast<double *>(a.krad) + (int64_t)f * a.krad_stride;
  for (int64_t sidx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; sidx < a.krad_stride;
       sidx += (int64_t)gridDim.x * blockDim.x) {
    const double ksq = k2 * (double)sidx;
    double K = 0.0;
    for (int m = 0; m < a.M; ++m) K += kpar(a.amp, a.p32, m) * exp(-0.5 * kpar(a.bw2, a.p32, m) * ksq);
    out[sidx] = K;
  }
}

// Column `col` of the spectrum rows -> (mx, local y); false for the pad
// columns (mx >= nx/2+1) of the chunked layout.
template <typename T>
__device__ __forceinline__ bool col_mode(const KsArgs<T> &a, int64_t col, int &mx, int &yl) {
  if (a.cw == 0) {
    mx = (int)(col % a.nxh);
    yl = (int)(col / a.nxh);
    return true;
  }
  const int64_t q = col / a.cw;
  const int xw = (int)(col - q * a.cw);
  const int xc = (int)(q / a.nyl);
  yl = (int)(q - (int64_t)xc * a.nyl);
  mx = xc * a.cw + xw;
  return mx < a.nxh;
}

// columns per z plane of the spectrum rows held by this call
template <typename T>
__host__ __device__ __forceinline__ int64_t cols_inner(const KsArgs<T> &a) {
  return a.cw == 0 ? (int64_t)a.nyl * a.nxh : (int64_t)((a.nxh + a.cw - 1) / a.cw) * a.nyl * a.cw;
}

// Per-axis Gaussian factors of the frame (the per-axis tables of
// lmp/sog.cpp:1391-1430): K(k^2) = sum_m amp_m Bx_m By_m Bz_m when k_a
// depends on m_a only.
template <typename T>
__global__ void k_axis_tables(const FrameGeom *__restrict__ geom, const T *__restrict__ bw2, int M, int nx,
                              int ny, int nz, double *__restrict__ btab) {
  const int f = blockIdx.y;
  const FrameGeom &g = geom[f];
  if (!g.ortho) return;
  const int nxh = nx / 2 + 1;
  const int per = nxh + ny + nz;
  const int64_t total = (int64_t)M * per;
  double *bt = btab + (int64_t)f * total;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    int i = (int)idx, axis, m;
    double k;
    if (i < M * nxh) {
      m = i / nxh; const int mx = i - m * nxh; axis = 0; k = g.kmat[0] * mx;
    } else if (i < M * (nxh + ny)) {
      i -= M * nxh; m = i / ny; const int iy = i - m * ny; axis = 1; k = g.kmat[4] * signed_mode(iy, ny);
    } else {
      i -= M * (nxh + ny); m = i / nz; const int iz = i - m * nz; axis = 2; k = g.kmat[8] * signed_mode(iz, nz);
    }
    (void)axis;
    bt[idx] = exp(-0.5 * (double)bw2[m] * k * k);
  }
}

// Green factors of one half-spectrum mode.
struct ModeGreen {
  double k[3], ksq, K, Kv, gE, gF, gS, gV;
  bool live;
};

__device__ __forceinline__ double sinc2p_dev(int mode, int n, int order, int j) {
  const double arg = kPi * (double)mode / (double)n + kPi * (double)j;
  const double s = fabs(arg) < 1e-14 ? 1.0 : sin(arg) / arg;
  double r = 1.0;
  for (int i = 0; i < 2 * order; ++i) r *= s;
  return r;
}

template <typename T>
__device__ __forceinline__ double kernel_sum(const double *amp, const double *bw2, int M, double ksq,
                                             double *Kv) {
  double K = 0.0, V = 0.0;
  for (int m = 0; m < M; ++m) {
    const double e = exp(-0.5 * bw2[m] * ksq);
    K += amp[m] * e;
    V += amp[m] * bw2[m] * e;
  }
  *Kv = V;
  return K;
}

// Per-Gaussian factors of a mode without alias sums: exp(-bw2 k^2 / 2) times
// the deconvolution D (gE) or alone (gS), and their bw2 derivatives.
__device__ __forceinline__ void principal_em(double bw2m, double ksq, double D, double *em) {
  const double e = exp(-0.5 * bw2m * ksq), h = -0.5 * ksq;
  em[0] = e * D;
  em[1] = e;
  em[2] = h * em[0];
  em[3] = h * e;
  em[4] = h * em[2];
  em[5] = h * em[3];
}

// B-spline alias sums of lmp/sog.cpp:1516-1578, pruned to the aliases that
// can fall inside the k_max sphere (rarely taken, kept out of line).
template <typename T>
__device__ __noinline__ void alias_green(const KsArgs<T> &a, const FrameGeom &g, const double *amp,
                                         const double *bw2, int mx, int my, int mz, int iy, int iz,
                                         int mfor, double *em, ModeGreen &r) {
  const double dl = a.sx[mx] * a.sy[iy] * a.sz[iz];
  const double denom = dl * dl;
  const int m3[3] = {mx, my, mz};
  const int n3[3] = {a.nx, a.ny, a.nz};
  int jlo[3], jhi[3];
  for (int c = 0; c < 3; ++c) {
    int lo = (int)ceil((-g.abound[c] - (double)m3[c]) / (double)n3[c]);
    int hi = (int)floor((g.abound[c] - (double)m3[c]) / (double)n3[c]);
    lo = max(min(lo, 0), -a.alias_extent);
    hi = min(max(hi, 0), a.alias_extent);
    jlo[c] = lo;
    jhi[c] = hi;
  }
  const double w0 = sinc2p_dev(mx, a.nx, a.order, 0) * sinc2p_dev(my, a.ny, a.order, 0) *
                    sinc2p_dev(mz, a.nz, a.order, 0);
  double s0 = 0.0, s1 = 0.0, sv = 0.0;
  double e6[6] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0};
  for (int jx = jlo[0]; jx <= jhi[0]; ++jx)
    for (int jy = jlo[1]; jy <= jhi[1]; ++jy)
      for (int jz = jlo[2]; jz <= jhi[2]; ++jz) {
        const double ax = mx + a.nx * jx, ay = my + a.ny * jy, az = mz + a.nz * jz;
        double q[3];
        for (int c = 0; c < 3; ++c) q[c] = g.kmat[c * 3 + 0] * ax + g.kmat[c * 3 + 1] * ay + g.kmat[c * 3 + 2] * az;
        const double qsq = q[0] * q[0] + q[1] * q[1] + q[2] * q[2];
        if (!(qsq > 0.0 && qsq <= g.k_sq_max)) continue;
        double Kvq;
        const double Kq = kernel_sum<T>(amp, bw2, a.M, qsq, &Kvq);
        const double wp = sinc2p_dev(mx, a.nx, a.order, jx) * sinc2p_dev(my, a.ny, a.order, jy) *
                          sinc2p_dev(mz, a.nz, a.order, jz);
        s0 += Kq * wp;
        s1 += (r.k[0] * q[0] + r.k[1] * q[1] + r.k[2] * q[2]) * Kq * wp;
        sv += Kvq * wp;
        if (em) {
          // d/d bw2_m of an alias term brings its own -|q|^2 / 2
          const double e = exp(-0.5 * bw2[mfor] * qsq);
          const double eDq = e * wp / denom, eSq = (w0 > 1e-20) ? e * wp / w0 : 0.0;
          const double h = -0.5 * qsq;
          e6[0] += eDq; e6[1] += eSq;
          e6[2] += h * eDq; e6[3] += h * eSq;
          e6[4] += h * h * eDq; e6[5] += h * h * eSq;
        }
      }
  r.gE = s0 / denom;
  r.gF = s1 / (r.ksq * denom);
  r.gS = (w0 > 1e-20) ? s0 / w0 : 0.0;
  r.gV = sv / denom;
  if (em)
    for (int i = 0; i < 6; ++i) em[i] = e6[i];
}

// Green function of a mode; with `alias` the B-spline alias sums of
// lmp/sog.cpp:1516-1578 (pruned to aliases inside the k_max sphere), else the
// principal (separable) form.  If em is given, the per-Gaussian factors of
// Gaussian mfor are returned too: em[0] = d gE / d amp_m, em[1] = d gS / d amp_m,
// em[2..3] their first and em[4..5] their second derivatives w.r.t. bw2_m.
template <typename T>
__device__ ModeGreen mode_green(const KsArgs<T> &a, const FrameGeom &g, const double *amp,
                                const double *bw2, int mx, int iy, int iz, int mfor, double *em,
                                const double *bt = nullptr) {
  ModeGreen r;
  const int my = signed_mode(iy, a.ny), mz = signed_mode(iz, a.nz);
  for (int c = 0; c < 3; ++c)
    r.k[c] = g.kmat[c * 3 + 0] * mx + g.kmat[c * 3 + 1] * my + g.kmat[c * 3 + 2] * mz;
  r.ksq = r.k[0] * r.k[0] + r.k[1] * r.k[1] + r.k[2] * r.k[2];
  r.live = !((mx | my | mz) == 0) && r.ksq <= g.k_sq_max;
  r.K = r.Kv = r.gE = r.gF = r.gS = r.gV = 0.0;
  if (!r.live) return r;
  if (bt) {
    const int nxh = a.nxh;
    const double *bx = bt, *by = bt + a.M * nxh, *bz = by + a.M * a.ny;
    double K = 0.0, V = 0.0;
    for (int m = 0; m < a.M; ++m) {
      const double e = bx[m * nxh + mx] * by[m * a.ny + iy] * bz[m * a.nz + iz];
      K += amp[m] * e;
      V += amp[m] * bw2[m] * e;
    }
    r.K = K;
    r.Kv = V;
  } else {
    r.K = kernel_sum<T>(amp, bw2, a.M, r.ksq, &r.Kv);
  }
  if (a.spline == SOG_SPLINE_CUBES2) {
    // variance subtraction: G = K exp(sum_a sig_a^2 k_a^2) over the Cartesian
    // components (cubes2_fft.py:1039-1049); no aliasing, no deconvolution
    const double D = exp(g.sig2[0] * r.k[0] * r.k[0] + g.sig2[1] * r.k[1] * r.k[1] + g.sig2[2] * r.k[2] * r.k[2]);
    r.gE = r.gF = r.K * D;
    r.gS = r.K;
    r.gV = r.Kv * D;
    if (em) principal_em(bw2[mfor], r.ksq, D, em);
    return r;
  }
  if (a.spline == SOG_SPLINE_QUADS) {
    double infl = a.tx[mx] * a.ty[iy] * a.tz[iz];
    if (infl < 1e-20) infl = 1e-20;  // quads_fft.py:194
    const double D = 1.0 / infl;
    r.gE = r.gF = r.K * D;
    r.gS = r.K;
    r.gV = r.Kv * D;
    if (em) principal_em(bw2[mfor], r.ksq, D, em);
    return r;
  }
  if (!g.pad) {
    const double D = a.tx[mx] * a.ty[iy] * a.tz[iz];
    r.gE = r.gF = r.K * D;
    r.gS = r.K;
    r.gV = r.Kv * D;
    if (em) principal_em(bw2[mfor], r.ksq, D, em);
    return r;
  }
  alias_green<T>(a, g, amp, bw2, mx, my, mz, iy, iz, mfor, em, r);
  return r;
}


// k-space step with the Green function read from k_green's tables (any nz):
// thread per (iy, mx) column walking its share of the z planes, energy
// partial sum and the ik / potential field spectra.  Same arithmetic as the
// field step of k_zfused_g.
template <typename T, typename TO = T>
__global__ void __launch_bounds__(256) k_kspace_tab(KsArgs<T> a) {
  using C = cplx_t<T>;
  using CO = cplx_t<TO>;
  __shared__ double red[8];
  const int f = blockIdx.y;
  const FrameGeom &g = a.geom[f];
  const int64_t inner = (int64_t)a.ny * a.nxh;
  const int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int zper = (a.nz + gridDim.z - 1) / gridDim.z;
  const int izb = blockIdx.z * zper, ize = min(a.nz, izb + zper);
  double accE = 0.0;
  if (col < inner) {
    const int iy = (int)(col / a.nxh), mx = (int)(col - (int64_t)iy * a.nxh);
    const int my = signed_mode(iy, a.ny);
    const double w = (mx == 0 || ((a.nx & 1) == 0 && mx == a.nx / 2)) ? 1.0 : 2.0;
    const double inv = 1.0 / ((double)a.nx * a.ny * a.nz);
    const C *sp = a.spec + (int64_t)f * a.nh + col;
    const double *ge = a.gtab + (int64_t)f * a.nh + col;
    const double *gf = (g.pad && a.gtabF) ? a.gtabF + (int64_t)f * a.nh + col : nullptr;
    CO *out = a.nfield ? static_cast<CO *>(a.fspec) + (int64_t)f * a.nfield * a.nh + col : nullptr;
    double kxy[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) kxy[c] = g.kmat[c * 3 + 0] * mx + g.kmat[c * 3 + 1] * my;
    for (int iz = izb; iz < ize; ++iz) {
      const int64_t o = (int64_t)iz * inner;
      const C r = sp[o];
      const double gE = ge[o];
      const double rr = (double)r.x, ri = (double)r.y;
      accE += w * gE * (rr * rr + ri * ri);
      if (out) {
        int fo = 0;
        if (a.want_force) {
          const double gF = gf ? gf[o] : gE;
          const double sre = gF * inv * rr, sim = gF * inv * ri;
          const int mz = signed_mode(iz, a.nz);
#pragma unroll
          for (int c = 0; c < 3; ++c) {
            const double kc = kxy[c] + g.kmat[c * 3 + 2] * mz;
            out[(int64_t)c * a.nh + o] = cmk<CO, TO>((TO)(-kc * sim), (TO)(kc * sre));
          }
          fo = 3;
        }
        if (a.nfield > fo) out[(int64_t)fo * a.nh + o] = cmk<CO, TO>((TO)(gE * inv * rr), (TO)(gE * inv * ri));
      }
    }
  }
  accE = warp_sum(accE);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = accE;
  __syncthreads();
  if (threadIdx.x == 0) {
    double e = 0.0;
    for (int wi = 0; wi < (int)(blockDim.x >> 5); ++wi) e += red[wi];
    double *p = a.part + ((int64_t)f * gridDim.z * gridDim.x + (int64_t)blockIdx.z * gridDim.x + blockIdx.x) * 2;
    p[0] = e;
    p[1] = 0.0;
  }
}

// Fused z pass for a power-of-two nz: forward z-FFT of a tile of ic spectrum
// columns, the k-space step of k_kspace on the registers, and the inverse z-FFT
// of every output field, so neither the z-transformed spectrum nor the field
// spectra make an extra round trip through HBM.  Energy / self partial sums per
// CTA go to a.part[(f*nchunks + chunk)*2].  With write_spec the transformed
// spectrum is also stored (for k_kspace_extra).
template <typename T, typename TO = T>
__global__ void __launch_bounds__(256, 2) k_zfused(KsArgs<T> a, int ic, RadixPlan rpz,
                                                 const cplx_t<T> *__restrict__ twz, int write_spec) {
  using C = cplx_t<T>;
  using CO = cplx_t<TO>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  C *sm = reinterpret_cast<C *>(smem_raw);
  __shared__ double s_amp[kMaxGauss], s_bw2[kMaxGauss];
  __shared__ double red[2][32];
  for (int m = threadIdx.x; m < a.M; m += blockDim.x) {
    s_amp[m] = kpar(a.amp, a.p32, m);
    s_bw2[m] = kpar(a.bw2, a.p32, m);
  }
  __syncthreads();
  const int n = rpz.n, TPT = n / kEPT;
  const int c = threadIdx.x % ic, t = threadIdx.x / ic;
  const int64_t inner = (int64_t)a.ny * a.nxh;
  const int64_t nchunks = (inner + ic - 1) / ic;
  const int f = (int)(blockIdx.x / nchunks);
  const int64_t chunk = blockIdx.x - (int64_t)f * nchunks;
  const int64_t col = chunk * ic + c;
  const bool ok = col < inner;
  const FrameGeom &g = a.geom[f];
  C *sp = const_cast<C *>(a.spec) + (int64_t)f * a.nh + (ok ? col : 0);
  C v[kEPT];
#pragma unroll
  for (int e = 0; e < kEPT; ++e) v[e] = ok ? sp[(int64_t)(t + e * TPT) * inner] : cmk<C, T>(T(0), T(0));
  reg_fft<T, -1, true>(v, t, rpz, twz, sm + c, ic);
  if (write_spec && ok) {
#pragma unroll
    for (int e = 0; e < kEPT; ++e) sp[(int64_t)(t + e * TPT) * inner] = v[e];
  }
  // keep rho-hat and the two Green scalars of the thread's modes in shared
  // memory (after the FFT buffer) so the field loop runs with few registers
  const int nthr = blockDim.x;
  C *s_rho = sm + (size_t)padded_row(n) * ic;                       // [kEPT][nthr]
  double *s_g = reinterpret_cast<double *>(s_rho + (size_t)kEPT * nthr);  // [kEPT][2][nthr]
  const int mx = ok ? (int)(col % a.nxh) : 0;
  const int iy = ok ? (int)(col / a.nxh) : 0;
  const int my = signed_mode(iy, a.ny);
  const double w = (mx == 0 || ((a.nx & 1) == 0 && mx == a.nx / 2)) ? 1.0 : 2.0;
  const double inv = 1.0 / ((double)a.nx * a.ny * a.nz);
  double accE = 0.0, accD = 0.0;
  const double *bt = (g.ortho && a.btab) ? a.btab + (int64_t)f * a.btab_stride : nullptr;
#pragma unroll
  for (int e = 0; e < kEPT; ++e) s_rho[e * nthr + threadIdx.x] = v[e];
#pragma unroll 1
  for (int e = 0; e < kEPT; ++e) {
    const int iz = t + e * TPT;
    const ModeGreen mg = mode_green<T>(a, g, s_amp, s_bw2, mx, iy, iz, 0, nullptr, bt);
    const bool live = ok && mg.live;
    const C r = s_rho[e * nthr + threadIdx.x];
    if (live) {
      const double rr = (double)r.x, ri = (double)r.y;
      accE += w * mg.gE * (rr * rr + ri * ri);
      accD += w * mg.gS;
    }
    s_g[(2 * e) * nthr + threadIdx.x] = live ? mg.gF * inv : 0.0;
    s_g[(2 * e + 1) * nthr + threadIdx.x] = live ? mg.gE * inv : 0.0;
  }
  const int nfield = a.nfield;
  CO *out = a.fspec ? static_cast<CO *>(a.fspec) + (int64_t)f * nfield * a.nh + (ok ? col : 0) : nullptr;
  for (int fl = 0; fl < nfield; ++fl) {
    const bool force = a.want_force && fl < 3;
    double km = 0.0, kz = 0.0;
    if (force) {
      km = g.kmat[fl * 3 + 0] * mx + g.kmat[fl * 3 + 1] * my;
      kz = g.kmat[fl * 3 + 2];
    }
    C wv[kEPT];
#pragma unroll
    for (int e = 0; e < kEPT; ++e) {
      const C r = s_rho[e * nthr + threadIdx.x];
      const double rr = (double)r.x, ri = (double)r.y;
      if (force) {
        const double kc = km + kz * signed_mode(t + e * TPT, a.nz);
        const double sc = s_g[(2 * e) * nthr + threadIdx.x];
        wv[e] = cmk<C, T>((T)(-kc * sc * ri), (T)(kc * sc * rr));
      } else {
        const double sc = s_g[(2 * e + 1) * nthr + threadIdx.x];
        wv[e] = cmk<C, T>((T)(sc * rr), (T)(sc * ri));
      }
    }
    reg_fft<T, +1, true>(wv, t, rpz, twz, sm + c, ic);
    if (ok) {
      CO *o = out + (int64_t)fl * a.nh;
#pragma unroll
      for (int e = 0; e < kEPT; ++e) o[(int64_t)(t + e * TPT) * inner] = to_field<TO>(wv[e]);
    }
  }
  accE = warp_sum(accE);
  accD = warp_sum(accD);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { red[0][warp] = accE; red[1][warp] = accD; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double e = 0.0, d = 0.0;
    for (int wi = 0; wi < (int)(blockDim.x >> 5); ++wi) { e += red[0][wi]; d += red[1][wi]; }
    double *p = a.part + ((int64_t)f * nchunks + chunk) * 2;
    p[0] = e;
    p[1] = d;
  }
}

// Green tables: one thread per half-spectrum mode writes gE(k) (and gF(k)
// for alias frames) and the block's share of the self sum sum_w gS.  The
// Green function depends on the box and the kernel parameters only, so the
// fused z pass below just streams it next to the spectrum.
// SEP: the separable fast path (orthorhombic frames without aliases inside
// the cutoff, M <= 16); !SEP: every other frame.  Both are launched on the
// same grid and each leaves the frames of the other, so the fast path gets
// a register allocation of its own.
template <typename T, bool SEP>
__global__ void __launch_bounds__(256) k_green(KsArgs<T> a) {
  extern __shared__ __align__(16) double s_bzt[];   // separable path: [z][m] z factors
  __shared__ double s_amp[kMaxGauss], s_bw2[kMaxGauss];
  __shared__ double red[8];
  for (int m = threadIdx.x; m < a.M; m += blockDim.x) {
    s_amp[m] = kpar(a.amp, a.p32, m);
    s_bw2[m] = kpar(a.bw2, a.p32, m);
  }
  __syncthreads();
  const int f = blockIdx.y;
  const FrameGeom &g = a.geom[f];
  // block-uniform: radial frames belong to the fused z pass (which sums
  // their self term: a zero partial here, written by one of the two
  // launches), separable ones to the SEP launch, the rest to the other
  if (green_radial(a, g)) {
    if (!SEP && threadIdx.x == 0) a.partD[((int64_t)f * gridDim.z + blockIdx.z) * gridDim.x + blockIdx.x] = 0.0;
    return;
  }
  const bool sep = green_separable(a, g);
  if (sep != SEP) return;
  const int64_t inner = cols_inner(a);
  const int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // (iy, mx) column
  // z planes of this block: the columns are split over gridDim.z
  const int zper = (a.nz + gridDim.z - 1) / gridDim.z;
  const int izb = blockIdx.z * zper, ize = min(a.nz, izb + zper);
  if constexpr (SEP) {
    // the frame's z factors of this block's planes, transposed to [z][m]
    const int M = a.M, mp = (M + 1) & ~1;
    const double *bz = a.btab + (int64_t)f * a.btab_stride + (int64_t)M * (a.nxh + a.ny);
    for (int i = threadIdx.x; i < (ize - izb) * mp; i += blockDim.x) {
      const int zl = i / mp, m = i - zl * mp;
      s_bzt[i] = m < M ? bz[m * a.nz + izb + zl] : 0.0;
    }
    __syncthreads();
  }
  double accD = 0.0;
  int mx = 0, yl = 0;
  const bool valid = col < inner && col_mode(a, col, mx, yl);
  if (col < inner && !valid) {
    // pad column of the chunked layout: a zero table entry
    for (int iz = izb; iz < ize; ++iz) a.gtab[(int64_t)f * a.nh + col + (int64_t)iz * inner] = 0.0;
  }
  if (valid) {
    const int iy = a.y0 + yl;
    const double w = (mx == 0 || ((a.nx & 1) == 0 && mx == a.nx / 2)) ? 1.0 : 2.0;
    double *gout = a.gtab + (int64_t)f * a.nh + col;
    if constexpr (SEP) {
      // separable path: K = sum_m amp_m (Bx_m By_m) Bz_m with the x-y
      // products of up to 16 Gaussians held in registers and the block's z
      // factors in shared memory, [z][m] (two per 16-byte load)
      const int M = a.M;
      const double *bt = a.btab + (int64_t)f * a.btab_stride;
      const double *bx = bt, *by = bt + M * a.nxh;
      double axy[16];
#pragma unroll
      for (int m = 0; m < 16; ++m) axy[m] = m < M ? s_amp[m] * bx[m * a.nxh + mx] * by[m * a.ny + iy] : 0.0;
      const double kx = g.kmat[0] * mx, ky = g.kmat[4] * signed_mode(iy, a.ny);
      const double kxy2 = kx * kx + ky * ky;
      const double txy = a.tx[mx] * a.ty[iy];
      const bool quads = a.spline == SOG_SPLINE_QUADS;
      const int mp = (M + 1) & ~1;
      for (int iz = izb; iz < ize; ++iz) {
        const int mz = signed_mode(iz, a.nz);
        const double kz = g.kmat[8] * mz;
        const double ksq = kxy2 + kz * kz;
        const bool live = !((mx | iy | mz) == 0) && ksq <= g.k_sq_max;
        double K = 0.0;
        if (live) {
          const double2 *row = reinterpret_cast<const double2 *>(s_bzt + (size_t)(iz - izb) * mp);
#pragma unroll
          for (int m2 = 0; m2 < 8; ++m2)
            if (2 * m2 < M) {
              const double2 v = row[m2];
              K += axy[2 * m2] * v.x;
              if (2 * m2 + 1 < M) K += axy[2 * m2 + 1] * v.y;
            }
        }
        double D = txy * a.tz[iz];
        if (quads) D = 1.0 / (D < 1e-20 ? 1e-20 : D);
        gout[(int64_t)iz * inner] = live ? K * D : 0.0;
        if (live) accD += w * K;
      }
    } else {
      double *gfout = (g.pad && a.gtabF) ? a.gtabF + (int64_t)f * a.nh + col : nullptr;
      const double *bt = (g.ortho && a.btab) ? a.btab + (int64_t)f * a.btab_stride : nullptr;
      for (int iz = izb; iz < ize; ++iz) {
        const ModeGreen mg = mode_green<T>(a, g, s_amp, s_bw2, mx, iy, iz, 0, nullptr, bt);
        gout[(int64_t)iz * inner] = mg.live ? mg.gE : 0.0;
        if (gfout) gfout[(int64_t)iz * inner] = mg.live ? mg.gF : 0.0;
        if (mg.live) accD += w * mg.gS;
      }
    }
  }
  accD = warp_sum(accD);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = accD;
  __syncthreads();
  if (threadIdx.x == 0) {
    double d = 0.0;
    for (int wi = 0; wi < (int)(blockDim.x >> 5); ++wi) d += red[wi];
    a.partD[((int64_t)f * gridDim.z + blockIdx.z) * gridDim.x + blockIdx.x] = d;
  }
}

// Fused z pass (power-of-two nz) with the Green function read from k_green's
// table: forward z-FFT of ic spectrum columns, energy partial sum, and for
// every field the scaled spectrum (i k_a gF rho / N or gE rho / N) inverse
// z-transformed.  Spectrum and gE tiles are double-buffered with cp.async.
// NTH threads per CTA: 256 (two CTAs per SM) or 512 (tiles of 8 columns of
// a 512-point transform, so that every field row it stores is 128
// contiguous bytes); see SOG_ZTHR.
template <typename T, int L, int NTH = 256, typename TO = T>
__global__ void __launch_bounds__(NTH, NTH == 512 ? 1 : SOG_ZFUSED_MINB) k_zfused_g(KsArgs<T> a, int ic,
                                                                                  int64_t ntiles,
                                                     const cplx_t<T> *__restrict__ twz, int write_spec) {
  using C = cplx_t<T>;
  using CO = cplx_t<TO>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ double red[2][NTH / 32];
  constexpr int n = 1 << L, TPT = n / kEPT;
  C *buf0 = reinterpret_cast<C *>(smem_raw);
  C *buf1 = buf0 + (size_t)n * ic;
  C *xbuf = buf1 + (size_t)n * ic;
  C *stg = xbuf + (size_t)padded_row(n) * ic;
  load_stage_twiddles<T, L, 0>(stg, twz);
  const int c = threadIdx.x % ic, t = threadIdx.x / ic;
  const int64_t inner = cols_inner(a);
  const int64_t nchunks = (inner + ic - 1) / ic;
  const int nfield = a.nfield;
  const double inv = 1.0 / ((double)a.nx * a.ny * a.nz);
  auto issue = [&](C *buf, int64_t tile) {
    const int64_t f = tile / nchunks;
    cols_issue<T>(buf, a.spec + f * a.nh, inner, n, ic, nchunks, tile - f * nchunks);
  };
  int64_t tile = blockIdx.x;
  if (tile < ntiles) issue(buf0, tile);
  cp_async_commit();
  for (int it = 0; tile < ntiles; ++it, tile += gridDim.x) {
    C *cur = (it & 1) ? buf1 : buf0;
    const int64_t next = tile + gridDim.x;
    if (next < ntiles) issue((it & 1) ? buf0 : buf1, next);
    cp_async_commit();
    const int f = (int)(tile / nchunks);
    const int64_t chunk = tile - (int64_t)f * nchunks;
    const int64_t col = chunk * ic + c;
    int mx = 0, yl = 0;
    const bool ok = col < inner && col_mode(a, col, mx, yl);
    const FrameGeom &g = a.geom[f];
    const int iy = a.y0 + yl;
    const int my = signed_mode(iy, a.ny);
    const double w = (mx == 0 || ((a.nx & 1) == 0 && mx == a.nx / 2)) ? 1.0 : 2.0;
    // Green values of this thread's modes, ready before the tile is: on the
    // fly for separable frames (K = sum_m amp_m Bx_m By_m Bz_m from the
    // per-axis factors of lmp/sog.cpp:1375-1476, times the per-axis
    // deconvolution; the same products in the same order as k_green's
    // table), else loads from the table, in flight during the FFT
    double gs[kEPT];
    double accD = 0.0;
    if (green_radial(a, g)) {   // frame-uniform
      const double *kr = a.krad + (int64_t)f * a.krad_stride;
      const double kx = g.kmat[0] * mx, ky = g.kmat[4] * my;
      const double kxy2 = kx * kx + ky * ky;
      const int sxy = mx * mx + my * my;
      const double txy = ok ? a.tx[mx] * a.ty[iy] : 0.0;
      const bool quads = a.spline == SOG_SPLINE_QUADS;
#pragma unroll
      for (int e = 0; e < kEPT; ++e) {
        const int iz = t + e * TPT;
        const int mz = signed_mode(iz, a.nz);
        const double kz = g.kmat[8] * mz;
        const bool live = ok && !((mx | my | mz) == 0) && kxy2 + kz * kz <= g.k_sq_max;
        const double K = live ? kr[sxy + mz * mz] : 0.0;
        double D = txy * a.tz[iz];
        if (quads) D = 1.0 / (D < 1e-20 ? 1e-20 : D);
        gs[e] = live ? K * D : 0.0;
        if (live) accD += w * K;
      }
    } else {
      const double *gp = a.gtab + (int64_t)f * a.nh + (ok ? col : 0);
#pragma unroll
      for (int e = 0; e < kEPT; ++e) gs[e] = ok ? gp[(int64_t)(t + e * TPT) * inner] : 0.0;
    }
    cp_async_wait<1>();
    __syncthreads();
    C v[kEPT];
#pragma unroll
    for (int e = 0; e < kEPT; ++e) v[e] = cur[(t + e * TPT) * ic + c];
    ct_fft<T, -1, L, true, 0, false, true>(v, t, stg, xbuf + c, ic);
    double accE = 0.0;
#pragma unroll
    for (int e = 0; e < kEPT; ++e) {
      const int slot = (t + e * TPT) * ic + c;
      const double rr = (double)v[e].x, ri = (double)v[e].y;
      if (ok) accE += w * gs[e] * (rr * rr + ri * ri);
      cur[slot] = v[e];             // own slots: no race
      gs[e] *= inv;
    }
    if (write_spec && ok) {
      C *sp = const_cast<C *>(a.spec) + (int64_t)f * a.nh + col;
#pragma unroll
      for (int e = 0; e < kEPT; ++e) sp[(int64_t)(t + e * TPT) * inner] = v[e];
    }
    const double *gFp = (g.pad && a.gtabF) ? a.gtabF + (int64_t)f * a.nh + (ok ? col : 0) : nullptr;
    CO *out = a.fspec ? static_cast<CO *>(a.fspec) + (int64_t)f * nfield * a.nh + (ok ? col : 0) : nullptr;
    const int64_t zbs = (int64_t)a.zblk * inner;   // one field's z block
    auto store_field = [&](int fl, const C (&wv)[kEPT]) {
      if (!ok) return;
#pragma unroll
      for (int e = 0; e < kEPT; ++e) {
        const int iz = t + e * TPT, b = iz / a.zblk, zl = iz - b * a.zblk;
        if (a.cw) {
          // chunked: this tile's cw columns are contiguous for every z
          const int64_t q = col / a.cw;
          static_cast<CO *>(a.zdst[b])[(int64_t)fl * zbs + (q * a.zblk + zl) * a.cw + (col - q * a.cw)] =
              to_field<TO>(wv[e]);
        } else {
          CO *ob = a.zdst[0] ? static_cast<CO *>(a.zdst[b]) + (int64_t)fl * zbs + col
                             : out + ((int64_t)b * nfield + fl) * zbs;
          ob[(int64_t)zl * inner] = to_field<TO>(wv[e]);
        }
      }
    };
    // The ik field spectra along this column are i k_a s rho with
    // k_a = kxy_a + kz_a mz and kxy_a fixed on the column, so two inverse
    // transforms serve all three: Y1 = IFFT(s rho), Y2 = IFFT(i mz s rho),
    // field a = i kxy_a Y1 + kz_a Y2.  The potential field (s = gE) is Y1
    // itself unless the force uses the alias-summed gF.
    // With two_slot, orthorhombic frames store Y1 and Y2 as they are (slots
    // 0 and 2): each field is then one of them times a factor that depends on
    // mx or my only, which k_cols_fields applies around the inverse y
    // transform, so a third of the field bytes never go to HBM.  Y2's input
    // waits in the tile buffer (in this thread's own slots) while Y1 is
    // transformed, so one transform's data is in registers at a time.
    bool pot_done = !(nfield > (a.want_force ? 3 : 0));
    const bool two = a.two_slot && g.ortho && a.want_force;   // frame-uniform
    if (a.want_force) {
      if (!pot_done && gFp) {
        // alias frame: the potential's own Green function, from the spectrum
        // while it is still in the tile buffer
        C wv[kEPT];
#pragma unroll
        for (int e = 0; e < kEPT; ++e) {
          const C r = cur[(t + e * TPT) * ic + c];
          wv[e] = cmk<C, T>((T)(gs[e] * (double)r.x), (T)(gs[e] * (double)r.y));
        }
        ct_fft<T, +1, L, true, 0, false, true>(wv, t, stg, xbuf + c, ic);
        store_field(3, wv);
        pot_done = true;
      }
      C y[kEPT];
#pragma unroll
      for (int e = 0; e < kEPT; ++e) {
        const int slot = (t + e * TPT) * ic + c;
        const C r = cur[slot];
        const double sc = gFp ? (ok ? gFp[(int64_t)(t + e * TPT) * inner] * inv : 0.0) : gs[e];
        y[e] = cmk<C, T>((T)(sc * (double)r.x), (T)(sc * (double)r.y));
        const double mzs = (double)signed_mode(t + e * TPT, a.nz) * sc;
        cur[slot] = cmk<C, T>((T)(-mzs * (double)r.y), (T)(mzs * (double)r.x));   // Y2's input
      }
      ct_fft<T, +1, L, true, 0, false, true>(y, t, stg, xbuf + c, ic);
      if (two) {
        store_field(0, y);
#pragma unroll
        for (int e = 0; e < kEPT; ++e) y[e] = cur[(t + e * TPT) * ic + c];
        ct_fft<T, +1, L, true, 0, false, true>(y, t, stg, xbuf + c, ic);
        store_field(2, y);
        pot_done = true;   // k_cols_fields takes the potential from Y1
      } else {
        if (!pot_done) {
          store_field(3, y);
          pot_done = true;
        }
        C w[kEPT];
#pragma unroll
        for (int e = 0; e < kEPT; ++e) {
          const int slot = (t + e * TPT) * ic + c;
          w[e] = cur[slot];
          cur[slot] = y[e];   // Y1 waits in the tile buffer
        }
        ct_fft<T, +1, L, true, 0, false, true>(w, t, stg, xbuf + c, ic);
        for (int fl = 0; fl < 3; ++fl) {
          const double kxy = g.kmat[fl * 3 + 0] * mx + g.kmat[fl * 3 + 1] * my;
          const double kz = g.kmat[fl * 3 + 2];
          C wv[kEPT];
#pragma unroll
          for (int e = 0; e < kEPT; ++e) {
            const C y1 = cur[(t + e * TPT) * ic + c];
            wv[e] = cmk<C, T>((T)(-kxy * (double)y1.y + kz * (double)w[e].x),
                              (T)(kxy * (double)y1.x + kz * (double)w[e].y));
          }
          store_field(fl, wv);
        }
      }
    }
    if (!pot_done) {
      C wv[kEPT];
#pragma unroll
      for (int e = 0; e < kEPT; ++e) {
        const C r = cur[(t + e * TPT) * ic + c];
        wv[e] = cmk<C, T>((T)(gs[e] * (double)r.x), (T)(gs[e] * (double)r.y));
      }
      ct_fft<T, +1, L, true, 0, false, true>(wv, t, stg, xbuf + c, ic);
      store_field(0, wv);
    }
    accE = warp_sum(accE);
    accD = warp_sum(accD);
    if ((threadIdx.x & 31) == 0) {
      red[0][threadIdx.x >> 5] = accE;
      red[1][threadIdx.x >> 5] = accD;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      double e = 0.0, d = 0.0;
      for (int wi = 0; wi < (int)(blockDim.x >> 5); ++wi) {
        e += red[0][wi];
        d += red[1][wi];
      }
      double *p = a.part + ((int64_t)f * nchunks + chunk) * 2;
      p[0] = e;
      p[1] = d;   // self sum of on-the-fly frames (zero for table frames)
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  if (a.zdst[0]) __threadfence_system();
}

// Inverse y transform of the field spectra [nf][F][nz][ny][nx/2+1], in place,
// forming the fields of two-slot frames (k_zfused_g): tile = (plane o =
// (f*F + s)*nz + z, ic columns mx).  An orthorhombic frame holds Y1 in slot 0
// and Y2 in slot 2: slot 0 yields field x = i kx mx IFFT(Y1) (and the
// potential IFFT(Y1) into slot 3, unless the z pass stored the frame's own
// potential there) and field y = ky IFFT(i my Y1) into slot 1; slot 2 yields
// field z = kz IFFT(Y2).  Slot 1, and slot 3 when it was not stored, have no
// input and are skipped.  Other frames: a plain inverse transform of every
// slot.  Same pipeline as k_cols_pipe.
template <typename T, bool PAD, int L, bool MAP = false>
__global__ void k_cols_fields(cplx_t<T> *__restrict__ data, const FrameGeom *__restrict__ geom, int F, int nz,
                              int64_t inner, int ic, int64_t ntiles, const cplx_t<T> *__restrict__ tw,
                              int two_slot, int want_pot, RowMap<cplx_t<T>> in = {}, RowMap<cplx_t<T>> out = {}) {
  using C = cplx_t<T>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int n = 1 << L, TPT = n / kEPT;
  C *buf0 = reinterpret_cast<C *>(smem_raw);
  C *buf1 = buf0 + (size_t)n * ic;
  C *xbuf = buf1 + (size_t)n * ic;
  C *stg = xbuf + (size_t)(PAD ? padded_row(n) : n) * ic;
  load_stage_twiddles<T, L, 0>(stg, tw);
  const int c = threadIdx.x % ic, t = threadIdx.x / ic;
  const int64_t nchunks = (inner + ic - 1) / ic;
  // role of a tile: 0 skip, 1 plain, 2 slot 0 (fields x, y, potential), 3 slot 2 (field z)
  auto role = [&](int64_t tile) -> int {
    const int64_t fs = tile / nchunks / nz;
    const int f = (int)(fs / F), sl = (int)(fs - (int64_t)f * F);
    const FrameGeom &g = geom[f];
    if (!(two_slot && g.ortho)) return 1;
    if (sl == 0) return 2;
    if (sl == 2) return 3;
    if (sl == 3 && g.pad) return 1;
    return 0;
  };
  // tile loads: in place, or through the input row map (MAP: the z-slab's
  // received blocks)
  auto issue = [&](C *buf, int64_t tile) {
    if constexpr (MAP) {
      const int64_t o = tile / nchunks;
      const int64_t i0 = (tile - o * nchunks) * ic;
      const int ic_sh = __ffs(ic) - 1;   // ic: a power of two
      for (int q = threadIdx.x; q < n * ic; q += blockDim.x) {
        const int r = q >> ic_sh, col = q - (r << ic_sh);
        const bool ok = i0 + col < inner;
        cp_async_elem(buf + q, ok ? in.at(o, r, i0 + col) : in.tab[0], ok);
      }
    } else {
      cols_issue<T>(buf, data, inner, n, ic, nchunks, tile);
    }
  };
  int64_t tile = blockIdx.x;
  if (tile < ntiles && role(tile)) issue(buf0, tile);
  cp_async_commit();
  for (int it = 0; tile < ntiles; ++it, tile += gridDim.x) {
    C *cur = (it & 1) ? buf1 : buf0;
    C *nxt = (it & 1) ? buf0 : buf1;
    const int64_t next = tile + gridDim.x;
    if (next < ntiles && role(next)) issue(nxt, next);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int rl = role(tile);   // block-uniform
    if (rl) {
      const int64_t o = tile / nchunks;
      const int64_t i0 = (tile - o * nchunks) * ic;
      const int64_t fs = o / nz;
      const int f = (int)(fs / F);
      const FrameGeom &g = geom[f];
      const bool okc = i0 + c < inner;
      const int mx = (int)(i0 + c);
      const int64_t sl = fs - (int64_t)f * F;
      const int64_t o0 = o - sl * nz;          // plane of slot 0, same (frame, z)
      // element e of this thread's column in plane `po` (slot k: po = o0 + k nz)
      auto put = [&](int64_t po, int e, C val) {
        if constexpr (MAP) *out.at(po, t + e * TPT, i0 + c) = val;
        else data[po * ((int64_t)n * inner) + (int64_t)(t + e * TPT) * inner + i0 + c] = val;
      };
      C v[kEPT];
#pragma unroll
      for (int e = 0; e < kEPT; ++e) v[e] = cur[(t + e * TPT) * ic + c];
      ct_fft<T, +1, L, PAD>(v, t, stg, xbuf + c, ic);
      if (rl == 1) {
        if (okc) {
#pragma unroll
          for (int e = 0; e < kEPT; ++e) put(o, e, v[e]);
        }
      } else if (rl == 3) {
        const double kz = g.kmat[8];
        if (okc) {
#pragma unroll
          for (int e = 0; e < kEPT; ++e) put(o, e, cmk<C, T>((T)(kz * (double)v[e].x), (T)(kz * (double)v[e].y)));
        }
      } else {
        const double kxm = g.kmat[0] * mx;
        if (okc) {
#pragma unroll
          for (int e = 0; e < kEPT; ++e) put(o0, e, cmk<C, T>((T)(-kxm * (double)v[e].y), (T)(kxm * (double)v[e].x)));
          if (want_pot && !g.pad) {
#pragma unroll
            for (int e = 0; e < kEPT; ++e) put(o0 + 3 * (int64_t)nz, e, v[e]);
          }
        }
        // field y: ky IFFT(i my Y1), Y1 still in the tile buffer
#pragma unroll
        for (int e = 0; e < kEPT; ++e) {
          const C r = cur[(t + e * TPT) * ic + c];
          const double my = (double)signed_mode(t + e * TPT, n);
          v[e] = cmk<C, T>((T)(-my * (double)r.y), (T)(my * (double)r.x));
        }
        ct_fft<T, +1, L, PAD>(v, t, stg, xbuf + c, ic);
        const double ky = g.kmat[4];
        if (okc) {
#pragma unroll
          for (int e = 0; e < kEPT; ++e)
            put(o0 + nz, e, cmk<C, T>((T)(ky * (double)v[e].x), (T)(ky * (double)v[e].y)));
        }
      }
    }
    __syncthreads();  // every thread is done with `cur` before it is refilled
  }
  cp_async_wait<0>();
}

// Extras: dE/d(amp_m, bw2_m) partial sums (cubes2_fft.py:822-862) and the
// reciprocal virial sums (cubes2_fft.py:874-921).  Layout of one partial:
//   [0, M)        sum w e_m D |rho|^2         (gA main)
//   [M, 2M)       sum w e_m                   (gA self)
//   [2M, 3M)      sum w (-k^2/2) amp_m e_m D |rho|^2
//   [3M, 4M)      sum w (-k^2/2) amp_m e_m
//   [4M]          sum w |rho|^2 gE            (virial diagonal)
//   [4M+1, 4M+7)  sum w |rho|^2 gV k_a k_b    (xx yy zz xy xz yz)
//   [4M+7, 4M+13) sum w Kv k_a k_b            (self-energy strain)
template <typename T>
__global__ void __launch_bounds__(256) k_kspace_extra(KsArgs<T> a, int want_grad, int want_vir) {
  using C = cplx_t<T>;
  __shared__ double s_amp[kMaxGauss], s_bw2[kMaxGauss];
  __shared__ double red[8][4 * kMaxGauss + 13];
  for (int m = threadIdx.x; m < a.M; m += blockDim.x) {
    s_amp[m] = kpar(a.amp, a.p32, m);
    s_bw2[m] = kpar(a.bw2, a.p32, m);
  }
  __syncthreads();
  const int f = blockIdx.y;
  const FrameGeom &g = a.geom[f];
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = a.M;
  bool valid = idx < a.nh;
  int mx = 0, iy = 0, iz = 0;
  double rho2 = 0.0, w = 0.0;
  if (valid) {
    mx = (int)(idx % a.nxh);
    const int64_t zy = idx / a.nxh;
    iy = (int)(zy % a.ny);
    iz = (int)(zy / a.ny);
    const C r = a.spec[(int64_t)f * a.nh + idx];
    rho2 = (double)r.x * r.x + (double)r.y * r.y;
    w = (mx == 0 || ((a.nx & 1) == 0 && mx == a.nx / 2)) ? 1.0 : 2.0;
  }
  ModeGreen mg;
  mg.live = false;
  if (valid) mg = mode_green<T>(a, g, s_amp, s_bw2, mx, iy, iz, 0, nullptr);
  const bool live = valid && mg.live;
  if (want_grad) {
    for (int m = 0; m < M; ++m) {
      double eD = 0.0, eS = 0.0;
      // bw2 derivatives: -k^2/2 times eD, eS, except with alias sums, whose
      // terms carry their own |q|^2
      double hD = -0.5 * mg.ksq, hS = hD;
      if (live) {
        if (a.spline == SOG_SPLINE_BSPLINE && g.pad) {
          double em[6];
          mode_green<T>(a, g, s_amp, s_bw2, mx, iy, iz, m, em);
          eD = em[0];
          eS = em[1];
          hD = eD != 0.0 ? em[2] / eD : 0.0;
          hS = eS != 0.0 ? em[3] / eS : 0.0;
        } else {
          const double e = exp(-0.5 * s_bw2[m] * mg.ksq);
          eS = e;
          eD = (mg.K != 0.0) ? e * (mg.gE / mg.K) : 0.0;
          if (mg.K == 0.0) {
            // D recomputed when K underflows to zero
            if (a.spline == SOG_SPLINE_QUADS) {
              double infl = a.tx[mx] * a.ty[iy] * a.tz[iz];
              if (infl < 1e-20) infl = 1e-20;
              eD = e / infl;
            } else {
              eD = e * a.tx[mx] * a.ty[iy] * a.tz[iz];
            }
          }
        }
      }
      const double v0 = warp_sum(live ? w * eD * rho2 : 0.0);
      const double v1 = warp_sum(live ? w * eS : 0.0);
      const double v2 = warp_sum(live ? w * (hD * s_amp[m]) * eD * rho2 : 0.0);
      const double v3 = warp_sum(live ? w * (hS * s_amp[m]) * eS : 0.0);
      if (lane == 0) {
        red[warp][m] = v0;
        red[warp][M + m] = v1;
        red[warp][2 * M + m] = v2;
        red[warp][3 * M + m] = v3;
      }
    }
  }
  if (want_vir) {
    double kk[6] = {0, 0, 0, 0, 0, 0};
    if (live) {
      kk[0] = mg.k[0] * mg.k[0]; kk[1] = mg.k[1] * mg.k[1]; kk[2] = mg.k[2] * mg.k[2];
      kk[3] = mg.k[0] * mg.k[1]; kk[4] = mg.k[0] * mg.k[2]; kk[5] = mg.k[1] * mg.k[2];
    }
    double v = warp_sum(live ? w * rho2 * mg.gE : 0.0);
    if (lane == 0) red[warp][4 * M] = v;
    for (int c = 0; c < 6; ++c) {
      v = warp_sum(live ? w * rho2 * mg.gV * kk[c] : 0.0);
      if (lane == 0) red[warp][4 * M + 1 + c] = v;
      v = warp_sum(live ? w * mg.Kv * kk[c] : 0.0);
      if (lane == 0) red[warp][4 * M + 7 + c] = v;
    }
  }
  __syncthreads();
  const int nacc = 4 * M + 13;
  double *p = a.partx + ((int64_t)f * gridDim.x + blockIdx.x) * a.nx_acc;
  for (int i = threadIdx.x; i < nacc; i += blockDim.x) {
    const bool used = (i < 4 * M) ? want_grad : want_vir;
    double s = 0.0;
    if (used)
      for (int wv = 0; wv < (int)(blockDim.x >> 5); ++wv) s += red[wv][i];
    p[i] = s;
  }
}

// Hessian-vector product, k-space step of one channel (separable splines).
// From the spectra of the mesh charge rho^ and of its derivative drho^ along
// the direction: the potential spectra
//   Phi^ = gE rho^ / N_g,   Psi^ = (gE drho^ + dgE rho^) / N_g,
//   dgE = sum_m (da_m eD_m + amp_m db_m deD_m/dbw2_m)
// in field slots 0 and 1 ([nf][2][nh]), and per block the parameter rows of
// H d (scaled by V^2 / N_g^2: rho^ = (N_g / V) S(k), the structure factor the
// shared finalize is written for) and, for channel 0, the self sums
// D0..D2 = sum w eS_m (1, d/dbw2, d2/dbw2^2).  part: [nf][nch][blocks][5M].
template <typename TP>
__global__ void __launch_bounds__(256) k_kspace_hvp(KsArgs<double> a, const cplx_t<double> *__restrict__ dspec,
                                                    const void *damp, const void *dbw2, int ch, int nch,
                                                    double *__restrict__ part) {
  __shared__ double s_amp[kMaxGauss], s_bw2[kMaxGauss], s_da[kMaxGauss], s_db[kMaxGauss];
  __shared__ double red[8][5 * kMaxGauss];
  const int f = blockIdx.y;
  const int M = a.M;
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    s_amp[m] = kpar(a.amp, a.p32, m);
    s_bw2[m] = kpar(a.bw2, a.p32, m);
    s_da[m] = ldir<TP>(damp, (int64_t)f * M + m);
    s_db[m] = ldir<TP>(dbw2, (int64_t)f * M + m);
  }
  __syncthreads();
  const FrameGeom &g = a.geom[f];
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool valid = idx < a.nh;
  int mx = 0, iy = 0, iz = 0;
  cplx_t<double> r = {0.0, 0.0}, d = {0.0, 0.0};
  double w = 0.0;
  if (valid) {
    mx = (int)(idx % a.nxh);
    const int64_t zy = idx / a.nxh;
    iy = (int)(zy % a.ny);
    iz = (int)(zy / a.ny);
    r = a.spec[(int64_t)f * a.nh + idx];
    d = dspec[(int64_t)f * a.nh + idx];
    w = (mx == 0 || ((a.nx & 1) == 0 && mx == a.nx / 2)) ? 1.0 : 2.0;
  }
  ModeGreen mg;
  mg.live = false;
  mg.gE = mg.ksq = 0.0;
  if (valid) mg = mode_green<double>(a, g, s_amp, s_bw2, mx, iy, iz, 0, nullptr);
  const bool live = valid && mg.live;
  double Dfac = 0.0;   // deconvolution of the principal form
  if (live && !(a.spline == SOG_SPLINE_BSPLINE && g.pad)) {
    if (a.spline == SOG_SPLINE_QUADS) {
      double infl = a.tx[mx] * a.ty[iy] * a.tz[iz];
      if (infl < 1e-20) infl = 1e-20;
      Dfac = 1.0 / infl;
    } else {
      Dfac = a.tx[mx] * a.ty[iy] * a.tz[iz];
    }
  }
  const double rr = r.x * r.x + r.y * r.y, rd = 2.0 * (r.x * d.x + r.y * d.y);
  double dG = 0.0;
  for (int m = 0; m < M; ++m) {
    double em[6] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0};
    if (live) {
      if (a.spline == SOG_SPLINE_BSPLINE && g.pad) mode_green<double>(a, g, s_amp, s_bw2, mx, iy, iz, m, em);
      else principal_em(s_bw2[m], mg.ksq, Dfac, em);
    }
    dG += s_da[m] * em[0] + s_amp[m] * s_db[m] * em[2];
    const double xa = warp_sum(w * (em[0] * rd + s_db[m] * em[2] * rr));
    const double xb = warp_sum(w * (s_amp[m] * (em[2] * rd + s_db[m] * em[4] * rr) + s_da[m] * em[2] * rr));
    const double d0 = warp_sum(ch == 0 ? w * em[1] : 0.0);
    const double d1 = warp_sum(ch == 0 ? w * em[3] : 0.0);
    const double d2 = warp_sum(ch == 0 ? w * em[5] : 0.0);
    if (lane == 0) {
      red[warp][m] = xa;
      red[warp][M + m] = xb;
      red[warp][2 * M + m] = d0;
      red[warp][3 * M + m] = d1;
      red[warp][4 * M + m] = d2;
    }
  }
  if (valid) {
    const double inv = 1.0 / ((double)a.nx * a.ny * a.nz);
    const double gE = live ? mg.gE : 0.0;
    cplx_t<double> *out = static_cast<cplx_t<double> *>(a.fspec) + (int64_t)f * 2 * a.nh + idx;
    out[0] = cplx_t<double>{gE * inv * r.x, gE * inv * r.y};
    out[a.nh] = cplx_t<double>{(gE * d.x + dG * r.x) * inv, (gE * d.y + dG * r.y) * inv};
  }
  __syncthreads();
  const double vs = g.vol / ((double)a.nx * a.ny * a.nz);
  const double v2 = vs * vs;
  double *p = part + (((int64_t)f * nch + ch) * gridDim.x + blockIdx.x) * 5 * M;
  for (int i = threadIdx.x; i < 5 * M; i += blockDim.x) {
    double s = 0.0;
    for (int wv = 0; wv < (int)(blockDim.x >> 5); ++wv) s += red[wv][i];
    p[i] = i < 2 * M ? s * v2 : s;
  }
}

// ------------------------------------------------------------------------
// gather
// ------------------------------------------------------------------------
template <typename T>
struct GatherArgs {
  const int4 *s_anchor;
  const T *s_t;
  const T *s_q;       // channel slice
  const int32_t *s_atom;
  const T *freal;     // [nf][F][ng]
  int nfield, want_force, want_pot;
  int64_t nslots, ng;
  AtomGrid ag;
  int spline;
  QuadsCoef qc;
  double norm;
  int channel, nch, accumulate;
  T *forces;          // [N,3]
  T *pot_raw;         // [N,C]
  // slots slot_lo .. slot_lo+nslots-1; field plane of anchor plane z + c is
  // z - zlo + c, wrapped at zwrap (nz when the fields hold the whole mesh)
  int64_t slot_lo;
  int zlo, zwrap;
  // when set, the slot range is [*range_lo, *range_hi) read on the device
  // (the sorted-atom bin offsets of a z slab) and nslots bounds the grid
  const uint32_t *range_lo, *range_hi;
  // exact dE/dr (k_gather_dedr): frame geometry and the [N,3] output
  const FrameGeom *geom;
  T *dedr;
};

// NT stencil terms as in k_spread (the weight of node (k, b, c) is
// sum_t X_t[k] Y_t[b] Z_t[c]).
template <typename T, int P, int NT = 1>
__global__ void __launch_bounds__(256, SOG_GATHER_MINB) k_gather(GatherArgs<T> a) {
  using ST = StencilTerms<NT>;
  const int64_t si = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (si >= a.nslots) return;
  int64_t s = a.slot_lo + si;
  if (a.range_lo) {
    s = (int64_t)*a.range_lo + si;
    if (s >= (int64_t)*a.range_hi) return;
  }
  const int4 an = a.s_anchor[s];
  T wx[ST::K][P], wy[ST::K][P], wz[ST::K][P];
  axis_kinds<T, P, NT>(a.spline, a.s_t[s * 3 + 0], wx, a.qc);
  axis_kinds<T, P, NT>(a.spline, a.s_t[s * 3 + 1], wy, a.qc);
  axis_kinds<T, P, NT>(a.spline, a.s_t[s * 3 + 2], wz, a.qc);
  const AtomGrid &ag = a.ag;
  int ix[P];
#pragma unroll
  for (int k = 0; k < P; ++k) { int v = an.x + k; ix[k] = v >= ag.nx ? v - ag.nx : v; }
  const int F = a.nfield;
  const T *base = a.freal + (int64_t)an.w * F * a.ng;
  T acc[4] = {T(0), T(0), T(0), T(0)};
#pragma unroll 1
  for (int c = 0; c < P; ++c) {
    int gz = an.z - a.zlo + c;
    if (gz >= a.zwrap) gz -= a.zwrap;
#pragma unroll
    for (int b = 0; b < P; ++b) {
      int gy = an.y + b;
      if (gy >= ag.ny) gy -= ag.ny;
      const int64_t row = ((int64_t)gz * ag.ny + gy) * ag.nx;
      T wzy[NT];
#pragma unroll
      for (int tt = 0; tt < NT; ++tt) wzy[tt] = wy[ST::y(tt)][b] * wz[ST::z(tt)][c];
#pragma unroll
      for (int k = 0; k < P; ++k) {
        T wv = T(0);
#pragma unroll
        for (int tt = 0; tt < NT; ++tt) wv += wx[ST::x(tt)][k] * wzy[tt];
        const T *pt = base + (row + ix[k]) * F;
        if (F == 3) {
          acc[0] += wv * pt[0]; acc[1] += wv * pt[1]; acc[2] += wv * pt[2];
        } else if (F == 4) {
          acc[0] += wv * pt[0]; acc[1] += wv * pt[1]; acc[2] += wv * pt[2]; acc[3] += wv * pt[3];
        } else {
          acc[0] += wv * pt[0];
        }
      }
    }
  }
  const int64_t atom = a.s_atom[s];
  const T q = a.s_q[s];
  if (a.want_force) {
    const T sc = -q * (T)a.norm;
    for (int c = 0; c < 3; ++c) {
      const T v = sc * acc[c];
      if (a.accumulate) a.forces[atom * 3 + c] += v; else a.forces[atom * 3 + c] = v;
    }
  }
  if (a.want_pot) a.pot_raw[atom * a.nch + a.channel] = acc[a.want_force ? 3 : 0];
}

// Exact gradient of the mesh energy w.r.t. the positions (separable
// splines): the potential field (the last of the F interleaved fields)
// gathered with the derivatives of the spline weights,
//   dE/dr_i = q_i norm sum_g grad_r w_i(g) Phi(g),  d t_a / d r_b = n_a (cell^-1)_{ba},
// the derivative of the energy the forward returns (as autograd through
// quads_fft.py's spread gives it).  Summed over the channels (accumulate).
template <typename T, int P>
__global__ void __launch_bounds__(256) k_gather_dedr(GatherArgs<T> a) {
  const int64_t si = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (si >= a.nslots) return;
  const int64_t s = a.slot_lo + si;
  const int4 an = a.s_anchor[s];
  double w[3][P], dw[3][P];
#pragma unroll
  for (int ax = 0; ax < 3; ++ax) {
    const double t = (double)a.s_t[s * 3 + ax];
    spline_w<double, P>(a.spline, t, w[ax], a.qc);
    spline_dw<P>(a.spline, t, dw[ax], a.qc);
  }
  const AtomGrid &ag = a.ag;
  const int F = a.nfield;
  const T *base = a.freal + (int64_t)an.w * F * a.ng + (F - 1);
  double g3[3] = {0.0, 0.0, 0.0};
#pragma unroll 1
  for (int c = 0; c < P; ++c) {
    int gz = an.z - a.zlo + c;
    if (gz >= a.zwrap) gz -= a.zwrap;
#pragma unroll
    for (int b = 0; b < P; ++b) {
      int gy = an.y + b;
      if (gy >= ag.ny) gy -= ag.ny;
      const int64_t row = ((int64_t)gz * ag.ny + gy) * ag.nx;
      const double wyz = w[1][b] * w[2][c], dyz = dw[1][b] * w[2][c], ydz = w[1][b] * dw[2][c];
#pragma unroll
      for (int k = 0; k < P; ++k) {
        int gx = an.x + k;
        if (gx >= ag.nx) gx -= ag.nx;
        const double phi = (double)base[(row + gx) * F];
        g3[0] += dw[0][k] * wyz * phi;
        g3[1] += w[0][k] * dyz * phi;
        g3[2] += w[0][k] * ydz * phi;
      }
    }
  }
  const FrameGeom &g = a.geom[an.w];
  const double n3[3] = {(double)ag.nx, (double)ag.ny, (double)ag.nz};
  const int64_t atom = a.s_atom[s];
  const double qn = (double)a.s_q[s] * a.norm;
#pragma unroll
  for (int b = 0; b < 3; ++b) {
    double v = 0.0;
#pragma unroll
    for (int ax = 0; ax < 3; ++ax) v += n3[ax] * g.cinv[b * 3 + ax] * g3[ax];
    v *= qn;
    if (a.accumulate) a.dedr[atom * 3 + b] += (T)v; else a.dedr[atom * 3 + b] = (T)v;
  }
}

// Hessian-vector product, gather of one channel (separable splines): the
// potential fields Phi (slot 0) and Psi (slot 1, [nf][ng][2]) over the
// atom's stencil with the spline weights and their first and second
// derivatives (u: mesh coordinates, J_cx = du_x / dr_c = n_x (cell^-1)_cx,
// bt = J^T b the position direction in mesh units):
//   (H d)_q  = norm [sum_g W Psi + sum_x bt_x G_x(Phi)]
//   (H d)_r += norm J [a G(Phi) + q G(Psi) + q S(Phi) bt]
// with G_x(f) = sum_g dW/du_x f and S_xy = sum_g d2W/du_x du_y Phi.  The
// charge rows are written per channel, the position rows summed over the
// channels (accumulate).
template <typename T, int P>
__global__ void __launch_bounds__(256) k_gather_hvp(GatherArgs<T> a, const double *__restrict__ fields,
                                                    const void *dir_q, const void *dir_r, T *__restrict__ out_q,
                                                    T *__restrict__ out_r) {
  const int64_t si = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (si >= a.nslots) return;
  const int64_t s = a.slot_lo + si;
  const int4 an = a.s_anchor[s];
  double w[3][P], dw[3][P], d2[3][P];
#pragma unroll
  for (int ax = 0; ax < 3; ++ax) {
    const double t = (double)a.s_t[s * 3 + ax];
    spline_w<double, P>(a.spline, t, w[ax], a.qc);
    spline_dw<P>(a.spline, t, dw[ax], a.qc);
    spline_d2w<P>(a.spline, t, d2[ax], a.qc);
  }
  const AtomGrid &ag = a.ag;
  const double *base = fields + (int64_t)an.w * 2 * a.ng;
  double sp = 0.0, gp[3] = {0.0, 0.0, 0.0}, gs[3] = {0.0, 0.0, 0.0};
  double hs[6] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0};   // xx yy zz xy xz yz
#pragma unroll 1
  for (int c = 0; c < P; ++c) {
    int gz = an.z + c;
    if (gz >= ag.nz) gz -= ag.nz;
#pragma unroll
    for (int b = 0; b < P; ++b) {
      int gy = an.y + b;
      if (gy >= ag.ny) gy -= ag.ny;
      const int64_t row = ((int64_t)gz * ag.ny + gy) * ag.nx;
      const double wyz = w[1][b] * w[2][c], dyz = dw[1][b] * w[2][c], ydz = w[1][b] * dw[2][c];
      const double yyz = d2[1][b] * w[2][c], yzz = w[1][b] * d2[2][c], dydz = dw[1][b] * dw[2][c];
#pragma unroll
      for (int k = 0; k < P; ++k) {
        int gx = an.x + k;
        if (gx >= ag.nx) gx -= ag.nx;
        const double phi = base[(row + gx) * 2], psi = base[(row + gx) * 2 + 1];
        const double wx = w[0][k], dx = dw[0][k];
        sp += wx * wyz * psi;
        gp[0] += dx * wyz * phi;
        gp[1] += wx * dyz * phi;
        gp[2] += wx * ydz * phi;
        gs[0] += dx * wyz * psi;
        gs[1] += wx * dyz * psi;
        gs[2] += wx * ydz * psi;
        hs[0] += d2[0][k] * wyz * phi;
        hs[1] += wx * yyz * phi;
        hs[2] += wx * yzz * phi;
        hs[3] += dx * dyz * phi;
        hs[4] += dx * ydz * phi;
        hs[5] += wx * dydz * phi;
      }
    }
  }
  const FrameGeom &g = a.geom[an.w];
  const double n3[3] = {(double)ag.nx, (double)ag.ny, (double)ag.nz};
  const int64_t atom = a.s_atom[s];
  const double qv = (double)a.s_q[s];
  const double av = ldir<T>(dir_q, atom * a.nch + a.channel);
  double br[3], bt[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) br[c] = ldir<T>(dir_r, atom * 3 + c);
#pragma unroll
  for (int x = 0; x < 3; ++x)
    bt[x] = n3[x] * (br[0] * g.cinv[0 * 3 + x] + br[1] * g.cinv[1 * 3 + x] + br[2] * g.cinv[2 * 3 + x]);
  out_q[atom * a.nch + a.channel] = (T)(a.norm * (sp + bt[0] * gp[0] + bt[1] * gp[1] + bt[2] * gp[2]));
  const double S[3][3] = {{hs[0], hs[3], hs[4]}, {hs[3], hs[1], hs[5]}, {hs[4], hs[5], hs[2]}};
  double v[3];
#pragma unroll
  for (int x = 0; x < 3; ++x)
    v[x] = av * gp[x] + qv * (gs[x] + S[x][0] * bt[0] + S[x][1] * bt[1] + S[x][2] * bt[2]);
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const double o = a.norm * (n3[0] * g.cinv[c * 3 + 0] * v[0] + n3[1] * g.cinv[c * 3 + 1] * v[1] +
                               n3[2] * g.cinv[c * 3 + 2] * v[2]);
    if (a.accumulate) out_r[atom * 3 + c] += (T)o; else out_r[atom * 3 + c] = (T)o;
  }
}

// fp64 gather of the three force fields (single-term splines, even P):
// an atom's stencil row of P points x 3 interleaved fields is 3P contiguous
// doubles when it does not wrap in x.  The row is read as 3P/2 16-byte loads
// from its 16-byte-aligned start below it, plus one 8-byte load for rows that
// start on an odd word, and the lane picks its 3P words from those: 3P/2 + 1
// load instructions a row instead of 3P, for every lane of a warp alike.
// Every load stays inside the row [start, start + 3P).  Rows that wrap take
// the per-point loads of k_gather.
template <int P>
__global__ void __launch_bounds__(256, SOG_GATHER_MINB) k_gather_f3v(GatherArgs<double> a) {
  static_assert(P % 2 == 0, "even stencil widths");
  const int64_t si = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (si >= a.nslots) return;
  int64_t s = a.slot_lo + si;
  if (a.range_lo) {
    s = (int64_t)*a.range_lo + si;
    if (s >= (int64_t)*a.range_hi) return;
  }
  const int4 an = a.s_anchor[s];
  double wx[1][P], wy[1][P], wz[1][P];
  axis_kinds<double, P, 1>(a.spline, a.s_t[s * 3 + 0], wx, a.qc);
  axis_kinds<double, P, 1>(a.spline, a.s_t[s * 3 + 1], wy, a.qc);
  axis_kinds<double, P, 1>(a.spline, a.s_t[s * 3 + 2], wz, a.qc);
  const AtomGrid &ag = a.ag;
  int ix[P];
#pragma unroll
  for (int k = 0; k < P; ++k) { int v = an.x + k; ix[k] = v >= ag.nx ? v - ag.nx : v; }
  const double *base = a.freal + (int64_t)an.w * 3 * a.ng;
  // aligned field block: a row's aligned-down start never precedes it
  const bool nowrap = an.x + P <= ag.nx && (reinterpret_cast<uintptr_t>(base) & 15) == 0;
  double acc0 = 0.0, acc1 = 0.0, acc2 = 0.0;
#pragma unroll 1
  for (int c = 0; c < P; ++c) {
    int gz = an.z - a.zlo + c;
    if (gz >= a.zwrap) gz -= a.zwrap;
#pragma unroll
    for (int b = 0; b < P; ++b) {
      int gy = an.y + b;
      if (gy >= ag.ny) gy -= ag.ny;
      const int64_t row = ((int64_t)gz * ag.ny + gy) * ag.nx;
      const double wzy = wy[0][b] * wz[0][c];
      if (nowrap) {
        const double *p0 = base + (row + an.x) * 3;
        const int par = (int)((reinterpret_cast<uintptr_t>(p0) >> 3) & 1);
        const double2 *q = reinterpret_cast<const double2 *>(p0 - par);
        double A[3 * P + 1];
#pragma unroll
        for (int u = 0; u < 3 * P / 2; ++u) {
          const double2 t = q[u];
          A[2 * u] = t.x;
          A[2 * u + 1] = t.y;
        }
        A[3 * P] = par ? p0[3 * P - 1] : 0.0;
#pragma unroll
        for (int k = 0; k < P; ++k) {
          const double wv = wx[0][k] * wzy;
          const double v0 = par ? A[3 * k + 1] : A[3 * k];
          const double v1 = par ? A[3 * k + 2] : A[3 * k + 1];
          const double v2 = par ? A[3 * k + 3] : A[3 * k + 2];
          acc0 += wv * v0;
          acc1 += wv * v1;
          acc2 += wv * v2;
        }
      } else {
#pragma unroll
        for (int k = 0; k < P; ++k) {
          const double wv = wx[0][k] * wzy;
          const double *pt = base + (row + ix[k]) * 3;
          acc0 += wv * pt[0];
          acc1 += wv * pt[1];
          acc2 += wv * pt[2];
        }
      }
    }
  }
  const int64_t atom = a.s_atom[s];
  const double q = a.s_q[s];
  const double sc = -q * a.norm;
  const double v[3] = {sc * acc0, sc * acc1, sc * acc2};
  for (int c = 0; c < 3; ++c) {
    if (a.accumulate) a.forces[atom * 3 + c] += v[c]; else a.forces[atom * 3 + c] = v[c];
  }
}

// Forces-only fp64 gather (even orders, three interleaved fields) with the
// stencil rows loaded by the whole warp.  One thread still owns one sorted
// atom (weights, sums, output), but the rows are fetched cooperatively: for
// every stencil row (c, b) the warp copies the 32 atoms' rows -- C 16-byte
// chunks each, from the row's 16-byte-aligned-down start, plus the odd tail
// double -- into a warp-private staging area with cp.async, lane l taking
// chunks j*32 + l.  One copy instruction then covers about three atoms'
// rows (a few cache lines) instead of 32 rows on 32 lines, and the copies of
// the next row are in flight while the current one is summed (two staging
// rows per warp, odd stride S so that the lanes' chunk reads hit distinct
// banks).  Atoms whose stencil wraps in x (or an unaligned field block) take
// the per-element loads of k_gather_f3v afterwards.  Same products and sums
// in the same order as k_gather_f3v: the same numbers.
template <int P>
struct GatherCoop {
  static constexpr int C = 3 * P / 2 + 1;   // chunks per staged row
  static constexpr int S = C | 1;           // staging stride (chunks)
  static constexpr size_t smem = (size_t)8 * 2 * 32 * S * sizeof(double2);
};

template <int P>
__global__ void __launch_bounds__(256, 2) k_gather_f3c(GatherArgs<double> a) {
  static_assert(P % 2 == 0, "even stencil widths");
  constexpr int C = GatherCoop<P>::C, S = GatherCoop<P>::S;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31;
  double2 *stg = reinterpret_cast<double2 *>(smem_raw) + (size_t)(threadIdx.x >> 5) * 2 * 32 * S;
  const int64_t si = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  bool active = si < a.nslots;
  int64_t s = a.slot_lo + si;
  if (a.range_lo) {
    s = (int64_t)*a.range_lo + si;
    active = active && s < (int64_t)*a.range_hi;
  }
  // warps without an atom leave at once (a slab's grid covers every slot but
  // only its range is live); the others keep all lanes for the shared copies
  if (!__any_sync(0xffffffffu, active)) return;
  int4 an = make_int4(0, 0, 0, 0);
  double wx[1][P], wy[1][P], wz[1][P];
#pragma unroll
  for (int k = 0; k < P; ++k) wx[0][k] = wy[0][k] = wz[0][k] = 0.0;
  if (active) {
    an = a.s_anchor[s];
    axis_kinds<double, P, 1>(a.spline, a.s_t[s * 3 + 0], wx, a.qc);
    axis_kinds<double, P, 1>(a.spline, a.s_t[s * 3 + 1], wy, a.qc);
    axis_kinds<double, P, 1>(a.spline, a.s_t[s * 3 + 2], wz, a.qc);
  }
  const AtomGrid &ag = a.ag;
  const double *base = a.freal + (int64_t)an.w * 3 * a.ng;
  const bool coop = active && an.x + P <= ag.nx && (reinterpret_cast<uintptr_t>(base) & 15) == 0;
  // this lane's row (c, b): aligned-down address | parity bit | staged bit
  auto packed_row = [&](int c, int b) -> unsigned long long {
    int gz = an.z - a.zlo + c;
    if (gz >= a.zwrap) gz -= a.zwrap;
    int gy = an.y + b;
    if (gy >= ag.ny) gy -= ag.ny;
    const uintptr_t u = reinterpret_cast<uintptr_t>(base + (((int64_t)gz * ag.ny + gy) * ag.nx + an.x) * 3);
    const unsigned long long par = (u >> 3) & 1;
    return coop ? ((unsigned long long)(u - 8 * par) | par | 2ull) : 0ull;
  };
  // chunk j*32 + lane of the warp's row: atom (lane) at_j, chunk u_j
  int at[C], uu[C];
#pragma unroll
  for (int j = 0; j < C; ++j) {
    const int idx = j * 32 + lane;
    at[j] = idx / C;
    uu[j] = idx - at[j] * C;
  }
  auto issue = [&](double2 *buf, unsigned long long pk) {
#pragma unroll
    for (int j = 0; j < C; ++j) {
      const unsigned long long q = __shfl_sync(0xffffffffu, pk, at[j]);
      const double *src = reinterpret_cast<const double *>(q & ~15ull);
      double2 *dst = buf + at[j] * S + uu[j];
      if (uu[j] < C - 1) {
        const bool use = (q & 2ull) != 0;
        cp_async16(dst, use ? (const void *)(src + 2 * uu[j]) : (const void *)a.freal, use);
      } else {
        const bool tail = (q & 3ull) == 3ull;   // staged row with an odd start: its last double
        cp_async8(dst, tail ? (const void *)(src + 2 * uu[j]) : (const void *)a.freal, tail);
      }
    }
  };
  double acc0 = 0.0, acc1 = 0.0, acc2 = 0.0;
  issue(stg, packed_row(0, 0));
  cp_async_commit();
#pragma unroll 1
  for (int c = 0; c < P; ++c) {
#pragma unroll
    for (int b = 0; b < P; ++b) {
      const int nc = b + 1 < P ? c : c + 1, nb = b + 1 < P ? b + 1 : 0;
      if (nc < P) issue(stg + ((b + 1) & 1) * 32 * S, packed_row(nc, nb));
      cp_async_commit();
      cp_async_wait<1>();
      __syncwarp();
      const double2 *mine = stg + (b & 1) * 32 * S + lane * S;
      const int par = (int)(packed_row(c, b) & 1ull);
      double A[3 * P + 1];
#pragma unroll
      for (int u = 0; u < 3 * P / 2; ++u) {
        const double2 t = mine[u];
        A[2 * u] = t.x;
        A[2 * u + 1] = t.y;
      }
      A[3 * P] = mine[C - 1].x;
      const double wzy = wy[0][b] * wz[0][c];
#pragma unroll
      for (int k = 0; k < P; ++k) {
        const double wv = wx[0][k] * wzy;
        const double v0 = par ? A[3 * k + 1] : A[3 * k];
        const double v1 = par ? A[3 * k + 2] : A[3 * k + 1];
        const double v2 = par ? A[3 * k + 3] : A[3 * k + 2];
        acc0 += wv * v0;
        acc1 += wv * v1;
        acc2 += wv * v2;
      }
      __syncwarp();
    }
  }
  cp_async_wait<0>();
  if (!active) return;
  if (!coop) {
    // stencil wrapping in x (or an unaligned field block): element loads
    int ix[P];
#pragma unroll
    for (int k = 0; k < P; ++k) { int v = an.x + k; ix[k] = v >= ag.nx ? v - ag.nx : v; }
    acc0 = acc1 = acc2 = 0.0;
#pragma unroll 1
    for (int c = 0; c < P; ++c) {
      int gz = an.z - a.zlo + c;
      if (gz >= a.zwrap) gz -= a.zwrap;
#pragma unroll
      for (int b = 0; b < P; ++b) {
        int gy = an.y + b;
        if (gy >= ag.ny) gy -= ag.ny;
        const int64_t row = ((int64_t)gz * ag.ny + gy) * ag.nx;
        const double wzy = wy[0][b] * wz[0][c];
#pragma unroll
        for (int k = 0; k < P; ++k) {
          const double wv = wx[0][k] * wzy;
          const double *pt = base + (row + ix[k]) * 3;
          acc0 += wv * pt[0];
          acc1 += wv * pt[1];
          acc2 += wv * pt[2];
        }
      }
    }
  }
  const int64_t atom = a.s_atom[s];
  const double q = a.s_q[s];
  const double sc = -q * a.norm;
  const double v[3] = {sc * acc0, sc * acc1, sc * acc2};
  for (int c = 0; c < 3; ++c) {
    if (a.accumulate) a.forces[atom * 3 + c] += v[c]; else a.forces[atom * 3 + c] = v[c];
  }
}

// ---- z-slab decomposition: transpose packing and slab dE/dq ----
// plain copy into another rank's halo planes (peer transport)
template <typename T>
__global__ void k_halo_push(const T *__restrict__ src, T *__restrict__ dst, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
  __threadfence_system();
}

// spec [zs][ny][nxh] -> send [rank d][zs][ys][nxh]; one CTA per send row
template <typename C>
__global__ void k_slab_pack(const C *__restrict__ src, C *__restrict__ dst, int zs, int ny, int ys, int nxh) {
  const int r = blockIdx.x;                 // (d * zs + z) * ys + yl
  const int yl = r % ys, dz = r / ys;
  const int z = dz % zs, d = dz / zs;
  const C *s = src + ((int64_t)z * ny + (int64_t)d * ys + yl) * nxh;
  C *o = dst + (int64_t)r * nxh;
  for (int x = threadIdx.x; x < nxh; x += blockDim.x) o[x] = s[x];
}

// receive [rank s][F][zs][ys][nxh] -> fspec [F][zs][ny][nxh]; one CTA per row
template <typename C>
__global__ void k_slab_unpack(const C *__restrict__ src, C *__restrict__ dst, int F, int zs, int ny, int ys,
                              int nxh) {
  const int r = blockIdx.x;                 // (f * zs + z) * ny + y
  const int y = r % ny, fz = r / ny;
  const int z = fz % zs, f = fz / zs;
  const int s = y / ys, yl = y - s * ys;
  const C *in = src + ((((int64_t)s * F + f) * zs + z) * ys + yl) * nxh;
  C *o = dst + (int64_t)r * nxh;
  for (int x = threadIdx.x; x < nxh; x += blockDim.x) o[x] = in[x];
}

// dE/dq finalisation for the atoms of this rank's slab (slots [*lo, *hi))
template <typename T>
__global__ void k_finalize_slab(const FrameGeom *__restrict__ geom, const double *__restrict__ fscal,
                                const double *__restrict__ qsum, const T *__restrict__ q, T *__restrict__ pot,
                                const int32_t *__restrict__ s_atom, const uint32_t *lo, const uint32_t *hi,
                                int64_t bound, int nch, double norm, double self_coeff, double lambda,
                                int remove_self, int k0) {
  const int64_t si = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (si >= bound) return;
  const int64_t s = (int64_t)*lo + si;
  if (s >= (int64_t)*hi) return;
  finalize_atom_pot<T>(geom[0], fscal, 0, qsum, q, pot, s_atom[s], nch, norm, self_coeff, lambda, remove_self, k0);
}

}  // namespace sogb

// ==========================================================================
// host side
// ==========================================================================
using namespace sogb;

namespace {

inline unsigned nblocks(int64_t n, int b) { return (unsigned)((n + b - 1) / b); }

// bookkeeping after a launch: launch counter and optional timing event
inline void after(Tracer *tr, cudaStream_t st, const char *name, int n = 1) {
  count_launch(n);
  if (tr) tr->mark(st, name);
}

void make_twiddles(int n, int dtype, std::vector<unsigned char> &buf) {
  if (dtype == SOG_DTYPE_F64) {
    buf.resize(sizeof(double2) * n);
    double2 *t = reinterpret_cast<double2 *>(buf.data());
    for (int m = 0; m < n; ++m) {
      const long double a = -2.0L * 3.141592653589793238462643383279502884L * (long double)m / (long double)n;
      t[m].x = (double)cosl(a);
      t[m].y = (double)sinl(a);
    }
  } else {
    buf.resize(sizeof(float2) * n);
    float2 *t = reinterpret_cast<float2 *>(buf.data());
    for (int m = 0; m < n; ++m) {
      const long double a = -2.0L * 3.141592653589793238462643383279502884L * (long double)m / (long double)n;
      t[m].x = (float)cosl(a);
      t[m].y = (float)sinl(a);
    }
  }
}

int upload(DevBuf &b, const void *src, size_t bytes) {
  if (b.reserve(bytes) != SOG_OK) return fail(SOG_ERR_NOMEM, "device allocation failed");
  SOG_CUDA_TRY(cudaMemcpy(b.p, src, bytes, cudaMemcpyHostToDevice));
  return SOG_OK;
}

bool smooth235(int n) {
  for (int p : {2, 3, 5})
    while (n % p == 0) n /= p;
  return n == 1;
}

// exclusive scan of n uint32 (in -> out), temp buffer sized by scan_temp_elems
int64_t scan_temp_elems(int64_t n) { return (n + kScanBlock - 1) / kScanBlock + 1; }

void launch_scan(const uint32_t *in, uint32_t *out, int64_t n, uint32_t *tmp, cudaStream_t st,
                 Tracer *tr) {
  const int64_t nb = (n + kScanBlock - 1) / kScanBlock;
  if (nb == 0) return;
  k_scan_local<<<(unsigned)nb, kScanBlock, 0, st>>>(in, out, n, tmp);
  k_scan_sums<<<1, kScanBlock, 0, st>>>(tmp, nb);
  k_scan_add<<<(unsigned)nb, kScanBlock, 0, st>>>(out, n, tmp);
  after(tr, st, "scan", 3);
}

template <typename T>
size_t fft_rows_smem(int n, int rows) { return 2 * (size_t)rows * n * sizeof(cplx_t<T>); }

template <typename T>
int rows_per_cta(int n) {
  const size_t budget = 64 * 1024;
  int r = (int)(budget / (2 * (size_t)n * sizeof(cplx_t<T>)));
  return std::max(1, std::min(r, 64));
}

// columns per CTA of the generic strided pass: a power of two (the smem
// transform maps lanes to columns with a mask)
template <typename T>
int cols_per_cta(int n) {
  const size_t budget = 64 * 1024;
  const int r = (int)(budget / (2 * (size_t)n * sizeof(cplx_t<T>)));
  int ic = 1;
  while (ic * 2 <= std::min(r, 16)) ic *= 2;
  return ic;
}

// Persistent grids: one wave of resident CTAs looping over the tiles.
template <typename K>
unsigned persistent_grid(K kernel, int threads, size_t smem, int64_t ntiles) {
  static std::atomic<int> sm_count[64];
  int dev = 0;
  cudaGetDevice(&dev);
  int nsm = sm_count[dev & 63].load(std::memory_order_relaxed);
  if (!nsm) {
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    if (nsm <= 0) nsm = 1;
    sm_count[dev & 63].store(nsm, std::memory_order_relaxed);
  }
  // resident CTAs per SM, cached per (kernel, threads, smem, device)
  static std::mutex mu;
  static std::map<std::tuple<const void *, int, size_t, int>, int> cache;
  const auto key = std::make_tuple(reinterpret_cast<const void *>(kernel), threads, smem, dev);
  int per = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto it = cache.find(key);
    if (it != cache.end()) per = it->second;
  }
  if (per == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, threads, smem) != cudaSuccess) {
      cudaGetLastError();
      per = 1;
    }
    per = std::max(per, 1);
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = per;
  }
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(ntiles, (int64_t)nsm * per));
}

// Calls f(std::integral_constant<int, L>) for n = 2^L, 8 <= n <= 1024.
template <typename Fn>
bool with_pow2(int n, Fn &&f) {
  switch (n) {
    case 8: f(std::integral_constant<int, 3>{}); return true;
    case 16: f(std::integral_constant<int, 4>{}); return true;
    case 32: f(std::integral_constant<int, 5>{}); return true;
    case 64: f(std::integral_constant<int, 6>{}); return true;
    case 128: f(std::integral_constant<int, 7>{}); return true;
    case 256: f(std::integral_constant<int, 8>{}); return true;
    case 512: f(std::integral_constant<int, 9>{}); return true;
    case 1024: f(std::integral_constant<int, 10>{}); return true;
    default: return false;
  }
}

// Raises the dynamic shared-memory limit of `kernel` once per device (the
// attribute is per device); later calls only look the pair up.
template <typename K>
void allow_smem(K kernel, int bytes = 220 * 1024) {
  static std::mutex mu;
  static std::set<std::pair<const void *, int>> seen;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (seen.insert({reinterpret_cast<const void *>(kernel), dev}).second)
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// The plan's roots of unity of axis 0/1/2 in the transform type T (an fp32
// plan keeps an fp64 copy for its fp64 forward transforms).
template <typename T>
const cplx_t<T> *tw_of(const sog_plan *p, int axis) {
  const bool wide = sizeof(T) == 8 && p->d.dtype == SOG_DTYPE_F32;
  const DevBuf &b = axis == 0 ? (wide ? p->twx64 : p->twx) : axis == 1 ? (wide ? p->twy64 : p->twy)
                                                                        : (wide ? p->twz64 : p->twz);
  return b.as<cplx_t<T>>();
}

// ---- FFT passes: register-resident kernels for power-of-two axes, the
// generic shared-memory Stockham otherwise ----
template <typename T>
int reg_width(int n, int max_threads, size_t smem_budget) {
  const int tpt = n / kEPT;
  const int by_threads = std::max(1, max_threads / tpt);
  const int by_smem = std::max(1, (int)(smem_budget / ((size_t)n * sizeof(cplx_t<T>))));
  int w = std::max(1, std::min(by_threads, by_smem));
  while (w & (w - 1)) w &= w - 1;   // a power of two (the column loads shift and mask)
  return w;
}

template <typename T>
void pass_x_fwd(sog_plan *p, T *rho, cplx_t<T> *spec, int64_t rows, cudaStream_t st) {
  using C = cplx_t<T>;
  const int nx = p->d.nx;
  if constexpr (sizeof(T) == 8 && SOG_COLS_TMA) {
    // fp64 512-point rows: bulk-copied rows, one warp per row
    if (nx == 512 && launch_r2c_tma(reinterpret_cast<const double *>(rho), reinterpret_cast<double2 *>(spec), rows, nx,
                                    reinterpret_cast<const double2 *>(tw_of<T>(p, 0)), p->status.as<unsigned>(), st)) {
      after(&p->tr, st, "fft_r2c_x");
      return;
    }
  }
  const bool done = nx >= 16 && with_pow2(nx, [&](auto lc) {
    constexpr int L = decltype(lc)::value < 4 ? 4 : decltype(lc)::value;
    constexpr int n = 1 << L;
    const int tpt = n / 2 / kEPT;
    const int rpc = std::max(1, 256 / tpt);
    const int64_t ntiles = (rows + rpc - 1) / rpc;
    const int thr = tpt * rpc;
    const size_t sm = 2 * (size_t)rpc * n * sizeof(T) + ((size_t)rpc * padded_row(n / 2) + n + n / 2) * sizeof(C);
    allow_smem(k_r2c_pipe<T, L>);
    k_r2c_pipe<T, L><<<persistent_grid(k_r2c_pipe<T, L>, thr, sm, ntiles), thr, sm, st>>>(
        rho, spec, rows, rpc, ntiles, tw_of<T>(p, 0));
  });
  if (!done) {
    if (is_pow2(nx)) {
      const int rpc = reg_width<T>(nx, 256, 64 * 1024);
      k_rows_r2c_reg<T><<<nblocks(rows, rpc), (nx / kEPT) * rpc, (size_t)rpc * padded_row(nx) * sizeof(C), st>>>(
          rho, spec, rows, rpc, p->rpx, tw_of<T>(p, 0));
    } else if (nx % 2 == 0) {
      const int rpc = rows_per_cta<T>(nx / 2);
      k_fft_r2c_xh<T><<<nblocks(rows, rpc), 256, fft_rows_smem<T>(nx / 2, rpc), st>>>(
          rho, spec, nx, rows, rpc, p->rpxh, tw_of<T>(p, 0));
    } else {
      const int rpc = rows_per_cta<T>(nx);
      k_fft_r2c_x<T><<<nblocks(rows, rpc), 256, fft_rows_smem<T>(nx, rpc), st>>>(
          rho, spec, nx, rows, rpc, p->rpx, tw_of<T>(p, 0));
    }
  }
  after(&p->tr, st, "fft_r2c_x");
}

// F fields of nframes frames -> interleaved real fields [frame][zy][x][F]
template <typename T>
// nzy rows per field and frame: fspec [nframes][F][nzy][nx/2+1] -> freal
// [nframes][nzy][nx][F]
void pass_x_inv(sog_plan *p, cplx_t<T> *fspec, T *freal, int64_t nframes, int64_t nzy, int F, cudaStream_t st) {
  using C = cplx_t<T>;
  const int nx = p->d.nx;
  if constexpr (sizeof(T) == 8 && SOG_COLS_TMA) {
    // fp64 512-point rows: bulk-copied rows, one warp per row and field
    if (nx == 512 && launch_c2r_tma(reinterpret_cast<const double2 *>(fspec), reinterpret_cast<double *>(freal), F,
                                    nzy, nframes * nzy, nx, reinterpret_cast<const double2 *>(tw_of<T>(p, 0)),
                                    p->status.as<unsigned>(), st)) {
      after(&p->tr, st, "fft_c2r_x");
      return;
    }
  }
  const bool done = nx >= 16 && with_pow2(nx, [&](auto lc) {
    constexpr int L = decltype(lc)::value < 4 ? 4 : decltype(lc)::value;
    constexpr int n = 1 << L;
    const int tpt = n / 2 / kEPT;
    const int rpc = std::max(1, 256 / (tpt * F));
    const int64_t rows = nframes * nzy;
    const int64_t ntiles = (rows + rpc - 1) / rpc;
    const int nxh = n / 2 + 1;
    const int thr = tpt * F * rpc;
    const size_t rowsz = std::max<size_t>(nxh, padded_row(n / 2));
    const size_t sm = (2 * (size_t)rpc * F * rowsz + n + n / 2) * sizeof(C);
    allow_smem(k_c2r_pipe<T, L>);
    k_c2r_pipe<T, L><<<persistent_grid(k_c2r_pipe<T, L>, thr, sm, ntiles), thr, sm, st>>>(
        fspec, freal, F, nzy, rows, rpc, ntiles, tw_of<T>(p, 0));
  });
  if (!done) {
    if (is_pow2(nx)) {
      const int tpt = nx / kEPT;
      const int rpc = std::max(1, 256 / (tpt * F));
      const int64_t rows = nframes * nzy;
      const size_t sm = std::max((size_t)rpc * F * padded_row(nx) * sizeof(C), (size_t)rpc * nx * F * sizeof(T));
      k_rows_c2r_il<T><<<nblocks(rows, rpc), tpt * F * rpc, sm, st>>>(fspec, freal, F, nzy, rows, rpc, p->rpx,
                                                                        tw_of<T>(p, 0));
    } else if (nx % 2 == 0) {
      const int rpc = std::max(1, std::min(256 / F, rows_per_cta<T>(nx / 2 + 1) / F));
      const int64_t rows = nframes * nzy;
      k_fft_c2r_xh<T><<<nblocks(rows, rpc), 256, fft_rows_smem<T>(nx / 2 + 1, rpc * F), st>>>(
          fspec, freal, nx, rows, rpc, p->rpxh, tw_of<T>(p, 0), F, nzy);
    } else {
      const int rpc = std::max(1, rows_per_cta<T>(nx + 1) / F);
      const int64_t rows = nframes * nzy;
      k_fft_c2r_x<T><<<nblocks(rows, rpc), 256, fft_rows_smem<T>(nx + 1, rpc * F), st>>>(
          fspec, freal, nx, rows, rpc, p->rpx, tw_of<T>(p, 0), F, nzy);
    }
  }
  after(&p->tr, st, "fft_c2r_x");
}

// C2C over an axis of length n with `inner` contiguous columns per slab.
template <typename T, int DIR>
void pass_cols(sog_plan *p, cplx_t<T> *data, int n, int64_t inner, int64_t outer, const RadixPlan &rp,
               const cplx_t<T> *tw, cudaStream_t st, const char *name) {
  using C = cplx_t<T>;
  if constexpr (sizeof(T) == 8 && SOG_COLS_TMA) {
    // fp64 256- and 512-point axes: warp-resident transforms fed by TMA tiles
    if ((n == 256 || n == 512) &&
        launch_cols_tma(reinterpret_cast<double2 *>(data), n, inner, outer, DIR,
                        reinterpret_cast<const double2 *>(tw), p->status.as<unsigned>(), st)) {
      after(&p->tr, st, name);
      return;
    }
  }
  const bool done = with_pow2(n, [&](auto lc) {
    constexpr int L = decltype(lc)::value;
    constexpr int nn = 1 << L;
    // fp32 columns are 8 bytes: 512-thread tiles keep each tile row of the
    // long axes at 64 bytes or more
    constexpr int thr_cap = sizeof(T) == 4 ? 512 : SOG_COLS_THR64;
    const int ic = reg_width<T>(nn, thr_cap, thr_cap * 256);
    const int64_t nchunks = (inner + ic - 1) / ic;
    const int64_t ntiles = outer * nchunks;
    const int thr = (nn / kEPT) * ic;
    if (ic >= 8) {
      const size_t sm = (3 * (size_t)nn * ic + nn) * sizeof(C);
      allow_smem(k_cols_pipe<T, DIR, false, L>);
      k_cols_pipe<T, DIR, false, L><<<persistent_grid(k_cols_pipe<T, DIR, false, L>, thr, sm, ntiles), thr, sm,
                                      st>>>(data, inner, ic, ntiles, tw);
    } else {
      const size_t sm = ((2 * (size_t)nn + padded_row(nn)) * ic + nn) * sizeof(C);
      allow_smem(k_cols_pipe<T, DIR, true, L>);
      k_cols_pipe<T, DIR, true, L><<<persistent_grid(k_cols_pipe<T, DIR, true, L>, thr, sm, ntiles), thr, sm,
                                     st>>>(data, inner, ic, ntiles, tw);
    }
  });
  if (!done) {
    if (is_pow2(n)) {
      const int ic = reg_width<T>(n, 256, 64 * 1024);
      const int64_t nchunks = (inner + ic - 1) / ic;
      if (ic >= 8)
        k_cols_reg<T, DIR, false><<<(unsigned)(outer * nchunks), (n / kEPT) * ic, (size_t)n * ic * sizeof(C), st>>>(
            data, inner, ic, rp, tw);
      else
        k_cols_reg<T, DIR, true><<<(unsigned)(outer * nchunks), (n / kEPT) * ic,
                                   (size_t)padded_row(n) * ic * sizeof(C), st>>>(data, inner, ic, rp, tw);
    } else {
      const int ic = cols_per_cta<T>(n);
      const int64_t nchunks = (inner + ic - 1) / ic;
      k_fft_strided<T, DIR><<<(unsigned)(outer * nchunks), 256, fft_rows_smem<T>(n, ic), st>>>(
          data, inner, outer, ic, rp, tw);
    }
  }
  after(&p->tr, st, name);
}

// Inverse y pass of the field spectra with the field formation of two-slot
// frames (k_cols_fields); power-of-two ny.
template <typename T>
void pass_cols_fields(sog_plan *p, cplx_t<T> *fspec, const FrameGeom *geom, int nf, int F, int two_slot,
                      int want_pot, cudaStream_t st) {
  using C = cplx_t<T>;
  const int ny = p->d.ny, nz = p->d.nz;
  const int64_t inner = p->nxh;
  if constexpr (sizeof(T) == 8 && SOG_COLS_TMA) {
    if ((ny == 256 || ny == 512) &&
        launch_cols_fields_tma(reinterpret_cast<double2 *>(fspec), geom, nf, F, nz, ny, inner,
                               reinterpret_cast<const double2 *>(tw_of<T>(p, 1)), two_slot, want_pot,
                               p->status.as<unsigned>(), st)) {
      after(&p->tr, st, "fft_y_inv");
      return;
    }
  }
  with_pow2(ny, [&](auto lc) {
    constexpr int L = decltype(lc)::value;
    constexpr int nn = 1 << L;
    constexpr int thr_cap = sizeof(T) == 4 ? 512 : SOG_COLS_THR64;
    const int ic = reg_width<T>(nn, thr_cap, thr_cap * 256);
    const int64_t ntiles = (int64_t)nf * F * nz * ((inner + ic - 1) / ic);
    const int thr = (nn / kEPT) * ic;
    if (ic >= 8) {
      const size_t sm = (3 * (size_t)nn * ic + nn) * sizeof(C);
      allow_smem(k_cols_fields<T, false, L>);
      k_cols_fields<T, false, L><<<persistent_grid(k_cols_fields<T, false, L>, thr, sm, ntiles), thr, sm, st>>>(
          fspec, geom, F, nz, inner, ic, ntiles, tw_of<T>(p, 1), two_slot, want_pot);
    } else {
      const size_t sm = ((2 * (size_t)nn + padded_row(nn)) * ic + nn) * sizeof(C);
      allow_smem(k_cols_fields<T, true, L>);
      k_cols_fields<T, true, L><<<persistent_grid(k_cols_fields<T, true, L>, thr, sm, ntiles), thr, sm, st>>>(
          fspec, geom, F, nz, inner, ic, ntiles, tw_of<T>(p, 1), two_slot, want_pot);
    }
  });
  after(&p->tr, st, "fft_y_inv");
}

template <typename T>
void set_fft_smem_attrs() {
  const int big = 200 * 1024;
  allow_smem(k_fft_r2c_x<T>, big);
  allow_smem(k_fft_c2r_x<T>, big);
  allow_smem(k_fft_r2c_xh<T>, big);
  allow_smem(k_fft_c2r_xh<T>, big);
  allow_smem(k_fft_strided<T, -1>, big);
  allow_smem(k_fft_strided<T, +1>, big);
  allow_smem(k_cols_reg<T, -1, false>, big);
  allow_smem(k_cols_reg<T, +1, false>, big);
  allow_smem(k_cols_reg<T, -1, true>, big);
  allow_smem(k_cols_reg<T, +1, true>, big);
  allow_smem(k_rows_r2c_reg<T>, big);
  allow_smem(k_rows_c2r_il<T>, big);
  allow_smem(k_zfused<T>, big);
}

template <typename T, int P, int NT = 1>
size_t spread_smem() {
  constexpr int KK = StencilTerms<NT>::K;
  constexpr int CH = KK == 3 ? kSpreadThreads / 2 : kSpreadThreads;
  return (size_t)CH * (KK * (kTileZ + 2 * P) + 1) * sizeof(T) + (size_t)CH * sizeof(int);
}

template <typename T, int P, int NT, typename TG>
void launch_spread(const SpreadArgs<T> &sa, int nframes, cudaStream_t st, Tracer *tr) {
  const size_t sm = spread_smem<T, P, NT>();
  allow_smem(k_spread<T, P, NT, TG>, (int)sm);
  const int64_t tiles = (int64_t)sa.ntx * sa.nty * sa.ntz * nframes;
  k_spread<T, P, NT, TG><<<(unsigned)tiles, kSpreadThreads, sm, st>>>(sa);
  after(tr, st, "spread");
}

// z split of the Green-table pass when its (mx, y) columns do not fill one
// wave of resident CTAs (two per SM); splitting a full wave further costs
// more (the x-y kernel products are rebuilt per split) than it gains
// Launches both Green kernels (separable frames, others) on one grid; the
// separable one holds its planes' z factors in shared memory.
template <typename T>
void launch_green(const KsArgs<T> &ka, unsigned gblocks, int nf, unsigned gz, cudaStream_t st);

inline unsigned green_zsplit(unsigned gblocks, int nf, int nz) {
  const int64_t have = (int64_t)gblocks * nf;
  const int64_t want = 2 * 148;
  int64_t gz = std::max<int64_t>(1, std::min<int64_t>({8, (want + have - 1) / have, (int64_t)nz}));
  // a block's z factors ([zper][16] doubles at most) stay within 96 KB
  while ((nz + gz - 1) / gz * 16 * (int64_t)sizeof(double) > 96 * 1024) ++gz;
  return (unsigned)gz;
}

// Separable splines: one warp per 8^3 block of mesh points (k_spread_blk).
template <typename T, int P, typename TG>
void launch_spread_blk(const SpreadArgs<T> &sa, int nframes, cudaStream_t st, Tracer *tr) {
  const int nbx = (sa.ag.nx + 7) / 8, nby = (sa.ag.ny + 7) / 8, nbz = (sa.zcnt + 7) / 8;
  const int64_t nblk = (int64_t)nbx * nby * nbz * nframes;
  const unsigned grid = (unsigned)((nblk + kWarpsPerSpreadCta - 1) / kWarpsPerSpreadCta);
  if (grid) k_spread_blk<T, P, TG><<<grid, 32 * kWarpsPerSpreadCta, 0, st>>>(sa, nbx, nby, nbz, nblk);
  after(tr, st, "spread");
}

template <typename T, typename TG = T>
void dispatch_spread(const SpreadArgs<T> &sa, int order, int nframes, cudaStream_t st, Tracer *tr) {
  if (SOG_SPREAD_BLK && sa.spline != SOG_SPLINE_CUBES2) {
    switch (order) {
      case 4: launch_spread_blk<T, 4, TG>(sa, nframes, st, tr); break;
      case 5: launch_spread_blk<T, 5, TG>(sa, nframes, st, tr); break;
      default: launch_spread_blk<T, 6, TG>(sa, nframes, st, tr); break;
    }
    return;
  }
  if (sa.spline == SOG_SPLINE_CUBES2) {
    if (order == 4) launch_spread<T, 4, 3, TG>(sa, nframes, st, tr);
    else launch_spread<T, 6, 4, TG>(sa, nframes, st, tr);
    return;
  }
  switch (order) {
    case 4: launch_spread<T, 4, 1, TG>(sa, nframes, st, tr); break;
    case 5: launch_spread<T, 5, 1, TG>(sa, nframes, st, tr); break;
    default: launch_spread<T, 6, 1, TG>(sa, nframes, st, tr); break;
  }
}

template <typename T>
void dispatch_gather(const GatherArgs<T> &ga, int order, cudaStream_t st, Tracer *tr) {
  const unsigned nb = nblocks(ga.nslots, 256);
  if (nb == 0) return;
  if (ga.spline == SOG_SPLINE_CUBES2) {
    if (order == 4) k_gather<T, 4, 3><<<nb, 256, 0, st>>>(ga);
    else k_gather<T, 6, 4><<<nb, 256, 0, st>>>(ga);
    after(tr, st, "gather");
    return;
  }
  if constexpr (std::is_same<T, double>::value) {
    // forces only (three interleaved fields): vector row loads
    if (SOG_GATHER_VEC && ga.nfield == 3 && ga.want_force && !ga.want_pot && (order == 4 || order == 6)) {
      if (SOG_GATHER_COOP) {
        if (order == 4) {
          allow_smem(k_gather_f3c<4>, (int)GatherCoop<4>::smem);
          k_gather_f3c<4><<<nb, 256, GatherCoop<4>::smem, st>>>(ga);
        } else {
          allow_smem(k_gather_f3c<6>, (int)GatherCoop<6>::smem);
          k_gather_f3c<6><<<nb, 256, GatherCoop<6>::smem, st>>>(ga);
        }
      } else if (order == 4) {
        k_gather_f3v<4><<<nb, 256, 0, st>>>(ga);
      } else {
        k_gather_f3v<6><<<nb, 256, 0, st>>>(ga);
      }
      after(tr, st, "gather");
      return;
    }
  }
  switch (order) {
    case 4: k_gather<T, 4><<<nb, 256, 0, st>>>(ga); break;
    case 5: k_gather<T, 5><<<nb, 256, 0, st>>>(ga); break;
    default: k_gather<T, 6><<<nb, 256, 0, st>>>(ga); break;
  }
  after(tr, st, "gather");
}

template <typename T>
void dispatch_gather_dedr(const GatherArgs<T> &ga, int order, cudaStream_t st, Tracer *tr) {
  const unsigned nb = nblocks(ga.nslots, 256);
  if (nb == 0) return;
  switch (order) {
    case 4: k_gather_dedr<T, 4><<<nb, 256, 0, st>>>(ga); break;
    case 5: k_gather_dedr<T, 5><<<nb, 256, 0, st>>>(ga); break;
    default: k_gather_dedr<T, 6><<<nb, 256, 0, st>>>(ga); break;
  }
  after(tr, st, "gather_dedr");
}

// Frames, geometry, cell sort and charge sums of one call (shared by the
// single-device and the slab paths).
struct Prep {
  FrameGeom *geom = nullptr;
  unsigned *status = nullptr;
  AtomGrid ag{};
  int64_t nslots = 0, maxat = 0;
};

template <typename T>
int prepare_atoms(sog_plan *p, const sog_mesh_args *a, cudaStream_t st, Prep &pr, int zb = SOG_BIN_ZB) {
  const int nf = a->nframes, nch = a->nchannels;
  const int nx = p->d.nx, ny = p->d.ny, nz = p->d.nz, P = p->d.order;
  Tracer *tr = &p->tr;
  // ---- frames ----
  std::vector<FrameHost> fh(nf);
  int64_t nslots = 0, maxat = 0;
  for (int f = 0; f < nf; ++f) {
    if (a->atom_count[f] < 0 || a->atom_begin[f] < 0) return fail(SOG_ERR_INVALID, "negative atom range");
    fh[f].atom_begin = a->atom_begin[f];
    fh[f].natoms = a->atom_count[f];
    fh[f].slot_base = nslots;
    fh[f].k_sq_max = a->k_sq_max[f];
    nslots += a->atom_count[f];
    maxat = std::max<int64_t>(maxat, a->atom_count[f]);
  }
  if (nslots >= (int64_t)1 << 31) return fail(SOG_ERR_INVALID, "more than 2^31 atoms in one call");
  int rc;
  if (p->frames_host_dev.reserve(sizeof(FrameHost) * nf) || p->geom.reserve(sizeof(FrameGeom) * nf) ||
      p->status.reserve(sizeof(unsigned) * 4))
    return fail(SOG_ERR_NOMEM, "device allocation failed");
  if (nf <= kFramesByValue) {
    // small frame tables travel as a kernel parameter: no host wait
    FrameTable ft;
    std::memset(&ft, 0, sizeof(ft));
    std::memcpy(ft.fh, fh.data(), sizeof(FrameHost) * nf);
    ft.nf = nf;
    k_store_frames<<<1, 32, 0, st>>>(ft, p->frames_host_dev.as<FrameHost>());
    count_launch();
  } else {
    // larger tables through the pinned staging buffer (waits for its previous copy)
    if ((rc = p->up.reserve(sizeof(FrameHost) * nf)) != SOG_OK) return rc;
    if ((rc = p->up.wait()) != SOG_OK) return rc;
    std::memcpy(p->up.p, fh.data(), sizeof(FrameHost) * nf);
    SOG_CUDA_TRY(cudaMemcpyAsync(p->frames_host_dev.p, p->up.p, sizeof(FrameHost) * nf,
                                 cudaMemcpyHostToDevice, st));
    SOG_CUDA_TRY(cudaEventRecord(p->up.done, st));
    p->up.pending = true;
  }
  FrameGeom *geom = p->geom.as<FrameGeom>();
  unsigned *status = p->status.as<unsigned>();
  tr->begin(st);
  k_frame_setup<T><<<nblocks(nf, 128), 128, 0, st>>>((const T *)a->cells, p->frames_host_dev.as<FrameHost>(),
                                                     geom, nf, p->d.kconv, nx, ny, nz, status,
                                                     p->d.spline == SOG_SPLINE_CUBES2 ? cubes2_xi(P) : 0.0);
  after(tr, st, "frame_setup");

  // ---- atom sort ----
  AtomGrid ag;
  ag.nx = nx; ag.ny = ny; ag.nz = nz;
  // first stencil node: floor index + 1 - P/2 for QuadS (quads_fft.py) and
  // CubeS2 (offsets -1..2 / -2..3, cubes2_spline.py), - (P-1)/2 for B-splines
  ag.first = (p->d.spline == SOG_SPLINE_BSPLINE) ? -((P - 1) / 2) : (1 - P / 2);
  ag.nbx = p->nb_x; ag.nby = p->nb_y; ag.nbz = p->nb_z;
  ag.zb = std::max(1, std::min(zb, ag.nbz));
  ag.bins_per_frame = (uint32_t)ag.nbx * ag.nby * ag.nbz;
  const uint64_t nbins64 = (uint64_t)ag.bins_per_frame * nf;
  if (nbins64 >= (1ull << 32) - 1) return fail(SOG_ERR_INVALID, "too many sort bins in one call");
  const uint32_t nbins = (uint32_t)nbins64;
  const int64_t sort_blocks = std::max<int64_t>(1, (nslots + kSortTile - 1) / kSortTile);
  const int64_t hist_n = sort_blocks * kRadixBuckets;
  const int64_t scan_n = std::max<int64_t>(hist_n, (int64_t)nbins + 1);
  if (p->keys0.reserve(4 * std::max<int64_t>(nslots, 1)) || p->vals0.reserve(4 * std::max<int64_t>(nslots, 1)) ||
      p->keys1.reserve(4 * std::max<int64_t>(nslots, 1)) || p->vals1.reserve(4 * std::max<int64_t>(nslots, 1)) ||
      p->hist.reserve(4 * scan_n) || p->scan_tmp.reserve(4 * scan_temp_elems(scan_n)) ||
      p->bin_start.reserve(4 * ((int64_t)nbins + 1)) ||
      p->s_anchor.reserve(sizeof(int4) * std::max<int64_t>(nslots, 1)) ||
      p->s_t.reserve(sizeof(T) * 3 * std::max<int64_t>(nslots, 1)) ||
      p->s_q.reserve(sizeof(T) * nch * std::max<int64_t>(nslots, 1)) ||
      p->s_atom.reserve(4 * std::max<int64_t>(nslots, 1)) ||
      p->qsum.reserve(sizeof(double) * 2 * nf * nch))
    return fail(SOG_ERR_NOMEM, "device allocation failed");
  uint32_t *k0 = p->keys0.as<uint32_t>(), *k1 = p->keys1.as<uint32_t>();
  int32_t *v0 = p->vals0.as<int32_t>(), *v1 = p->vals1.as<int32_t>();
  if (maxat > 0)
    k_atom_bin<T><<<dim3(nblocks(maxat, 256), nf), 256, 0, st>>>(
        (const T *)a->positions, (const T *)a->charges, nch, geom, ag, k0, v0, status);
  if (maxat > 0) after(tr, st, "atom_bin");
  int keybits = 1;
  while (keybits < 32 && (1ull << keybits) <= (uint64_t)nbins) ++keybits;
  for (int shift = 0; shift < keybits; shift += kRadixBits) {
    if (nslots == 0) break;
    k_radix_hist<<<(unsigned)sort_blocks, kSortThreads, 0, st>>>(k0, nslots, shift, p->hist.as<uint32_t>(),
                                                                 (int)sort_blocks);
    after(tr, st, "radix_hist");
    launch_scan(p->hist.as<uint32_t>(), p->hist.as<uint32_t>(), hist_n, p->scan_tmp.as<uint32_t>(), st, tr);
    k_radix_scatter<<<(unsigned)sort_blocks, kSortThreads, 0, st>>>(k0, v0, k1, v1, nslots, shift,
                                                                    p->hist.as<uint32_t>(), (int)sort_blocks);
    after(tr, st, "radix_scatter");
    std::swap(k0, k1);
    std::swap(v0, v1);
  }
  k_bin_starts<<<nblocks(nslots + 1, 256), 256, 0, st>>>(k0, nslots, nbins, p->bin_start.as<uint32_t>());
  after(tr, st, "bin_starts");
  if (nslots > 0)
    k_atom_sorted<T><<<nblocks(nslots, 256), 256, 0, st>>>(
        (const T *)a->positions, (const T *)a->charges, nch, geom, ag, k0, v0, nslots,
        p->s_anchor.as<int4>(), p->s_t.as<T>(), p->s_q.as<T>(), p->s_atom.as<int32_t>());
  if (nslots > 0) after(tr, st, "atom_sorted");
  {
    const int qs = (int)std::max<int64_t>(1, std::min<int64_t>(256, (maxat + 16383) / 16384));
    if (p->qpart.reserve(sizeof(double) * 2 * (int64_t)nf * nch * qs))
      return fail(SOG_ERR_NOMEM, "device allocation failed");
    k_qsums<T><<<dim3(nf, nch, qs), 256, 0, st>>>((const T *)a->charges, nch, geom, p->qpart.as<double>());
    k_reduce_parts<<<dim3(nf, nch, 1), 256, 0, st>>>(p->qpart.as<double>(), nf, nch, qs, 2, 2,
                                                    p->qsum.as<double>());
    after(tr, st, "qsums", 2);
  }

  pr.geom = geom;
  pr.status = status;
  pr.ag = ag;
  pr.nslots = nslots;
  pr.maxat = maxat;
  return SOG_OK;
}

// Both Green kernels on one grid (each takes its frames); with ka.krad the
// radial frames are left to the fused z pass.
template <typename T>
void launch_green(const KsArgs<T> &ka, unsigned gblocks, int nf, unsigned gz, cudaStream_t st) {
  const int zper = (ka.nz + (int)gz - 1) / (int)gz;
  const size_t sm = ka.M <= 16 ? (size_t)zper * ((ka.M + 1) & ~1) * sizeof(double) : 0;
  allow_smem(k_green<T, true>);
  k_green<T, true><<<dim3(gblocks, nf, gz), 256, sm, st>>>(ka);
  count_launch();
  k_green<T, false><<<dim3(gblocks, nf, gz), 256, 0, st>>>(ka);
}

// Radial tables of the call's cubic frames (sized for the mesh's largest
// mx^2 + my^2 + mz^2), before the Green tables.
template <typename T>
int setup_radial(sog_plan *p, KsArgs<T> &ka, int nf, cudaStream_t st) {
  const int64_t hx = p->d.nx / 2, hy = p->d.ny / 2, hz = p->d.nz / 2;
  ka.krad_stride = hx * hx + hy * hy + hz * hz + 1;
  if (p->krad.reserve(sizeof(double) * ka.krad_stride * nf)) return fail(SOG_ERR_NOMEM, "device allocation failed");
  ka.krad = p->krad.as<double>();
  k_radial_table<T><<<dim3((unsigned)std::min<int64_t>((ka.krad_stride + 255) / 256, 1024), nf), 256, 0, st>>>(ka);
  after(&p->tr, st, "radial_table");
  return SOG_OK;
}

// Precision: the charge grid, the forward transforms, the Green multiply and
// the energy sums run in fp64 for every plan; an fp32 plan computes its
// atom data, field spectra, inverse transforms and gather in fp32.  (The
// k-space energy is a difference of two large sums, the mesh term and the
// self term, so the forward transform's rounding is amplified by their
// ratio: in fp32 it alone gave relative energy errors near 2e-5 on the
// 131,072-atom 256^3 system.)
template <typename T>
int mesh_forward_impl(sog_plan *p, const sog_mesh_args *a, cudaStream_t st) {
  using C = cplx_t<T>;       // field spectra
  using TF = double;         // grid, forward spectrum, k-space
  using CF = cplx_t<TF>;
  const int nf = a->nframes, nch = a->nchannels, M = a->n_gauss;
  const int nx = p->d.nx, ny = p->d.ny, nz = p->d.nz, nxh = p->nxh, P = p->d.order;
  const int64_t ng = p->ng, nh = p->nh;
  Prep pr;
  int rc = prepare_atoms<T>(p, a, st, pr);
  if (rc != SOG_OK) return rc;
  FrameGeom *geom = pr.geom;
  const AtomGrid ag = pr.ag;
  const int64_t nslots = pr.nslots, maxat = pr.maxat;
  Tracer *tr = &p->tr;

  // ---- buffers ----
  const bool want_force = a->forces != nullptr;
  const bool want_pot = a->potential != nullptr;
  const bool want_grad = a->grad_amp != nullptr || a->grad_bw2 != nullptr;
  const bool want_vir = a->virial != nullptr;
  const bool want_dedr = a->dedr != nullptr;
  const bool pot_field = want_pot || want_dedr;   // the exact gradient gathers the potential field
  const int nfield = (want_force ? 3 : 0) + (pot_field ? 1 : 0);
  const unsigned ks_blocks = nblocks(nh, 256);
  // the fused z pass writes one partial per tile; the generic k-space kernel one per block
  const int64_t part_blocks = std::max<int64_t>(ks_blocks, (int64_t)ny * nxh);
  const int nx_acc = 4 * M + 13;
  if (p->rho.reserve(sizeof(TF) * ng * nf) || p->spec.reserve(sizeof(CF) * nh * nf) ||
      p->partE.reserve(sizeof(double) * 2 * part_blocks * nf * nch) ||
      (nfield && (p->fspec.reserve(sizeof(C) * nh * nf * nfield) ||
                  p->freal.reserve(sizeof(T) * ng * nf * nfield))) ||
      ((want_grad || want_vir) && p->partX.reserve(sizeof(double) * nx_acc * (int64_t)ks_blocks * nf * nch)) ||
      p->red.reserve(sizeof(double) * ((int64_t)nf * nch * (2 + nx_acc) + (int64_t)nf * 4)) ||
      p->redtmp.reserve(sizeof(double) * std::max(reduce_tmp_elems(nf, nch, part_blocks, 2),
                                                  reduce_tmp_elems(nf, nch, ks_blocks, nx_acc))))
    return fail(SOG_ERR_NOMEM, "device allocation failed (mesh buffers)");

  QuadsCoef qc;
  std::memset(&qc, 0, sizeof(qc));
  if (p->d.spline == SOG_SPLINE_QUADS) quads_coeffs(P, qc.c);

  SpreadArgs<T> sa;
  sa.s_anchor = p->s_anchor.as<int4>();
  sa.s_t = p->s_t.as<T>();
  sa.bin_start = p->bin_start.as<uint32_t>();
  sa.geom = geom;
  sa.rho = p->rho.p;
  sa.ag = ag;
  sa.spline = p->d.spline;
  sa.ntx = (nx + kTileX - 1) / kTileX;
  sa.nty = (ny + kTileY - 1) / kTileY;
  sa.ntz = (nz + kTileZ - 1) / kTileZ;
  sa.qc = qc;
  sa.zlo = 0;
  sa.zcnt = nz;

  KsArgs<TF> ka;
  std::memset(&ka, 0, sizeof(ka));
  ka.spec = p->spec.as<CF>();
  ka.fspec = nfield ? p->fspec.p : nullptr;
  ka.geom = geom;
  ka.tx = p->tab.fx.as<double>(); ka.ty = p->tab.fy.as<double>(); ka.tz = p->tab.fz.as<double>();
  ka.sx = p->tab.sx.as<double>(); ka.sy = p->tab.sy.as<double>(); ka.sz = p->tab.sz.as<double>();
  ka.amp = a->amp;
  ka.bw2 = a->bw2;
  ka.p32 = p->d.dtype == SOG_DTYPE_F32;
  ka.M = M;
  ka.spline = p->d.spline;
  ka.order = P;
  ka.alias_extent = p->d.alias_extent;
  ka.nx = nx; ka.ny = ny; ka.nz = nz; ka.nxh = nxh;
  ka.nh = nh;
  ka.y0 = 0;
  ka.nyl = ny;
  ka.zblk = nz;
  ka.nfield = nfield;
  ka.want_force = want_force;
  ka.nx_acc = nx_acc;
  ka.btab_stride = (int64_t)M * (nxh + ny + nz);
  if (p->btab.reserve(sizeof(double) * ka.btab_stride * nf)) return fail(SOG_ERR_NOMEM, "device allocation failed");
  ka.btab = p->btab.as<double>();
  k_axis_tables<T><<<dim3(nblocks(ka.btab_stride, 256), nf), 256, 0, st>>>(geom, (const T *)a->bw2, M, nx, ny,
                                                                          nz, p->btab.as<double>());
  after(tr, st, "axis_tables");
  ka.gtab = ka.gtabF = ka.partD = nullptr;

  GatherArgs<T> gar;
  gar.s_anchor = p->s_anchor.as<int4>();
  gar.s_t = p->s_t.as<T>();
  gar.s_atom = p->s_atom.as<int32_t>();
  gar.freal = p->freal.as<T>();
  gar.nfield = nfield;
  gar.want_force = want_force;
  gar.want_pot = want_pot;
  gar.nslots = nslots;
  gar.ng = ng;
  gar.ag = ag;
  gar.spline = p->d.spline;
  gar.qc = qc;
  gar.norm = a->norm_factor;
  gar.nch = nch;
  gar.forces = (T *)a->forces;
  gar.pot_raw = (T *)a->potential;
  gar.slot_lo = 0;
  gar.zlo = 0;
  gar.zwrap = nz;
  gar.range_lo = gar.range_hi = nullptr;
  gar.geom = geom;
  gar.dedr = (T *)a->dedr;

  set_fft_smem_attrs<T>();
  if (!std::is_same<T, TF>::value) set_fft_smem_attrs<TF>();
  // power-of-two nz: fused z pass, which evaluates the Green function of
  // separable frames itself and reads k_green's tables for the others;
  // otherwise separate z passes around k_kspace_tab, which reads the tables
  // of every frame.
  const bool zfuse = is_pow2(nz);
  const bool zgeneric = zfuse && nz > 1024;  // runtime-plan fused pass, Green on the fly
  if (zfuse && !zgeneric && (rc = setup_radial<TF>(p, ka, nf, st)) != SOG_OK) return rc;
  // two-slot field spectra (fused z pass -> k_cols_fields) for power-of-two ny
  ka.two_slot = (zfuse && !zgeneric && want_force && is_pow2(ny) && ny <= 1024) ? 1 : 0;
  // fused z pass: 512 threads (8-column tiles) for 512 and 1024 points
  const int zic = zfuse ? (SOG_ZTHR == 512 && nz >= 512 && nz <= 1024 ? reg_width<TF>(nz, 512, 64 * 1024)
                                                   : reg_width<TF>(nz, 256, 32 * 1024))
                        : 0;
  const int64_t zchunks = zfuse ? ((int64_t)ny * nxh + zic - 1) / zic : 0;
  const unsigned tblocks = nblocks((int64_t)ny * nxh, 256);
  const unsigned tz = green_zsplit(tblocks, nf, nz);
  const int64_t nblk_e = zfuse ? zchunks : (int64_t)tblocks * tz;
  double *redD = nullptr;
  if (!zgeneric) {
    // Green tables and the self sum, once per call (independent of the charges)
    const bool aliasable = p->d.spline == SOG_SPLINE_BSPLINE;
    const unsigned gblocks = nblocks((int64_t)ny * nxh, 256);
    const unsigned gz = green_zsplit(gblocks, nf, nz);
    const int64_t gparts = (int64_t)gblocks * gz;
    if (p->gtab.reserve(sizeof(double) * nh * nf) ||
        (aliasable && p->gtabF.reserve(sizeof(double) * nh * nf)) ||
        p->partD.reserve(sizeof(double) * (gparts * nf + nf + reduce_tmp_elems(nf, 1, gparts, 1))))
      return fail(SOG_ERR_NOMEM, "device allocation failed (Green tables)");
    ka.gtab = p->gtab.as<double>();
    ka.gtabF = aliasable ? p->gtabF.as<double>() : nullptr;
    ka.partD = p->partD.as<double>();
    launch_green<TF>(ka, gblocks, nf, gz, st);
    after(tr, st, "green");
    redD = ka.partD + gparts * nf;
    reduce_parts(ka.partD, nf, 1, gparts, 1, 1, redD, redD + nf, st);
    after(tr, st, "reduce_green", reduce_split(gparts) > 1 ? 2 : 1);
  }
  auto launch_zfused = [&]() {
    const int write_spec = (want_grad || want_vir) ? 1 : 0;
    const CF *twz = tw_of<TF>(p, 2);
    const bool done = with_pow2(nz, [&](auto lc) {
      constexpr int L = decltype(lc)::value;
      constexpr int n = 1 << L;
      const int zthr = (n / kEPT) * zic;
      const size_t zsm = ((2 * (size_t)n + padded_row(n)) * zic + n) * sizeof(CF);
      const int64_t ztiles = zchunks * nf;
      if (zthr == 512) {
        allow_smem(k_zfused_g<TF, L, 512, T>);
        k_zfused_g<TF, L, 512, T><<<persistent_grid(k_zfused_g<TF, L, 512, T>, zthr, zsm, ztiles), zthr, zsm,
                                    st>>>(ka, zic, ztiles, twz, write_spec);
      } else {
        allow_smem(k_zfused_g<TF, L, 256, T>);
        k_zfused_g<TF, L, 256, T><<<persistent_grid(k_zfused_g<TF, L, 256, T>, zthr, zsm, ztiles), zthr, zsm,
                                    st>>>(ka, zic, ztiles, twz, write_spec);
      }
    });
    if (!done) {
      const size_t zsm = (size_t)padded_row(nz) * zic * sizeof(CF) +
                         (size_t)(nz / kEPT) * zic * kEPT * (sizeof(CF) + 2 * sizeof(double));
      allow_smem(k_zfused<TF, T>, 200 * 1024);
      k_zfused<TF, T><<<(unsigned)(zchunks * nf), (nz / kEPT) * zic, zsm, st>>>(ka, zic, p->rpz, twz, write_spec);
    }
  };
  for (int c = 0; c < nch; ++c) {
    sa.s_q = p->s_q.as<T>() + (int64_t)c * nslots;
    dispatch_spread<T, TF>(sa, P, nf, st, tr);
    pass_x_fwd<TF>(p, p->rho.as<TF>(), p->spec.as<CF>(), (int64_t)nf * nz * ny, st);
    pass_cols<TF, -1>(p, p->spec.as<CF>(), ny, nxh, (int64_t)nf * nz, p->rpy, tw_of<TF>(p, 1), st, "fft_y_fwd");
    ka.part = p->partE.as<double>() + (int64_t)c * nf * nblk_e * 2;
    if (zfuse) {
      launch_zfused();
      after(tr, st, "zfused");
    } else {
      pass_cols<TF, -1>(p, p->spec.as<CF>(), nz, (int64_t)ny * nxh, nf, p->rpz, tw_of<TF>(p, 2), st, "fft_z_fwd");
      k_kspace_tab<TF, T><<<dim3(tblocks, nf, tz), 256, 0, st>>>(ka);
      after(tr, st, "kspace");
    }
    if (want_grad || want_vir) {
      ka.partx = p->partX.as<double>() + (int64_t)c * nf * ks_blocks * nx_acc;
      k_kspace_extra<TF><<<dim3(ks_blocks, nf), 256, 0, st>>>(ka, want_grad, want_vir);
      after(tr, st, "kspace_extra");
    }
    if (nfield) {
      const int64_t nb = (int64_t)nf * nfield;
      if (!zfuse)
        pass_cols<T, +1>(p, p->fspec.as<C>(), nz, (int64_t)ny * nxh, nb, p->rpz, tw_of<T>(p, 2), st,
                         "fft_z_inv");
      if (ka.two_slot)
        pass_cols_fields<T>(p, p->fspec.as<C>(), geom, nf, nfield, 1, pot_field ? 1 : 0, st);
      else
        pass_cols<T, +1>(p, p->fspec.as<C>(), ny, nxh, nb * nz, p->rpy, tw_of<T>(p, 1), st, "fft_y_inv");
      pass_x_inv<T>(p, p->fspec.as<C>(), p->freal.as<T>(), nf, (int64_t)nz * ny, nfield, st);
      gar.s_q = p->s_q.as<T>() + (int64_t)c * nslots;
      gar.channel = c;
      gar.accumulate = c > 0;
      if (want_force || want_pot) dispatch_gather<T>(gar, P, st, tr);
      if (want_dedr) dispatch_gather_dedr<T>(gar, P, st, tr);
    }
  }
  // ---- reductions / finalisation ----
  double *redE = p->red.as<double>();
  double *redX = redE + (int64_t)nf * nch * 2;
  double *fscal = redX + (int64_t)nf * nch * nx_acc;
  reduce_parts(p->partE.as<double>(), nf, nch, nblk_e, 2, 2, redE, p->redtmp.as<double>(), st);
  after(tr, st, "reduce", reduce_split(nblk_e) > 1 ? 2 : 1);
  if (want_grad || want_vir)
    reduce_parts(p->partX.as<double>(), nf, nch, ks_blocks, nx_acc, nx_acc, redX, p->redtmp.as<double>(), st);
  if (want_grad || want_vir) after(tr, st, "reduce_extra", reduce_split(ks_blocks) > 1 ? 2 : 1);
  FinalArgs fa;
  fa.geom = geom;
  fa.redE = redE;
  fa.redX = redX;
  fa.redD = zgeneric ? nullptr : redD;
  fa.qsum = p->qsum.as<double>();
  fa.amp = a->amp;
  fa.bw2 = a->bw2;
  fa.M = M; fa.nch = nch; fa.nx = nx; fa.ny = ny; fa.nz = nz;
  fa.norm = a->norm_factor;
  fa.self_coeff = a->self_coeff;
  fa.lambda = a->charge_neutral_lambda;
  fa.remove_self = a->remove_self;
  fa.k0 = a->k0_correction;
  fa.want_grad = want_grad;
  fa.want_vir = want_vir;
  fa.direct = 0;
  fa.energy = a->energy;
  fa.grad_amp = a->grad_amp;
  fa.grad_bw2 = a->grad_bw2;
  fa.virial = a->virial;
  fa.fscal = fscal;
  k_finalize_frames<T><<<nblocks(nf, 64), 64, 0, st>>>(fa, nf);
  after(tr, st, "finalize_frames");
  if (want_pot && maxat > 0)
    k_finalize_atoms<T><<<dim3(nblocks(maxat, 256), nf), 256, 0, st>>>(
        geom, fscal, p->qsum.as<double>(), (const T *)a->charges, (T *)a->potential, nch,
        a->norm_factor, a->self_coeff, a->charge_neutral_lambda, a->remove_self, a->k0_correction);
  if (want_pot && maxat > 0) after(tr, st, "finalize_atoms");
  SOG_CUDA_TRY(cudaGetLastError());
  return SOG_OK;
}

// Hessian-vector product of the mesh energy (B-spline and QuadS, whose
// position gradient is the derivative of the spread weights).  Per channel:
// the charge mesh and its derivative along the direction (k_spread_dip)
// through the forward transforms, the k-space step k_kspace_hvp, the inverse
// transforms of the two potential fields and the gather k_gather_hvp; then
// the parameter rows and the self / k=0 / penalty terms by the finalize
// kernels every solver shares.  Grids, spectra and fields are fp64 for
// every plan.
template <typename T>
int mesh_hvp_impl(sog_plan *p, const sog_mesh_args *a, const sog_hvp_args *hv, cudaStream_t st) {
  using CF = cplx_t<double>;
  const int nf = a->nframes, nch = a->nchannels, M = a->n_gauss;
  const int nx = p->d.nx, ny = p->d.ny, nz = p->d.nz, nxh = p->nxh, P = p->d.order;
  const int64_t ng = p->ng, nh = p->nh;
  Prep pr;
  int rc = prepare_atoms<T>(p, a, st, pr);
  if (rc != SOG_OK) return rc;
  FrameGeom *geom = pr.geom;
  const int64_t nslots = pr.nslots, maxat = pr.maxat;
  Tracer *tr = &p->tr;
  const unsigned kb = nblocks(nh, 256);
  const int nw = 5 * M;
  if (p->rho.reserve(sizeof(double) * ng * nf) || p->spec.reserve(sizeof(CF) * nh * nf) ||
      p->hspec.reserve(sizeof(CF) * nh * nf) || p->fspec.reserve(sizeof(CF) * nh * nf * 2) ||
      p->freal.reserve(sizeof(double) * ng * nf * 2) ||
      p->hpart.reserve(sizeof(double) * nw * (int64_t)kb * nf * nch) || p->hred.reserve(sizeof(double) * nw * nf) ||
      p->hdsum.reserve(sizeof(double) * 2 * nf * nch) || p->hscal.reserve(sizeof(double) * 8 * nf) ||
      p->redtmp.reserve(sizeof(double) * std::max<int64_t>(1, reduce_tmp_elems(nf, 1, (int64_t)kb * nch, nw))))
    return fail(SOG_ERR_NOMEM, "device allocation failed (mesh HVP)");

  QuadsCoef qc;
  std::memset(&qc, 0, sizeof(qc));
  if (p->d.spline == SOG_SPLINE_QUADS) quads_coeffs(P, qc.c);
  SpreadArgs<T> sa;
  std::memset(&sa, 0, sizeof(sa));
  sa.s_anchor = p->s_anchor.as<int4>();
  sa.s_t = p->s_t.as<T>();
  sa.bin_start = p->bin_start.as<uint32_t>();
  sa.geom = geom;
  sa.rho = p->rho.p;
  sa.ag = pr.ag;
  sa.spline = p->d.spline;
  sa.ntx = (nx + kTileX - 1) / kTileX;
  sa.nty = (ny + kTileY - 1) / kTileY;
  sa.ntz = (nz + kTileZ - 1) / kTileZ;
  sa.qc = qc;
  sa.zlo = 0;
  sa.zcnt = nz;
  sa.dir_q = hv->dir_q;
  sa.dir_r = hv->dir_r;
  sa.s_atom = p->s_atom.as<int32_t>();
  sa.nch = nch;

  KsArgs<double> ka;
  std::memset(&ka, 0, sizeof(ka));
  ka.spec = p->spec.as<CF>();
  ka.fspec = p->fspec.p;
  ka.geom = geom;
  ka.tx = p->tab.fx.as<double>(); ka.ty = p->tab.fy.as<double>(); ka.tz = p->tab.fz.as<double>();
  ka.sx = p->tab.sx.as<double>(); ka.sy = p->tab.sy.as<double>(); ka.sz = p->tab.sz.as<double>();
  ka.amp = a->amp;
  ka.bw2 = a->bw2;
  ka.p32 = p->d.dtype == SOG_DTYPE_F32;
  ka.M = M;
  ka.spline = p->d.spline;
  ka.order = P;
  ka.alias_extent = p->d.alias_extent;
  ka.nx = nx; ka.ny = ny; ka.nz = nz; ka.nxh = nxh;
  ka.nh = nh;
  ka.nyl = ny;
  ka.zblk = nz;
  ka.nfield = 2;

  GatherArgs<T> gar;
  std::memset(&gar, 0, sizeof(gar));
  gar.s_anchor = p->s_anchor.as<int4>();
  gar.s_t = p->s_t.as<T>();
  gar.s_atom = p->s_atom.as<int32_t>();
  gar.nfield = 2;
  gar.nslots = nslots;
  gar.ng = ng;
  gar.ag = pr.ag;
  gar.spline = p->d.spline;
  gar.qc = qc;
  gar.norm = a->norm_factor;
  gar.nch = nch;
  gar.zwrap = nz;
  gar.geom = geom;

  set_fft_smem_attrs<double>();
  auto forward = [&](CF *spec) {
    pass_x_fwd<double>(p, p->rho.as<double>(), spec, (int64_t)nf * nz * ny, st);
    pass_cols<double, -1>(p, spec, ny, nxh, (int64_t)nf * nz, p->rpy, tw_of<double>(p, 1), st, "fft_y_fwd");
    pass_cols<double, -1>(p, spec, nz, (int64_t)ny * nxh, nf, p->rpz, tw_of<double>(p, 2), st, "fft_z_fwd");
  };
  const int nbx = (nx + 7) / 8, nby = (ny + 7) / 8, nbz = (nz + 7) / 8;
  const int64_t nblk = (int64_t)nbx * nby * nbz * nf;
  const unsigned dgrid = (unsigned)((nblk + kWarpsPerDipCta - 1) / kWarpsPerDipCta);
  for (int c = 0; c < nch; ++c) {
    sa.s_q = p->s_q.as<T>() + (int64_t)c * nslots;
    sa.channel = c;
    dispatch_spread<T, double>(sa, P, nf, st, tr);
    forward(p->spec.as<CF>());
    if (dgrid) {
      switch (P) {
        case 4: k_spread_dip<T, 4><<<dgrid, 32 * kWarpsPerDipCta, 0, st>>>(sa, nbx, nby, nbz, nblk); break;
        case 5: k_spread_dip<T, 5><<<dgrid, 32 * kWarpsPerDipCta, 0, st>>>(sa, nbx, nby, nbz, nblk); break;
        default: k_spread_dip<T, 6><<<dgrid, 32 * kWarpsPerDipCta, 0, st>>>(sa, nbx, nby, nbz, nblk); break;
      }
      after(tr, st, "spread_dip");
    }
    forward(p->hspec.as<CF>());
    k_kspace_hvp<T><<<dim3(kb, nf), 256, 0, st>>>(ka, p->hspec.as<CF>(), hv->dir_amp, hv->dir_bw2, c, nch,
                                                  p->hpart.as<double>());
    after(tr, st, "kspace_hvp");
    pass_cols<double, +1>(p, p->fspec.as<CF>(), nz, (int64_t)ny * nxh, (int64_t)nf * 2, p->rpz,
                          tw_of<double>(p, 2), st, "fft_z_inv");
    pass_cols<double, +1>(p, p->fspec.as<CF>(), ny, nxh, (int64_t)nf * 2 * nz, p->rpy, tw_of<double>(p, 1), st,
                          "fft_y_inv");
    pass_x_inv<double>(p, p->fspec.as<CF>(), p->freal.as<double>(), nf, (int64_t)nz * ny, 2, st);
    gar.s_q = p->s_q.as<T>() + (int64_t)c * nslots;
    gar.channel = c;
    gar.accumulate = c > 0;
    const unsigned gb = nblocks(nslots, 256);
    if (gb) {
      const double *fl = p->freal.as<double>();
      T *oq = (T *)hv->out_q, *orr = (T *)hv->out_r;
      switch (P) {
        case 4: k_gather_hvp<T, 4><<<gb, 256, 0, st>>>(gar, fl, hv->dir_q, hv->dir_r, oq, orr); break;
        case 5: k_gather_hvp<T, 5><<<gb, 256, 0, st>>>(gar, fl, hv->dir_q, hv->dir_r, oq, orr); break;
        default: k_gather_hvp<T, 6><<<gb, 256, 0, st>>>(gar, fl, hv->dir_q, hv->dir_r, oq, orr); break;
      }
      after(tr, st, "gather_hvp");
    }
  }
  // the channels' block partials of a frame are contiguous: one reduction
  reduce_parts(p->hpart.as<double>(), nf, 1, (int64_t)kb * nch, nw, nw, p->hred.as<double>(),
               p->redtmp.as<double>(), st);
  after(tr, st, "reduce", reduce_split((int64_t)kb * nch) > 1 ? 2 : 1);
  k_hvp_dsums<T><<<dim3(nf, nch), 256, 0, st>>>((const T *)a->charges, hv->dir_q, nch, geom, p->hdsum.as<double>());
  after(tr, st, "hvp_dsums");
  HvpFinal hf;
  hf.geom = geom;
  hf.hred = p->hred.as<double>();
  hf.qsum = p->qsum.as<double>();
  hf.dsum = p->hdsum.as<double>();
  hf.amp = a->amp;
  hf.bw2 = a->bw2;
  hf.damp = hv->dir_amp;
  hf.dbw2 = hv->dir_bw2;
  hf.oamp = hv->out_amp;
  hf.obw2 = hv->out_bw2;
  hf.scal = p->hscal.as<double>();
  hf.M = M;
  hf.nch = nch;
  hf.norm = a->norm_factor;
  hf.self_coeff = a->self_coeff;
  hf.lambda = a->charge_neutral_lambda;
  hf.remove_self = a->remove_self;
  hf.k0 = a->k0_correction;
  k_hvp_finalize_frames<T><<<nblocks(nf, 64), 64, 0, st>>>(hf, nf);
  after(tr, st, "hvp_finalize_frames");
  if (maxat > 0) {
    k_hvp_finalize_atoms<T><<<dim3(nblocks(maxat, 256), nf), 256, 0, st>>>(
        geom, p->hscal.as<double>(), p->hdsum.as<double>(), (const T *)a->charges, hv->dir_q, (T *)hv->out_q, nch,
        a->norm_factor, a->charge_neutral_lambda);
    after(tr, st, "hvp_finalize_atoms");
  }
  SOG_CUDA_TRY(cudaGetLastError());
  return SOG_OK;
}

// ==========================================================================
// z-slab decomposition of one frame over `size` ranks
// ==========================================================================
struct SlabLayout {
  int zs = 0, ys = 0, F = 0;
  size_t fs = 0, fr = 0, is = 0, ir = 0, fe = 0, red = 0, total = 0;  // workspace byte offsets
};

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Workspace: forward send / receive (one rank's share of the spectrum each),
// inverse send / receive (nfield shares), the real fields with order-1 halo
// planes, and the scalars summed over ranks.
// With the peer transport the receive buffers belong to the plan (exported
// to the other ranks) and the workspace holds only the IPC handles being
// swapped and the summed scalars.
SlabLayout slab_layout(const sog_plan *p, int nfield, int size, int transport) {
  SlabLayout L;
  const size_t sc = p->d.dtype == SOG_DTYPE_F64 ? 16 : 8, sr = sc / 2;
  L.zs = p->d.nz / size;
  L.ys = p->d.ny / size;
  L.F = nfield;
  size_t off = 0;
  if (transport == SOG_SLAB_PEER) {
    L.fs = off; off += align256(3 * sizeof(cudaIpcMemHandle_t));                       // own handles
    L.fr = off; off += align256(3 * sizeof(cudaIpcMemHandle_t) * (size_t)size);        // everyone's
  } else {
    const size_t share = (size_t)L.zs * p->d.ny * p->nxh * sc;
    L.fs = off; off += align256(share);
    L.fr = off; off += align256(share);
    L.is = off; off += align256(share * nfield);
    L.ir = off; off += align256(share * nfield);
    L.fe = off; off += align256((size_t)(L.zs + p->d.order - 1) * p->d.ny * p->d.nx * nfield * sr);
  }
  L.red = off; off += 4096;
  L.total = off;
  return L;
}

void close_peers(sog_plan *p) {
  for (int s = 0; s < p->peer_size; ++s) {
    if (s == p->peer_rank) continue;
    for (void **pp : {&p->peer_fwd[s], &p->peer_inv[s], &p->peer_fe[s]})
      if (*pp) {
        cudaIpcCloseMemHandle(*pp);
        *pp = nullptr;
      }
  }
  for (int s = 0; s < 8; ++s) p->peer_fwd[s] = p->peer_inv[s] = p->peer_fe[s] = nullptr;
  p->peer_rank = -1;
  p->peer_size = 0;
}

// Peer transport set-up, once per (plan, group): receive buffers of the
// largest field count, their IPC handles swapped with ALLGATHER, the peers'
// buffers opened.  Every rank learns through SUM_F64 whether all ranks
// succeeded, so a failure returns the same error everywhere.
// recv_el: complex elements of one spectrum's receive buffer (nz x the
// chunked columns of this rank's rows).
template <typename T>
int peer_setup(sog_plan *p, const sog_slab_desc *sd, unsigned char *ws, const SlabLayout &L, int64_t recv_el,
               cudaStream_t st, const std::function<int(int, size_t, size_t, size_t)> &exchange) {
  if (p->peer_rank == sd->rank && p->peer_size == sd->size && p->xr_fwd.bytes >= sizeof(cplx_t<T>) * recv_el)
    return SOG_OK;
  close_peers(p);
  using C = cplx_t<T>;
  const sog_plan_desc &d = p->d;
  if (p->xr_fwd.reserve(sizeof(C) * recv_el) || p->xr_inv.reserve(sizeof(C) * recv_el * 4) ||
      p->xr_fe.reserve(sizeof(T) * (int64_t)(L.zs + d.order - 1) * d.ny * d.nx * 4))
    return fail(SOG_ERR_NOMEM, "device allocation failed (slab receive buffers)");
  // the pad columns of the chunked layout are never written: keep them zero
  SOG_CUDA_TRY(cudaMemsetAsync(p->xr_fwd.p, 0, p->xr_fwd.bytes, st));
  SOG_CUDA_TRY(cudaMemsetAsync(p->xr_inv.p, 0, p->xr_inv.bytes, st));
  cudaIpcMemHandle_t own[3];
  SOG_CUDA_TRY(cudaIpcGetMemHandle(&own[0], p->xr_fwd.p));
  SOG_CUDA_TRY(cudaIpcGetMemHandle(&own[1], p->xr_inv.p));
  SOG_CUDA_TRY(cudaIpcGetMemHandle(&own[2], p->xr_fe.p));
  SOG_CUDA_TRY(cudaMemcpyAsync(ws + L.fs, own, sizeof(own), cudaMemcpyHostToDevice, st));
  int rc = exchange(SOG_EXCH_ALLGATHER, L.fs, L.fr, sizeof(own));
  if (rc != SOG_OK) return rc;
  std::vector<cudaIpcMemHandle_t> all(3 * (size_t)sd->size);
  SOG_CUDA_TRY(cudaMemcpyAsync(all.data(), ws + L.fr, sizeof(own) * sd->size, cudaMemcpyDeviceToHost, st));
  SOG_CUDA_TRY(cudaStreamSynchronize(st));
  p->peer_rank = sd->rank;
  p->peer_size = sd->size;
  double failed = 0.0;
  for (int s = 0; s < sd->size; ++s) {
    void **dst[3] = {&p->peer_fwd[s], &p->peer_inv[s], &p->peer_fe[s]};
    void *local[3] = {p->xr_fwd.p, p->xr_inv.p, p->xr_fe.p};
    for (int i = 0; i < 3; ++i) {
      if (s == sd->rank) {
        *dst[i] = local[i];
      } else if (cudaIpcOpenMemHandle(dst[i], all[3 * (size_t)s + i], cudaIpcMemLazyEnablePeerAccess) !=
                 cudaSuccess) {
        cudaGetLastError();
        *dst[i] = nullptr;
        failed += 1.0;
      }
    }
  }
  double *flag = reinterpret_cast<double *>(ws + L.red);
  SOG_CUDA_TRY(cudaMemcpyAsync(flag, &failed, sizeof(double), cudaMemcpyHostToDevice, st));
  if ((rc = exchange(SOG_EXCH_SUM_F64, L.red, L.red, sizeof(double))) != SOG_OK) return rc;
  double total = 0.0;
  SOG_CUDA_TRY(cudaMemcpyAsync(&total, flag, sizeof(double), cudaMemcpyDeviceToHost, st));
  SOG_CUDA_TRY(cudaStreamSynchronize(st));
  if (total > 0.0) {
    close_peers(p);
    return fail(SOG_ERR_UNSUPPORTED, "peer memory between the ranks is not available (CUDA IPC open failed on " +
                                         std::to_string((int)total) + " buffers); use the exchange transport");
  }
  return SOG_OK;
}

// Row-mapped column FFT pass (power-of-two n only).
template <typename T, int DIR>
void pass_cols_map(sog_plan *p, RowMap<cplx_t<T>> in, RowMap<cplx_t<T>> out, int n, int64_t inner,
                   int64_t outer, const cplx_t<T> *tw, cudaStream_t st, const char *name) {
  using C = cplx_t<T>;
  with_shifts(in);
  with_shifts(out);
  with_pow2(n, [&](auto lc) {
    constexpr int L = decltype(lc)::value;
    constexpr int nn = 1 << L;
    constexpr int thr_cap = sizeof(T) == 4 ? 512 : SOG_SLAB_COLS_THR64;
    const int ic = reg_width<T>(nn, thr_cap, thr_cap * 256);
    const int64_t ntiles = outer * ((inner + ic - 1) / ic);
    const int thr = (nn / kEPT) * ic;
    if (ic >= 8) {
      const size_t sm = (3 * (size_t)nn * ic + nn) * sizeof(C);
      allow_smem(k_cols_map<T, DIR, false, L>);
      k_cols_map<T, DIR, false, L><<<persistent_grid(k_cols_map<T, DIR, false, L>, thr, sm, ntiles), thr, sm, st>>>(
          in, out, inner, ic, ntiles, tw);
    } else {
      const size_t sm = ((2 * (size_t)nn + padded_row(nn)) * ic + nn) * sizeof(C);
      allow_smem(k_cols_map<T, DIR, true, L>);
      k_cols_map<T, DIR, true, L><<<persistent_grid(k_cols_map<T, DIR, true, L>, thr, sm, ntiles), thr, sm, st>>>(
          in, out, inner, ic, ntiles, tw);
    }
  });
  after(&p->tr, st, name);
}

// Inverse y pass of the z-slab's received field spectra (k_cols_fields
// through row maps): F slots of zs planes each, two-slot frames' fields formed
// on the way (power-of-two ny only).
template <typename T>
void pass_cols_fields_map(sog_plan *p, RowMap<cplx_t<T>> in, RowMap<cplx_t<T>> out,
                          const FrameGeom *geom, int F, int zs, int two_slot, int want_pot, cudaStream_t st) {
  using C = cplx_t<T>;
  with_shifts(in);
  with_shifts(out);
  const int64_t inner = p->nxh;
  with_pow2(p->d.ny, [&](auto lc) {
    constexpr int L = decltype(lc)::value;
    constexpr int nn = 1 << L;
    constexpr int thr_cap = sizeof(T) == 4 ? 512 : SOG_SLAB_COLS_THR64;
    const int ic = reg_width<T>(nn, thr_cap, thr_cap * 256);
    const int64_t ntiles = (int64_t)F * zs * ((inner + ic - 1) / ic);
    const int thr = (nn / kEPT) * ic;
    if (ic >= 8) {
      const size_t sm = (3 * (size_t)nn * ic + nn) * sizeof(C);
      allow_smem(k_cols_fields<T, false, L, true>);
      k_cols_fields<T, false, L, true><<<persistent_grid(k_cols_fields<T, false, L, true>, thr, sm, ntiles), thr, sm,
                                         st>>>(nullptr, geom, F, zs, inner, ic, ntiles, tw_of<T>(p, 1), two_slot,
                                               want_pot, in, out);
    } else {
      const size_t sm = ((2 * (size_t)nn + padded_row(nn)) * ic + nn) * sizeof(C);
      allow_smem(k_cols_fields<T, true, L, true>);
      k_cols_fields<T, true, L, true><<<persistent_grid(k_cols_fields<T, true, L, true>, thr, sm, ntiles), thr, sm,
                                        st>>>(nullptr, geom, F, zs, inner, ic, ntiles, tw_of<T>(p, 1), two_slot,
                                              want_pot, in, out);
    }
  });
  after(&p->tr, st, "fft_y_inv");
}

template <typename T>
int mesh_slab_impl(sog_plan *p, const sog_mesh_args *a, const sog_slab_desc *sd, cudaStream_t st) {
  using C = cplx_t<T>;
  const int nch = a->nchannels, M = a->n_gauss;
  const int nx = p->d.nx, ny = p->d.ny, nz = p->d.nz, nxh = p->nxh, P = p->d.order;
  const int rank = sd->rank, size = sd->size;
  const bool want_force = a->forces != nullptr;
  const bool want_pot = a->potential != nullptr;
  const int nfield = (want_force ? 3 : 0) + (want_pot ? 1 : 0);
  const bool peer = sd->transport == SOG_SLAB_PEER;
  const SlabLayout L = slab_layout(p, nfield, size, sd->transport);
  if (sd->workspace_bytes < L.total) return fail(SOG_ERR_INVALID, "slab workspace smaller than sog_mesh_slab_workspace()");
  unsigned char *ws = static_cast<unsigned char *>(sd->workspace);
  const int zs = L.zs, ys = L.ys, zlo = rank * zs, y0 = rank * ys;
  std::function<int(int, size_t, size_t, size_t)> exchange = [&](int kind, size_t so, size_t ro,
                                                                 size_t bytes) -> int {
    const int r = sd->exchange(sd->ctx, kind, (int64_t)so, (int64_t)ro, (int64_t)bytes, st);
    if (r != 0) return fail(SOG_ERR_COMM, "exchange callback returned " + std::to_string(r));
    return SOG_OK;
  };
  // stream-ordered barrier of the peer transport: a one-double sum (all
  // ranks' earlier kernels, and so their stores into this rank's buffers,
  // are complete when it completes)
  const size_t barrier_off = L.red + 2048;
  auto barrier = [&](const char *name) -> int {
    const int r = exchange(SOG_EXCH_SUM_F64, barrier_off, barrier_off, sizeof(double));
    if (r == SOG_OK) after(&p->tr, st, name, 0);
    return r;
  };
  // spectrum rows of this rank after the transpose: plain [nz][ys][nxh], or
  // with the peer transport chunked into tiles of W = (fused z tile width)
  // columns, [nz][nxh/W][ys][W], so that every tile a peer stores is contiguous.
  const bool z512 = SOG_SLAB_ZTHR == 512 && nz >= 512 && nz <= 1024;
  const int zic = z512 ? reg_width<T>(nz, 512, 64 * 1024) : reg_width<T>(nz, 256, 32 * 1024);
  const int W = peer ? zic : 0;
  const int64_t inner_loc = peer ? (int64_t)((nxh + W - 1) / W) * ys * W : (int64_t)ys * nxh;
  if (peer) {
    const int r = peer_setup<T>(p, sd, ws, L, (int64_t)nz * inner_loc, st, exchange);
    if (r != SOG_OK) return r;
  }

  Prep pr;
  // slab ranks take z ranges of bins: plain z-major bin order
  int rc = prepare_atoms<T>(p, a, st, pr, 1);
  if (rc != SOG_OK) return rc;
  FrameGeom *geom = pr.geom;
  const AtomGrid ag = pr.ag;
  const int64_t nslots = pr.nslots;
  Tracer *tr = &p->tr;

  const int64_t nh_loc = (int64_t)nz * inner_loc;      // spectrum rows of this rank after the transpose
  const int64_t spec_loc = (int64_t)zs * ny * nxh;     // spectrum of this rank's planes
  const int64_t zchunks = (inner_loc + zic - 1) / zic;
  if (p->rho.reserve(sizeof(T) * (int64_t)zs * ny * nx) || p->spec.reserve(sizeof(C) * spec_loc) ||
      p->partE.reserve(sizeof(double) * 2 * zchunks * nch) ||
      (nfield && p->fspec.reserve(sizeof(C) * spec_loc * nfield)) ||
      p->redtmp.reserve(sizeof(double) * std::max<int64_t>(reduce_tmp_elems(1, nch, zchunks, 2), 1)) ||
      p->red.reserve(sizeof(double) * (4 * 1 + 8)))
    return fail(SOG_ERR_NOMEM, "device allocation failed (slab buffers)");

  QuadsCoef qc;
  std::memset(&qc, 0, sizeof(qc));
  if (p->d.spline == SOG_SPLINE_QUADS) quads_coeffs(P, qc.c);
  SpreadArgs<T> sa;
  sa.s_anchor = p->s_anchor.as<int4>();
  sa.s_t = p->s_t.as<T>();
  sa.bin_start = p->bin_start.as<uint32_t>();
  sa.geom = geom;
  sa.rho = p->rho.as<T>();
  sa.ag = ag;
  sa.spline = p->d.spline;
  sa.ntx = (nx + kTileX - 1) / kTileX;
  sa.nty = (ny + kTileY - 1) / kTileY;
  sa.ntz = (zs + kTileZ - 1) / kTileZ;
  sa.qc = qc;
  sa.zlo = zlo;
  sa.zcnt = zs;

  KsArgs<T> ka;
  std::memset(&ka, 0, sizeof(ka));
  ka.spec = peer ? p->xr_fwd.as<C>() : reinterpret_cast<C *>(ws + L.fr);
  ka.fspec = nfield ? (peer ? p->xr_inv.as<C>() : reinterpret_cast<C *>(ws + L.is)) : nullptr;
  ka.cw = W;
  if (peer && nfield) {
    // block b of the fields goes to rank b's receive buffer, slot of this rank
    const int64_t blk = (int64_t)nfield * zs * inner_loc;
    for (int b = 0; b < size; ++b) ka.zdst[b] = static_cast<C *>(p->peer_inv[b]) + (int64_t)rank * blk;
  }
  ka.geom = geom;
  ka.tx = p->tab.fx.as<double>(); ka.ty = p->tab.fy.as<double>(); ka.tz = p->tab.fz.as<double>();
  ka.sx = p->tab.sx.as<double>(); ka.sy = p->tab.sy.as<double>(); ka.sz = p->tab.sz.as<double>();
  ka.amp = a->amp;
  ka.bw2 = a->bw2;
  ka.p32 = p->d.dtype == SOG_DTYPE_F32;
  ka.M = M;
  ka.spline = p->d.spline;
  ka.order = P;
  ka.alias_extent = p->d.alias_extent;
  ka.nx = nx; ka.ny = ny; ka.nz = nz; ka.nxh = nxh;
  ka.nh = nh_loc;
  ka.nfield = nfield;
  ka.want_force = want_force;
  // two-slot field spectra over the peer transport (orthorhombic frames):
  // two thirds of the force fields' NVLink bytes
  ka.two_slot = (SOG_SLAB_TWO_SLOT && peer && want_force && is_pow2(ny) && ny <= 1024) ? 1 : 0;
  ka.nx_acc = 4 * M + 13;
  ka.y0 = y0;
  ka.nyl = ys;
  ka.zblk = zs;
  ka.btab_stride = (int64_t)M * (nxh + ny + nz);
  if (p->btab.reserve(sizeof(double) * ka.btab_stride)) return fail(SOG_ERR_NOMEM, "device allocation failed");
  ka.btab = p->btab.as<double>();
  k_axis_tables<T><<<dim3(nblocks(ka.btab_stride, 256), 1), 256, 0, st>>>(geom, (const T *)a->bw2, M, nx, ny, nz,
                                                                         p->btab.as<double>());
  after(tr, st, "axis_tables");
  set_fft_smem_attrs<T>();

  // Green table of this rank's spectrum rows and its self-sum partials
  double *red = reinterpret_cast<double *>(ws + L.red);   // [nch][2] energy sums, then the self sum
  {
    const bool aliasable = p->d.spline == SOG_SPLINE_BSPLINE;
    const unsigned gblocks = nblocks(inner_loc, 256);
    const unsigned gz = green_zsplit(gblocks, 1, nz);
    const int64_t gparts = (int64_t)gblocks * gz;
    if (p->gtab.reserve(sizeof(double) * nh_loc) || (aliasable && p->gtabF.reserve(sizeof(double) * nh_loc)) ||
        p->partD.reserve(sizeof(double) * (gparts + 1 + reduce_tmp_elems(1, 1, gparts, 1))))
      return fail(SOG_ERR_NOMEM, "device allocation failed (Green tables)");
    ka.gtab = p->gtab.as<double>();
    ka.gtabF = aliasable ? p->gtabF.as<double>() : nullptr;
    ka.partD = p->partD.as<double>();
    if ((rc = setup_radial<T>(p, ka, 1, st)) != SOG_OK) return rc;
    launch_green<T>(ka, gblocks, 1, gz, st);
    after(tr, st, "green");
    reduce_parts(ka.partD, 1, 1, gparts, 1, 1, red + 2 * nch, ka.partD + gparts + 1, st);
    after(tr, st, "reduce_green", reduce_split(gparts) > 1 ? 2 : 1);
  }

  GatherArgs<T> gar;
  std::memset(&gar, 0, sizeof(gar));
  gar.s_anchor = p->s_anchor.as<int4>();
  gar.s_t = p->s_t.as<T>();
  gar.s_atom = p->s_atom.as<int32_t>();
  T *fields = peer ? p->xr_fe.as<T>() : reinterpret_cast<T *>(ws + L.fe);
  gar.freal = fields;
  gar.nfield = nfield;
  gar.want_force = want_force;
  gar.want_pot = want_pot;
  gar.nslots = nslots;
  gar.ng = 0;
  gar.ag = ag;
  gar.spline = p->d.spline;
  gar.qc = qc;
  gar.norm = a->norm_factor;
  gar.nch = nch;
  gar.forces = (T *)a->forces;
  gar.pot_raw = (T *)a->potential;
  gar.slot_lo = 0;
  gar.zlo = zlo;
  gar.zwrap = INT_MAX;
  const uint32_t *bs = p->bin_start.as<uint32_t>();
  const int64_t bins_per_z = (int64_t)ag.nbx * ag.nby;
  gar.range_lo = bs + (int64_t)(zlo / kBin) * bins_per_z;
  gar.range_hi = bs + (int64_t)((zlo + zs) / kBin) * bins_per_z;

  // outputs of atoms outside the slab stay zero
  const int64_t natoms = a->atom_begin[0] + a->atom_count[0];
  if (want_force) {
    k_zero<T><<<nblocks(3 * natoms, 256), 256, 0, st>>>((T *)a->forces, 3 * natoms);
    count_launch();
  }
  if (want_pot) {
    k_zero<T><<<nblocks(natoms * nch, 256), 256, 0, st>>>((T *)a->potential, natoms * nch);
    count_launch();
  }

  const size_t share = (size_t)zs * ys * nxh * sizeof(C);
  for (int c = 0; c < nch; ++c) {
    sa.s_q = p->s_q.as<T>() + (int64_t)c * nslots;
    dispatch_spread<T>(sa, P, 1, st, tr);
    pass_x_fwd<T>(p, p->rho.as<T>(), p->spec.as<C>(), (int64_t)zs * ny, st);
    if (peer) {
      // y transform stored straight into every rank's receive buffer:
      // rows [d*ys, (d+1)*ys) of plane z go to rank d at [this rank][z][..]
      const RowMap<C> in = plain_map(p->spec.as<C>(), ny, nxh);
      RowMap<C> out = plain_map<C>(nullptr, ny, nxh);
      for (int d = 0; d < size; ++d) out.tab[d] = static_cast<C *>(p->peer_fwd[d]) + (int64_t)rank * zs * inner_loc;
      out.rb = ys;
      out.olo = inner_loc;            // plane zl
      out.rstride = W;                // row yl
      out.cw = W;
      out.cstride = (int64_t)ys * W;  // column chunk xc
      pass_cols_map<T, -1>(p, in, out, ny, nxh, zs, p->twy.as<C>(), st, "fft_y_fwd");
      if ((rc = barrier("barrier_fwd")) != SOG_OK) return rc;
    } else {
      pass_cols<T, -1>(p, p->spec.as<C>(), ny, nxh, zs, p->rpy, p->twy.as<C>(), st, "fft_y_fwd");
      k_slab_pack<C><<<(unsigned)((int64_t)zs * ny), 256, 0, st>>>(
          p->spec.as<C>(), reinterpret_cast<C *>(ws + L.fs), zs, ny, ys, nxh);
      after(tr, st, "slab_pack");
      if ((rc = exchange(SOG_EXCH_ALLTOALL, L.fs, L.fr, share)) != SOG_OK) return rc;
      after(tr, st, "exchange_fwd", 0);
    }
    ka.part = p->partE.as<double>() + (int64_t)c * zchunks * 2;
    {
      const int write_spec = 0;
      const bool done = with_pow2(nz, [&](auto lc) {
        constexpr int Lz = decltype(lc)::value;
        constexpr int n = 1 << Lz;
        const int zthr = (n / kEPT) * zic;
        const size_t zsm = ((2 * (size_t)n + padded_row(n)) * zic + n) * sizeof(C);
        if (zthr == 512) {
          allow_smem(k_zfused_g<T, Lz, 512>);
          k_zfused_g<T, Lz, 512><<<persistent_grid(k_zfused_g<T, Lz, 512>, zthr, zsm, zchunks), zthr, zsm, st>>>(
              ka, zic, zchunks, p->twz.as<C>(), write_spec);
        } else {
          allow_smem(k_zfused_g<T, Lz>);
          k_zfused_g<T, Lz><<<persistent_grid(k_zfused_g<T, Lz>, zthr, zsm, zchunks), zthr, zsm, st>>>(
              ka, zic, zchunks, p->twz.as<C>(), write_spec);
        }
      });
      if (!done) return fail(SOG_ERR_UNSUPPORTED, "slab mode needs a power-of-two nz up to 1024");
      after(tr, st, "zfused");
    }
    if (nfield) {
      const size_t plane = (size_t)ny * nx * nfield * sizeof(T);
      if (peer) {
        if ((rc = barrier("barrier_inv")) != SOG_OK) return rc;
        // y inverse read in place from the received blocks [src][F][zs][ys][..]
        // received blocks [src][F][xc*ys + yl][zs][W], read in place
        RowMap<C> in = plain_map<C>(nullptr, ny, nxh);
        for (int s = 0; s < size; ++s) in.tab[s] = p->xr_inv.as<C>();
        in.rb = ys;
        in.bstride = (int64_t)nfield * zs * inner_loc;   // source rank
        in.osplit = zs;
        in.ohi = (int64_t)zs * inner_loc;                // field
        in.olo = W;                                      // plane zl
        in.rstride = (int64_t)zs * W;                    // row yl
        in.cw = W;
        in.cstride = (int64_t)ys * zs * W;               // column chunk xc
        const RowMap<C> out = plain_map(p->fspec.as<C>(), ny, nxh);
        if (ka.two_slot)
          pass_cols_fields_map<T>(p, in, out, geom, nfield, zs, 1, want_pot ? 1 : 0, st);
        else
          pass_cols_map<T, +1>(p, in, out, ny, nxh, (int64_t)nfield * zs, p->twy.as<C>(), st, "fft_y_inv");
        pass_x_inv<T>(p, p->fspec.as<C>(), fields, 1, (int64_t)zs * ny, nfield, st);
        // first order-1 planes to the halo of rank r-1
        const int prev = (rank + size - 1) % size;
        const int64_t nh_el = (int64_t)(P - 1) * ny * nx * nfield;
        k_halo_push<T><<<nblocks(nh_el, 256), 256, 0, st>>>(
            fields, static_cast<T *>(p->peer_fe[prev]) + (int64_t)zs * ny * nx * nfield, nh_el);
        after(tr, st, "halo_push");
        if ((rc = barrier("barrier_halo")) != SOG_OK) return rc;
      } else {
        if ((rc = exchange(SOG_EXCH_ALLTOALL, L.is, L.ir, share * nfield)) != SOG_OK) return rc;
        after(tr, st, "exchange_inv", 0);
        k_slab_unpack<C><<<(unsigned)((int64_t)nfield * zs * ny), 256, 0, st>>>(
            reinterpret_cast<const C *>(ws + L.ir), p->fspec.as<C>(), nfield, zs, ny, ys, nxh);
        after(tr, st, "slab_unpack");
        pass_cols<T, +1>(p, p->fspec.as<C>(), ny, nxh, (int64_t)nfield * zs, p->rpy, p->twy.as<C>(), st,
                         "fft_y_inv");
        pass_x_inv<T>(p, p->fspec.as<C>(), fields, 1, (int64_t)zs * ny, nfield, st);
        if ((rc = exchange(SOG_EXCH_HALO, L.fe, L.fe + plane * zs, plane * (P - 1))) != SOG_OK) return rc;
        after(tr, st, "exchange_halo", 0);
      }
      gar.s_q = p->s_q.as<T>() + (int64_t)c * nslots;
      gar.channel = c;
      gar.accumulate = c > 0;
      dispatch_gather<T>(gar, P, st, tr);
    }
  }
  // energy sums of this rank's spectrum rows, summed over ranks
  reduce_parts(p->partE.as<double>(), 1, nch, zchunks, 2, 2, red, p->redtmp.as<double>(), st);
  after(tr, st, "reduce", reduce_split(zchunks) > 1 ? 2 : 1);
  if ((rc = exchange(SOG_EXCH_SUM_F64, L.red, L.red, sizeof(double) * (2 * nch + 1))) != SOG_OK) return rc;
  after(tr, st, "exchange_sum", 0);
  FinalArgs fa;
  std::memset(&fa, 0, sizeof(fa));
  fa.geom = geom;
  fa.redE = red;
  fa.redX = nullptr;
  fa.redD = red + 2 * nch;
  fa.qsum = p->qsum.as<double>();
  fa.amp = a->amp;
  fa.bw2 = a->bw2;
  fa.M = M; fa.nch = nch; fa.nx = nx; fa.ny = ny; fa.nz = nz;
  fa.norm = a->norm_factor;
  fa.self_coeff = a->self_coeff;
  fa.lambda = a->charge_neutral_lambda;
  fa.remove_self = a->remove_self;
  fa.k0 = a->k0_correction;
  fa.direct = 0;
  fa.energy = a->energy;
  double *fscal = p->red.as<double>();
  fa.fscal = fscal;
  k_finalize_frames<T><<<1, 64, 0, st>>>(fa, 1);
  after(tr, st, "finalize_frames");
  if (want_pot && nslots > 0) {
    k_finalize_slab<T><<<nblocks(nslots, 256), 256, 0, st>>>(
        geom, fscal, p->qsum.as<double>(), (const T *)a->charges, (T *)a->potential, p->s_atom.as<int32_t>(),
        gar.range_lo, gar.range_hi, nslots, nch, a->norm_factor, a->self_coeff, a->charge_neutral_lambda,
        a->remove_self, a->k0_correction);
    after(tr, st, "finalize_atoms");
  }
  SOG_CUDA_TRY(cudaGetLastError());
  return SOG_OK;
}

}  // namespace

// ==========================================================================
// C ABI
// ==========================================================================
extern "C" int sog_plan_create(sog_plan **out, const sog_plan_desc *desc) {
  if (!out || !desc) return fail(SOG_ERR_INVALID, "null argument");
  *out = nullptr;
  const sog_plan_desc &d = *desc;
  if (d.dtype != SOG_DTYPE_F64 && d.dtype != SOG_DTYPE_F32) return fail(SOG_ERR_INVALID, "dtype must be F64 or F32");
  if (d.spline == SOG_SPLINE_BSPLINE) {
    if (d.order < 4 || d.order > 6) return fail(SOG_ERR_INVALID, "B-spline order must be 4, 5 or 6");
  } else if (d.spline == SOG_SPLINE_QUADS) {
    if (d.order != 4 && d.order != 6) return fail(SOG_ERR_INVALID, "QuadS order must be 4 or 6");
  } else if (d.spline == SOG_SPLINE_CUBES2) {
    if (d.order != 4 && d.order != 6) return fail(SOG_ERR_INVALID, "CubeS2 order must be 4 or 6");
  } else {
    return fail(SOG_ERR_INVALID, "unknown spline family");
  }
  if (d.nx < 8 || d.ny < 8 || d.nz < 8) return fail(SOG_ERR_INVALID, "mesh dims must be >= 8");
  if (!smooth235(d.nx) || !smooth235(d.ny) || !smooth235(d.nz))
    return fail(SOG_ERR_INVALID, "mesh dims must be 2,3,5-smooth");
  if (d.nx > 4096 || d.ny > 4096 || d.nz > 4096) return fail(SOG_ERR_UNSUPPORTED, "mesh dim above 4096");
  if (d.kconv != SOG_KCONV_PHYSICAL && d.kconv != SOG_KCONV_REFERENCE)
    return fail(SOG_ERR_INVALID, "kconv must be PHYSICAL or REFERENCE");
  DeviceGuard dg(d.device);
  sog_plan *p = new sog_plan();
  p->d = d;
  if (p->d.alias_extent <= 0) p->d.alias_extent = 8;
  p->nxh = d.nx / 2 + 1;
  p->ng = (int64_t)d.nx * d.ny * d.nz;
  p->nh = (int64_t)d.nz * d.ny * p->nxh;
  build_radix_plan(d.nx, &p->rpx);
  if (d.nx % 2 == 0) build_radix_plan(d.nx / 2, &p->rpxh);
  build_radix_plan(d.ny, &p->rpy);
  build_radix_plan(d.nz, &p->rpz);
  p->nb_x = (d.nx + kBin - 1) / kBin;
  p->nb_y = (d.ny + kBin - 1) / kBin;
  p->nb_z = (d.nz + kBin - 1) / kBin;
  int rc = SOG_OK;
  std::vector<unsigned char> tw;
  make_twiddles(d.nx, d.dtype, tw);
  if ((rc = upload(p->twx, tw.data(), tw.size())) != SOG_OK) goto bad;
  make_twiddles(d.ny, d.dtype, tw);
  if ((rc = upload(p->twy, tw.data(), tw.size())) != SOG_OK) goto bad;
  make_twiddles(d.nz, d.dtype, tw);
  if ((rc = upload(p->twz, tw.data(), tw.size())) != SOG_OK) goto bad;
  if (d.dtype == SOG_DTYPE_F32) {
    make_twiddles(d.nx, SOG_DTYPE_F64, tw);
    if ((rc = upload(p->twx64, tw.data(), tw.size())) != SOG_OK) goto bad;
    make_twiddles(d.ny, SOG_DTYPE_F64, tw);
    if ((rc = upload(p->twy64, tw.data(), tw.size())) != SOG_OK) goto bad;
    make_twiddles(d.nz, SOG_DTYPE_F64, tw);
    if ((rc = upload(p->twz64, tw.data(), tw.size())) != SOG_OK) goto bad;
  }
  {
    // per-axis Green factors and alias sums over mode indices of each axis
    auto axis = [&](int n, int len, bool half, DevBuf &fb, DevBuf &sb) -> int {
      std::vector<double> fv(len), sv(len);
      for (int i = 0; i < len; ++i) {
        const int m = half ? i : (i <= n / 2 ? i : i - n);
        sv[i] = bspline_sinc_sum(m, n, d.order, p->d.alias_extent);
        if (d.spline == SOG_SPLINE_QUADS) fv[i] = quads_influence_1d(m, n, d.order);
        else fv[i] = bspline_sinc2p(m, n, d.order, 0) / (sv[i] * sv[i]);
      }
      int r = upload(fb, fv.data(), sizeof(double) * len);
      if (r == SOG_OK) r = upload(sb, sv.data(), sizeof(double) * len);
      return r;
    };
    if ((rc = axis(d.nx, p->nxh, true, p->tab.fx, p->tab.sx)) != SOG_OK) goto bad;
    if ((rc = axis(d.ny, d.ny, false, p->tab.fy, p->tab.sy)) != SOG_OK) goto bad;
    if ((rc = axis(d.nz, d.nz, false, p->tab.fz, p->tab.sz)) != SOG_OK) goto bad;
  }
  if ((rc = p->up.reserve(4096)) != SOG_OK) goto bad;
  *out = p;
  return SOG_OK;
bad:
  sog_plan_destroy(p);
  return rc;
}

extern "C" int sog_plan_destroy(sog_plan *p) {
  if (!p) return SOG_OK;
  DeviceGuard dg(p->d.device);
  DevBuf *bufs[] = {&p->twx, &p->twy, &p->twz, &p->twx64, &p->twy64, &p->twz64, &p->tab.fx, &p->tab.fy, &p->tab.fz, &p->tab.sx,
                    &p->tab.sy, &p->tab.sz, &p->frames_host_dev, &p->geom, &p->status, &p->keys0,
                    &p->vals0, &p->keys1, &p->vals1, &p->hist, &p->scan_tmp, &p->bin_start,
                    &p->s_atom, &p->s_anchor, &p->s_t, &p->s_q, &p->qsum, &p->rho, &p->spec,
                    &p->fspec, &p->freal, &p->partE, &p->partX, &p->red, &p->redtmp, &p->qpart, &p->btab, &p->gtab, &p->gtabF, &p->partD, &p->krad,
                    &p->hspec, &p->hpart, &p->hred, &p->hdsum, &p->hscal};
  for (DevBuf *b : bufs) b->release();
  close_peers(p);
  p->xr_fwd.release();
  p->xr_inv.release();
  p->xr_fe.release();
  p->up.release();
  p->tr.release();
  delete p;
  return SOG_OK;
}

extern "C" int sog_plan_status(sog_plan *p, unsigned *bits) {
  if (!p || !bits) return fail(SOG_ERR_INVALID, "null argument");
  *bits = 0;
  if (!p->status.p) return SOG_OK;
  DeviceGuard dg(p->d.device);
  SOG_CUDA_TRY(cudaDeviceSynchronize());
  SOG_CUDA_TRY(cudaMemcpy(bits, p->status.p, sizeof(unsigned), cudaMemcpyDeviceToHost));
  SOG_CUDA_TRY(cudaMemset(p->status.p, 0, sizeof(unsigned)));
  return SOG_OK;
}

extern "C" int sog_mesh_forward(sog_plan *p, const sog_mesh_args *a, void *stream) {
  if (!p || !a) return fail(SOG_ERR_INVALID, "null argument");
  if (a->nframes <= 0) return SOG_OK;
  if (!a->atom_begin || !a->atom_count || !a->k_sq_max || !a->positions || !a->charges || !a->cells ||
      !a->amp || !a->bw2)
    return fail(SOG_ERR_INVALID, "missing input array");
  if (a->nchannels < 1) return fail(SOG_ERR_INVALID, "nchannels must be >= 1");
  if (a->n_gauss < 1 || a->n_gauss > kMaxGauss) return fail(SOG_ERR_INVALID, "n_gauss must be in [1, 64]");
  if (a->dedr && p->d.spline == SOG_SPLINE_CUBES2)
    return fail(SOG_ERR_UNSUPPORTED, "exact dE/dr is computed for the B-spline and QuadS meshes");
  DeviceGuard dg(p->d.device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p->d.dtype == SOG_DTYPE_F64) return mesh_forward_impl<double>(p, a, st);
  return mesh_forward_impl<float>(p, a, st);
}

extern "C" int sog_mesh_hvp(sog_plan *p, const sog_mesh_args *a, const sog_hvp_args *h, void *stream) {
  if (!p || !a || !h) return fail(SOG_ERR_INVALID, "null argument");
  if (a->nframes <= 0) return SOG_OK;
  if (!a->atom_begin || !a->atom_count || !a->k_sq_max || !a->positions || !a->charges || !a->cells ||
      !a->amp || !a->bw2)
    return fail(SOG_ERR_INVALID, "missing input array");
  if (!h->out_q || !h->out_r || !h->out_amp || !h->out_bw2) return fail(SOG_ERR_INVALID, "missing HVP output array");
  if (a->nchannels < 1) return fail(SOG_ERR_INVALID, "nchannels must be >= 1");
  if (a->n_gauss < 1 || a->n_gauss > kMaxGauss) return fail(SOG_ERR_INVALID, "n_gauss must be in [1, 64]");
  if (p->d.spline == SOG_SPLINE_CUBES2)
    return fail(SOG_ERR_UNSUPPORTED, "second derivatives are computed for the B-spline and QuadS meshes");
  DeviceGuard dg(p->d.device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p->d.dtype == SOG_DTYPE_F64) return mesh_hvp_impl<double>(p, a, h, st);
  return mesh_hvp_impl<float>(p, a, h, st);
}

// Checks the slab constraints of a plan for `size` ranks ("" when valid).
static std::string slab_check(const sog_plan *p, int size, int transport) {
  const sog_plan_desc &d = p->d;
  if (size < 1) return "slab size must be >= 1";
  if (transport == SOG_SLAB_PEER) {
    if (size > kMaxSlabRanks) return "the peer transport spans at most 8 ranks (one node)";
    if (!is_pow2(d.ny) || d.ny > 1024) return "the peer transport needs a power-of-two ny up to 1024";
  }
  if (!is_pow2(d.nz) || d.nz > 1024) return "slab mode needs a power-of-two nz up to 1024";
  if (d.nz % size || d.ny % size) return "nz and ny must be divisible by the number of ranks";
  const int zs = d.nz / size;
  if (zs % kBin) return "nz / ranks must be a multiple of 8";
  if (zs < d.order - 1) return "nz / ranks must be at least order - 1 (halo from one neighbour)";
  return "";
}

extern "C" int sog_mesh_slab_workspace(const sog_plan *p, int nfield, int size, int transport, size_t *bytes) {
  if (!p || !bytes) return fail(SOG_ERR_INVALID, "null argument");
  if (nfield < 0 || nfield > 4) return fail(SOG_ERR_INVALID, "nfield must be in [0, 4]");
  if (transport != SOG_SLAB_EXCHANGE && transport != SOG_SLAB_PEER) return fail(SOG_ERR_INVALID, "bad transport");
  const std::string why = slab_check(p, size, transport);
  if (!why.empty()) return fail(SOG_ERR_UNSUPPORTED, why);
  *bytes = slab_layout(p, nfield, size, transport).total;
  return SOG_OK;
}

extern "C" int sog_mesh_slab_forward(sog_plan *p, const sog_mesh_args *a, const sog_slab_desc *sd, void *stream) {
  if (!p || !a || !sd) return fail(SOG_ERR_INVALID, "null argument");
  if (a->nframes != 1) return fail(SOG_ERR_UNSUPPORTED, "slab mode solves exactly one frame per call");
  if (!a->atom_begin || !a->atom_count || !a->k_sq_max || !a->positions || !a->charges || !a->cells ||
      !a->amp || !a->bw2)
    return fail(SOG_ERR_INVALID, "missing input array");
  if (a->nchannels < 1 || a->nchannels > 8) return fail(SOG_ERR_INVALID, "slab mode takes 1..8 charge channels");
  if (a->n_gauss < 1 || a->n_gauss > kMaxGauss) return fail(SOG_ERR_INVALID, "n_gauss must be in [1, 64]");
  if (a->dedr) return fail(SOG_ERR_UNSUPPORTED, "slab mode computes explicit (ik) forces; exact dE/dr needs one device");
  if (a->grad_amp || a->grad_bw2 || a->virial)
    return fail(SOG_ERR_UNSUPPORTED, "slab mode computes energy, forces and dE/dq only");
  if (!sd->exchange || !sd->workspace) return fail(SOG_ERR_INVALID, "slab needs an exchange callback and a workspace");
  if (sd->rank < 0 || sd->rank >= sd->size) return fail(SOG_ERR_INVALID, "slab rank out of range");
  if (sd->transport != SOG_SLAB_EXCHANGE && sd->transport != SOG_SLAB_PEER) return fail(SOG_ERR_INVALID, "bad transport");
  const std::string why = slab_check(p, sd->size, sd->transport);
  if (!why.empty()) return fail(SOG_ERR_UNSUPPORTED, why);
  DeviceGuard dg(p->d.device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p->d.dtype == SOG_DTYPE_F64) return mesh_slab_impl<double>(p, a, sd, st);
  return mesh_slab_impl<float>(p, a, sd, st);
}
