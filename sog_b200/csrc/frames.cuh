// Per-frame kernels shared by the mesh and direct solvers: geometry set-up,
// charge sums, deterministic partial-sum reduction, energy / gradient /
// virial finalisation and the per-atom potential epilogue.
#pragma once
#include <algorithm>
#include <cfloat>

#include "common.cuh"

namespace sogb {
namespace {

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------------
// frame set-up
// ------------------------------------------------------------------------
// c2xi > 0: CubeS2 with that xi (its Green factor exp(sum_a sig2_a k_a^2)
// uses sig_a = xi |a_alpha| / n_alpha, cubes2_fft.py:1039-1045; no aliasing).
template <typename T>
__global__ void k_frame_setup(const T *__restrict__ cells, const FrameHost *__restrict__ fh,
                              FrameGeom *__restrict__ geom, int nf, int kconv, int nx, int ny,
                              int nz, unsigned *status, double c2xi = 0.0) {
  const int f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= nf) return;
  FrameGeom g;
  double c[9];
  for (int i = 0; i < 9; ++i) c[i] = (double)cells[(int64_t)f * 9 + i];
  const double A = c[4] * c[8] - c[5] * c[7], B = -(c[3] * c[8] - c[5] * c[6]),
               Cc = c[3] * c[7] - c[4] * c[6];
  const double det = c[0] * A + c[1] * B + c[2] * Cc;
  double vol = fabs(det);
  if (!(vol > DBL_EPSILON) || !isfinite(vol)) {
    raise_status(status, kStatusBadCell);
    vol = 1.0;
  }
  const double id = (det != 0.0 && isfinite(det)) ? 1.0 / det : 0.0;
  double ci[9];
  ci[0] = A * id;  ci[1] = -(c[1] * c[8] - c[2] * c[7]) * id; ci[2] = (c[1] * c[5] - c[2] * c[4]) * id;
  ci[3] = B * id;  ci[4] = (c[0] * c[8] - c[2] * c[6]) * id;  ci[5] = -(c[0] * c[5] - c[2] * c[3]) * id;
  ci[6] = Cc * id; ci[7] = -(c[0] * c[7] - c[1] * c[6]) * id; ci[8] = (c[0] * c[4] - c[1] * c[3]) * id;
  const double tp = 2.0 * kPi;
  for (int i = 0; i < 9; ++i) { g.cell[i] = c[i]; g.cinv[i] = ci[i]; }
  for (int a = 0; a < 3; ++a)
    for (int b = 0; b < 3; ++b) g.kmat[a * 3 + b] = tp * (kconv ? ci[b * 3 + a] : ci[a * 3 + b]);
  g.vol = vol;
  // reciprocal vectors b_i = 2 pi (a_j x a_k) / V   (gaussian.py:774-782)
  const double *a1 = c, *a2 = c + 3, *a3 = c + 6;
  double bb[3][3] = {{a2[1] * a3[2] - a2[2] * a3[1], a2[2] * a3[0] - a2[0] * a3[2], a2[0] * a3[1] - a2[1] * a3[0]},
                     {a3[1] * a1[2] - a3[2] * a1[1], a3[2] * a1[0] - a3[0] * a1[2], a3[0] * a1[1] - a3[1] * a1[0]},
                     {a1[1] * a2[2] - a1[2] * a2[1], a1[2] * a2[0] - a1[0] * a2[2], a1[0] * a2[1] - a1[1] * a2[0]}};
  double kmin2 = 1e300;
  for (int i = 0; i < 3; ++i) {
    double s = 0.0;
    for (int k = 0; k < 3; ++k) { const double v = tp * bb[i][k] / vol; s += v * v; }
    kmin2 = fmin(kmin2, s);
  }
  g.kmin2 = kmin2;
  g.k_sq_max = fh[f].k_sq_max;
  const double kmax = sqrt(fmax(g.k_sq_max, 0.0));
  for (int a = 0; a < 3; ++a) {
    double s = 0.0;
    for (int b = 0; b < 3; ++b) { const double v = kconv ? c[b * 3 + a] : c[a * 3 + b]; s += v * v; }
    g.abound[a] = sqrt(s) * kmax / tp + 1e-9;
  }
  g.scale = (double)nx * (double)ny * (double)nz / vol;
  g.atom_begin = fh[f].atom_begin;
  g.slot_base = fh[f].slot_base;
  g.natoms = (int32_t)fh[f].natoms;
  // Alias flag.  Every non-zero alias displacement 2 pi (N o j) has length at
  // least min_a 2 pi N_a / |v_a| (v_a: lattice row, or cell column for the
  // reference convention).  If that exceeds 2 k_max no alias of a mode inside
  // the k_max sphere is inside it, and the B-spline Green reduces to its
  // principal term: the plugin's alias fast path (lmp/sog.cpp:1370-1374).
  {
    const int n3[3] = {nx, ny, nz};
    double lmin = 1e300;
    for (int a = 0; a < 3; ++a) {
      double s = 0.0;
      for (int b = 0; b < 3; ++b) { const double v = kconv ? c[b * 3 + a] : c[a * 3 + b]; s += v * v; }
      lmin = fmin(lmin, tp * (double)n3[a] / sqrt(s));
    }
    g.pad = (lmin > 2.0 * kmax) ? 0 : 1;
  }
  g.ortho = (g.kmat[1] == 0.0 && g.kmat[2] == 0.0 && g.kmat[3] == 0.0 && g.kmat[5] == 0.0 &&
             g.kmat[6] == 0.0 && g.kmat[7] == 0.0) ? 1 : 0;
  g.pad2 = 0;
  {
    const int n3[3] = {nx, ny, nz};
    for (int a = 0; a < 3; ++a) {
      const double la = sqrt(c[3 * a] * c[3 * a] + c[3 * a + 1] * c[3 * a + 1] + c[3 * a + 2] * c[3 * a + 2]);
      const double s = c2xi * la / (double)n3[a];
      g.sig2[a] = s * s;
    }
    if (c2xi > 0.0) g.pad = 0;
  }
  geom[f] = g;
}

// per (frame, channel, split): partial sums of q and q^2 over a contiguous
// chunk of the frame's atoms (fixed-order tree); reduced by reduce_parts.
template <typename T>
__global__ void k_qsums(const T *__restrict__ q, int nch, const FrameGeom *__restrict__ geom,
                        double *__restrict__ part, const T *__restrict__ pos = nullptr,
                        unsigned *status = nullptr) {
  const int f = blockIdx.x, c = blockIdx.y, z = blockIdx.z, nz = gridDim.z;
  const FrameGeom &g = geom[f];
  const int64_t chunk = ((int64_t)g.natoms + nz - 1) / nz;
  const int64_t i0 = (int64_t)z * chunk, i1 = min((int64_t)g.natoms, i0 + chunk);
  double s1 = 0.0, s2 = 0.0;
  bool bad = false;
  for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    double v = (double)q[(g.atom_begin + i) * nch + c];
    if (!isfinite(v)) { v = 0.0; bad = true; }
    // positions checked once, by the channel-0 blocks (when a status word is given)
    if (status && c == 0) {
      const T *r = pos + (g.atom_begin + i) * 3;
      if (!isfinite((double)r[0]) || !isfinite((double)r[1]) || !isfinite((double)r[2])) bad = true;
    }
    s1 += v;
    s2 += v * v;
  }
  if (bad && status) raise_status(status, kStatusNonFinite);
  __shared__ double r1[256], r2[256];
  r1[threadIdx.x] = s1;
  r2[threadIdx.x] = s2;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) { r1[threadIdx.x] += r1[threadIdx.x + o]; r2[threadIdx.x] += r2[threadIdx.x + o]; }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    double *p = part + (((int64_t)c * gridDim.x + f) * nz + z) * 2;
    p[0] = r1[0];
    p[1] = r2[0];
  }
}

// ------------------------------------------------------------------------
// reductions and finalisation
// ------------------------------------------------------------------------
// Sums partial results part[((c*nf + f)*nblk + b)*stride + i] over b in fixed
// order.  With gridDim.z > 1 each z sums a contiguous chunk of b and writes
// the same partial layout (nblk = gridDim.z, stride = nacc) for a second pass;
// with gridDim.z == 1 it writes out[(f*nch + c)*nacc + i].
__global__ void k_reduce_parts(const double *__restrict__ part, int nf, int nch, int64_t nblk,
                               int stride, int nacc, double *__restrict__ out) {
  const int f = blockIdx.x, c = blockIdx.y, z = blockIdx.z, nz = gridDim.z;
  const int64_t chunk = (nblk + nz - 1) / nz;
  const int64_t b0 = (int64_t)z * chunk, b1 = min(nblk, b0 + chunk);
  __shared__ double sh[256];
  for (int i = 0; i < nacc; ++i) {
    double s = 0.0;
    const double *p = part + (((int64_t)c * nf + f) * nblk) * stride + i;
    for (int64_t b = b0 + threadIdx.x; b < b1; b += blockDim.x) s += p[b * stride];
    sh[threadIdx.x] = s;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
      if (threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      if (nz > 1) out[(((int64_t)c * nf + f) * nz + z) * nacc + i] = sh[0];
      else out[((int64_t)f * nch + c) * nacc + i] = sh[0];
    }
    __syncthreads();
  }
}

// Two-level deterministic reduction (split chosen from the sizes only).
inline int reduce_split(int64_t nblk) {
  int64_t s = (nblk + 2047) / 2048;
  return (int)std::max<int64_t>(1, std::min<int64_t>(s, 512));
}

// Few partials per (frame, channel): one thread per accumulated value adds its
// nblk partials in order (many small frames would otherwise spend a
// 256-thread tree and its barriers on each of nacc values).
__global__ void k_reduce_parts_few(const double *__restrict__ part, int nf, int nch, int64_t nblk,
                                   int stride, int nacc, double *__restrict__ out) {
  const int f = blockIdx.x, c = blockIdx.y;
  const double *p = part + (((int64_t)c * nf + f) * nblk) * stride;
  for (int i = threadIdx.x; i < nacc; i += blockDim.x) {
    double s = 0.0;
    for (int64_t b = 0; b < nblk; ++b) s += p[b * stride + i];
    out[((int64_t)f * nch + c) * nacc + i] = s;
  }
}

inline void reduce_parts(const double *part, int nf, int nch, int64_t nblk, int stride, int nacc,
                         double *out, double *tmp, cudaStream_t st) {
  const int split = reduce_split(nblk);
  if (nblk <= 16) {
    k_reduce_parts_few<<<dim3(nf, nch, 1), 64, 0, st>>>(part, nf, nch, nblk, stride, nacc, out);
    return;
  }
  if (split == 1) {
    k_reduce_parts<<<dim3(nf, nch, 1), 256, 0, st>>>(part, nf, nch, nblk, stride, nacc, out);
    return;
  }
  k_reduce_parts<<<dim3(nf, nch, split), 256, 0, st>>>(part, nf, nch, nblk, stride, nacc, tmp);
  k_reduce_parts<<<dim3(nf, nch, 1), 256, 0, st>>>(tmp, nf, nch, split, nacc, nacc, out);
}

inline int64_t reduce_tmp_elems(int nf, int nch, int64_t nblk, int nacc) {
  return (int64_t)nf * nch * reduce_split(nblk) * nacc;
}

struct FinalArgs {
  const FrameGeom *geom;
  const double *redE;    // [nf][C][2]
  const double *redX;    // [nf][C][4M+13] or null
  const double *redD;    // [nf] self sums (sum_w gS) when not in redE, or null
  const double *qsum;    // [nf][C][2]
  const void *amp, *bw2;
  int M, nch, nx, ny, nz;
  double norm, self_coeff, lambda;
  int remove_self, k0;
  int want_grad, want_vir;
  int direct;            // 1: sums are sum_half 2 K |S|^2 (scale 1/2V); 0: mesh (V/2 N^-2)
  void *energy, *grad_amp, *grad_bw2, *virial;
  double *fscal;         // [nf][4]: diag, kfe, Q, (unused)
};

template <typename T>
__global__ void k_finalize_frames(FinalArgs a, int nf) {
  const int f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= nf) return;
  const FrameGeom &g = a.geom[f];
  const double V = g.vol;
  const double N3 = (double)a.nx * a.ny * a.nz;
  const double sc = a.direct ? 1.0 / (2.0 * V) : 0.5 * V / (N3 * N3);
  const T *amp = (const T *)a.amp;
  const T *bw2 = (const T *)a.bw2;
  // self sum sum_w gS: from the Green-table pass (redD) and / or from the
  // pass that evaluated the Green function on the fly (channel 0's second sum)
  const double diag = ((a.redD ? a.redD[f] : 0.0) + a.redE[((int64_t)f * a.nch + 0) * 2 + 1]) / (2.0 * V);
  double E = 0.0, Q = 0.0, QQ = 0.0, pen = 0.0;
  for (int c = 0; c < a.nch; ++c) {
    const double qs = a.qsum[((int64_t)f * a.nch + c) * 2 + 0];
    const double qq = a.qsum[((int64_t)f * a.nch + c) * 2 + 1];
    double e = sc * a.redE[((int64_t)f * a.nch + c) * 2 + 0];
    if (a.remove_self) e -= qq * diag;
    if (a.self_coeff != 0.0) e -= qq * a.self_coeff;
    E += e;
    Q += qs;
    QQ += qq;
    if (g.natoms > 0) { const double mean = qs / g.natoms; pen += mean * mean; }
  }
  E *= a.norm;
  double kfe = 0.0;
  if (a.k0) {
    for (int m = 0; m < a.M; ++m) kfe += (double)amp[m] * exp(-0.5 * (double)bw2[m] * g.kmin2);
    E += kfe * Q * Q / (2.0 * V) * a.norm;
    if (a.remove_self) E -= kfe * QQ / (2.0 * V) * a.norm;
  }
  if (a.lambda > 0.0) E += a.lambda * pen;
  if (a.energy) ((T *)a.energy)[f] = (T)E;
  a.fscal[f * 4 + 0] = diag;
  a.fscal[f * 4 + 1] = kfe;
  a.fscal[f * 4 + 2] = Q;
  a.fscal[f * 4 + 3] = 0.0;
  const int M = a.M;
  const int nacc = 4 * M + 13;
  if (a.want_grad) {
    for (int m = 0; m < M; ++m) {
      double ga = 0.0, gb = 0.0;
      for (int c = 0; c < a.nch; ++c) {
        const double *x = a.redX + ((int64_t)f * a.nch + c) * nacc;
        const double qq = a.qsum[((int64_t)f * a.nch + c) * 2 + 1];
        double va = sc * x[m], vb = sc * x[2 * M + m];
        if (a.remove_self) {
          va -= qq * x[M + m] / (2.0 * V);
          vb -= qq * x[3 * M + m] / (2.0 * V);
        }
        ga += va;
        gb += vb;
      }
      ga *= a.norm;
      gb *= a.norm;
      if (a.k0) {
        const double em = exp(-0.5 * (double)bw2[m] * g.kmin2);
        double cA = Q * Q / (2.0 * V) * a.norm;
        if (a.remove_self) cA -= QQ / (2.0 * V) * a.norm;
        ga += em * cA;
        gb += (double)amp[m] * em * (-0.5 * g.kmin2) * cA;
      }
      if (a.grad_amp) ((T *)a.grad_amp)[(int64_t)f * M + m] = (T)ga;
      if (a.grad_bw2) ((T *)a.grad_bw2)[(int64_t)f * M + m] = (T)gb;
    }
  }
  if (a.want_vir && a.virial) {
    const int comp[3][3] = {{0, 3, 4}, {3, 1, 5}, {4, 5, 2}};
    double W[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
    const double pref = a.norm * sc;
    for (int c = 0; c < a.nch; ++c) {
      const double *x = a.redX + ((int64_t)f * a.nch + c) * nacc + 4 * M;
      const double qq = a.qsum[((int64_t)f * a.nch + c) * 2 + 1];
      for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) {
          double w = -pref * x[1 + comp[i][j]];
          if (i == j) w += pref * x[0];
          if (a.remove_self) {
            w += qq * a.norm / (2.0 * V) * x[7 + comp[i][j]];
            if (i == j) w -= qq * a.norm * diag;
          }
          W[i * 3 + j] += w;
        }
    }
    for (int i = 0; i < 9; ++i) ((T *)a.virial)[(int64_t)f * 9 + i] = (T)W[i];
  }
}

// potential: dE/dq = norm * (gathered - 2 q (rsi*diag + self)) + k=0 / penalty terms
// dE/dq of one atom from its raw potential (all channels): self and k=0
// terms, the neutrality penalty, times norm (cubes2_fft.py:536-583,
// gaussian.py:784-798).
template <typename T>
__device__ __forceinline__ void finalize_atom_pot(const FrameGeom &g, const double *__restrict__ fscal, int f,
                                                  const double *__restrict__ qsum, const T *__restrict__ q,
                                                  T *__restrict__ pot, int64_t atom, int nch, double norm,
                                                  double self_coeff, double lambda, int remove_self, int k0) {
  const double diag = fscal[f * 4 + 0], kfe = fscal[f * 4 + 1], Q = fscal[f * 4 + 2];
  for (int c = 0; c < nch; ++c) {
    const double qi = (double)q[atom * nch + c];
    double v = (double)pot[atom * nch + c];
    if (remove_self) v -= 2.0 * qi * diag;
    if (self_coeff != 0.0) v -= 2.0 * qi * self_coeff;
    v *= norm;
    if (k0) {
      v += kfe * 2.0 * Q / (2.0 * g.vol) * norm;
      if (remove_self) v -= kfe * 2.0 * qi / (2.0 * g.vol) * norm;
    }
    if (lambda > 0.0 && g.natoms > 0) {
      const double mean = qsum[((int64_t)f * nch + c) * 2 + 0] / g.natoms;
      v += lambda * 2.0 * mean / g.natoms;
    }
    pot[atom * nch + c] = (T)v;
  }
}

template <typename T>
__global__ void k_finalize_atoms(const FrameGeom *__restrict__ geom, const double *__restrict__ fscal,
                                 const double *__restrict__ qsum, const T *__restrict__ q,
                                 T *__restrict__ pot, int nch, double norm, double self_coeff,
                                 double lambda, int remove_self, int k0) {
  const int f = blockIdx.y;
  const FrameGeom &g = geom[f];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= g.natoms) return;
  finalize_atom_pot<T>(g, fscal, f, qsum, q, pot, g.atom_begin + i, nch, norm, self_coeff, lambda, remove_self,
                       k0);
}

// Frame table passed by value (small calls): written to device memory by
// the first kernel of the call, with no pinned staging buffer and no host wait.
constexpr int kFramesByValue = 32;
struct FrameTable {
  FrameHost fh[kFramesByValue];
  int nf;
};

__global__ void k_store_frames(const FrameTable t, FrameHost *__restrict__ dst) {
  for (int f = threadIdx.x; f < t.nf; f += blockDim.x) dst[f] = t.fh[f];
}

template <typename T>
__global__ void k_zero(T *p, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = T(0);
}


}  // namespace

// ------------------------------------------------------------------------
// Hessian-vector products: the terms every solver shares (direction sums,
// the self / k=0 / penalty terms, parameter rows).  The per-frame mode sums
// D0..D2 of exp(-bw2_m k^2 / 2) (weights as the solver's own self sum) come
// with the solver's core parameter rows in hred.
// ------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ double ldir(const void *p, int64_t i) {
  return p ? (double)static_cast<const T *>(p)[i] : 0.0;
}

// direction sums per frame and channel: sum a, sum q a
template <typename T>
__global__ void k_hvp_dsums(const T *__restrict__ q, const void *dq, int nch, const FrameGeom *__restrict__ geom,
                            double *__restrict__ out) {
  const int f = blockIdx.x, c = blockIdx.y;
  const FrameGeom &g = geom[f];
  double s1 = 0.0, s2 = 0.0;
  for (int64_t i = threadIdx.x; i < g.natoms; i += blockDim.x) {
    const int64_t o = (g.atom_begin + i) * nch + c;
    const double av = ldir<T>(dq, o);
    s1 += av;
    s2 += (double)q[o] * av;
  }
  __shared__ double r1[256], r2[256];
  r1[threadIdx.x] = s1;
  r2[threadIdx.x] = s2;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) { r1[threadIdx.x] += r1[threadIdx.x + o]; r2[threadIdx.x] += r2[threadIdx.x + o]; }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    out[((int64_t)f * nch + c) * 2 + 0] = r1[0];
    out[((int64_t)f * nch + c) * 2 + 1] = r2[0];
  }
}

struct HvpFinal {
  const FrameGeom *geom;
  const double *hred;   // [nf][5M]: theta rows (amp, bw2), D0, D1, D2 (half-space weight 2)
  const double *qsum;   // [nf][C][2] sum q, sum q^2
  const double *dsum;   // [nf][C][2] sum a, sum q a
  const void *amp, *bw2, *damp, *dbw2;
  void *oamp, *obw2;
  double *scal;         // [nf][8] per-frame scalars for the atom pass
  int M, nch;
  double norm, self_coeff, lambda;
  int remove_self, k0;
};

// Parameter rows of H d per frame (core + self + k=0 terms) and the scalars
// of the charge rows' self / k=0 / penalty terms.
//   self:  E_s = -norm (rs D + self_coeff) sum_c |q_c|^2,  D = sum_m amp_m D0_m / 2V
//   k=0:   E_0 = norm kfe (Q^2 - rs QQ) / 2V,  kfe = sum_m amp_m exp(-bw2_m kmin^2 / 2)
//   pen:   E_p = lambda sum_c mean_c(q)^2
template <typename T>
__global__ void k_hvp_finalize_frames(HvpFinal a, int nf) {
  const int f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= nf) return;
  const FrameGeom &g = a.geom[f];
  const double V = g.vol, i2v = 1.0 / (2.0 * V);
  const int M = a.M;
  const T *amp = (const T *)a.amp, *bw2 = (const T *)a.bw2;
  const double *x = a.hred + (int64_t)f * 5 * M;
  const double *D0 = x + 2 * M, *D1 = x + 3 * M, *D2 = x + 4 * M;
  double Q = 0, QQ = 0, A = 0, QA = 0;
  for (int c = 0; c < a.nch; ++c) {
    Q += a.qsum[((int64_t)f * a.nch + c) * 2 + 0];
    QQ += a.qsum[((int64_t)f * a.nch + c) * 2 + 1];
    A += a.dsum[((int64_t)f * a.nch + c) * 2 + 0];
    QA += a.dsum[((int64_t)f * a.nch + c) * 2 + 1];
  }
  const double rs = a.remove_self ? 1.0 : 0.0;
  const double kmin2 = g.kmin2;
  double diag = 0.0, ddiag = 0.0, kfe = 0.0, dkfe = 0.0;
  for (int m = 0; m < M; ++m) {
    const double am = (double)amp[m], ca = ldir<T>(a.damp, (int64_t)f * M + m), cb = ldir<T>(a.dbw2, (int64_t)f * M + m);
    const double Em = exp(-0.5 * (double)bw2[m] * kmin2);
    diag += am * D0[m] * i2v;
    ddiag += (ca * D0[m] + cb * am * D1[m]) * i2v;
    kfe += am * Em;
    dkfe += ca * Em + cb * am * (-0.5 * kmin2) * Em;
  }
  for (int m = 0; m < M; ++m) {
    const double am = (double)amp[m], ca = ldir<T>(a.damp, (int64_t)f * M + m), cb = ldir<T>(a.dbw2, (int64_t)f * M + m);
    const double Em = exp(-0.5 * (double)bw2[m] * kmin2);
    // core rows (the half-space sums carry 2, E carries 1/2V)
    double ga = a.norm * i2v * x[m], gb = a.norm * i2v * x[M + m];
    // self term: d/dtheta of -norm rs QQ D, along the direction
    const double dD_a = D0[m] * i2v, dD_b = am * D1[m] * i2v;          // dD/damp_m, dD/dbw2_m
    const double hD_a = cb * D1[m] * i2v;                               // (d2 D . c)_amp_m
    const double hD_b = (ca * D1[m] + cb * am * D2[m]) * i2v;           // (d2 D . c)_bw2_m
    ga += -a.norm * rs * (2.0 * QA * dD_a + QQ * hD_a);
    gb += -a.norm * rs * (2.0 * QA * dD_b + QQ * hD_b);
    if (a.k0) {
      const double dk_a = Em, dk_b = am * (-0.5 * kmin2) * Em;
      const double hk_a = cb * (-0.5 * kmin2) * Em;
      const double hk_b = ca * (-0.5 * kmin2) * Em + cb * am * 0.25 * kmin2 * kmin2 * Em;
      const double lin = 2.0 * Q * A - 2.0 * rs * QA, quad = Q * Q - rs * QQ;
      ga += a.norm * i2v * (dk_a * lin + hk_a * quad);
      gb += a.norm * i2v * (dk_b * lin + hk_b * quad);
    }
    ((T *)a.oamp)[(int64_t)f * M + m] = (T)ga;
    ((T *)a.obw2)[(int64_t)f * M + m] = (T)gb;
  }
  double *s = a.scal + (int64_t)f * 8;
  s[0] = rs * diag + a.self_coeff;
  s[1] = rs * ddiag;
  s[2] = a.k0 ? kfe : 0.0;
  s[3] = a.k0 ? dkfe : 0.0;
  s[4] = Q;
  s[5] = A;
  s[6] = rs;
  s[7] = 0.0;
}

// Charge rows: self, k=0 and penalty terms added to the core term.
template <typename T>
__global__ void k_hvp_finalize_atoms(const FrameGeom *__restrict__ geom, const double *__restrict__ scal,
                                     const double *__restrict__ dsum, const T *__restrict__ q, const void *dq,
                                     T *__restrict__ oq, int nch, double norm, double lambda) {
  const int f = blockIdx.y;
  const FrameGeom &g = geom[f];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= g.natoms) return;
  const double *s = scal + (int64_t)f * 8;
  const double i2v = 1.0 / (2.0 * g.vol);
  const int64_t atom = g.atom_begin + i;
  for (int c = 0; c < nch; ++c) {
    const int64_t o = atom * nch + c;
    const double qi = (double)q[o], ai = ldir<T>(dq, o);
    double v = (double)oq[o];
    v += -2.0 * norm * (ai * s[0] + qi * s[1]);
    v += norm * i2v * (s[2] * (2.0 * s[5] - 2.0 * s[6] * ai) + s[3] * (2.0 * s[4] - 2.0 * s[6] * qi));
    if (lambda > 0.0 && g.natoms > 0)
      v += 2.0 * lambda * dsum[((int64_t)f * nch + c) * 2 + 0] / ((double)g.natoms * g.natoms);
    oq[o] = (T)v;
  }
}

}  // namespace sogb
